// dit_forward.cu — the parts of one RF-DiT Euler step around the blocks
// (sampler.c:238-297, dit.c:488-541, 1070-1090), resident on the device:
//
//   conditioner  timestep embedding -> linear, silu -> linear, silu -> linear
//                (dit.c:488-530), computed once per step: every row of a step
//                shares the timestep (sampler.c:246-253)
//   input        x_t [R*S, 32] -> [R*S, D] (dit.c:532-541), each output row
//                stored to the request's CFG rows (sampler.c:256-262)
//   blocks       iro_dit_block_dev, one context block per request shared by
//                its CFG rows (sampler.c:219-224)
//   output       RMSNorm + linear D -> 32 (dit.c:1070-1090)
//   update       CFG combination and Euler step (sampler.c:283-297)
//
// The plain fp32 linears (conditioner, input, output) sum each output in the
// reference's order (iro_linear_scalar, ops.c:221-234: a running sum over k,
// then the bias), without fused multiply-adds, so they reproduce the IEEE
// build of the reference bit for bit given the same inputs; the timestep
// embedding and silu go through CUDA's expf/cosf/sinf.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "dit_block.cuh"
#include "runtime.cuh"

namespace iro {
namespace {

// y[M, N] = x[M, K] . w[N, K]^T (+ bias), optional silu on y (in place of
// the reference's separate iro_silu_inplace).  BM x BN output tile per
// 256-thread block, TM x TN outputs per thread, k in increasing order.
constexpr int kLK = 16;

template <int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__(256) linear_ref_kernel(const float* __restrict__ x,
                                                         const float* __restrict__ w,
                                                         const float* __restrict__ bias,
                                                         float* __restrict__ y, int M, int N, int K,
                                                         int silu, int ex_cfg, int ex_S) {
  static_assert((BM / TM) * (BN / TN) == 256, "256 threads");
  __shared__ float xs[kLK][BM + 1];
  __shared__ float ws[kLK][BN + 1];
  const int tx = threadIdx.x % (BN / TN), ty = threadIdx.x / (BN / TN);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += kLK) {
    for (int i = threadIdx.x; i < BM * kLK; i += 256) {
      const int r = i / kLK, kk = i % kLK;
      const int m = m0 + r, k = k0 + kk;
      xs[kk][r] = (m < M && k < K) ? x[(size_t)m * K + k] : 0.0f;
    }
    for (int i = threadIdx.x; i < BN * kLK; i += 256) {
      const int r = i / kLK, kk = i % kLK;
      const int n = n0 + r, k = k0 + kk;
      ws[kk][r] = (n < N && k < K) ? w[(size_t)n * K + k] : 0.0f;
    }
    __syncthreads();
    const int kn = min(kLK, K - k0);
    for (int kk = 0; kk < kn; kk++) {
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++)
          acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xs[kk][ty * TM + i], ws[kk][tx * TN + j]));
    }
    __syncthreads();
  }
  // A thread's TN consecutive outputs of a row go out as one vector store
  // when they are whole and aligned (TN = 4, N % 4 == 0).
  const bool vec = TN == 4 && (N & 3) == 0 && n0 + tx * TN + TN <= N &&
                   (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
#pragma unroll
  for (int i = 0; i < TM; i++) {
    const int m = m0 + ty * TM + i;
    if (m >= M) continue;
    float v[TN];
#pragma unroll
    for (int j = 0; j < TN; j++) {
      const int n = n0 + tx * TN + j;
      v[j] = 0.0f;
      if (n >= N) continue;
      v[j] = __fadd_rn(acc[i][j], bias ? bias[n] : 0.0f);
      if (silu) v[j] = __fdiv_rn(v[j], __fadd_rn(1.0f, expf(-v[j])));
    }
    const int c0 = n0 + tx * TN;
    const size_t r = (size_t)(m / ex_S), t = (size_t)(m % ex_S);
    const int copies = ex_cfg <= 1 ? 1 : ex_cfg;
    for (int c = 0; c < copies; c++) {
      float* yrow = ex_cfg <= 1 ? y + (size_t)m * N : y + ((r * ex_cfg + c) * ex_S + t) * N;
      if (vec) {
        *reinterpret_cast<float4*>(yrow + c0) = make_float4(v[0], v[1 % TN], v[2 % TN], v[3 % TN]);
      } else {
#pragma unroll
        for (int j = 0; j < TN; j++)
          if (c0 + j < N) yrow[c0 + j] = v[j];
      }
    }
  }
}

// y[M, N] = x[M, K] . w[N, K]^T (+ bias) for a few rows (the conditioner):
// one warp per (row, 32 outputs) and one warp per block, so the warps spread
// over the SMs; lane j sums output n0 + j in increasing k (the reference's
// order) with float4 loads of its own weight row and the broadcast input row.
__global__ void __launch_bounds__(32) linear_rows_kernel(const float* __restrict__ x,
                                                          const float* __restrict__ w,
                                                          const float* __restrict__ bias,
                                                          float* __restrict__ y, int M, int N,
                                                          int K, int silu) {
  const int ngroups = (N + 31) / 32;
  const long long gw = blockIdx.x;
  if (gw >= (long long)M * ngroups) return;
  const int m = (int)(gw / ngroups), n = (int)(gw % ngroups) * 32 + (threadIdx.x & 31);
  const bool active = n < N;
  const float* xr = x + (size_t)m * K;
  const float* wr = w + (size_t)(active ? n : 0) * K;
  float acc = 0.0f;
  if ((K & 3) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const float4* w4 = reinterpret_cast<const float4*>(wr);
#pragma unroll 8
    for (int k = 0; k < K / 4; k++) {
      const float4 a = x4[k], b = w4[k];
      acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
      acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
      acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
      acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
    }
  } else {
    for (int k = 0; k < K; k++) acc = __fadd_rn(acc, __fmul_rn(xr[k], wr[k]));
  }
  if (!active) return;
  float v = __fadd_rn(acc, bias ? bias[n] : 0.0f);
  if (silu) v = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
  y[(size_t)m * N + n] = v;
}

// y[M, 32] = x[M, K] . w[32, K]^T (+ bias), the output head, on a persistent
// grid: W^T staged in shared memory once per block ([K][32], 128 KB for
// K = 1024); groups of 128 input rows stream through shared memory in chunks
// of 32 k by cp.async, double-buffered so the next chunk lands while this one
// is summed.  Each warp sums 8 rows: lane j holds output j of its rows, in
// increasing k (the reference's order), reading W^T[k][j] from a
// conflict-free 128-byte row and the rows' x[k .. k+3] as broadcasts.
constexpr size_t kNarrowSmemMax = 160 * 1024;  // W^T
constexpr int kNarrowRows = 128;               // rows per group (16 warps x 8)
constexpr int kNarrowKC = 32;                  // k per staged chunk
constexpr int kNarrowThreads = 512;
constexpr size_t kNarrowXBytes = 2 * kNarrowRows * kNarrowKC * sizeof(float);  // 32 KB

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

__global__ void __launch_bounds__(kNarrowThreads, 1) linear_narrow_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
    float* __restrict__ y, int M, int K, int silu) {
  extern __shared__ float4 narrow_smem[];
  float* wt = reinterpret_cast<float*>(narrow_smem);  // [K][32]
  float* xs = wt + (size_t)K * 32;                    // [2][kNarrowRows][kNarrowKC]
  for (int i = threadIdx.x; i < K * 32; i += kNarrowThreads) {
    const int n = i & 31, k = i >> 5;
    wt[i] = w[(size_t)n * K + k];
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float b = bias ? bias[lane] : 0.0f;
  const int nk = (K + kNarrowKC - 1) / kNarrowKC;
  // Each block owns one contiguous share of the rows (the last group of a
  // share may be partial), so no block sums more than ceil(M / grid) rows.
  const int share = (M + gridDim.x - 1) / gridDim.x;
  const int rbeg = blockIdx.x * share, rend = min(M, rbeg + share);
  // One chunk: 128 rows x 32 floats = 1024 16-byte pieces, two per thread
  // (rows past the share repeat its last row; their sums are not stored).
  auto stage = [&](int g0, int kc, int buf) {
    const int kw = min(kNarrowKC, K - kc * kNarrowKC) / 4;  // float4 per row in this chunk
    for (int i = threadIdx.x; i < kNarrowRows * (kNarrowKC / 4); i += kNarrowThreads) {
      const int r = i / (kNarrowKC / 4), c4 = i % (kNarrowKC / 4);
      if (c4 < kw) {
        const int row = min(g0 + r, rend - 1);
        cp_async16(xs + ((size_t)buf * kNarrowRows + r) * kNarrowKC + 4 * c4,
                   x + (size_t)row * K + (size_t)kc * kNarrowKC + 4 * c4);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int g0 = rbeg; g0 < rend; g0 += kNarrowRows) {
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; r++) acc[r] = 0.0f;
    __syncthreads();  // W^T staged; the previous group's last chunk is read
    stage(g0, 0, 0);
    for (int kc = 0; kc < nk; kc++) {
      if (kc + 1 < nk) {
        stage(g0, kc + 1, (kc + 1) & 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      }
      __syncthreads();
      const float* xb = xs + ((size_t)(kc & 1) * kNarrowRows + warp * 8) * kNarrowKC;
      const float* wb = wt + (size_t)kc * kNarrowKC * 32 + lane;
      const int kl = min(kNarrowKC, K - kc * kNarrowKC);
      // Warps whose 8 rows all lie past the block's share (the tail of a
      // partial group) skip the sums.
      if (g0 + warp * 8 < rend) {
        for (int k = 0; k < kl; k += 4) {
          const float w0 = wb[(k + 0) * 32], w1 = wb[(k + 1) * 32];
          const float w2 = wb[(k + 2) * 32], w3 = wb[(k + 3) * 32];
#pragma unroll
          for (int r = 0; r < 8; r++) {
            const float4 a = *reinterpret_cast<const float4*>(xb + r * kNarrowKC + k);
            acc[r] = __fadd_rn(acc[r], __fmul_rn(a.x, w0));
            acc[r] = __fadd_rn(acc[r], __fmul_rn(a.y, w1));
            acc[r] = __fadd_rn(acc[r], __fmul_rn(a.z, w2));
            acc[r] = __fadd_rn(acc[r], __fmul_rn(a.w, w3));
          }
        }
      }
      __syncthreads();  // this buffer is staged over two chunks from now
    }
#pragma unroll
    for (int r = 0; r < 8; r++) {
      const int m = g0 + warp * 8 + r;
      if (m >= rend) break;
      float v = __fadd_rn(acc[r], b);
      if (silu) v = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
      y[(size_t)m * 32 + lane] = v;
    }
  }
}

// ex_cfg > 1: output row m is written to the ex_cfg rows
// ((m / ex_S) * ex_cfg + c) * ex_S + m % ex_S (one request's row broadcast to
// its CFG rows, sampler.c:256-262).
int linear_ref(const float* x, const float* w, const float* bias, float* y, int M, int N, int K,
               int silu, cudaStream_t s, int ex_cfg = 1, int ex_S = 1) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15u) == 0;
  if (ex_cfg <= 1 && aligned && N == 32 && (size_t)K * 32 * 4 <= kNarrowSmemMax &&
      (K & 3) == 0 && M > 64) {
    static bool attr = false;
    const int smem = K * 32 * 4 + (int)kNarrowXBytes;
    if (!attr) {
      cudaFuncSetAttribute(linear_narrow_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(kNarrowSmemMax + kNarrowXBytes));
      attr = true;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = std::min(sms, cdiv(M, 64));
    linear_narrow_kernel<<<grid, kNarrowThreads, smem, s>>>(x, w, bias, y, M, K, silu);
  } else if (ex_cfg <= 1 && aligned && M <= 64) {
    const long long warps = (long long)M * cdiv(N, 32);
    linear_rows_kernel<<<(unsigned)warps, 32, 0, s>>>(x, w, bias, y, M, N, K, silu);
  } else
    linear_ref_kernel<64, 64, 4, 4><<<dim3(cdiv(N, 64), cdiv(M, 64)), 256, 0, s>>>(
        x, w, bias, y, M, N, K, silu, ex_cfg, ex_S);
  return check_launch();
}

// dit.c:488-500: [cos(t f_i) | sin(t f_i)], f_i = 1000 exp(-ln(1e4) i / half).
// Row b = blockIdx.y takes its timestep from t_dev[b], or t_scalar when
// t_dev is null.
__global__ void timestep_embedding_kernel(const float* __restrict__ t_dev, float t_scalar,
                                          int dim, float* __restrict__ emb_rows) {
  const int half = dim / 2;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= half) return;
  const float t = t_dev ? t_dev[blockIdx.y] : t_scalar;
  float* emb = emb_rows + (size_t)blockIdx.y * dim;
  const float log_theta = logf(10000.0f);
  const float freq = __fmul_rn(1000.0f, expf(__fdiv_rn(__fmul_rn(-log_theta, (float)i), (float)half)));
  const float arg = __fmul_rn(t, freq);
  emb[i] = cosf(arg);
  emb[half + i] = sinf(arg);
}

// dit.c:1078 / ops.c:738-747: y = x * inv * w, inv = 1 / sqrt(mean(x^2) + eps),
// the mean of squares summed in the reference's order by one thread per row.
// 32 rows per block; each 128-column slice of those rows is staged through
// shared memory with coalesced loads, then every thread walks its own row.
constexpr int kNR = 32, kNC = 128;

__global__ void __launch_bounds__(256) rmsnorm_ref_kernel(const float* x,
                                                          const float* __restrict__ w, float* y,
                                                          int M, int D, float eps) {
  __shared__ float tile[kNR][kNC + 1];
  __shared__ float inv_s[kNR];
  const int r0 = blockIdx.x * kNR;
  const int t = threadIdx.x;
  float ms = 0.0f;
  for (int c0 = 0; c0 < D; c0 += kNC) {
    const int nc = min(kNC, D - c0);
    __syncthreads();
    for (int i = t; i < kNR * kNC; i += 256) {
      const int rr = i / kNC, cc = i % kNC;
      const int m = r0 + rr;
      tile[rr][cc] = (m < M && cc < nc) ? x[(size_t)m * D + c0 + cc] : 0.0f;
    }
    __syncthreads();
    if (t < kNR)
      for (int cc = 0; cc < nc; cc++) ms = __fadd_rn(ms, __fmul_rn(tile[t][cc], tile[t][cc]));
  }
  if (t < kNR) inv_s[t] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ms, (float)D), eps)));
  __syncthreads();
  for (int rr = 0; rr < kNR; rr++) {
    const int m = r0 + rr;
    if (m >= M) break;
    const float inv = inv_s[rr];
    const float* xm = x + (size_t)m * D;
    float* ym = y + (size_t)m * D;
    for (int d = t; d < D; d += 256) ym[d] = __fmul_rn(__fmul_rn(xm[d], inv), w[d]);
  }
}

// sampler.c:283-297: guided = v_cond + sum_i scale_i (v_cond - v_uncond_i),
// added in the reference's branch order, then state += guided * dt.
__global__ void euler_cfg_kernel(float* __restrict__ state, const float* __restrict__ v, int R,
                                 int cfg, long long one, float dt, float s1, float s2, float s3) {
  const long long n = (long long)R * one;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / one, e = i - r * one;
    const float* vr = v + (size_t)r * cfg * one;
    const float vc = vr[e];
    float g = vc;
    if (cfg > 1) g = __fadd_rn(g, __fmul_rn(s1, __fsub_rn(vc, vr[one + e])));
    if (cfg > 2) g = __fadd_rn(g, __fmul_rn(s2, __fsub_rn(vc, vr[2 * one + e])));
    if (cfg > 3) g = __fadd_rn(g, __fmul_rn(s3, __fsub_rn(vc, vr[3 * one + e])));
    state[i] = __fadd_rn(state[i], __fmul_rn(g, dt));
  }
}


// The conditional rows' mask [R, C] out of the full CFG mask [R*cfg, C].
__global__ void cond_mask_kernel(const uint8_t* __restrict__ mask, uint8_t* __restrict__ out,
                                 int R, int cfg, int C) {
  const long long n = (long long)R * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / C, cc = i - r * C;
    out[i] = mask[(r * cfg) * C + cc];
  }
}

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

// Workspace: RoPE tables and the conditional-row mask first (written once
// per sampling run), then the per-step scratch.
struct StepBufs {
  float* rcos;
  float* rsin;
  float* rope_t;  // grouped copy for the QKVG epilogue: cos [8][S][4], then sin
  uint8_t* cond_mask;
  uint8_t* rest;
};

size_t head_bytes(int R, int S, int C) {
  return 4 * al256(sizeof(float) * (size_t)S * 32) + al256((size_t)R * C);
}

StepBufs carve(uint8_t* ws, int S) {
  StepBufs b;
  const size_t tab = al256(sizeof(float) * (size_t)S * 32);
  b.rcos = reinterpret_cast<float*>(ws);
  b.rsin = reinterpret_cast<float*>(ws + tab);
  b.rope_t = reinterpret_cast<float*>(ws + 2 * tab);
  b.cond_mask = ws + 4 * tab;
  b.rest = nullptr;
  return b;
}

bool valid_model(const IroDiTModelDev* m) {
  if (!m || m->layers <= 0 || m->layers > IRO_DIT_MAX_LAYERS || !m->cond_w0 || !m->cond_w1 ||
      !m->cond_w2 || !m->in_w || !m->in_b || !m->out_norm || !m->out_w || !m->out_b ||
      m->timestep_dim <= 0 || m->timestep_dim % 2 || m->latent_dim <= 0)
    return false;
  const IroDiTBlockDev& b0 = m->block[0];
  for (int l = 1; l < m->layers; l++) {
    const IroDiTBlockDev& b = m->block[l];
    if (b.model_dim != b0.model_dim || b.heads != b0.heads || b.head_dim != b0.head_dim ||
        b.adaln_rank != b0.adaln_rank || b.mlp_dim != b0.mlp_dim)
      return false;
  }
  return b0.head_dim == 64;
}

// RoPE tables (the host recurrence, dit.c:560-586) into the workspace;
// synchronous, so the host vectors may go when it returns.
int upload_rope(const StepBufs& b, int S, cudaStream_t s) {
  std::vector<float> hc((size_t)S * 32), hs((size_t)S * 32);
  int st = iro_dit_rope_table(hc.data(), hs.data(), S, 64);
  if (st) return st;
  std::vector<float> ht((size_t)S * 64);
  for (int tok = 0; tok < S; tok++)
    for (int j = 0; j < 32; j++) {
      const size_t o = ((size_t)(j >> 2) * S + tok) * 4 + (j & 3);
      ht[o] = hc[(size_t)tok * 32 + j];
      ht[(size_t)32 * S + o] = hs[(size_t)tok * 32 + j];
    }
  cudaError_t e = cudaMemcpyAsync(b.rcos, hc.data(), sizeof(float) * hc.size(),
                                  cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(b.rsin, hs.data(), sizeof(float) * hs.size(), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(b.rope_t, ht.data(), sizeof(float) * ht.size(), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

// Conditioning of `n` timesteps at once (dit.c:502-530): cond [n, 3D] and
// every layer's AdaLN parameters, params [2L sets][3][n][D].  The sampler
// calls it once for all its steps; a single step calls it with n = 1.
struct CondBufs {
  float* t;       // [n] timesteps (device)
  float* emb;     // [n, TD]
  float* h0;      // [n, D]
  float* h1;      // [n, D]
  float* cond;    // [n, 3D]
  float* params;  // [2L][3][n][D]
  void* scratch;
  int n;
};

size_t cond_bytes(const IroDiTModelDev* m, int n) {
  const size_t D = (size_t)m->block[0].model_dim;
  return al256(sizeof(float) * n) + al256(sizeof(float) * n * m->timestep_dim) +
         2 * al256(sizeof(float) * n * D) + al256(sizeof(float) * n * 3 * D) +
         al256(sizeof(float) * 6 * (size_t)m->layers * n * D) +
         dit_adaln_scratch_bytes(2 * m->layers, n, (int)D, m->block[0].adaln_rank);
}

CondBufs carve_cond(const IroDiTModelDev* m, int n, uint8_t* ws) {
  const size_t D = (size_t)m->block[0].model_dim;
  CondBufs b;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = ws + off;
    off += al256(bytes);
    return p;
  };
  b.t = reinterpret_cast<float*>(take(sizeof(float) * n));
  b.emb = reinterpret_cast<float*>(take(sizeof(float) * n * m->timestep_dim));
  b.h0 = reinterpret_cast<float*>(take(sizeof(float) * n * D));
  b.h1 = reinterpret_cast<float*>(take(sizeof(float) * n * D));
  b.cond = reinterpret_cast<float*>(take(sizeof(float) * n * 3 * D));
  b.params = reinterpret_cast<float*>(take(sizeof(float) * 6 * (size_t)m->layers * n * D));
  b.scratch = ws + off;
  b.n = n;
  return b;
}

int condition_all(const IroDiTModelDev* m, const float* t_host, const CondBufs& b,
                  cudaStream_t s) {
  const int D = m->block[0].model_dim, TD = m->timestep_dim, n = b.n;
  // Pageable source: staged before the call returns.
  cudaError_t e = cudaMemcpyAsync(b.t, t_host, sizeof(float) * n, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  timestep_embedding_kernel<<<dim3(cdiv(TD / 2, 128), n), 128, 0, s>>>(b.t, 0.0f, TD, b.emb);
  int st = check_launch();
  if (st) return st;
  if ((st = linear_ref(b.emb, m->cond_w0, nullptr, b.h0, n, D, TD, 1, s))) return st;
  if ((st = linear_ref(b.h0, m->cond_w1, nullptr, b.h1, n, D, D, 1, s))) return st;
  if ((st = linear_ref(b.h1, m->cond_w2, nullptr, b.cond, n, 3 * D, D, 0, s))) return st;
  const IroDiTBlockDev* blks[IRO_DIT_MAX_LAYERS];
  for (int l = 0; l < m->layers; l++) blks[l] = &m->block[l];
  return dit_adaln_params(blks, m->layers, b.cond, n, b.params, b.scratch, s);
}

// One step with `cfg` active rows per request, `mask` [R*cfg, C] for those
// rows; `full_cfg` is the width the scratch was sized for; the step's
// conditioning is row `row` of `cb`.  With `vel_out` the per-row velocities
// [R*cfg, S, L] go there and the state is not updated.
int step_impl(Ctx* c, const IroDiTModelDev* m, float* state, int R, int cfg, int full_cfg,
              int S, float t, float t_next, const float* scales, const float* const* ctx_k,
              const float* const* ctx_v, const uint8_t* mask, int C, const StepBufs& tb,
              const CondBufs& cb, int row, cudaStream_t s, float* vel_out = nullptr) {
  const int D = m->block[0].model_dim, L = m->latent_dim;
  const int B = R * cfg, Bfull = R * full_cfg;
  uint8_t* ws = tb.rest;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = ws + off;
    off += al256(bytes);
    return p;
  };
  float* x = reinterpret_cast<float*>(take(sizeof(float) * (size_t)Bfull * S * D));
  float* vel = reinterpret_cast<float*>(take(sizeof(float) * (size_t)Bfull * S * L));
  if (vel_out) vel = vel_out;
  void* blk_ws = ws + off;
  int st;
  // Input projection per request, each row stored to its CFG rows.
  if ((st = linear_ref(state, m->in_w, m->in_b, x, R * S, D, L, 0, s, cfg, S))) return st;
  for (int l = 0; l < m->layers; l++) {
    const float* ada[6];
    for (int i = 0; i < 6; i++)
      ada[i] = cb.params + (((size_t)(2 * l) * 3 + i) * cb.n + row) * D;
    st = dit_block_run(c, &m->block[l], x, ada, 1, ctx_k[l], ctx_v[l], mask, R, B, S, C, tb.rcos,
                       tb.rsin, blk_ws, s, l, tb.rope_t);
    if (st) return st;
  }
  // Output head (normalised in place: x is rebuilt from the state next
  // step) into the velocity, then the guided Euler update.
  rmsnorm_ref_kernel<<<cdiv(B * S, kNR), 256, 0, s>>>(x, m->out_norm, x, B * S, D, m->norm_eps);
  if ((st = check_launch())) return st;
  if ((st = linear_ref(x, m->out_w, m->out_b, vel, B * S, L, D, 0, s))) return st;
  if (vel_out) return IRO_OK;
  const float dt = t_next - t;
  const float s1 = cfg > 1 ? scales[0] : 0.0f, s2 = cfg > 2 ? scales[1] : 0.0f;
  const float s3 = cfg > 3 ? scales[2] : 0.0f;
  const long long one = (long long)S * L;
  const int ub = (int)std::min<long long>((R * one + 255) / 256, c->num_sms * 16LL);
  euler_cfg_kernel<<<ub, 256, 0, s>>>(state, vel, R, cfg, one, dt, s1, s2, s3);
  return check_launch();
}

bool valid_run(const IroDiTModelDev* m, const float* state, int R, int cfg, int S,
               const float* cfg_scales, const float* const* ctx_k, const float* const* ctx_v,
               const uint8_t* mask, int C) {
  if (!valid_model(m) || !state || R <= 0 || cfg < 1 || cfg > 4 || S <= 0 || C <= 0 || !ctx_k ||
      !ctx_v || !mask || (cfg > 1 && !cfg_scales))
    return false;
  for (int l = 0; l < m->layers; l++)
    if (!ctx_k[l] || !ctx_v[l]) return false;
  return true;
}

// Block-level checks at the step's shapes (one row of conditioning).
int check_blocks(const IroDiTModelDev* m, const float* state, int R, int cfg, int S,
                 const float* const* ctx_k, const float* const* ctx_v, const uint8_t* mask,
                 int C) {
  // The step's own buffers (x, RoPE tables) live in the workspace, 256-byte
  // aligned; an aligned stand-in passes the pointer checks.
  alignas(16) static const float stand_in[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  (void)state;
  for (int l = 0; l < m->layers; l++) {
    int st = dit_block_check(&m->block[l], stand_in, 1, ctx_k[l], ctx_v[l], mask, R, R * cfg, S,
                             C, stand_in, stand_in);
    if (st) return st;
  }
  return IRO_OK;
}

}  // namespace
}  // namespace iro

using namespace iro;

extern "C" {

size_t iro_dit_step_workspace_bytes(const IroDiTModelDev* m, int R, int cfg, int S, int C) {
  return iro_dit_sample_workspace_bytes(m, R, cfg, S, C, 1);
}

size_t iro_dit_sample_workspace_bytes(const IroDiTModelDev* m, int R, int cfg, int S, int C,
                                      int steps) {
  if (!valid_model(m) || R <= 0 || cfg <= 0 || S <= 0 || C <= 0 || steps <= 0) return 0;
  const int D = m->block[0].model_dim, B = R * cfg;
  size_t t = head_bytes(R, S, C) + cond_bytes(m, steps);
  t += al256(sizeof(float) * (size_t)B * S * D);                       // x
  t += al256(sizeof(float) * (size_t)B * S * m->latent_dim);           // velocity
  // Blocks may differ in their policies (two-term groups, diagnostic modes),
  // so the shared block workspace is the largest any layer needs.
  size_t body = 0;
  for (int l = 0; l < m->layers; l++)
    body = std::max(body, dit_block_body_bytes(&m->block[l], B, S, C, R));
  return t + body;
}

int iro_dit_euler_step_dev(const IroDiTModelDev* m, float* state, int R, int cfg, int S,
                           float t, float t_next, const float* cfg_scales, const float* const* ctx_k,
                           const float* const* ctx_v, const uint8_t* mask, int C,
                           void* workspace, void* stream) {
  if (!valid_run(m, state, R, cfg, S, cfg_scales, ctx_k, ctx_v, mask, C)) return IRO_ERR_INVALID;
  int st = check_blocks(m, state, R, cfg, S, ctx_k, ctx_v, mask, C);
  if (st) return st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!ws) {
    ws = static_cast<uint8_t*>(arena_get(c, iro_dit_step_workspace_bytes(m, R, cfg, S, C), &st));
    if (!ws) return st;
  }
  StepBufs tb = carve(ws, S);
  const CondBufs cb = carve_cond(m, 1, ws + head_bytes(R, S, C));
  tb.rest = ws + head_bytes(R, S, C) + cond_bytes(m, 1);
  if ((st = upload_rope(tb, S, s))) return st;
  if ((st = condition_all(m, &t, cb, s))) return st;
  return step_impl(c, m, state, R, cfg, cfg, S, t, t_next, cfg_scales, ctx_k, ctx_v, mask, C, tb,
                   cb, 0, s);
}

int iro_dit_velocity_dev(const IroDiTModelDev* m, const float* state, int R, int cfg, int S,
                         float t, const float* const* ctx_k, const float* const* ctx_v,
                         const uint8_t* mask, int C, float* velocity, void* workspace,
                         void* stream) {
  static const float no_scales[3] = {0.0f, 0.0f, 0.0f};
  if (!velocity ||
      !valid_run(m, state, R, cfg, S, no_scales, ctx_k, ctx_v, mask, C))
    return IRO_ERR_INVALID;
  int st = check_blocks(m, state, R, cfg, S, ctx_k, ctx_v, mask, C);
  if (st) return st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!ws) {
    ws = static_cast<uint8_t*>(arena_get(c, iro_dit_step_workspace_bytes(m, R, cfg, S, C), &st));
    if (!ws) return st;
  }
  StepBufs tb = carve(ws, S);
  const CondBufs cb = carve_cond(m, 1, ws + head_bytes(R, S, C));
  tb.rest = ws + head_bytes(R, S, C) + cond_bytes(m, 1);
  if ((st = upload_rope(tb, S, s))) return st;
  if ((st = condition_all(m, &t, cb, s))) return st;
  return step_impl(c, m, const_cast<float*>(state), R, cfg, cfg, S, t, t, no_scales, ctx_k, ctx_v,
                   mask, C, tb, cb, 0, s, velocity);
}

int iro_dit_cfg_update_dev(const IroDiTModelDev* m, float* state, const float* velocity, int R,
                           int cfg, int S, float t, float t_next, const float* cfg_scales,
                           void* stream) {
  if (!valid_model(m) || !state || !velocity || R <= 0 || cfg < 1 || cfg > 4 || S <= 0 ||
      (cfg > 1 && !cfg_scales))
    return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  const long long one = (long long)S * m->latent_dim;
  const float s1 = cfg > 1 ? cfg_scales[0] : 0.0f, s2 = cfg > 2 ? cfg_scales[1] : 0.0f;
  const float s3 = cfg > 3 ? cfg_scales[2] : 0.0f;
  const int ub = (int)std::min<long long>((R * one + 255) / 256, c->num_sms * 16LL);
  euler_cfg_kernel<<<ub, 256, 0, s>>>(state, velocity, R, cfg, one, t_next - t, s1, s2, s3);
  return check_launch();
}

int iro_dit_sample_euler_dev(const IroDiTModelDev* m, float* state, int R, int cfg, int S,
                             int steps, float init_scale, float cfg_min_t, float cfg_max_t,
                             const float* cfg_scales, const float* const* ctx_k,
                             const float* const* ctx_v, const uint8_t* mask, int C,
                             void* workspace, void* stream) {
  if (!valid_run(m, state, R, cfg, S, cfg_scales, ctx_k, ctx_v, mask, C) || steps <= 0)
    return IRO_ERR_INVALID;
  int st = check_blocks(m, state, R, cfg, S, ctx_k, ctx_v, mask, C);
  if (st) return st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!ws) {
    ws = static_cast<uint8_t*>(
        arena_get(c, iro_dit_sample_workspace_bytes(m, R, cfg, S, C, steps), &st));
    if (!ws) return st;
  }
  // sampler.c:244-249: the timestep schedule, in the reference's float
  // arithmetic; all steps' conditioning is computed up front.
  std::vector<float> ts(steps), tn(steps);
  for (int step = 0; step < steps; step++) {
    const float u = (float)step / (float)steps;
    const float u_next = (float)(step + 1) / (float)steps;
    ts[step] = (1.0f - u) * init_scale;
    tn[step] = (1.0f - u_next) * init_scale;
  }
  StepBufs tb = carve(ws, S);
  const CondBufs cb = carve_cond(m, steps, ws + head_bytes(R, S, C));
  tb.rest = ws + head_bytes(R, S, C) + cond_bytes(m, steps);
  if ((st = upload_rope(tb, S, s))) return st;
  if ((st = condition_all(m, ts.data(), cb, s))) return st;
  if (cfg > 1) {
    const int mb = (int)std::min<long long>(((long long)R * C + 255) / 256, c->num_sms * 4LL);
    cond_mask_kernel<<<mb, 256, 0, s>>>(mask, tb.cond_mask, R, cfg, C);
    if ((st = check_launch())) return st;
  }
  // sampler.c:142-144, 312-321: one IRO_GEMM_PROFILE record per sampling run.
  iro_cuda_gemm_profile_reset();
  for (int step = 0; step < steps; step++) {
    const float t = ts[step];
    const bool use_cfg = cfg > 1 && t >= cfg_min_t && t <= cfg_max_t;
    st = step_impl(c, m, state, R, use_cfg ? cfg : 1, cfg, S, t, tn[step], cfg_scales, ctx_k,
                   ctx_v, use_cfg ? mask : (cfg > 1 ? tb.cond_mask : mask), C, tb, cb, step, s);
    if (st) {
      iro_cuda_gemm_profile_emit_json("error", steps, S, C);
      return st;
    }
  }
  iro_cuda_gemm_profile_emit_json("ok", steps, S, C);
  return IRO_OK;
}

// The reference's public DiT pieces on device buffers, for callers that
// compose their own loop and for stage-level parity.

size_t iro_dit_stage_workspace_bytes(const IroDiTModelDev* m, int rows) {
  if (!valid_model(m) || rows <= 0) return 0;
  const size_t D = (size_t)m->block[0].model_dim;
  return al256(sizeof(float) * rows) + al256(sizeof(float) * rows * m->timestep_dim) +
         2 * al256(sizeof(float) * rows * D) + al256(sizeof(float) * rows * D);
}

int iro_dit_condition_dev(const IroDiTModelDev* m, const float* t, int B, float* cond,
                          void* workspace, void* stream) {
  if (!valid_model(m) || !t || B <= 0 || !cond) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  const int D = m->block[0].model_dim, TD = m->timestep_dim;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!ws) {
    ws = static_cast<uint8_t*>(arena_get(c, iro_dit_stage_workspace_bytes(m, B), &st));
    if (!ws) return st;
  }
  float* td = reinterpret_cast<float*>(ws);
  float* emb = reinterpret_cast<float*>(ws + al256(sizeof(float) * B));
  float* h0 = emb + al256(sizeof(float) * (size_t)B * TD) / sizeof(float);
  float* h1 = h0 + al256(sizeof(float) * (size_t)B * D) / sizeof(float);
  // Pageable source: the copy is staged before the call returns.
  cudaError_t e = cudaMemcpyAsync(td, t, sizeof(float) * B, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  timestep_embedding_kernel<<<dim3(cdiv(TD / 2, 128), B), 128, 0, s>>>(td, 0.0f, TD, emb);
  if ((st = check_launch())) return st;
  if ((st = linear_ref(emb, m->cond_w0, nullptr, h0, B, D, TD, 1, s))) return st;
  if ((st = linear_ref(h0, m->cond_w1, nullptr, h1, B, D, D, 1, s))) return st;
  return linear_ref(h1, m->cond_w2, nullptr, cond, B, 3 * D, D, 0, s);
}

int iro_dit_input_dev(const IroDiTModelDev* m, const float* x, int B, int S, float* projected,
                      void* stream) {
  if (!valid_model(m) || !x || B <= 0 || S <= 0 || !projected) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  return linear_ref(x, m->in_w, m->in_b, projected, B * S, m->block[0].model_dim, m->latent_dim,
                    0, pick_stream(c, stream));
}

int iro_dit_output_dev(const IroDiTModelDev* m, const float* x, int B, int S, float* velocity,
                       void* workspace, void* stream) {
  if (!valid_model(m) || !x || B <= 0 || S <= 0 || !velocity) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  const int D = m->block[0].model_dim, rows = B * S;
  float* norm = static_cast<float*>(workspace);
  if (!norm) {
    norm = static_cast<float*>(arena_get(c, sizeof(float) * (size_t)rows * D, &st));
    if (!norm) return st;
  }
  rmsnorm_ref_kernel<<<cdiv(rows, kNR), 256, 0, s>>>(x, m->out_norm, norm, rows, D, m->norm_eps);
  if ((st = check_launch())) return st;
  return linear_ref(norm, m->out_w, m->out_b, velocity, rows, m->latent_dim, D, 0, s);
}

}  // extern "C"
