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

// y[M, N] = x[M, K] . w[N, K]^T (+ bias) for a few rows (the conditioner,
// M <= 8 per block): one warp per block and 32 outputs, lane j summing output
// n0 + j of every row in increasing k (the reference's order, ops.c:221-234).
// The reference's order makes each output one chain of K dependent adds, so
// what bounds the kernel is how early the weights arrive: the block's 32
// weight rows stream through shared memory in chunks of 64 k by cp.async,
// kGemvStages chunks in flight (coalesced 16-byte pieces; rows padded to 68
// floats so that lane j's 16-byte reads of its own row are conflict-free).
constexpr int kGemvKC = 64;
constexpr int kGemvLd = kGemvKC + 4;
constexpr int kGemvRows = 8;  // input rows per block
constexpr int kGemvStages = 6;
constexpr size_t kGemvStageFloats = 32 * kGemvLd + kGemvRows * kGemvKC;
constexpr size_t kGemvSmem = kGemvStages * kGemvStageFloats * sizeof(float);

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int MR>
__global__ void __launch_bounds__(32) gemv_rows_kernel(const float* __restrict__ x,
                                                        const float* __restrict__ w,
                                                        const float* __restrict__ bias,
                                                        float* __restrict__ y, int M, int N,
                                                        int K, int silu) {
  extern __shared__ float4 gemv_smem[];
  float* sm = reinterpret_cast<float*>(gemv_smem);
  const int lane = threadIdx.x;
  const int n0 = blockIdx.x * 32, m0 = blockIdx.y * MR;
  const int mr = min(MR, M - m0);
  const int nk = (K + kGemvKC - 1) / kGemvKC;
  // Chunk kc into stage buffer b: weight rows n0 .. n0+31 (rows past N repeat
  // row N-1; their sums are not stored), then the block's input rows.
  auto stage = [&](int kc, int b) {
    float* ws = sm + (size_t)b * kGemvStageFloats;
    float* xs = ws + 32 * kGemvLd;
    const int k0 = kc * kGemvKC;
    const int p4 = min(kGemvKC, K - k0) / 4;  // 16-byte pieces per row in this chunk
    if (p4 == kGemvKC / 4) {
      // A whole chunk: lane l moves pieces l, l + 32, ... (row i / 16).
#pragma unroll
      for (int j = 0; j < 32 * (kGemvKC / 4) / 32; j++) {
        const int i = lane + 32 * j;
        const int r = i / (kGemvKC / 4), c = i % (kGemvKC / 4);
        const int n = min(n0 + r, N - 1);
        cp_async16(ws + r * kGemvLd + 4 * c, w + (size_t)n * K + k0 + 4 * c);
      }
      for (int i = lane; i < mr * (kGemvKC / 4); i += 32) {
        const int r = i / (kGemvKC / 4), c = i % (kGemvKC / 4);
        cp_async16(xs + r * kGemvKC + 4 * c, x + (size_t)(m0 + r) * K + k0 + 4 * c);
      }
      return;
    }
    for (int i = lane; i < 32 * p4; i += 32) {
      const int r = i / p4, c = i - r * p4;
      const int n = min(n0 + r, N - 1);
      cp_async16(ws + r * kGemvLd + 4 * c, w + (size_t)n * K + k0 + 4 * c);
    }
    for (int i = lane; i < mr * p4; i += 32) {
      const int r = i / p4, c = i - r * p4;
      cp_async16(xs + r * kGemvKC + 4 * c, x + (size_t)(m0 + r) * K + k0 + 4 * c);
    }
  };
  float acc[MR];
#pragma unroll
  for (int r = 0; r < MR; r++) acc[r] = 0.0f;
#pragma unroll
  for (int b = 0; b < kGemvStages - 1; b++) {
    if (b < nk) stage(b, b);
    cp_async_commit();
  }
  for (int kc = 0; kc < nk; kc++) {
    // The buffer chunk kc + stages - 1 goes to was last read by chunk kc - 1,
    // which every lane finished before the barrier at the end of its turn.
    if (kc + kGemvStages - 1 < nk) stage(kc + kGemvStages - 1, (kc + kGemvStages - 1) % kGemvStages);
    cp_async_commit();
    cp_async_wait<kGemvStages - 1>();
    __syncwarp();
    const float* ws = sm + (size_t)(kc % kGemvStages) * kGemvStageFloats;
    const float* xs = ws + 32 * kGemvLd;
    const int kl = min(kGemvKC, K - kc * kGemvKC);
    auto step4 = [&](int k) {
      const float4 b4 = *reinterpret_cast<const float4*>(ws + lane * kGemvLd + k);
#pragma unroll
      for (int r = 0; r < MR; r++) {
        if (MR == 1 || r < mr) {
          const float4 a = *reinterpret_cast<const float4*>(xs + r * kGemvKC + k);
          acc[r] = __fadd_rn(acc[r], __fmul_rn(a.x, b4.x));
          acc[r] = __fadd_rn(acc[r], __fmul_rn(a.y, b4.y));
          acc[r] = __fadd_rn(acc[r], __fmul_rn(a.z, b4.z));
          acc[r] = __fadd_rn(acc[r], __fmul_rn(a.w, b4.w));
        }
      }
    };
    if (kl == kGemvKC) {
      // Unrolled so the shared-memory reads run ahead of the dependent adds.
#pragma unroll
      for (int k = 0; k < kGemvKC; k += 4) step4(k);
    } else {
      for (int k = 0; k < kl; k += 4) step4(k);
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  const int n = n0 + lane;
  if (n >= N) return;
  const float bn = bias ? bias[n] : 0.0f;
#pragma unroll
  for (int r = 0; r < MR; r++) {
    if (r >= mr) break;
    float v = __fadd_rn(acc[r], bn);
    if (silu) v = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    y[(size_t)(m0 + r) * N + n] = v;
  }
}

// The input projection y[M, N] = x[M, 32] . w[N, 32]^T + bias (dit.c:532-541),
// output row m stored to ex_cfg rows ((m / ex_S) * ex_cfg + c) * ex_S + m % ex_S
// (one request's row broadcast to its CFG rows, sampler.c:256-262).  Each
// thread keeps the weights of its two outputs in registers (64 floats) and
// walks the block's rows; the rows' inputs (128 bytes each) arrive through a
// ring of kInAhead rows in shared memory by cp.async, several rows ahead, and
// are read as broadcasts.  128 threads cover 256 outputs (blockIdx.y); each
// output sums k in increasing order, then adds the bias, as the reference
// does.
constexpr int kInK = 32;
constexpr int kInThreads = 128;
constexpr int kInAhead = 8;

__global__ void __launch_bounds__(kInThreads) input_proj_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               const float* __restrict__ bias,
                                                               float* __restrict__ y, int M,
                                                               int N, int ex_cfg, int ex_S) {
  __shared__ __align__(16) float xs[kInAhead][kInK];
  const int n = blockIdx.y * (2 * kInThreads) + 2 * threadIdx.x;
  // Row i of this block is blockIdx.x + i * gridDim.x; threads 0-7 move its
  // eight 16-byte pieces.
  const int nrows = M > (int)blockIdx.x ? (M - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto fetch = [&](int i) {
    if (i < nrows && threadIdx.x < kInK / 4) {
      const int m = blockIdx.x + i * gridDim.x;
      cp_async16(&xs[i % kInAhead][4 * threadIdx.x], x + (size_t)m * kInK + 4 * threadIdx.x);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < kInAhead - 1; i++) fetch(i);
  float w0[kInK], w1[kInK];
#pragma unroll
  for (int k4 = 0; k4 < kInK / 4; k4++) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(w + (size_t)n * kInK) + k4);
    const float4 b = __ldg(reinterpret_cast<const float4*>(w + (size_t)(n + 1) * kInK) + k4);
    w0[4 * k4] = a.x; w0[4 * k4 + 1] = a.y; w0[4 * k4 + 2] = a.z; w0[4 * k4 + 3] = a.w;
    w1[4 * k4] = b.x; w1[4 * k4 + 1] = b.y; w1[4 * k4 + 2] = b.z; w1[4 * k4 + 3] = b.w;
  }
  const float b0 = bias ? bias[n] : 0.0f, b1 = bias ? bias[n + 1] : 0.0f;
  const int copies = ex_cfg <= 1 ? 1 : ex_cfg;
  for (int i = 0; i < nrows; i++) {
    // The ring slot row i + kInAhead - 1 goes to was read for row i - 1,
    // which every thread finished before the barrier at the end of its turn.
    fetch(i + kInAhead - 1);
    cp_async_wait<kInAhead - 1>();
    __syncthreads();
    const float4* xr = reinterpret_cast<const float4*>(xs[i % kInAhead]);
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int k4 = 0; k4 < kInK / 4; k4++) {
      const float4 v = xr[k4];
      a0 = __fadd_rn(a0, __fmul_rn(v.x, w0[4 * k4]));
      a1 = __fadd_rn(a1, __fmul_rn(v.x, w1[4 * k4]));
      a0 = __fadd_rn(a0, __fmul_rn(v.y, w0[4 * k4 + 1]));
      a1 = __fadd_rn(a1, __fmul_rn(v.y, w1[4 * k4 + 1]));
      a0 = __fadd_rn(a0, __fmul_rn(v.z, w0[4 * k4 + 2]));
      a1 = __fadd_rn(a1, __fmul_rn(v.z, w1[4 * k4 + 2]));
      a0 = __fadd_rn(a0, __fmul_rn(v.w, w0[4 * k4 + 3]));
      a1 = __fadd_rn(a1, __fmul_rn(v.w, w1[4 * k4 + 3]));
    }
    __syncthreads();
    const int m = blockIdx.x + i * gridDim.x;
    const float2 out = make_float2(__fadd_rn(a0, b0), __fadd_rn(a1, b1));
    const size_t r = (size_t)(m / ex_S), t = (size_t)(m % ex_S);
    for (int c = 0; c < copies; c++) {
      float* yrow = ex_cfg <= 1 ? y + (size_t)m * N : y + ((r * ex_cfg + c) * ex_S + t) * N;
      *reinterpret_cast<float2*>(yrow + n) = out;
    }
  }
  cp_async_wait<0>();
}

// ex_cfg > 1: output row m is written to the ex_cfg rows
// ((m / ex_S) * ex_cfg + c) * ex_S + m % ex_S (one request's row broadcast to
// its CFG rows, sampler.c:256-262).
int linear_ref(const float* x, const float* w, const float* bias, float* y, int M, int N, int K,
               int silu, cudaStream_t s, int ex_cfg = 1, int ex_S = 1) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15u) == 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (K == kInK && !silu && aligned && N % (2 * kInThreads) == 0 &&
      (reinterpret_cast<uintptr_t>(y) & 7u) == 0 && M > 64) {
    // One wave of resident blocks; each walks its share of the rows.
    static int occ_dev[64] = {0};
    int& occ = occ_dev[dev & 63];
    if (occ <= 0 &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, input_proj_kernel, kInThreads, 0) !=
            cudaSuccess) {
      cudaGetLastError();
      occ = 4;
    }
    const int col_blocks = N / (2 * kInThreads);
    const int row_blocks = std::min(M, std::max(1, std::max(occ, 1) * sms / col_blocks));
    input_proj_kernel<<<dim3(row_blocks, col_blocks), kInThreads, 0, s>>>(x, w, bias, y, M, N,
                                                                          ex_cfg, ex_S);
  } else if (ex_cfg <= 1 && aligned && (K & 3) == 0 && M <= 64) {
    // Rows per block: the fewest that cover M in at most eight-row blocks
    // (each output's chain of adds is per row; idle row slots cost issue).
    // The shared-memory opt-in is a per-device attribute of each kernel (the
    // four instantiations share this lambda's type, hence the slot).
    auto go = [&](auto kernel, int mr) {
      static bool attr[4][64] = {};
      const int slot = mr == 1 ? 0 : mr == 2 ? 1 : mr == 4 ? 2 : 3;
      if (!attr[slot][dev & 63]) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvSmem);
        attr[slot][dev & 63] = true;
      }
      kernel<<<dim3(cdiv(N, 32), cdiv(M, mr)), 32, kGemvSmem, s>>>(x, w, bias, y, M, N, K, silu);
    };
    if (M == 1) go(gemv_rows_kernel<1>, 1);
    else if (M == 2) go(gemv_rows_kernel<2>, 2);
    else if (M <= 4) go(gemv_rows_kernel<4>, 4);
    else go(gemv_rows_kernel<8>, 8);
  } else {
    linear_ref_kernel<64, 64, 4, 4><<<dim3(cdiv(N, 64), cdiv(M, 64)), 256, 0, s>>>(
        x, w, bias, y, M, N, K, silu, ex_cfg, ex_S);
  }
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

// The output head, vel[M, 32] = rmsnorm(x)[M, D] . w[32, D]^T + b
// (dit.c:1070-1090), in one kernel: rmsnorm(x)[d] = (x[d] * inv) * g[d] with
// inv = 1 / sqrt(mean of squares + eps), the squares summed in increasing d
// (ops.c:738-747), and each output summed in increasing k, then the bias
// (ops.c:221-234): the reference's operations in its order, so the result is
// bit-identical to its IEEE build.
//
// A persistent grid; each block owns one contiguous share of the rows and
// walks it in groups of up to 192 (8 warps x 24 rows; a group is the whole
// share at config-3 sizes, and 24-row warp tiles spread it evenly over the
// four schedulers).  W^T ([D][32],
// 128 KB at D = 1024) and g stay in shared memory.  A group's rows stream
// through a ring of STAGES chunks of 32 k (128 bytes per row, cp.async,
// several in flight) twice: the first pass sums each row's squares (thread t
// owns row t), the
// second normalises each landed chunk in place (thread t its row again) and
// accumulates the outputs.  In the second pass lane (g, q) = (lane / 4,
// lane % 4) of warp w owns rows 24w + g + 8i (i < 3) and outputs 8q .. 8q+7:
// each 16-byte read of a row's x serves 8 outputs and each 32-byte read of
// W^T[k] serves 3 rows, so the shared-memory reads per multiply-add are a
// fraction of one row per lane.  The second pass reads the group again from
// L2 (up to 768 KB per block), so the normalised rows are never written out.
//
// Chunk layout: row r's 16-byte piece c sits at piece c ^ (r & 7), so the
// reads of eight different rows at the same k (and of a thread's own row)
// are free of bank conflicts.
constexpr int kHeadRPL = 3;                            // rows per lane in the sums
constexpr int kHeadWarpRows = 8 * kHeadRPL;            // rows per warp
constexpr int kHeadThreads = 256;
constexpr int kHeadMaxRows = (kHeadThreads / 32) * kHeadWarpRows;  // 192
constexpr int kHeadKC = 32;

__device__ __forceinline__ int head_idx(int r, int k) {
  return r * kHeadKC + ((((k >> 2) ^ (r & 7))) << 2) + (k & 3);
}

template <int STAGES>
__global__ void __launch_bounds__(kHeadThreads, 1) out_head_kernel(
    const float* __restrict__ x, const float* __restrict__ g, const float* __restrict__ w,
    const float* __restrict__ bias, float* __restrict__ y, int M, int D, float eps, int GR) {
  extern __shared__ float4 head_smem[];
  float* wt = reinterpret_cast<float*>(head_smem);  // [D][32]
  float* gs = wt + (size_t)D * 32;                   // [D]
  float* xs = gs + D;                                // [STAGES][GR][kHeadKC]
  const size_t chunk_floats = (size_t)GR * kHeadKC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lg = lane >> 2, lq = lane & 3;
  // W^T in 32 x 32 tiles: lane l reads column k = 32t + l of all 32 rows
  // (coalesced), then writes its W^T row as eight 16-byte pieces.
  for (int t = warp; t < D / 32; t += kHeadThreads / 32) {
    const int k = 32 * t + lane;
    float v[32];
#pragma unroll
    for (int n = 0; n < 32; n++) v[n] = w[(size_t)n * D + k];
#pragma unroll
    for (int j = 0; j < 8; j++)
      *reinterpret_cast<float4*>(wt + (size_t)k * 32 + 4 * j) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  for (int i = tid; i < D; i += kHeadThreads) gs[i] = g[i];
  float bq[8];
#pragma unroll
  for (int j = 0; j < 8; j++) bq[j] = bias ? bias[8 * lq + j] : 0.0f;
  const int nk = (D + kHeadKC - 1) / kHeadKC;
  const int share = (M + gridDim.x - 1) / gridDim.x;
  const int rbeg = blockIdx.x * share, rend = min(M, rbeg + share);
  // One chunk: GR rows x 8 pieces of 16 bytes (rows past the share repeat its
  // last row; their results are not stored).
  auto stage = [&](int g0, int kc) {
    float* dst = xs + (size_t)(kc % STAGES) * chunk_floats;
    const int kw = min(kHeadKC, D - kc * kHeadKC) / 4;
    for (int i = tid; i < GR * (kHeadKC / 4); i += kHeadThreads) {
      const int r = i >> 3, c = i & 7;
      if (c < kw) {
        const int row = min(g0 + r, rend - 1);
        cp_async16(dst + r * kHeadKC + ((c ^ (r & 7)) << 2),
                   x + (size_t)row * D + (size_t)kc * kHeadKC + 4 * c);
      }
    }
  };
  // Streams chunks 0 .. nk-1 of the group through the ring; body(kc, buf)
  // runs once chunk kc has landed and is visible to every thread.
  auto stream = [&](int g0, auto&& body) {
#pragma unroll
    for (int j = 0; j < STAGES - 1; j++) {
      if (j < nk) stage(g0, j);
      cp_async_commit();
    }
    for (int kc = 0; kc < nk; kc++) {
      if (kc + STAGES - 1 < nk) stage(g0, kc + STAGES - 1);
      cp_async_commit();
      cp_async_wait<STAGES - 1>();
      __syncthreads();
      body(kc, xs + (size_t)(kc % STAGES) * chunk_floats);
      __syncthreads();  // the buffer is staged again STAGES - 1 chunks later
    }
    cp_async_wait<0>();
  };
  __syncthreads();  // W^T and g staged
  const bool own_row = tid < GR;  // thread t owns row t of each group
  for (int g0 = rbeg; g0 < rend; g0 += GR) {
    // Pass 1: thread t sums the squares of row t in increasing d.
    float ms = 0.0f;
    stream(g0, [&](int kc, float* buf) {
      if (!own_row) return;
      const int kl = min(kHeadKC, D - kc * kHeadKC);
      for (int k = 0; k < kl; k += 4) {
        const float4 v = *reinterpret_cast<const float4*>(buf + head_idx(tid, k));
        ms = __fadd_rn(ms, __fmul_rn(v.x, v.x));
        ms = __fadd_rn(ms, __fmul_rn(v.y, v.y));
        ms = __fadd_rn(ms, __fmul_rn(v.z, v.z));
        ms = __fadd_rn(ms, __fmul_rn(v.w, v.w));
      }
    });
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ms, (float)D), eps)));
    // Pass 2: normalise each chunk in place (thread t: row t), then the sums.
    float acc[kHeadRPL][8];
#pragma unroll
    for (int i = 0; i < kHeadRPL; i++)
#pragma unroll
      for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
    // A warp wholly past the group (or the share) skips the sums.
    const bool active = warp * kHeadWarpRows < GR && g0 + warp * kHeadWarpRows < rend;
    stream(g0, [&](int kc, float* buf) {
      const int k0 = kc * kHeadKC;
      const int kl = min(kHeadKC, D - k0);
      for (int k = 0; k < kl && own_row; k += 4) {
        float4* p = reinterpret_cast<float4*>(buf + head_idx(tid, k));
        float4 v = *p;
        const float4 gg = *reinterpret_cast<const float4*>(gs + k0 + k);
        v.x = __fmul_rn(__fmul_rn(v.x, inv), gg.x);
        v.y = __fmul_rn(__fmul_rn(v.y, inv), gg.y);
        v.z = __fmul_rn(__fmul_rn(v.z, inv), gg.z);
        v.w = __fmul_rn(__fmul_rn(v.w, inv), gg.w);
        *p = v;
      }
      __syncthreads();
      if (!active) return;
      for (int k = 0; k < kl; k += 4) {
        float4 a[kHeadRPL];
#pragma unroll
        for (int i = 0; i < kHeadRPL; i++)
          a[i] = *reinterpret_cast<const float4*>(
              buf + head_idx(min(warp * kHeadWarpRows + lg + 8 * i, GR - 1), k));
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const float4* wr = reinterpret_cast<const float4*>(wt + (size_t)(k0 + k + kk) * 32 + 8 * lq);
          const float4 wl = wr[0], wh = wr[1];
          const float wv[8] = {wl.x, wl.y, wl.z, wl.w, wh.x, wh.y, wh.z, wh.w};
#pragma unroll
          for (int i = 0; i < kHeadRPL; i++) {
            const float xv = kk == 0 ? a[i].x : kk == 1 ? a[i].y : kk == 2 ? a[i].z : a[i].w;
#pragma unroll
            for (int j = 0; j < 8; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xv, wv[j]));
          }
        }
      }
    });
    if (active) {
#pragma unroll
      for (int i = 0; i < kHeadRPL; i++) {
        const int m = g0 + warp * kHeadWarpRows + lg + 8 * i;
        if (m >= rend || warp * kHeadWarpRows + lg + 8 * i >= GR) continue;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; j++) o[j] = __fadd_rn(acc[i][j], bq[j]);
        float4* dst = reinterpret_cast<float4*>(y + (size_t)m * 32 + 8 * lq);
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
      }
    }
  }
}

size_t out_head_smem(int D, int stages, int GR) {
  return sizeof(float) * ((size_t)D * 32 + D + (size_t)stages * GR * kHeadKC);
}

constexpr size_t kHeadSmemCap = 227 * 1024;

// Launch geometry of the fused output head: one block per SM (at most one
// per 64 rows), each over a contiguous share of the rows in groups of GR.
struct HeadPlan {
  int grid, GR, stages;  // stages 0: the fused kernel does not apply
};

HeadPlan out_head_plan(const IroDiTModelDev* m, const float* x, const float* vel, int rows) {
  HeadPlan p{0, 0, 0};
  const int D = m->block[0].model_dim;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(m->out_w) |
                         reinterpret_cast<uintptr_t>(m->out_norm) |
                         reinterpret_cast<uintptr_t>(vel)) & 15u) == 0;
  if (m->latent_dim != 32 || !aligned || D % 32 != 0 || rows <= 0) return p;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  p.grid = std::min(sms, cdiv(rows, 64));
  p.GR = std::min(kHeadMaxRows, cdiv(rows, p.grid));
  if (out_head_smem(D, 4, p.GR) <= kHeadSmemCap) p.stages = 4;
  else if (out_head_smem(D, 3, p.GR) <= kHeadSmemCap) p.stages = 3;
  return p;
}

bool output_head_fused(const IroDiTModelDev* m, const float* x, const float* vel, int rows) {
  return out_head_plan(m, x, vel, rows).stages > 0;
}

template <int STAGES>
int launch_out_head(const IroDiTModelDev* m, const float* x, int rows, float* vel,
                    const HeadPlan& p, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {false};  // the shared-memory opt-in is per device
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(out_head_kernel<STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kHeadSmemCap);
    attr[dev & 63] = true;
  }
  const int D = m->block[0].model_dim;
  out_head_kernel<STAGES><<<p.grid, kHeadThreads, out_head_smem(D, STAGES, p.GR), s>>>(
      x, m->out_norm, m->out_w, m->out_b, vel, rows, D, m->norm_eps, p.GR);
  return check_launch();
}

// The output head on `rows` hidden rows into vel [rows, 32]: the fused kernel
// when its shared memory fits (D <= 1280 with 3-4 chunks in flight), else
// the RMSNorm into `scratch` [rows, D] (may be x itself) and the general
// linear.
int output_head(const IroDiTModelDev* m, const float* x, int rows, float* vel, float* scratch,
                cudaStream_t s) {
  const HeadPlan p = out_head_plan(m, x, vel, rows);
  if (p.stages == 4) return launch_out_head<4>(m, x, rows, vel, p, s);
  if (p.stages == 3) return launch_out_head<3>(m, x, rows, vel, p, s);
  const int D = m->block[0].model_dim;
  rmsnorm_ref_kernel<<<cdiv(rows, kNR), 256, 0, s>>>(x, m->out_norm, scratch, rows, D,
                                                     m->norm_eps);
  int st = check_launch();
  if (st) return st;
  return linear_ref(scratch, m->out_w, m->out_b, vel, rows, m->latent_dim, D, 0, s);
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
  if ((st = output_head(m, x, B * S, vel, x, s))) return st;
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
  if (!norm && !output_head_fused(m, x, velocity, rows)) {
    norm = static_cast<float*>(arena_get(c, sizeof(float) * (size_t)rows * D, &st));
    if (!norm) return st;
  }
  return output_head(m, x, rows, velocity, norm, s);
}

}  // extern "C"
