// dit_forward.cu — the parts of one RF-DiT Euler step around the blocks
// (sampler.c:238-297, dit.c:488-541, 1070-1090), resident on the device:
//
//   conditioner  timestep embedding -> linear, silu -> linear, silu -> linear
//                (dit.c:488-530), computed once per step: every row of a step
//                shares the timestep (sampler.c:246-253)
//   input        x_t [R*S, 32] -> [R*S, D] (dit.c:532-541), broadcast to the
//                request's CFG rows (sampler.c:256-262)
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
// 256-thread block, 4 x 4 outputs per thread, k in increasing order.
constexpr int kLK = 16;

template <int BM, int BN>
__global__ void __launch_bounds__(256) linear_ref_kernel(const float* __restrict__ x,
                                                         const float* __restrict__ w,
                                                         const float* __restrict__ bias,
                                                         float* __restrict__ y, int M, int N, int K,
                                                         int silu) {
  static_assert((BM / 4) * (BN / 4) == 256, "4 x 4 outputs per thread, 256 threads");
  __shared__ float xs[kLK][BM + 1];
  __shared__ float ws[kLK][BN + 1];
  const int tx = threadIdx.x % (BN / 4), ty = threadIdx.x / (BN / 4);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
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
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
          acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(xs[kk][ty * 4 + i], ws[kk][tx * 4 + j]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = __fadd_rn(acc[i][j], bias ? bias[n] : 0.0f);
      if (silu) v = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
      y[(size_t)m * N + n] = v;
    }
  }
}

int linear_ref(const float* x, const float* w, const float* bias, float* y, int M, int N, int K,
               int silu, cudaStream_t s) {
  if (N <= 32)
    linear_ref_kernel<128, 32><<<dim3(cdiv(N, 32), cdiv(M, 128)), 256, 0, s>>>(x, w, bias, y, M,
                                                                              N, K, silu);
  else
    linear_ref_kernel<64, 64><<<dim3(cdiv(N, 64), cdiv(M, 64)), 256, 0, s>>>(x, w, bias, y, M, N,
                                                                            K, silu);
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

// x[(r*cfg + c)*S + s] = p[r*S + s] for every CFG row c of request r.
__global__ void expand_rows_kernel(const float* __restrict__ p, float* __restrict__ x, int R,
                                   int cfg, int S, int D) {
  const long long n = (long long)R * cfg * S * D;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / D;
    const int d = (int)(i - row * D);
    const long long s = row % S;
    const long long r = row / ((long long)S * cfg);
    x[i] = p[(r * S + s) * D + d];
  }
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
  for (int i = t; i < kNR * D; i += 256) {
    const int rr = i / D, d = i % D;
    const int m = r0 + rr;
    if (m < M) {
      const size_t o = (size_t)m * D + d;
      y[o] = __fmul_rn(__fmul_rn(x[o], inv_s[rr]), w[d]);
    }
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
  uint8_t* cond_mask;
  uint8_t* rest;
};

size_t head_bytes(int R, int S, int C) {
  return 2 * al256(sizeof(float) * (size_t)S * 32) + al256((size_t)R * C);
}

StepBufs carve(uint8_t* ws, int S) {
  StepBufs b;
  const size_t tab = al256(sizeof(float) * (size_t)S * 32);
  b.rcos = reinterpret_cast<float*>(ws);
  b.rsin = reinterpret_cast<float*>(ws + tab);
  b.cond_mask = ws + 2 * tab;
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
  cudaError_t e = cudaMemcpyAsync(b.rcos, hc.data(), sizeof(float) * hc.size(),
                                  cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(b.rsin, hs.data(), sizeof(float) * hs.size(), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

// One step with `cfg` active rows per request, `mask` [R*cfg, C] for those
// rows; `full_cfg` is the width the scratch was sized for.
int step_impl(Ctx* c, const IroDiTModelDev* m, float* state, int R, int cfg, int full_cfg,
              int S, float t, float t_next, const float* scales, const float* const* ctx_k,
              const float* const* ctx_v, const uint8_t* mask, int C, const StepBufs& tb,
              cudaStream_t s) {
  const int D = m->block[0].model_dim, L = m->latent_dim, TD = m->timestep_dim;
  const int B = R * cfg, Bfull = R * full_cfg;
  uint8_t* ws = tb.rest;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = ws + off;
    off += al256(bytes);
    return p;
  };
  float* emb = reinterpret_cast<float*>(take(sizeof(float) * TD));
  float* h0 = reinterpret_cast<float*>(take(sizeof(float) * D));
  float* h1 = reinterpret_cast<float*>(take(sizeof(float) * D));
  float* cond = reinterpret_cast<float*>(take(sizeof(float) * 3 * (size_t)D));
  float* proj = reinterpret_cast<float*>(take(sizeof(float) * (size_t)R * S * D));
  float* x = reinterpret_cast<float*>(take(sizeof(float) * (size_t)Bfull * S * D));
  float* vel = reinterpret_cast<float*>(take(sizeof(float) * (size_t)Bfull * S * L));
  float* params = reinterpret_cast<float*>(take(sizeof(float) * 6 * (size_t)m->layers * D));
  void* ada_scratch = take(dit_adaln_scratch_bytes(2 * m->layers, 1, D, m->block[0].adaln_rank));
  void* blk_ws = ws + off;
  int st;
  // Conditioner, once: every row shares the timestep.
  timestep_embedding_kernel<<<cdiv(TD / 2, 128), 128, 0, s>>>(nullptr, t, TD, emb);
  if ((st = check_launch())) return st;
  if ((st = linear_ref(emb, m->cond_w0, nullptr, h0, 1, D, TD, 1, s))) return st;
  if ((st = linear_ref(h0, m->cond_w1, nullptr, h1, 1, D, D, 1, s))) return st;
  if ((st = linear_ref(h1, m->cond_w2, nullptr, cond, 1, 3 * D, D, 0, s))) return st;
  // Input projection per request, broadcast to its CFG rows.
  if ((st = linear_ref(state, m->in_w, m->in_b, proj, R * S, D, L, 0, s))) return st;
  const int eb = (int)std::min<long long>(((long long)B * S * D + 255) / 256, c->num_sms * 16LL);
  expand_rows_kernel<<<eb, 256, 0, s>>>(proj, x, R, cfg, S, D);
  if ((st = check_launch())) return st;
  // Every layer's AdaLN parameters in one batch: the step's rows share cond.
  const IroDiTBlockDev* blks[IRO_DIT_MAX_LAYERS];
  for (int l = 0; l < m->layers; l++) blks[l] = &m->block[l];
  if ((st = dit_adaln_params(blks, m->layers, cond, 1, params, ada_scratch, s))) return st;
  for (int l = 0; l < m->layers; l++) {
    st = dit_block_run(c, &m->block[l], x, params + (size_t)l * 6 * D, 1, ctx_k[l], ctx_v[l],
                       mask, R, B, S, C, tb.rcos, tb.rsin, blk_ws, s);
    if (st) return st;
  }
  // Output head (normalised in place: x is rebuilt from the state next
  // step) into the velocity, then the guided Euler update.
  rmsnorm_ref_kernel<<<cdiv(B * S, kNR), 256, 0, s>>>(x, m->out_norm, x, B * S, D, m->norm_eps);
  if ((st = check_launch())) return st;
  if ((st = linear_ref(x, m->out_w, m->out_b, vel, B * S, L, D, 0, s))) return st;
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
  if (!valid_model(m) || R <= 0 || cfg <= 0 || S <= 0 || C <= 0) return 0;
  const int D = m->block[0].model_dim, B = R * cfg;
  size_t t = head_bytes(R, S, C);
  t += al256(sizeof(float) * (size_t)m->timestep_dim);                 // embedding
  t += 2 * al256(sizeof(float) * (size_t)D) + al256(sizeof(float) * 3 * (size_t)D);  // cond
  t += al256(sizeof(float) * (size_t)R * S * D);                       // projected
  t += al256(sizeof(float) * (size_t)B * S * D);                       // x
  t += al256(sizeof(float) * (size_t)B * S * m->latent_dim);           // velocity
  t += al256(sizeof(float) * 6 * (size_t)m->layers * D);               // AdaLN params
  t += dit_adaln_scratch_bytes(2 * m->layers, 1, D, m->block[0].adaln_rank);
  return t + dit_block_body_bytes(&m->block[0], B, S, C, R);
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
  tb.rest = ws + head_bytes(R, S, C);
  if ((st = upload_rope(tb, S, s))) return st;
  return step_impl(c, m, state, R, cfg, cfg, S, t, t_next, cfg_scales, ctx_k, ctx_v, mask, C, tb,
                   s);
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
    ws = static_cast<uint8_t*>(arena_get(c, iro_dit_step_workspace_bytes(m, R, cfg, S, C), &st));
    if (!ws) return st;
  }
  StepBufs tb = carve(ws, S);
  tb.rest = ws + head_bytes(R, S, C);
  if ((st = upload_rope(tb, S, s))) return st;
  if (cfg > 1) {
    const int mb = (int)std::min<long long>(((long long)R * C + 255) / 256, c->num_sms * 4LL);
    cond_mask_kernel<<<mb, 256, 0, s>>>(mask, tb.cond_mask, R, cfg, C);
    if ((st = check_launch())) return st;
  }
  for (int step = 0; step < steps; step++) {
    // sampler.c:244-249, in the reference's float arithmetic.
    const float u = (float)step / (float)steps;
    const float u_next = (float)(step + 1) / (float)steps;
    const float t = (1.0f - u) * init_scale;
    const float t_next = (1.0f - u_next) * init_scale;
    const bool use_cfg = cfg > 1 && t >= cfg_min_t && t <= cfg_max_t;
    st = step_impl(c, m, state, R, use_cfg ? cfg : 1, cfg, S, t, t_next, cfg_scales, ctx_k, ctx_v,
                   use_cfg ? mask : (cfg > 1 ? tb.cond_mask : mask), C, tb, s);
    if (st) return st;
  }
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
