// dit_block.cu — one RF-DiT transformer block (dit.c:983-1051) resident on the
// device: the int8 projections run through the tcgen05 GEMMs, the fp32
// support work through the kernels below.
//
//   AdaLN params   (dit.c:543-559, 585-593)  adaln_params_kernel
//   AdaLN apply    (dit.c:597-609)           adaln_apply_kernel
//   QKVG           (dit.c:785-792)           one int8 GEMM, four outputs
//   head RMSNorm + half RoPE (dit.c:638-706) qk_norm_rope_kernel
//   joint attention, sigmoid gate (dit.c:806-862)  attention_kernel
//   Wo             (dit.c:876-884)           int8 GEMM
//   gated residual (dit.c:1013-1020)         gated_residual_kernel
//   SwiGLU         (dit.c:913-969)           iro_int8_swiglu_dev
//
// The fp32 parts follow the reference's formulas and per-element operation
// order; reductions (row mean squares, dot products, softmax sums) are summed
// in a different order than the reference's sequential loops, so their
// results agree to rounding, not bit for bit.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "gemm_i8.cuh"
#include "quantize.cuh"

namespace iro {
namespace {

constexpr int kHD = 64;  // head dimension (IRO_DIT_HEAD_DIM)

__device__ __forceinline__ float silu_ref(float x) {
  // ops.c iro_silu: x / (1 + expf(-x)).
  return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

// The nine AdaLN matrices of one block half, in IroAdaLN order
// (dit.h: shift down/up/bias, scale down/up/bias, gate down/up/bias).
struct AdaMats {
  const float* m[9];
};

// One (batch row, branch) per block.  out = up(down(silu(c))) + bias + c for
// c = cond[b, branch*D .. +D]; the gate branch (2) ends in tanhf.
__global__ void __launch_bounds__(256) adaln_params_kernel(
    const float* __restrict__ cond, int D, int R, const AdaMats mats,
    float* __restrict__ shift, float* __restrict__ scale, float* __restrict__ gate) {
  extern __shared__ float sh[];
  float* act = sh;       // [D]
  float* low = sh + D;   // [R]
  const int b = blockIdx.x, br = blockIdx.y;
  const float* c = cond + (size_t)b * 3 * D + (size_t)br * D;
  const float* down = mats.m[3 * br + 0];  // [R, D]
  const float* up = mats.m[3 * br + 1];    // [D, R]
  const float* bias = mats.m[3 * br + 2];  // [D]
  for (int d = threadIdx.x; d < D; d += blockDim.x) act[d] = silu_ref(c[d]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < R; r += nw) {
    const float* row = down + (size_t)r * D;
    float s = 0.0f;
    for (int d = lane; d < D; d += 32) s = __fmaf_rn(act[d], row[d], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) low[r] = s;
  }
  __syncthreads();
  float* out = (br == 0 ? shift : br == 1 ? scale : gate) + (size_t)b * D;
  for (int d = warp; d < D; d += nw) {
    const float* row = up + (size_t)d * R;
    float s = 0.0f;
    for (int r = lane; r < R; r += 32) s = __fmaf_rn(low[r], row[r], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      float v = __fadd_rn(__fadd_rn(s, bias[d]), c[d]);
      out[d] = br == 2 ? tanhf(v) : v;
    }
  }
}

// h = x * inv * (1 + scale) + shift per row (dit.c:597-609), one warp per row.
// The AdaLN parameters of batch row b are row (b / prow) of shift/scale.
__global__ void __launch_bounds__(256) adaln_apply_kernel(const float* __restrict__ x, int rows,
                                                          int S, int D, float eps, int prow,
                                                          const float* __restrict__ shift,
                                                          const float* __restrict__ scale,
                                                          float* __restrict__ h) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * D;
  float ms = 0.0f;
  for (int d = lane; d < D; d += 32) ms = __fmaf_rn(xr[d], xr[d], ms);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ms += __shfl_xor_sync(0xffffffffu, ms, o);
  const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ms, (float)D), eps)));
  const int b = row / S / prow;
  const float* sh = shift + (size_t)b * D;
  const float* sc = scale + (size_t)b * D;
  float* hr = h + (size_t)row * D;
  for (int d = lane; d < D; d += 32)
    hr[d] = __fadd_rn(__fmul_rn(__fmul_rn(xr[d], inv), __fadd_rn(1.0f, sc[d])), sh[d]);
}

// Per (row, head): RMSNorm of q and k with their weights, then RoPE on the
// first half of the heads (dit.c:638-706).  Lane p holds dims 2p, 2p+1.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    float* __restrict__ q, float* __restrict__ k, int rows, int S, int D, int heads, float eps,
    const float* __restrict__ qw, const float* __restrict__ kw, const float* __restrict__ rcos,
    const float* __restrict__ rsin) {
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= rows * heads) return;
  const int row = item / heads, hd = item % heads;
  const int s = row % S;
  const int d = 2 * lane;
  float* qr = q + (size_t)row * D + hd * kHD;
  float* kr = k + (size_t)row * D + hd * kHD;
  float2 qv = *reinterpret_cast<float2*>(qr + d);
  float2 kv = *reinterpret_cast<float2*>(kr + d);
  float qms = __fmaf_rn(qv.y, qv.y, __fmul_rn(qv.x, qv.x));
  float kms = __fmaf_rn(kv.y, kv.y, __fmul_rn(kv.x, kv.x));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    qms += __shfl_xor_sync(0xffffffffu, qms, o);
    kms += __shfl_xor_sync(0xffffffffu, kms, o);
  }
  const float qinv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(qms, (float)kHD), eps)));
  const float kinv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(kms, (float)kHD), eps)));
  const float* qwh = qw + hd * kHD;
  const float* kwh = kw + hd * kHD;
  const float q0 = __fmul_rn(qv.x, __fmul_rn(qinv, qwh[d]));
  const float q1 = __fmul_rn(qv.y, __fmul_rn(qinv, qwh[d + 1]));
  const float k0 = __fmul_rn(kv.x, __fmul_rn(kinv, kwh[d]));
  const float k1 = __fmul_rn(kv.y, __fmul_rn(kinv, kwh[d + 1]));
  if (hd >= heads / 2) {
    *reinterpret_cast<float2*>(qr + d) = make_float2(q0, q1);
    *reinterpret_cast<float2*>(kr + d) = make_float2(k0, k1);
    return;
  }
  const float c = rcos[(size_t)s * (kHD / 2) + lane], sn = rsin[(size_t)s * (kHD / 2) + lane];
  *reinterpret_cast<float2*>(qr + d) =
      make_float2(__fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, sn)),
                  __fadd_rn(__fmul_rn(q0, sn), __fmul_rn(q1, c)));
  *reinterpret_cast<float2*>(kr + d) =
      make_float2(__fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, sn)),
                  __fadd_rn(__fmul_rn(k0, sn), __fmul_rn(k1, c)));
}

// Valid context positions per batch row (dit.c:811-813, 828-839); the mask
// is [B, C] even when the context K/V are shared by the batch.
__global__ void context_list_kernel(const uint8_t* __restrict__ mask, int rows, int C,
                                    int* __restrict__ list, int* __restrict__ count) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= rows) return;
  int n = 0;
  for (int c = 0; c < C; c++)
    if (mask[(size_t)b * C + c]) list[(size_t)b * C + n++] = c;
  count[b] = n;
}

// Joint attention of one (64-query tile, head, batch row): keys are the S
// self tokens then the valid context tokens; softmax(q.k / 8) . v, then the
// sigmoid gate (dit.c:853, ops.c iro_sigmoid_mul_inplace).  Online softmax in
// fp32; two threads per query row, each holding 32 of the 64 output dims.
constexpr int kAQ = 64;   // queries per block
constexpr int kAK = 64;   // keys per tile
constexpr int kAThreads = 2 * kAQ;

struct AttnArgs {
  const float* q;
  const float* k;
  const float* v;
  const float* g;        // gate projection
  const float* ck;       // context keys [Cb, C, D]
  const float* cv;
  const int* clist;      // [B, C] valid context positions per batch row
  const int* ccount;     // [B]
  int ctx_group;         // batch rows per context block
  int S, C, D;
  float* mix;
};

__global__ void __launch_bounds__(kAThreads) attention_kernel(AttnArgs a) {
  // 48 KB: K and V tiles, and the probabilities with the key index XOR'ed by
  // the query row (conflict-free reads of one key across 16 query rows).
  __shared__ float ks[kAK][kHD];
  __shared__ float vs[kAK][kHD];
  __shared__ float ps[kAQ][kAK];
  const int b = blockIdx.z, hd = blockIdx.y;
  const int q0 = blockIdx.x * kAQ;
  const int t = threadIdx.x;
  const int qi = t >> 1;        // query within the tile
  const int half = t & 1;       // which 32 keys / 32 dims
  const int qrow = q0 + qi;
  const bool qok = qrow < a.S;
  const int cb = b / a.ctx_group;  // K/V row block
  const int nctx = a.ccount[b];
  const int joined = a.S + nctx;
  const size_t base = (size_t)b * a.S;

  float qv[kHD];
  {
    const float* qr = a.q + (base + (qok ? qrow : 0)) * a.D + hd * kHD;
#pragma unroll
    for (int d = 0; d < kHD; d += 4) {
      const float4 x = *reinterpret_cast<const float4*>(qr + d);
      qv[d] = x.x;
      qv[d + 1] = x.y;
      qv[d + 2] = x.z;
      qv[d + 3] = x.w;
    }
  }
  float o[kHD / 2];
#pragma unroll
  for (int i = 0; i < kHD / 2; i++) o[i] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  const float scale = __fdiv_rn(1.0f, sqrtf((float)kHD));

  for (int j0 = 0; j0 < joined; j0 += kAK) {
    const int nk = min(kAK, joined - j0);
    __syncthreads();
    for (int i = t; i < kAK * (kHD / 4); i += kAThreads) {
      const int kk = i / (kHD / 4), d4 = (i % (kHD / 4)) * 4;
      float4 kx = make_float4(0.f, 0.f, 0.f, 0.f), vx = kx;
      if (kk < nk) {
        const int j = j0 + kk;
        const float *kp, *vp;
        if (j < a.S) {
          kp = a.k + (base + j) * a.D + hd * kHD;
          vp = a.v + (base + j) * a.D + hd * kHD;
        } else {
          const size_t crow = (size_t)cb * a.C + a.clist[(size_t)b * a.C + (j - a.S)];
          kp = a.ck + crow * a.D + hd * kHD;
          vp = a.cv + crow * a.D + hd * kHD;
        }
        kx = *reinterpret_cast<const float4*>(kp + d4);
        vx = *reinterpret_cast<const float4*>(vp + d4);
      }
      ks[kk][d4] = kx.x;
      ks[kk][d4 + 1] = kx.y;
      ks[kk][d4 + 2] = kx.z;
      ks[kk][d4 + 3] = kx.w;
      *reinterpret_cast<float4*>(&vs[kk][d4]) = vx;
    }
    __syncthreads();
    // Scores of this thread's 32 keys.
    float sc[kAK / 2];
    float tmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < kAK / 2; i++) {
      const int kk = half * (kAK / 2) + i;
      float s = 0.0f;
#pragma unroll
      for (int d = 0; d < kHD; d++) s = __fmaf_rn(qv[d], ks[kk][d], s);
      s = kk < nk ? __fmul_rn(s, scale) : -INFINITY;
      sc[i] = s;
      tmax = fmaxf(tmax, s);
    }
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    const float mn = fmaxf(m, tmax);
    const float corr = expf(m - mn);  // 0 on the first tile (m = -inf)
    float tsum = 0.0f;
#pragma unroll
    for (int i = 0; i < kAK / 2; i++) {
      const float p = expf(sc[i] - mn);
      ps[qi][(half * (kAK / 2) + i) ^ (qi & 31)] = p;
      tsum += p;
    }
    tsum += __shfl_xor_sync(0xffffffffu, tsum, 1);
    l = l * corr + tsum;
    m = mn;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < kHD / 2; i++) o[i] *= corr;
    for (int kk = 0; kk < nk; kk++) {
      const float p = ps[qi][kk ^ (qi & 31)];
#pragma unroll
      for (int i = 0; i < kHD / 2; i++) o[i] = __fmaf_rn(p, vs[kk][half * (kHD / 2) + i], o[i]);
    }
  }
  if (!qok) return;
  const float* gr = a.g + (base + qrow) * a.D + hd * kHD + half * (kHD / 2);
  float* out = a.mix + (base + qrow) * a.D + hd * kHD + half * (kHD / 2);
  const float inv_l = __fdiv_rn(1.0f, l);
#pragma unroll
  for (int i = 0; i < kHD / 2; i++) {
    const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gr[i])));
    out[i] = __fmul_rn(__fmul_rn(o[i], inv_l), sg);
  }
}

// x += gate[b] * branch (dit.c:1013-1020); gate row b / prow.
__global__ void gated_residual_kernel(float* __restrict__ x, const float* __restrict__ branch,
                                      const float* __restrict__ gate, long long n, int S, int D,
                                      int prow) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / D;
    const int d = (int)(i - row * D);
    const int b = (int)(row / S) / prow;
    x[i] = __fadd_rn(x[i], __fmul_rn(gate[(size_t)b * D + d], branch[i]));
  }
}

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace
}  // namespace iro

using namespace iro;

extern "C" {

// dit.c:644-705: cos/sin of position s and pair p, produced by the
// reference's double-precision rotation recurrence (computed on the host with
// the same libm calls, so the tables are the reference's exact floats).
int iro_dit_rope_table(float* cos_out, float* sin_out, int S, int head_dim) {
  if (!cos_out || !sin_out || S <= 0 || head_dim <= 0 || head_dim % 2) return IRO_ERR_INVALID;
  const int P = head_dim / 2;
  std::vector<double> cs(P), ss(P), cp(P, 1.0), sp(P, 0.0);
  for (int p = 0; p < P; p++) {
    const double inv = 1.0 / pow(10000.0, (double)(2 * p) / head_dim);
    cs[p] = cos(inv);
    ss[p] = sin(inv);
  }
  for (int s = 0; s < S; s++) {
    for (int p = 0; p < P; p++) {
      cos_out[(size_t)s * P + p] = (float)cp[p];
      sin_out[(size_t)s * P + p] = (float)sp[p];
      const double c = cp[p], sn = sp[p];
      cp[p] = c * cs[p] - sn * ss[p];
      sp[p] = sn * cs[p] + c * ss[p];
    }
  }
  return IRO_OK;
}

size_t iro_dit_block_workspace_bytes(const IroDiTBlockDev* blk, int B, int S, int C,
                                     int context_batch) {
  if (!blk || B <= 0 || S <= 0 || C <= 0) return 0;
  const size_t M = (size_t)B * S, D = (size_t)blk->model_dim;
  size_t t = 0;
  t += 7 * al256(sizeof(float) * M * D);                           // h, q, k, v, g, mix, branch
  t += al256(M * D) + 2 * al256(sizeof(float) * M);                // codes + row params
  t += 6 * al256(sizeof(float) * (size_t)B * D);                   // AdaLN params
  t += al256(sizeof(int) * (size_t)B * C) + al256(sizeof(int) * B);
  t += iro_int8_swiglu_workspace_bytes((int)M, blk->model_dim, blk->mlp_dim,
                                       (blk->residual_mask & 8) != 0);
  return t;
}

int iro_dit_block_dev(const IroDiTBlockDev* blk, float* x, const float* cond, int cond_rows,
                      const float* ctx_k, const float* ctx_v, const uint8_t* ctx_mask,
                      int context_batch, int B, int S, int C, const float* rope_cos,
                      const float* rope_sin, void* workspace, void* stream) {
  if (!blk || !x || !cond || !ctx_k || !ctx_v || !ctx_mask || !rope_cos || !rope_sin ||
      B <= 0 || S <= 0 || C <= 0 || context_batch <= 0 || B % context_batch != 0 ||
      (cond_rows != 1 && cond_rows != B))
    return IRO_ERR_INVALID;
  const int D = blk->model_dim, NH = blk->heads, R = blk->adaln_rank, H = blk->mlp_dim;
  if (blk->head_dim != kHD || NH * kHD != D || R <= 0 || H <= 0 || D % 16 != 0)
    return IRO_ERR_UNSUPPORTED;
  // Residual (two-term) policy: the reference's default, W2 only (dit.c:
  // 429-436), or none; the QKVG, Wo and W1/W3 two-term forms are not built.
  if ((blk->residual_mask & ~8) != 0) return IRO_ERR_UNSUPPORTED;
  if (blk->qkvg.N != 4 * D || blk->qkvg.K != D || blk->wo.N != D || blk->wo.K != D ||
      blk->w13.layout != IRO_LAYOUT_GATED_PAIR || blk->w13.K != D || blk->w13.hidden != H ||
      blk->w2.N != D || blk->w2.K != H)
    return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  const size_t M = (size_t)B * S;
  const size_t need = iro_dit_block_workspace_bytes(blk, B, S, C, context_batch);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!ws) {
    ws = static_cast<uint8_t*>(arena_get(c, need, &st));
    if (!ws) return st;
  }
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = ws + off;
    off += al256(bytes);
    return p;
  };
  float* h = reinterpret_cast<float*>(take(sizeof(float) * M * D));
  float* q = reinterpret_cast<float*>(take(sizeof(float) * M * D));
  float* k = reinterpret_cast<float*>(take(sizeof(float) * M * D));
  float* v = reinterpret_cast<float*>(take(sizeof(float) * M * D));
  float* g = reinterpret_cast<float*>(take(sizeof(float) * M * D));
  float* mix = reinterpret_cast<float*>(take(sizeof(float) * M * D));
  float* branch = reinterpret_cast<float*>(take(sizeof(float) * M * D));
  uint8_t* codes = take(M * D);
  float* rs = reinterpret_cast<float*>(take(sizeof(float) * M));
  int32_t* rz = reinterpret_cast<int32_t*>(take(sizeof(float) * M));
  float* ada[6];
  for (int i = 0; i < 6; i++) ada[i] = reinterpret_cast<float*>(take(sizeof(float) * (size_t)B * D));
  int* clist = reinterpret_cast<int*>(take(sizeof(int) * (size_t)B * C));
  int* ccount = reinterpret_cast<int*>(take(sizeof(int) * B));
  void* sw_ws = ws + off;
  const float* rcos = rope_cos;
  const float* rsin = rope_sin;

  context_list_kernel<<<cdiv(B, 64), 64, 0, s>>>(ctx_mask, B, C, clist, ccount);
  if ((st = check_launch())) return st;

  const size_t ada_smem = sizeof(float) * (size_t)(D + R);
  const int prow = B / cond_rows;  // batch rows per AdaLN parameter row
  const long long n = (long long)M * D;
  const int res_blocks = (int)std::min<long long>((n + 255) / 256, (long long)c->num_sms * 16);
  for (int half = 0; half < 2; half++) {
    // AdaLN (attention: matrices 0..8, MLP: 9..17) and apply.
    AdaMats am;
    for (int i = 0; i < 9; i++) am.m[i] = blk->adaln[half][i];
    adaln_params_kernel<<<dim3(cond_rows, 3), 256, ada_smem, s>>>(cond, D, R, am, ada[0],
                                                                  ada[1], ada[2]);
    if ((st = check_launch())) return st;
    adaln_apply_kernel<<<cdiv((int)M, 8), 256, 0, s>>>(x, (int)M, S, D, blk->norm_eps, prow,
                                                       ada[0], ada[1], h);
    if ((st = check_launch())) return st;
    if (half == 0) {
      // QKVG on one quantised copy of h (dit.c:785-792).
      st = quantize_rows_launch(h, (int)M, D, codes, rs, rz, 0, s);
      if (st) return st;
      GemmRequest r;
      r.epi = EPI_SPLIT;
      r.M = (int)M;
      r.a = codes;
      r.lda = D;
      r.sx = rs;
      r.zp = rz;
      r.w = &blk->qkvg;
      r.bias = nullptr;
      r.nout = 4;
      r.seg = D;
      r.outs[0] = q;
      r.outs[1] = k;
      r.outs[2] = v;
      r.outs[3] = g;
      if ((st = gemm_launch(c, r, s))) return st;
      qk_norm_rope_kernel<<<cdiv((int)M * NH, 8), 256, 0, s>>>(
          q, k, (int)M, S, D, NH, blk->norm_eps, blk->q_norm, blk->k_norm, rcos, rsin);
      if ((st = check_launch())) return st;
      AttnArgs aa{q, k, v, g, ctx_k, ctx_v, clist, ccount, B / context_batch, S, C, D, mix};
      attention_kernel<<<dim3(cdiv(S, kAQ), NH, B), kAThreads, 0, s>>>(aa);
      if ((st = check_launch())) return st;
      // Wo on the quantised gated mix (dit.c:876-884).
      st = quantize_rows_launch(mix, (int)M, D, codes, rs, rz, 0, s);
      if (st) return st;
      GemmRequest o;
      o.epi = EPI_LINEAR;
      o.M = (int)M;
      o.a = codes;
      o.lda = D;
      o.sx = rs;
      o.zp = rz;
      o.w = &blk->wo;
      o.y = branch;
      o.ldy = D;
      if ((st = gemm_launch(c, o, s))) return st;
    } else {
      st = iro_int8_swiglu_dev(h, (int)M, &blk->w13, &blk->w2, nullptr, branch,
                               (blk->residual_mask & 8) != 0, sw_ws, s);
      if (st) return st;
    }
    gated_residual_kernel<<<res_blocks, 256, 0, s>>>(x, branch, ada[2], n, S, D, prow);
    if ((st = check_launch())) return st;
  }
  return IRO_OK;
}

}  // extern "C"
