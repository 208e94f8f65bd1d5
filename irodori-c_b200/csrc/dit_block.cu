// dit_block.cu — one RF-DiT transformer block (dit.c:983-1051) resident on the
// device: the int8 projections run through the tcgen05 GEMMs, the fp32
// support work through the kernels below.
//
//   AdaLN params   (dit.c:543-559, 585-593)  adaln_params_kernel
//   AdaLN apply    (dit.c:597-609)           adaln_apply_kernel
//   QKVG           (dit.c:785-792)           one int8 GEMM, four outputs
//   head RMSNorm + half RoPE (dit.c:638-706) qk_norm_rope_kernel
//   joint attention, sigmoid gate (dit.c:806-862)  attention_tc_kernel
//                  (dit_attention.cu; tensor cores, fp16 operands, fp32
//                  accumulation), or attention_kernel (fp32 CUDA cores)
//   Wo             (dit.c:876-884)           int8 GEMM
//   gated residual (dit.c:1013-1020)         in the Wo and W2 GEMM epilogues
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

#include "diag.cuh"
#include "dit_attention.cuh"
#include "dit_block.cuh"
#include "dit_diag32.cuh"
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

// A batch of AdaLN matrix sets and where each set's parameters go: out[set]
// holds [3][rows][D] (shift, scale, gate).
constexpr int kAdaMaxSets = 2 * IRO_DIT_MAX_LAYERS;
struct AdaBatch {
  const float* m[kAdaMaxSets][9];
  float* out[kAdaMaxSets];
};

// AdaLN parameters (dit.c:543-559, 585-593) for a batch of matrix sets (one
// set = one block half): out = up(down(silu(c))) + bias + c for each of the
// three branches c = cond[row, br*D .. +D], the gate branch ending in tanhf.
// Three launches over all sets at once, one warp per output, so that the 24
// sets of a 12-layer step take a few microseconds instead of 24 serial
// low-parallelism launches.
__global__ void __launch_bounds__(256) adaln_act_kernel(const float* __restrict__ cond, int n,
                                                        float* __restrict__ act) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    act[i] = silu_ref(cond[i]);
}

// low[set][row][br][r] = sum_d act[row][br*D + d] * down[r][d]
__global__ void __launch_bounds__(256) adaln_down_kernel(const AdaBatch bt,
                                                         const float* __restrict__ act, int D,
                                                         int R, float* __restrict__ low) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * 8 + warp;  // br * R + r
  const int set = blockIdx.y, row = blockIdx.z, rows = gridDim.z;
  if (o >= 3 * R) return;
  const int br = o / R, r = o - br * R;
  const float* a = act + ((size_t)row * 3 + br) * D;
  const float* w = bt.m[set][3 * br] + (size_t)r * D;
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  int d = lane;
  // Unrolled: four iterations' loads issue before their multiply-adds (each
  // accumulator still sums its elements in increasing d).
#pragma unroll 4
  for (; d + 96 < D; d += 128) {
    s0 = __fmaf_rn(a[d], w[d], s0);
    s1 = __fmaf_rn(a[d + 32], w[d + 32], s1);
    s2 = __fmaf_rn(a[d + 64], w[d + 64], s2);
    s3 = __fmaf_rn(a[d + 96], w[d + 96], s3);
  }
  for (; d < D; d += 32) s0 = __fmaf_rn(a[d], w[d], s0);
  float sum = (s0 + s1) + (s2 + s3);
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, k);
  if (lane == 0) low[(((size_t)set * rows + row) * 3 + br) * R + r] = sum;
}

// out[set][br][row][d] = sum_r low[set][row][br][r] * up[d][r] + bias[d] + c[d]
__global__ void __launch_bounds__(256) adaln_up_kernel(const AdaBatch bt,
                                                       const float* __restrict__ cond,
                                                       const float* __restrict__ low, int D,
                                                       int R) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * 8 + warp;  // br * D + d
  const int set = blockIdx.y, row = blockIdx.z, rows = gridDim.z;
  if (o >= 3 * D) return;
  const int br = o / D, d = o - br * D;
  const float* lw = low + (((size_t)set * rows + row) * 3 + br) * R;
  const float* u = bt.m[set][3 * br + 1] + (size_t)d * R;
  float sum = 0.0f;
  for (int r = lane; r < R; r += 32) sum = __fmaf_rn(lw[r], u[r], sum);
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, k);
  if (lane == 0) {
    const float c = cond[(size_t)row * 3 * D + (size_t)br * D + d];
    const float v = __fadd_rn(__fadd_rn(sum, bt.m[set][3 * br + 2][d]), c);
    bt.out[set][((size_t)br * rows + row) * D + d] = br == 2 ? tanhf(v) : v;
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

// AdaLN apply fused with the row quantiser that follows it (dit.c:597-609
// then ops.c:321-348): h = x * inv * (1 + scale) + shift is formed in
// registers and written only as u8 codes with the row's scale and zero
// point, so h never goes to HBM.  One warp per row, lane l holding float4
// elements l, l + 32, ...; the range and codes use the quantiser's own
// arithmetic (row_params, quant_code).
template <int V>
__global__ void __launch_bounds__(256) adaln_quant_kernel(const float* __restrict__ x, int rows,
                                                          int S, int D, float eps, int prow,
                                                          const float* __restrict__ shift,
                                                          const float* __restrict__ scale,
                                                          uint8_t* __restrict__ q,
                                                          float* __restrict__ qs,
                                                          int32_t* __restrict__ qz) {
  grid_dep_wait();  // launched with programmatic stream serialization
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int D4 = D >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * D);
  float4 v[V];
  float ms = 0.0f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int j = i * 32 + lane;
    v[i] = j < D4 ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
    ms = __fmaf_rn(v[i].x, v[i].x, ms);
    ms = __fmaf_rn(v[i].y, v[i].y, ms);
    ms = __fmaf_rn(v[i].z, v[i].z, ms);
    ms = __fmaf_rn(v[i].w, v[i].w, ms);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ms += __shfl_xor_sync(0xffffffffu, ms, o);
  const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ms, (float)D), eps)));
  const int b = row / S / prow;
  const float4* sh = reinterpret_cast<const float4*>(shift + (size_t)b * D);
  const float4* sc = reinterpret_cast<const float4*>(scale + (size_t)b * D);
  float lo = 0.0f, hi = 0.0f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int j = i * 32 + lane;
    if (j < D4) {
      const float4 s4 = sc[j], h4 = sh[j];
      v[i].x = __fadd_rn(__fmul_rn(__fmul_rn(v[i].x, inv), __fadd_rn(1.0f, s4.x)), h4.x);
      v[i].y = __fadd_rn(__fmul_rn(__fmul_rn(v[i].y, inv), __fadd_rn(1.0f, s4.y)), h4.y);
      v[i].z = __fadd_rn(__fmul_rn(__fmul_rn(v[i].z, inv), __fadd_rn(1.0f, s4.z)), h4.z);
      v[i].w = __fadd_rn(__fmul_rn(__fmul_rn(v[i].w, inv), __fadd_rn(1.0f, s4.w)), h4.w);
      lo = run_lo(v[i].x, lo); hi = run_hi(v[i].x, hi);
      lo = run_lo(v[i].y, lo); hi = run_hi(v[i].y, hi);
      lo = run_lo(v[i].z, lo); hi = run_hi(v[i].z, hi);
      lo = run_lo(v[i].w, lo); hi = run_hi(v[i].w, hi);
    }
  }
  warp_minmax(lo, hi);
  float s, qinv;
  int zp;
  row_params(lo, hi, s, qinv, zp);
  const float zpf = (float)zp;
  uint32_t* dst = reinterpret_cast<uint32_t*>(q + (size_t)row * D);
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int j = i * 32 + lane;
    if (j < D4)
      dst[j] = quant_code4(v[i], qinv, zpf);
  }
  if (lane == 0) {
    qs[row] = s;
    qz[row] = zp;
  }
}

int adaln_quant_launch(const float* x, int rows, int S, int D, float eps, int prow,
                       const float* shift, const float* scale, uint8_t* q, float* qs, int32_t* qz,
                       cudaStream_t s) {
  const int V = cdiv(D / 4, 32);
  const dim3 grid(cdiv(rows, 8)), block(256);
  cudaError_t e;
#define IRO_AQ(N)                                                                              \
  case N:                                                                                      \
    e = launch_pdl(adaln_quant_kernel<N>, grid, block, 0, s, x, rows, S, D, eps, prow, shift, \
                   scale, q, qs, qz);                                                          \
    break;
  switch (V) {
    IRO_AQ(4)
    IRO_AQ(8)
    IRO_AQ(10)
    IRO_AQ(12)
    IRO_AQ(16)
    default:
      return IRO_ERR_UNSUPPORTED;
  }
#undef IRO_AQ
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
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

// qk_norm_rope_kernel's work for a tile of 32 tokens of one batch row and one
// head, written as the tensor-core attention's fp16 operands (q16, k16
// [B*S, D], range-checked), plus that tile of V transposed into the per-head
// V^T rows (vt[((b * heads + h) * 64 + d) * ld + s], zero for s in [S, ld)).
// 8 warps x 4 tokens for q and k; V through a shared-memory transpose.
__global__ void __launch_bounds__(256) qk_norm_rope_half_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    __half* __restrict__ q16, __half* __restrict__ k16, __half* __restrict__ vt, int S, int D,
    int heads, int ld, float eps, const float* __restrict__ qw, const float* __restrict__ kw,
    const float* __restrict__ rcos, const float* __restrict__ rsin, DevError* err) {
  __shared__ float tile[kHD][33];
  const int s0 = blockIdx.x * 32, hd = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
  const int d = 2 * lane;
  // V loads first (8 per thread), so their latency overlaps the q/k work.
  float vv[8];
#pragma unroll
  for (int r = 0; r < 8; r++) {
    const int i = t + r * 256;
    const int ss = i / kHD, dd = i % kHD;
    const int s = s0 + ss;
    vv[r] = s < S ? v[((size_t)b * S + s) * D + (size_t)hd * kHD + dd] : 0.0f;
  }
  // q and k of this warp's four tokens, loaded together.
  float2 qv[4], kv[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int s = min(s0 + warp * 4 + i, S - 1);
    const size_t off = ((size_t)b * S + s) * D + hd * kHD + d;
    qv[i] = *reinterpret_cast<const float2*>(q + off);
    kv[i] = *reinterpret_cast<const float2*>(k + off);
  }
  const float* qwh = qw + hd * kHD;
  const float* kwh = kw + hd * kHD;
  const float qw0 = qwh[d], qw1 = qwh[d + 1], kw0 = kwh[d], kw1 = kwh[d + 1];
  float qms[4], kms[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    qms[i] = __fmaf_rn(qv[i].y, qv[i].y, __fmul_rn(qv[i].x, qv[i].x));
    kms[i] = __fmaf_rn(kv[i].y, kv[i].y, __fmul_rn(kv[i].x, kv[i].x));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      qms[i] += __shfl_xor_sync(0xffffffffu, qms[i], o);
      kms[i] += __shfl_xor_sync(0xffffffffu, kms[i], o);
    }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int s = s0 + warp * 4 + i;
    if (s >= S) break;  // warp-uniform
    const float qinv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(qms[i], (float)kHD), eps)));
    const float kinv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(kms[i], (float)kHD), eps)));
    const float q0 = __fmul_rn(qv[i].x, __fmul_rn(qinv, qw0));
    const float q1 = __fmul_rn(qv[i].y, __fmul_rn(qinv, qw1));
    const float k0 = __fmul_rn(kv[i].x, __fmul_rn(kinv, kw0));
    const float k1 = __fmul_rn(kv[i].y, __fmul_rn(kinv, kw1));
    const size_t off = ((size_t)b * S + s) * D + hd * kHD + d;
    float2 qo = make_float2(q0, q1), ko = make_float2(k0, k1);
    if (hd < heads / 2) {
      const float c = rcos[(size_t)s * (kHD / 2) + lane], sn = rsin[(size_t)s * (kHD / 2) + lane];
      qo = make_float2(__fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, sn)),
                       __fadd_rn(__fmul_rn(q0, sn), __fmul_rn(q1, c)));
      ko = make_float2(__fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, sn)),
                       __fadd_rn(__fmul_rn(k0, sn), __fmul_rn(k1, c)));
    }
    *reinterpret_cast<__half2*>(q16 + off) =
        __halves2half2(to_half_checked(qo.x, err, 105), to_half_checked(qo.y, err, 105));
    *reinterpret_cast<__half2*>(k16 + off) =
        __halves2half2(to_half_checked(ko.x, err, 106), to_half_checked(ko.y, err, 106));
  }
#pragma unroll
  for (int r = 0; r < 8; r++) {
    const int i = t + r * 256;
    tile[i % kHD][i / kHD] = vv[r];
  }
  __syncthreads();
  for (int i = t; i < 32 * kHD; i += 256) {
    const int dd = i / 32, ss = i % 32;
    const int s = s0 + ss;
    if (s < ld)
      vt[(((size_t)b * heads + hd) * kHD + dd) * ld + s] = to_half_checked(tile[dd][ss], err, 107);
  }
}

// RoPE tables [S][32] -> groups of four pairs [8][S][4] (cos block, then the
// sin block at 32 * S), the layout the QKVG epilogue reads (EPI_QKV).
__global__ void rope_group4_kernel(const float* __restrict__ rcos, const float* __restrict__ rsin,
                                   int S, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= S * 32) return;
  const int tok = i >> 5, pair = i & 31;
  const size_t o = ((size_t)(pair >> 2) * S + tok) * 4 + (pair & 3);
  out[o] = rcos[i];
  out[(size_t)32 * S + o] = rsin[i];
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

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

// IRO_DIT_ATTENTION=simt selects the fp32 CUDA-core attention kernel above
// (exact fp32 products) instead of the tensor-core one (fp16 operands); the
// CUDA-core kernel also serves requests the tensor-core one does not take
// (unaligned context buffers).
int attention_mode() {
  const char* e = getenv("IRO_DIT_ATTENTION");
  if (e && strcmp(e, "simt") == 0) return 1;
  return 0;
}

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

}  // extern "C"

namespace iro {

size_t dit_adaln_scratch_bytes(int sets, int rows, int D, int R) {
  return al256(sizeof(float) * (size_t)rows * 3 * D) +
         al256(sizeof(float) * (size_t)sets * rows * 3 * R);
}

int dit_adaln_params(const IroDiTBlockDev* const* blks, int n_blocks, const float* cond,
                     int rows, float* params, void* scratch, cudaStream_t s) {
  if (n_blocks <= 0 || 2 * n_blocks > kAdaMaxSets) return IRO_ERR_INVALID;
  const int D = blks[0]->model_dim, R = blks[0]->adaln_rank, sets = 2 * n_blocks;
  float* act = static_cast<float*>(scratch);
  float* low = act + al256(sizeof(float) * (size_t)rows * 3 * D) / sizeof(float);
  AdaBatch bt;
  for (int i = 0; i < sets; i++) {
    for (int k = 0; k < 9; k++) bt.m[i][k] = blks[i / 2]->adaln[i % 2][k];
    bt.out[i] = params + (size_t)i * 3 * rows * D;
  }
  const int n = rows * 3 * D;
  adaln_act_kernel<<<cdiv(n, 256), 256, 0, s>>>(cond, n, act);
  int st = check_launch();
  if (st) return st;
  adaln_down_kernel<<<dim3(cdiv(3 * R, 8), sets, rows), 256, 0, s>>>(bt, act, D, R, low);
  if ((st = check_launch())) return st;
  adaln_up_kernel<<<dim3(cdiv(3 * D, 8), sets, rows), 256, 0, s>>>(bt, cond, low, D, R);
  return check_launch();
}

namespace {

// Mode of one projection group under the block's diagnostic switches
// (dit.c:780-797, 876-883, 940-969): left out of the int8 mask -> fp32,
// else int8, or emulated when emulate is set (1 = weight-only, any other
// value = activation-only error, as int8_linear_emulated decides).
int group_mode(const IroDiTBlockDev* blk, int group) {
  if (blk->fp32_groups & group) return DIAG_FP32;
  if (blk->emulate == 0) return DIAG_INT8;
  return blk->emulate == 1 ? DIAG_EMULATE_WEIGHT : DIAG_EMULATE_ACTIVATION;
}

bool diag_active(const IroDiTBlockDev* blk) { return blk->fp32_groups != 0 || blk->emulate != 0; }

// The SwiGLU scratch is only live in the MLP half, the V^T copies only in
// the attention half: they share the tail of the workspace.
size_t block_tail_bytes(const IroDiTBlockDev* blk, int B, int S, int C, int context_batch) {
  const int M = B * S;
  return std::max(swiglu_workspace_bytes_ex(M, blk->model_dim, blk->mlp_dim,
                                            (blk->residual_mask & 8) != 0,
                                            (blk->residual_mask & 4) != 0),
                  attention_tc_workspace_bytes(B, S, C, context_batch, blk->model_dim));
}

// The diagnostic paths' region after the tail: the projections' scratch,
// then the hidden [M, H], the W3 output [M, H] and W2's codes (two terms)
// with their row parameters.
size_t diag_scratch_bytes(const IroDiTBlockDev* blk, int M) {
  const int D = blk->model_dim, H = blk->mlp_dim;
  return std::max(diag_linear_scratch_bytes(M, D, D),
                  std::max(diag_linear_scratch_bytes(M, D, H), diag_linear_scratch_bytes(M, H, D)));
}

size_t diag_region_bytes(const IroDiTBlockDev* blk, int M) {
  const size_t H = (size_t)blk->mlp_dim;
  return al256(diag_scratch_bytes(blk, M)) + 2 * al256(sizeof(float) * M * H) +
         2 * (al256((size_t)M * H) + 2 * al256(sizeof(float) * M));
}

}  // namespace

size_t dit_block_body_bytes(const IroDiTBlockDev* blk, int B, int S, int C, int context_batch) {
  const size_t M = (size_t)B * S, D = (size_t)blk->model_dim;
  size_t t = 0;
  t += 6 * al256(sizeof(float) * M * D);                           // h, q, k, v, g, mix
  t += 2 * (al256(M * D) + 2 * al256(sizeof(float) * M));          // codes (two terms) + row params
  t += al256(sizeof(int) * (size_t)B * C) + al256(sizeof(int) * B);
  t += al256(sizeof(float) * 2 * 32 * (size_t)S);                   // grouped RoPE tables
  const size_t tail = block_tail_bytes(blk, B, S, C, context_batch);
  if (!diag_active(blk)) return t + tail;
  return t + al256(tail) + diag_region_bytes(blk, (int)M);
}

int dit_block_check(const IroDiTBlockDev* blk, const float* x, int cond_rows, const float* ctx_k,
                    const float* ctx_v, const uint8_t* ctx_mask, int context_batch, int B, int S,
                    int C, const float* rope_cos, const float* rope_sin) {
  if (!blk || !x || !ctx_k || !ctx_v || !ctx_mask || !rope_cos || !rope_sin || B <= 0 ||
      S <= 0 || C <= 0 || context_batch <= 0 || B % context_batch != 0 ||
      (cond_rows != 1 && cond_rows != B))
    return IRO_ERR_INVALID;
  const int D = blk->model_dim, NH = blk->heads, R = blk->adaln_rank, H = blk->mlp_dim;
  if (blk->head_dim != kHD || NH * kHD != D || R <= 0 || H <= 0 || D % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return IRO_ERR_UNSUPPORTED;
  // Two-term activation policy: any combination of the four groups
  // (dit.c:429-436); the reference's default is W2 only (8).
  if ((blk->residual_mask & ~15) != 0 || (blk->fp32_groups & ~15) != 0) return IRO_ERR_INVALID;
  const int m_qkvg = group_mode(blk, 1), m_wo = group_mode(blk, 2);
  const int m_w13 = group_mode(blk, 4), m_w2 = group_mode(blk, 8);
  // The int8 weights where a group reads them (int8 and weight emulation),
  // the fp32 weights where it reads those (fp32 and activation emulation).
  auto int8_used = [](int m) { return m == DIAG_INT8 || m == DIAG_EMULATE_WEIGHT; };
  auto fp32_used = [](int m) { return m == DIAG_FP32 || m == DIAG_EMULATE_ACTIVATION; };
  if (int8_used(m_qkvg) &&
      (blk->qkvg.N != 4 * D || blk->qkvg.K != D || blk->qkvg.layout != IRO_LAYOUT_PLAIN))
    return IRO_ERR_INVALID;
  if (int8_used(m_wo) && (blk->wo.N != D || blk->wo.K != D)) return IRO_ERR_INVALID;
  if (int8_used(m_w13) &&
      (blk->w13.layout != IRO_LAYOUT_GATED_PAIR || blk->w13.K != D || blk->w13.hidden != H))
    return IRO_ERR_INVALID;
  if (int8_used(m_w2) && (blk->w2.N != D || blk->w2.K != H)) return IRO_ERR_INVALID;
  const int groups[8] = {m_qkvg, m_qkvg, m_qkvg, m_qkvg, m_wo, m_w13, m_w13, m_w2};
  for (int i = 0; i < 8; i++)
    if (fp32_used(groups[i]) && !blk->w_fp32[i]) return IRO_ERR_INVALID;
  // The two-term W1/W3 path runs inside the int8 SwiGLU only.
  if ((blk->residual_mask & 4) && m_w13 == DIAG_INT8 && m_w2 != DIAG_INT8)
    return IRO_ERR_UNSUPPORTED;
  return IRO_OK;
}

// The block with its AdaLN parameters precomputed: ada = shift, scale, gate
// of the attention half, then of the MLP half, each [cond_rows][D].
int dit_block_run(Ctx* c, const IroDiTBlockDev* blk, float* x, const float* const* ada,
                  int cond_rows, const float* ctx_k, const float* ctx_v,
                  const uint8_t* ctx_mask, int context_batch, int B, int S, int C,
                  const float* rcos, const float* rsin, void* workspace, cudaStream_t s,
                  int stats_layer, const float* rope_t) {
  const int D = blk->model_dim, NH = blk->heads;
  const size_t M = (size_t)B * S;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
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
  uint8_t* codes = take(M * D);
  float* rs = reinterpret_cast<float*>(take(sizeof(float) * M));
  int32_t* rz = reinterpret_cast<int32_t*>(take(sizeof(float) * M));
  // Second activation term of the two-term QKVG / Wo policies.
  uint8_t* codes2 = take(M * D);
  float* rs2 = reinterpret_cast<float*>(take(sizeof(float) * M));
  int32_t* rz2 = reinterpret_cast<int32_t*>(take(sizeof(float) * M));
  int* clist = reinterpret_cast<int*>(take(sizeof(int) * (size_t)B * C));
  int* ccount = reinterpret_cast<int*>(take(sizeof(int) * B));
  float* rope_ws = reinterpret_cast<float*>(take(sizeof(float) * 2 * 32 * (size_t)S));
  void* sw_ws = ws + off;
  int st;
  // Two-term activation policy per projection group (dit.c:429-436,
  // IRO_INT8_RESIDUAL bits: 1 QKVG, 2 Wo, 4 W1/W3, 8 W2).
  const bool res_qkvg = (blk->residual_mask & 1) != 0, res_wo = (blk->residual_mask & 2) != 0;
  const bool res_w13 = (blk->residual_mask & 4) != 0, res_w2 = (blk->residual_mask & 8) != 0;
  const int diag_layer = (stats_layer >= 0 && diag_enabled()) ? stats_layer : -1;
  // The diagnostic modes per group (fp32_groups / emulate) and their region
  // after the tail.
  const int m_qkvg = group_mode(blk, 1), m_wo = group_mode(blk, 2);
  const int m_w13 = group_mode(blk, 4), m_w2 = group_mode(blk, 8);
  const int H = blk->mlp_dim;
  uint8_t* dreg = static_cast<uint8_t*>(sw_ws) + al256(block_tail_bytes(blk, B, S, C, context_batch));
  void* dscratch = dreg;
  float* dhid = reinterpret_cast<float*>(dreg + al256(diag_scratch_bytes(blk, (int)M)));
  float* da3 = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(dhid) +
                                        al256(sizeof(float) * M * H));
  uint8_t* dq = reinterpret_cast<uint8_t*>(da3) + al256(sizeof(float) * M * H);
  float* dqs = reinterpret_cast<float*>(dq + al256(M * H));
  int32_t* dqz = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(dqs) + al256(sizeof(float) * M));
  uint8_t* dq2 = reinterpret_cast<uint8_t*>(dqz) + al256(sizeof(float) * M);
  float* dqs2 = reinterpret_cast<float*>(dq2 + al256(M * H));
  int32_t* dqz2 =
      reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(dqs2) + al256(sizeof(float) * M));

  const int prow = B / cond_rows;  // batch rows per AdaLN parameter row
  for (int half = 0; half < 2; half++) {
    const float* shift = ada[half * 3 + 0];
    const float* scale = ada[half * 3 + 1];
    const float* gate = ada[half * 3 + 2];
    // AdaLN apply and the row quantiser of its consumer (QKVG, or W1/W3 of
    // the SwiGLU) in one pass; h is materialised for the two-term policies
    // and for shapes the fused kernel does not take.
    const bool two_term = half == 0 ? res_qkvg : res_w13;
    const bool int8_in = (half == 0 ? m_qkvg : m_w13) == DIAG_INT8;
    st = (two_term || diag_layer >= 0 || !int8_in)
             ? (int)IRO_ERR_UNSUPPORTED
             : adaln_quant_launch(x, (int)M, S, D, blk->norm_eps, prow, shift, scale, codes, rs,
                                  rz, s);
    const bool fused = st == IRO_OK;
    if (st == IRO_ERR_UNSUPPORTED) {
      adaln_apply_kernel<<<cdiv((int)M, 8), 256, 0, s>>>(x, (int)M, S, D, blk->norm_eps, prow,
                                                         shift, scale, h);
      if ((st = check_launch())) return st;
      // Q/K/V/gate or W1/W3 input diagnostics (dit.c:787, 944), recorded on
      // the int8 path as the reference does.
      if (int8_in && diag_layer >= 0 &&
          (st = diag_record(diag_layer, half == 0 ? 0 : 2, h, (int)M, D, s)))
        return st;
      if (!int8_in)
        st = IRO_OK;
      else if (half == 0 && res_qkvg)
        st = quantize_rows_residual_launch(h, (int)M, D, codes, rs, rz, nullptr, codes2, rs2,
                                           rz2, s);
      else if (!(half == 1 && res_w13))
        st = quantize_rows_launch(h, (int)M, D, codes, rs, rz, 0, s);
      if (st) return st;
    } else if (st) {
      return st;
    }
    if (half == 0) {
      // QKVG on one quantised copy of h (dit.c:785-792).  With the
      // tensor-core attention and the single-term policy, the head norm,
      // RoPE and the V transpose run in the GEMM's epilogue (EPI_QKV).
      AttnTcRequest ar{g, ctx_k, ctx_v, ctx_mask, mix, B, S, C, context_batch, D, NH, sw_ws};
      const bool tc = attention_mode() != 1 && attention_tc_supported(ar);
      auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
      const bool fuse_heads =
          tc && !res_qkvg && m_qkvg == DIAG_INT8 && al16(blk->q_norm) && al16(blk->k_norm);
      // The tensor-core attention's fp16 operands (q, k, V^T) in the tail.
      const AttnTcOperands ao = attention_tc_operands(ar);
      if (m_qkvg != DIAG_INT8) {
        // The fp32 / emulated projections, one per output (dit.c:780-784,
        // 793-797).
        float* outs[4] = {q, k, v, g};
        for (int i = 0; i < 4; i++)
          if ((st = diag_linear(c, m_qkvg, h, (int)M, D, &blk->qkvg, i * D, 0, blk->w_fp32[i],
                                outs[i], D, dscratch, s)))
            return st;
      } else {
      GemmRequest r;
      r.epi = res_qkvg ? EPI_DUAL : fuse_heads ? EPI_QKV : EPI_SPLIT;
      r.M = (int)M;
      r.a = codes;
      r.lda = D;
      r.sx = rs;
      r.zp = rz;
      if (res_qkvg) {
        r.a2 = codes2;
        r.sx2 = rs2;
        r.zp2 = rz2;
      }
      r.w = &blk->qkvg;
      r.bias = nullptr;
      r.nout = 4;
      r.seg = D;
      r.outs[0] = q;
      r.outs[1] = k;
      r.outs[2] = v;
      r.outs[3] = g;
      if (fuse_heads) {
        if (!rope_t) {
          rope_group4_kernel<<<cdiv(S * 32, 256), 256, 0, s>>>(rcos, rsin, S, rope_ws);
          if ((st = check_launch())) return st;
          rope_t = rope_ws;
        }
        r.outs[0] = r.outs[1] = r.outs[2] = nullptr;
        r.hn_q = blk->q_norm;
        r.hn_k = blk->k_norm;
        r.rcos = rope_t;
        r.rsin = rope_t + 32 * (size_t)S;
        r.hq = ao.q;
        r.hk = ao.k;
        r.hvt = ao.vt;
        r.vt_ld = ao.ldv;
        r.tokens = S;
        r.eps = blk->norm_eps;
      }
      if ((st = gemm_launch(c, r, s))) return st;
      }
      if (tc) {
        if (!fuse_heads) {
          // Head norm + RoPE into the fp16 q, k, with the self V^T rows.
          qk_norm_rope_half_kernel<<<dim3(cdiv(S, 32), NH, B), 256, 0, s>>>(
              q, k, v, ao.q, ao.k, ao.vt, S, D, NH, ao.ldv, blk->norm_eps, blk->q_norm,
              blk->k_norm, rcos, rsin, c->err);
          if ((st = check_launch())) return st;
        }
        if ((st = attention_tc_launch(c, ar, s))) return st;
      } else {
        qk_norm_rope_kernel<<<cdiv((int)M * NH, 8), 256, 0, s>>>(
            q, k, (int)M, S, D, NH, blk->norm_eps, blk->q_norm, blk->k_norm, rcos, rsin);
        if ((st = check_launch())) return st;
        context_list_kernel<<<cdiv(B, 64), 64, 0, s>>>(ctx_mask, B, C, clist, ccount);
        if ((st = check_launch())) return st;
        AttnArgs aa{q, k, v, g, ctx_k, ctx_v, clist, ccount, B / context_batch, S, C, D, mix};
        attention_kernel<<<dim3(cdiv(S, kAQ), NH, B), kAThreads, 0, s>>>(aa);
        if ((st = check_launch())) return st;
      }
      if (m_wo != DIAG_INT8) {
        // The fp32 / emulated Wo (dit.c:876-877, 882-883), then the gated
        // residual x += gate * out (dit.c:1013-1020) on its own.
        if ((st = diag_linear(c, m_wo, mix, (int)M, D, &blk->wo, 0, 0, blk->w_fp32[4], q, D,
                              dscratch, s)))
          return st;
        if ((st = gated_residual_launch(c, x, q, gate, S * prow, (int)M, D, s))) return st;
        continue;
      }
      // Wo on the quantised gated mix (dit.c:876-884), with the gated
      // residual x += gate * Wo(mix) (dit.c:1013-1020) in its epilogue.
      if (diag_layer >= 0 && (st = diag_record(diag_layer, 1, mix, (int)M, D, s))) return st;
      st = res_wo ? quantize_rows_residual_launch(mix, (int)M, D, codes, rs, rz, nullptr, codes2,
                                                  rs2, rz2, s)
                  : quantize_rows_launch(mix, (int)M, D, codes, rs, rz, 0, s);
      if (st) return st;
      GemmRequest o;
      o.epi = res_wo ? EPI_DUAL : EPI_LINEAR;
      o.M = (int)M;
      o.a = codes;
      o.lda = D;
      o.sx = rs;
      o.zp = rz;
      if (res_wo) {
        o.a2 = codes2;
        o.sx2 = rs2;
        o.zp2 = rz2;
      }
      o.w = &blk->wo;
      o.y = x;
      o.ldy = D;
      o.rgate = gate;
      o.rgate_rows = S * prow;
      if ((st = gemm_launch(c, o, s))) return st;
    } else if (m_w13 != DIAG_INT8 || m_w2 != DIAG_INT8) {
      // SwiGLU with a diagnostic group (dit.c:940-969): W1/W3 into the plain
      // hidden [M, H], silu(w1) * w3, then W2 and the gated residual.
      if (m_w13 == DIAG_INT8) {
        // Single-term int8 W1/W3 with the gate in its epilogue (the two-term
        // one is rejected by the block check).
        GemmRequest gr;
        gr.epi = EPI_GATED;
        gr.M = (int)M;
        gr.a = codes;
        gr.lda = D;
        gr.sx = rs;
        gr.zp = rz;
        gr.w = &blk->w13;
        gr.hidden = dhid;
        gr.ldh = H;
        if ((st = gemm_launch(c, gr, s))) return st;
      } else {
        if ((st = diag_linear(c, m_w13, h, (int)M, D, &blk->w13, 0, 0, blk->w_fp32[5], dhid, H,
                              dscratch, s)) ||
            (st = diag_linear(c, m_w13, h, (int)M, D, &blk->w13, 0, 1, blk->w_fp32[6], da3, H,
                              dscratch, s)) ||
            (st = silu_mul_plain_launch(c, dhid, da3, (long long)M * H, dhid, s)))
          return st;
      }
      if (m_w2 == DIAG_INT8) {
        // W2 input diagnostics (dit.c:964), then the int8 W2 with the gated
        // residual in its epilogue.
        if (diag_layer >= 0 && (st = diag_record(diag_layer, 3, dhid, (int)M, H, s))) return st;
        st = res_w2 ? quantize_rows_residual_launch(dhid, (int)M, H, dq, dqs, dqz, nullptr, dq2,
                                                    dqs2, dqz2, s)
                    : quantize_rows_launch(dhid, (int)M, H, dq, dqs, dqz, 0, s);
        if (st) return st;
        GemmRequest o;
        o.epi = res_w2 ? EPI_DUAL : EPI_LINEAR;
        o.M = (int)M;
        o.a = dq;
        o.lda = H;
        o.sx = dqs;
        o.zp = dqz;
        if (res_w2) {
          o.a2 = dq2;
          o.sx2 = dqs2;
          o.zp2 = dqz2;
        }
        o.w = &blk->w2;
        o.bias = blk->w2.bias;
        o.y = x;
        o.ldy = D;
        o.rgate = gate;
        o.rgate_rows = S * prow;
        if ((st = gemm_launch(c, o, s))) return st;
      } else {
        if ((st = diag_linear(c, m_w2, dhid, (int)M, H, &blk->w2, 0, 0, blk->w_fp32[7], q, D,
                              dscratch, s)) ||
            (st = gated_residual_launch(c, x, q, gate, S * prow, (int)M, D, s)))
          return st;
      }
    } else {
      // SwiGLU (dit.c:913-969), x += gate * W2(...) in the W2 epilogue.
      if (res_w13)
        st = swiglu_run(c, h, (int)M, &blk->w13, &blk->w2, nullptr, x, res_w2, sw_ws, s, gate,
                        S * prow, nullptr, nullptr, nullptr, 1, diag_layer);
      else
        st = swiglu_run(c, fused ? nullptr : h, (int)M, &blk->w13, &blk->w2, nullptr, x, res_w2,
                        sw_ws, s, gate, S * prow, codes, rs, rz, 0, diag_layer);
      if (st) return st;
    }
  }
  return IRO_OK;
}

}  // namespace iro

extern "C" {

size_t iro_dit_block_workspace_bytes(const IroDiTBlockDev* blk, int B, int S, int C,
                                     int context_batch) {
  if (!blk || B <= 0 || S <= 0 || C <= 0) return 0;
  const size_t D = (size_t)blk->model_dim;
  return dit_block_body_bytes(blk, B, S, C, context_batch) +
         al256(sizeof(float) * 6 * (size_t)B * D) +
         dit_adaln_scratch_bytes(2, B, blk->model_dim, blk->adaln_rank);
}

int iro_dit_block_dev(const IroDiTBlockDev* blk, float* x, const float* cond, int cond_rows,
                      const float* ctx_k, const float* ctx_v, const uint8_t* ctx_mask,
                      int context_batch, int B, int S, int C, const float* rope_cos,
                      const float* rope_sin, void* workspace, void* stream) {
  int st = dit_block_check(blk, x, cond_rows, ctx_k, ctx_v, ctx_mask, context_batch, B, S, C,
                           rope_cos, rope_sin);
  if (st) return st;
  if (!cond) return IRO_ERR_INVALID;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!ws) {
    ws = static_cast<uint8_t*>(
        arena_get(c, iro_dit_block_workspace_bytes(blk, B, S, C, context_batch), &st));
    if (!ws) return st;
  }
  const size_t body = dit_block_body_bytes(blk, B, S, C, context_batch);
  float* params = reinterpret_cast<float*>(ws + body);
  void* scratch = ws + body + al256(sizeof(float) * 6 * (size_t)B * blk->model_dim);
  if ((st = dit_adaln_params(&blk, 1, cond, cond_rows, params, scratch, s))) return st;
  const float* ada[6];
  for (int i = 0; i < 6; i++) ada[i] = params + (size_t)i * cond_rows * blk->model_dim;
  return dit_block_run(c, blk, x, ada, cond_rows, ctx_k, ctx_v, ctx_mask, context_batch, B,
                       S, C, rope_cos, rope_sin, ws, s);
}

}  // extern "C"
