// quantize.cu — per-row activation quantisers and the weight quantiser.
//
// Activation rows (ops.c:321-348, ops.c:427-442, tests/bench_vnni_linear.c:
// 82-101) are memory-bound: one 128-thread block per row, the row held in
// registers as float4 (coalesced loads), a block min/max, then codes packed
// four per 32-bit store.  Rows that do not fit the register path (K > 4096,
// K % 4 != 0 or unaligned pointers) take a generic warp-per-row path that
// re-reads the row.
#include "quantize.cuh"

namespace iro {

enum QuantMode { QM_ASYM = 0, QM_SYM = 1, QM_RESID = 2 };

struct QuantArgs {
  const float* x;
  int M, K;
  uint8_t* q;
  float* scale;
  int32_t* zero;
  float* residual;  // QM_RESID, optional
  uint8_t* q2;
  float* scale2;
  int32_t* zero2;
};

// Symmetric code: clamp((int)lrintf(x/s), -127, 127) + 128, with lrintf's
// x86-64 result for NaN (the low 32 bits of LONG_MIN, i.e. 0).
__device__ __forceinline__ uint32_t sym_code(float x, float s) {
  float r = rintf(__fdiv_rn(x, s));
  int v = (r >= -2147483648.0f && r < 2147483648.0f) ? __float2int_rz(r) : 0;
  v = v > 127 ? 127 : v;
  v = v < -127 ? -127 : v;
  return (uint32_t)(v + 128);
}

// One 128-thread block per row: thread t holds float4 elements t, t+128, ...
// (at most V of them) in registers.  The row range is reduced across the
// block (warp shuffles, then four partials in shared memory).
constexpr int kQThreads = 128;

__device__ __forceinline__ void block_minmax(float& lo, float& hi, float* sm) {
  warp_minmax(lo, hi);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // sm may still be read from a previous reduction
  if (lane == 0) {
    sm[2 * w] = lo;
    sm[2 * w + 1] = hi;
  }
  __syncthreads();
  lo = fminf(fminf(sm[0], sm[2]), fminf(sm[4], sm[6]));
  hi = fmaxf(fmaxf(sm[1], sm[3]), fmaxf(sm[5], sm[7]));
}

__device__ __forceinline__ float block_max(float a, float* sm) {
  a = warp_max(a);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sm[w] = a;
  __syncthreads();
  return fmaxf(fmaxf(sm[0], sm[1]), fmaxf(sm[2], sm[3]));
}

template <int V, int MODE>
__global__ void __launch_bounds__(kQThreads) quant_rows_vec(QuantArgs a) {
  __shared__ float sm[8];
  grid_dep_wait();
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int K4 = a.K >> 2;
  const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)row * a.K);
  float4 v[V];
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int j = i * kQThreads + tid;
    v[i] = j < K4 ? __ldg(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (MODE == QM_SYM) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < V; i++) {
      if (i * kQThreads + tid < K4) {
        float t;
        t = fabsf(v[i].x); amax = t > amax ? t : amax;
        t = fabsf(v[i].y); amax = t > amax ? t : amax;
        t = fabsf(v[i].z); amax = t > amax ? t : amax;
        t = fabsf(v[i].w); amax = t > amax ? t : amax;
      }
    }
    amax = block_max(amax, sm);
    const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    uint32_t* dst = reinterpret_cast<uint32_t*>(a.q + (size_t)row * a.K);
#pragma unroll
    for (int i = 0; i < V; i++) {
      const int j = i * kQThreads + tid;
      if (j < K4)
        dst[j] = sym_code(v[i].x, s) | (sym_code(v[i].y, s) << 8) |
                 (sym_code(v[i].z, s) << 16) | (sym_code(v[i].w, s) << 24);
    }
    if (tid == 0) {
      a.scale[row] = s;
      a.zero[row] = 128;
    }
    return;
  }
  float lo = 0.0f, hi = 0.0f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    if (i * kQThreads + tid < K4) {
      lo = run_lo(v[i].x, lo); hi = run_hi(v[i].x, hi);
      lo = run_lo(v[i].y, lo); hi = run_hi(v[i].y, hi);
      lo = run_lo(v[i].z, lo); hi = run_hi(v[i].z, hi);
      lo = run_lo(v[i].w, lo); hi = run_hi(v[i].w, hi);
    }
  }
  block_minmax(lo, hi, sm);
  float s, inv;
  int zp;
  row_params(lo, hi, s, inv, zp);
  const float zpf = (float)zp;
  uint32_t* dst = reinterpret_cast<uint32_t*>(a.q + (size_t)row * a.K);
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int j = i * kQThreads + tid;
    if (j < K4) {
      float4 q;
      dst[j] = quant_code4(v[i], inv, zpf, q);
      if (MODE == QM_RESID) {
        // ops.c:436-439: r = x - s*((float)q - zp), in place of x.
        v[i].x = __fsub_rn(v[i].x, __fmul_rn(s, __fsub_rn(q.x, zpf)));
        v[i].y = __fsub_rn(v[i].y, __fmul_rn(s, __fsub_rn(q.y, zpf)));
        v[i].z = __fsub_rn(v[i].z, __fmul_rn(s, __fsub_rn(q.z, zpf)));
        v[i].w = __fsub_rn(v[i].w, __fmul_rn(s, __fsub_rn(q.w, zpf)));
      }
    }
  }
  if (tid == 0) {
    a.scale[row] = s;
    a.zero[row] = zp;
  }
  if (MODE != QM_RESID) return;
  float4* rdst = a.residual ? reinterpret_cast<float4*>(a.residual + (size_t)row * a.K) : nullptr;
  float lo2 = 0.0f, hi2 = 0.0f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int j = i * kQThreads + tid;
    if (j < K4) {
      if (rdst) rdst[j] = v[i];
      lo2 = run_lo(v[i].x, lo2); hi2 = run_hi(v[i].x, hi2);
      lo2 = run_lo(v[i].y, lo2); hi2 = run_hi(v[i].y, hi2);
      lo2 = run_lo(v[i].z, lo2); hi2 = run_hi(v[i].z, hi2);
      lo2 = run_lo(v[i].w, lo2); hi2 = run_hi(v[i].w, hi2);
    }
  }
  block_minmax(lo2, hi2, sm);
  float s2, inv2;
  int zp2;
  row_params(lo2, hi2, s2, inv2, zp2);
  const float zpf2 = (float)zp2;
  uint32_t* dst2 = reinterpret_cast<uint32_t*>(a.q2 + (size_t)row * a.K);
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int j = i * kQThreads + tid;
    if (j < K4) dst2[j] = quant_code4(v[i], inv2, zpf2);
  }
  if (tid == 0) {
    a.scale2[row] = s2;
    a.zero2[row] = zp2;
  }
}

// Any K / alignment: one warp per row, scalar loads, the row read per pass.
template <int MODE>
__global__ void __launch_bounds__(256) quant_rows_generic(QuantArgs a) {
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= a.M) return;
  const float* src = a.x + (size_t)row * a.K;
  uint8_t* dst = a.q + (size_t)row * a.K;
  if (MODE == QM_SYM) {
    float amax = 0.0f;
    for (int k = lane; k < a.K; k += 32) {
      float t = fabsf(src[k]);
      amax = t > amax ? t : amax;
    }
    amax = warp_max(amax);
    const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    for (int k = lane; k < a.K; k += 32) dst[k] = (uint8_t)sym_code(src[k], s);
    if (lane == 0) {
      a.scale[row] = s;
      a.zero[row] = 128;
    }
    return;
  }
  float lo = 0.0f, hi = 0.0f;
  for (int k = lane; k < a.K; k += 32) {
    lo = run_lo(src[k], lo);
    hi = run_hi(src[k], hi);
  }
  warp_minmax(lo, hi);
  float s, inv;
  int zp;
  row_params(lo, hi, s, inv, zp);
  const float zpf = (float)zp;
  float lo2 = 0.0f, hi2 = 0.0f;
  for (int k = lane; k < a.K; k += 32) {
    const uint32_t c = quant_code(src[k], inv, zpf);
    dst[k] = (uint8_t)c;
    if (MODE == QM_RESID) {
      const float r = __fsub_rn(src[k], __fmul_rn(s, __fsub_rn((float)c, zpf)));
      if (a.residual) a.residual[(size_t)row * a.K + k] = r;
      lo2 = run_lo(r, lo2);
      hi2 = run_hi(r, hi2);
    }
  }
  if (lane == 0) {
    a.scale[row] = s;
    a.zero[row] = zp;
  }
  if (MODE != QM_RESID) return;
  warp_minmax(lo2, hi2);
  float s2, inv2;
  int zp2;
  row_params(lo2, hi2, s2, inv2, zp2);
  const float zpf2 = (float)zp2;
  uint8_t* dst2 = a.q2 + (size_t)row * a.K;
  for (int k = lane; k < a.K; k += 32) {
    const uint32_t c = quant_code(src[k], inv, zpf);
    const float r = __fsub_rn(src[k], __fmul_rn(s, __fsub_rn((float)c, zpf)));
    dst2[k] = (uint8_t)quant_code(r, inv2, zpf2);
  }
  if (lane == 0) {
    a.scale2[row] = s2;
    a.zero2[row] = zp2;
  }
}

template <int MODE>
static int launch_mode(const QuantArgs& a, cudaStream_t s) {
  const int rows_per_block = 8;
  const dim3 grid((unsigned)cdiv(a.M, rows_per_block)), block(256);
  const bool aligned = (a.K % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) &&
                       ((reinterpret_cast<uintptr_t>(a.q) & 3u) == 0) &&
                       (MODE != QM_RESID ||
                        (((reinterpret_cast<uintptr_t>(a.q2) & 3u) == 0) &&
                         ((reinterpret_cast<uintptr_t>(a.residual) & 15u) == 0)));
  const int K4 = a.K / 4;
  if (aligned && K4 <= 8 * kQThreads) {
    const dim3 rg((unsigned)a.M), rb(kQThreads);
    cudaError_t e;
    if (K4 <= 1 * kQThreads) e = launch_pdl(quant_rows_vec<1, MODE>, rg, rb, 0, s, a);
    else if (K4 <= 2 * kQThreads) e = launch_pdl(quant_rows_vec<2, MODE>, rg, rb, 0, s, a);
    else if (K4 <= 4 * kQThreads) e = launch_pdl(quant_rows_vec<4, MODE>, rg, rb, 0, s, a);
    else if (K4 <= 6 * kQThreads) e = launch_pdl(quant_rows_vec<6, MODE>, rg, rb, 0, s, a);
    else e = launch_pdl(quant_rows_vec<8, MODE>, rg, rb, 0, s, a);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
  } else {
    cudaError_t e = launch_pdl(quant_rows_generic<MODE>, grid, block, 0, s, a);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
  }
  return check_launch();
}

int quantize_rows_launch(const float* x, int M, int K, uint8_t* q, float* scale, int32_t* zero,
                         int symmetric, cudaStream_t s) {
  if (M <= 0 || K <= 0) return M == 0 ? IRO_OK : IRO_ERR_INVALID;
  QuantArgs a{x, M, K, q, scale, zero, nullptr, nullptr, nullptr, nullptr};
  return symmetric ? launch_mode<QM_SYM>(a, s) : launch_mode<QM_ASYM>(a, s);
}

int quantize_rows_residual_launch(const float* x, int M, int K, uint8_t* q1, float* s1,
                                  int32_t* z1, float* residual, uint8_t* q2, float* s2,
                                  int32_t* z2, cudaStream_t s) {
  if (M <= 0 || K <= 0) return M == 0 ? IRO_OK : IRO_ERR_INVALID;
  QuantArgs a{x, M, K, q1, s1, z1, residual, q2, s2, z2};
  return launch_mode<QM_RESID>(a, s);
}

// ---------------------------------------------------------------------------
// Weight quantiser (ops.c:259-293): one warp per output row; codes written
// with row pitch `ld` and the pad [K, ld) zeroed so TMA tiles past K add 0.

__global__ void __launch_bounds__(256) weight_quant_kernel(const float* __restrict__ w, int N,
                                                           int K, int8_t* __restrict__ data,
                                                           int ld, float* __restrict__ scale,
                                                           int32_t* __restrict__ colsum) {
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (n >= N) return;
  const float* src = w + (size_t)n * K;
  float amax = 0.0f;
  for (int k = lane; k < K; k += 32) {
    const float t = fabsf(src[k]);
    amax = t > amax ? t : amax;
  }
  amax = warp_max(amax);
  const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, s);
  int total = 0;
  int8_t* dst = data + (size_t)n * ld;
  for (int k = lane; k < ld; k += 32) {
    int v = 0;
    if (k < K) {
      v = f2i_x86(rintf(__fmul_rn(src[k], inv)));
      v = v > 127 ? 127 : v;
      v = v < -127 ? -127 : v;
    }
    dst[k] = (int8_t)v;
    total += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  if (lane == 0) {
    scale[n] = s;
    colsum[n] = total;
  }
}

int weight_quantize_launch(const float* w, int N, int K, int8_t* data, int ld, float* scale,
                           int32_t* colsum, cudaStream_t s) {
  if (N <= 0 || K <= 0 || ld < K) return IRO_ERR_INVALID;
  weight_quant_kernel<<<cdiv(N, 8), 256, 0, s>>>(w, N, K, data, ld, scale, colsum);
  return check_launch();
}

// [K,N] -> [N,K] transpose through 32x32 shared tiles.
__global__ void transpose_f32_kernel(const float* __restrict__ in, int rows, int cols,
                                     float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = in[(size_t)r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (c < cols && r < rows) out[(size_t)c * rows + r] = tile[threadIdx.x][i];
  }
}

int transpose_f32_launch(const float* in, int rows, int cols, float* out, cudaStream_t s) {
  dim3 grid(cdiv(cols, 32), cdiv(rows, 32)), block(32, 8);
  transpose_f32_kernel<<<grid, block, 0, s>>>(in, rows, cols, out);
  return check_launch();
}

// Copy u8 rows of pitch `K` into rows of pitch `ld` (>= K), zero padded, so
// an operand whose K is not a multiple of 16 bytes can be read by TMA.
__global__ void repack_rows_kernel(const uint8_t* __restrict__ in, int M, int K,
                                   uint8_t* __restrict__ out, int ld) {
  const size_t total = (size_t)M * ld;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t m = i / ld;
    const int k = (int)(i - m * ld);
    out[i] = k < K ? in[m * K + k] : (uint8_t)0;
  }
}

int repack_rows_launch(const uint8_t* in, int M, int K, uint8_t* out, int ld, cudaStream_t s) {
  const size_t total = (size_t)M * ld;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  repack_rows_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(in, M, K, out, ld);
  return check_launch();
}

}  // namespace iro
