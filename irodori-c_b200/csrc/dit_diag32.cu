// dit_diag32.cu — the reference's error-attribution switches for the DiT's
// int8 projections, IRO_INT8_MASK and IRO_INT8_EMULATE (dit.c:273-335,
// 780-797, 876-883, 940-969), on the device.
//
// Per projection group the block runs one of:
//   int8       the normal path (quantised activations x int8 weights);
//   fp32       the group left out of the int8 mask: fp32 activations x the
//              fp32 weights (the reference's iro_linear);
//   emulate 1  fp32 activations x the dequantised int8 weights
//              (scale[n] * (float)q[n,k]; weight-only error);
//   emulate 2  fake-quantised activations (the row quantiser's codes turned
//              back into scale[m] * ((float)q - (float)zp)) x the fp32
//              weights (activation-only error).
// The fp32 products run through a plain tiled fp32 GEMM that sums each
// output the way the reference's scalar linear does (iro_linear_scalar,
// ops.c:221-234: a running sum over increasing k, each product and each
// addition rounded, no fused multiply-add, then + 0 for the absent bias), so
// a projection matches the IEEE build of the reference bit for bit given the
// same inputs.  These paths are diagnostics: correct, not tuned.
#include "dit_diag32.cuh"
#include <algorithm>

#include "quantize.cuh"

namespace iro {
namespace {

constexpr int kT = 64;   // output tile (rows and columns)
constexpr int kTK = 16;  // K step

// C[M, N] = A[M, K] . B[N, K]^T, fp32, row-major; 256 threads, 4x4 outputs
// per thread.  The loop stops at K: a zero-padded step would add +0 and turn
// a -0 sum into +0.
__global__ void __launch_bounds__(256) sgemm_nt_kernel(const float* __restrict__ A,
                                                       const float* __restrict__ B,
                                                       float* __restrict__ Cm, int M, int N,
                                                       int K) {
  __shared__ float sa[kTK][kT + 4];
  __shared__ float sb[kTK][kT + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kT, n0 = blockIdx.x * kT;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kTK) {
    for (int i = threadIdx.x; i < kT * kTK; i += 256) {
      const int r = i / kTK, kk = i % kTK;
      const int m = m0 + r, n = n0 + r, k = k0 + kk;
      sa[kk][r] = (m < M && k < K) ? A[(size_t)m * K + k] : 0.0f;
      sb[kk][r] = (n < N && k < K) ? B[(size_t)n * K + k] : 0.0f;
    }
    __syncthreads();
    const int kn = min(kTK, K - k0);
#pragma unroll 4
    for (int kk = 0; kk < kn; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        a[i] = sa[kk][ty * 4 + i];
        b[i] = sb[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
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
      if (n < N) Cm[(size_t)m * N + n] = __fadd_rn(acc[i][j], 0.0f);
    }
  }
}

// out[n, k] = scale[r] * (float)data[r, k] for rows r of a device weight:
// r = row0 + n (PLAIN), or the `part` half (0 = W1, 1 = W3) of the
// GATED_PAIR layout's hidden channel n.
__global__ void dequant_weight_kernel(IroInt8DevWeight w, int row0, int part, int N,
                                      float* __restrict__ out) {
  const long long total = (long long)N * w.K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / w.K), k = (int)(i - (long long)n * w.K);
    const int r = w.layout == IRO_LAYOUT_GATED_PAIR
                      ? (n / w.pair) * 2 * w.pair + part * w.pair + n % w.pair
                      : row0 + n;
    out[i] = __fmul_rn(w.scale[r], (float)w.data[(size_t)r * w.ld + k]);
  }
}

// x_fake[m, k] = scale[m] * ((float)q[m, k] - (float)zp[m]) (dit.c:326-328).
__global__ void fake_quant_kernel(const uint8_t* __restrict__ q, const float* __restrict__ sc,
                                  const int32_t* __restrict__ zp, int M, int K,
                                  float* __restrict__ out) {
  const long long total = (long long)M * K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / K);
    out[i] = __fmul_rn(sc[m], __fsub_rn((float)q[i], (float)zp[m]));
  }
}

int grid_for(long long n, int sms) {
  return (int)std::min<long long>((n + 255) / 256, (long long)sms * 16);
}

}  // namespace

// x += gate[row / rows_per_gate] * y, elementwise in the reference's order
// (dit.c:1013-1020: the branch value times the gate, then added).
__global__ void gated_residual_kernel(float* __restrict__ x, const float* __restrict__ y,
                                      const float* __restrict__ gate, int rows_per_gate, int M,
                                      int D) {
  const long long total = (long long)M * D;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / D), d = (int)(i - (long long)m * D);
    x[i] = __fadd_rn(x[i], __fmul_rn(gate[(size_t)(m / rows_per_gate) * D + d], y[i]));
  }
}

// h = (a / (1 + expf(-a))) * g (ops.c:781-784), a and g plain [M, H].
__global__ void silu_mul_plain_kernel(const float* __restrict__ a, const float* __restrict__ g,
                                      long long n, float* __restrict__ h) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    h[i] = __fmul_rn(__fdiv_rn(a[i], __fadd_rn(1.0f, expf(-a[i]))), g[i]);
}

size_t diag_linear_scratch_bytes(int M, int K, int N) {
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  // Emulate 1: the dequantised weight rows; emulate 2: the fake-quantised
  // activations plus the quantiser's codes and row parameters.
  const size_t e1 = al(sizeof(float) * (size_t)N * K);
  const size_t e2 = al(sizeof(float) * (size_t)M * K) + al((size_t)M * K) + 2 * al(4 * (size_t)M);
  return e1 > e2 ? e1 : e2;
}

int diag_linear(Ctx* c, int mode, const float* x, int M, int K, const IroInt8DevWeight* w,
                int row0, int part, const float* w_fp32, float* y, int N, void* scratch,
                cudaStream_t s) {
  if (M <= 0) return IRO_OK;
  const float* A = x;
  const float* Bw = w_fp32;
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  int st;
  if (mode == DIAG_EMULATE_WEIGHT) {
    float* deq = reinterpret_cast<float*>(sc);
    dequant_weight_kernel<<<grid_for((long long)N * K, c->num_sms), 256, 0, s>>>(*w, row0, part,
                                                                               N, deq);
    if ((st = check_launch())) return st;
    Bw = deq;
  } else if (mode == DIAG_EMULATE_ACTIVATION) {
    if (!w_fp32) return IRO_ERR_UNSUPPORTED;
    float* fake = reinterpret_cast<float*>(sc);
    uint8_t* q = sc + al(sizeof(float) * (size_t)M * K);
    float* rs = reinterpret_cast<float*>(q + al((size_t)M * K));
    int32_t* rz = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(rs) + al(4 * (size_t)M));
    if ((st = quantize_rows_launch(x, M, K, q, rs, rz, 0, s))) return st;
    fake_quant_kernel<<<grid_for((long long)M * K, c->num_sms), 256, 0, s>>>(q, rs, rz, M, K,
                                                                            fake);
    if ((st = check_launch())) return st;
    A = fake;
  } else if (!w_fp32) {
    return IRO_ERR_UNSUPPORTED;
  }
  sgemm_nt_kernel<<<dim3(cdiv(N, kT), cdiv(M, kT)), 256, 0, s>>>(A, Bw, y, M, N, K);
  return check_launch();
}

int gated_residual_launch(Ctx* c, float* x, const float* y, const float* gate,
                          int rows_per_gate, int M, int D, cudaStream_t s) {
  gated_residual_kernel<<<grid_for((long long)M * D, c->num_sms), 256, 0, s>>>(
      x, y, gate, rows_per_gate, M, D);
  return check_launch();
}

int silu_mul_plain_launch(Ctx* c, const float* a, const float* g, long long n, float* h,
                          cudaStream_t s) {
  silu_mul_plain_kernel<<<grid_for(n, c->num_sms), 256, 0, s>>>(a, g, n, h);
  return check_launch();
}

}  // namespace iro
