// dit_diag32.cuh — fp32 / emulated projection paths of the DiT block for the
// reference's IRO_INT8_MASK and IRO_INT8_EMULATE diagnostics (dit_diag32.cu).
#pragma once

#include "runtime.cuh"

namespace iro {

enum DiagMode {
  DIAG_INT8 = 0,               // the normal int8 path
  DIAG_FP32 = 1,               // group outside the int8 mask: fp32 x fp32 weights
  DIAG_EMULATE_WEIGHT = 2,     // IRO_INT8_EMULATE=1: fp32 x dequantised int8 weights
  DIAG_EMULATE_ACTIVATION = 3  // IRO_INT8_EMULATE=2: fake-quantised x fp32 weights
};

// Scratch of diag_linear for an [M, K] input and N outputs.
size_t diag_linear_scratch_bytes(int M, int K, int N);

// y[M, N] = (mode-dependent x)[M, K] . (mode-dependent W)^T: the int8
// weight's rows row0..row0+N-1 (PLAIN) or the `part` half of the GATED_PAIR
// layout (0 = W1, 1 = W3), or the fp32 weight w_fp32 [N, K].
int diag_linear(Ctx* c, int mode, const float* x, int M, int K, const IroInt8DevWeight* w,
                int row0, int part, const float* w_fp32, float* y, int N, void* scratch,
                cudaStream_t s);

// x += gate[row / rows_per_gate] * y (dit.c:1013-1020, 1032-1039 order).
int gated_residual_launch(Ctx* c, float* x, const float* y, const float* gate,
                          int rows_per_gate, int M, int D, cudaStream_t s);

// h = (a / (1 + expf(-a))) * g over n elements (ops.c:781-784).
int silu_mul_plain_launch(Ctx* c, const float* a, const float* g, long long n, float* h,
                          cudaStream_t s);

}  // namespace iro
