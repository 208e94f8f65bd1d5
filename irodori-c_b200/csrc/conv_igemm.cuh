// conv_igemm.cuh — host interface of the implicit-GEMM kernel-7 conv.
#pragma once

#include "runtime.cuh"

namespace iro {

// True when the fused implicit-GEMM kernel handles this convolution (stride
// 1, no residual term, 64-channel multiples, 512 output channels, window
// rows within one TMA box, aligned buffers); otherwise the caller uses the
// code-materialising path.
bool conv7_igemm_supported(int C, int N, int kernel, int stride, int dilation, int padding,
                           int residual, const void* input, const void* output);

// Launch on `s`.  scale/zero/inv are the per-output-row parameters
// [batch * T_out] from conv_row_params.
int conv7_igemm_launch(Ctx* c, const float* input, int batch, int T_in, int C,
                       const IroInt8DevWeight* w, int kernel, int dilation, int padding,
                       const float* bias, const float* scale, const int32_t* zero,
                       const float* inv, float* output, int T_out, cudaStream_t s);

}  // namespace iro
