// quantize.cuh — launchers of the quantiser kernels (quantize.cu).
#pragma once

#include <algorithm>

#include "runtime.cuh"

namespace iro {

int quantize_rows_launch(const float* x, int M, int K, uint8_t* q, float* scale, int32_t* zero,
                         int symmetric, cudaStream_t s);
int quantize_rows_residual_launch(const float* x, int M, int K, uint8_t* q1, float* s1,
                                  int32_t* z1, float* residual, uint8_t* q2, float* s2,
                                  int32_t* z2, cudaStream_t s);
int weight_quantize_launch(const float* w, int N, int K, int8_t* data, int ld, float* scale,
                           int32_t* colsum, cudaStream_t s);
int transpose_f32_launch(const float* in, int rows, int cols, float* out, cudaStream_t s);
int repack_rows_launch(const uint8_t* in, int M, int K, uint8_t* out, int ld, cudaStream_t s);

}  // namespace iro
