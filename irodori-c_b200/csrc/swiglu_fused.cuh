// swiglu_fused.cuh — host interface of the single-kernel SwiGLU block
// (swiglu_fused.cu).
#pragma once

#include "runtime.cuh"

namespace iro {

// Device buffers of one block invocation (carved from the caller's
// workspace): codes and row parameters of x and of the hidden, the fp32
// hidden, the per-row hidden ranges and the phase counters.
struct SwigluBuffers {
  uint8_t* qx;
  float* sx;
  int32_t* zx;
  float* hidden;
  uint8_t* qh;
  float* sh;
  int32_t* zh;
  int* hlo;
  int* hhi;
  int* ctr;
};

// Workspace bytes the fused kernel needs beyond the separate-kernel path's.
size_t swiglu_fused_extra_bytes(int M);

// Whether the fused kernel covers this block (single-term W2, 128-wide pair
// layout, 16-byte aligned rows) and is selected (IRO_SWIGLU_FUSED=1).
bool swiglu_fused_supported(Ctx* c, const float* x, int M, const IroInt8DevWeight* w13,
                            const IroInt8DevWeight* w2, const float* out, int residual_w2);

int swiglu_fused_launch(Ctx* c, const float* x, int M, const IroInt8DevWeight* w13,
                        const IroInt8DevWeight* w2, const float* b2, float* out,
                        const SwigluBuffers& b, cudaStream_t s);

}  // namespace iro
