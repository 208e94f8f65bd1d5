// dit_attention.cuh — tensor-core joint attention of the DiT block.
#pragma once

#include <cuda_fp16.h>

#include "runtime.cuh"

namespace iro {

// mix = softmax(q.k^T / 8) . v * sigmoid(g) per (batch row, head) over the
// row's S self keys and its valid context keys (dit.c:806-862).  g, mix:
// [B*S, D] row-major fp32 (D = heads * 64); ck, cv: [context_batch*C, D]
// fp32; mask: [B, C] per batch row; batch row b uses context block
// b / (B / context_batch).  The self operands are fp16 copies in the
// workspace (attention_tc_operands), written by the caller before the launch
// (the QKVG GEMM's EPI_QKV epilogue, or qk_norm_rope_half_kernel).
struct AttnTcRequest {
  const float* g;
  const float* ck;
  const float* cv;
  const uint8_t* mask;
  float* mix;
  int B, S, C, context_batch, D, heads;
  void* workspace;  // attention_tc_workspace_bytes(B, S, C, context_batch, D), 256-byte aligned
};

// The fp16 operand regions of the workspace:
//   q, k  [B*S, D]: head-normed, RoPE applied (row-major, like the fp32 q, k)
//   vt    [(b * heads + h) * 64 + d][ldv]: V^T per head, zero for s in [S, ldv)
//   ck    [context_batch*C, D]: the context keys
//   cvt   [(cb * heads + h) * 64 + d][ldc]: the context V^T, zero past C
// ck and cvt are filled by attention_tc_launch from the fp32 ck / cv.
struct AttnTcOperands {
  __half* q;
  __half* k;
  __half* vt;
  int ldv;
  __half* ck;
  __half* cvt;
  int ldc;
};
AttnTcOperands attention_tc_operands(const AttnTcRequest& r);

// Row pitch (halves) of the V^T rows for n tokens: 16-byte rows.
int attention_tc_vt_ld(int n);

// Scratch of the fp16 operands.
size_t attention_tc_workspace_bytes(int B, int S, int C, int context_batch, int D);

// Whether the tensor-core kernel takes this request (16-byte aligned
// buffers, 64-wide heads, C <= 8192).
bool attention_tc_supported(const AttnTcRequest& r);

// Stream-ordered launch: the context conversion, then the attention kernel
// (programmatic dependent launch; it waits for the previous kernel before
// touching memory).  IRO_OK or IRO_ERR_*; a context value beyond the fp16
// range is reported on the device error word as IRO_ERR_RANGE.
int attention_tc_launch(Ctx* c, const AttnTcRequest& r, cudaStream_t s);

}  // namespace iro
