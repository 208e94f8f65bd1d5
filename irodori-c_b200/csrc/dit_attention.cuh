// dit_attention.cuh — tensor-core joint attention of the DiT block.
#pragma once

#include "runtime.cuh"

namespace iro {

// q, k, v, g, mix: [B*S, D] row-major fp32 (D = heads * 64); ck, cv:
// [context_batch*C, D]; mask: [B, C] per batch row; batch row b uses context
// row b / (B / context_batch).  mix = softmax(q.k^T / 8) . v * sigmoid(g)
// over the row's S self keys and its valid context keys (dit.c:806-862).
struct AttnTcRequest {
  const float* q;
  const float* k;
  const float* v;
  const float* g;
  const float* ck;
  const float* cv;
  const uint8_t* mask;
  float* mix;
  int B, S, C, context_batch, D, heads;
  void* workspace;  // attention_tc_workspace_bytes(B, S, C, context_batch, D), 16-byte aligned
  // Optional: the self V^T rows already in the workspace's first region
  // (vt[((b * heads + h) * 64 + d) * attention_tc_vt_ld(S) + s], zero past S),
  // so the launch only transposes the context V.
  const float* vt_self;
  // One CTA per 128 query rows (M = 128 MMAs) instead of CTA pairs (M = 256).
  int single_cta;
};

// Row pitch (floats) of the V^T rows for n tokens.
int attention_tc_vt_ld(int n);

// Scratch for the per-head V^T copies of the self and context values.
size_t attention_tc_workspace_bytes(int B, int S, int C, int context_batch, int D);

// Whether the tensor-core kernel takes this request (16-byte aligned
// buffers, D a multiple of 64).
bool attention_tc_supported(const AttnTcRequest& r);

// Stream-ordered launch (programmatic dependent launch; the kernel waits for
// the previous kernel before touching memory).  IRO_OK or IRO_ERR_*.
int attention_tc_launch(Ctx* c, const AttnTcRequest& r, cudaStream_t s);

}  // namespace iro
