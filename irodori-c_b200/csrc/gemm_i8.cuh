// gemm_i8.cuh — host interface of the tcgen05 int8 GEMM (gemm_i8.cu).
#pragma once

#include "runtime.cuh"

namespace iro {

enum EpiKind {
  EPI_LINEAR = 0,  // y (=|+=) dequant (+bias); optional raw s32 sums
  EPI_SPLIT = 1,   // as LINEAR, column block g written to outs[g]
  EPI_GATED = 2,   // hidden = silu(dequant W1 + b1) * (dequant W3 + b3)
  EPI_DUAL = 3,    // y = (dequant(q1) + bias) + dequant(q2); with accumulate
                   // y = (y + (dequant(q1) + bias)) + dequant(q2)
  EPI_QKV = 4,     // the QKVG split (outs = q, k, -, gate) with the DiT's head
                   // RMSNorm + RoPE on q and k and v written as per-head V^T
  EPI_DUAL2 = 5    // EPI_DUAL into y (nout = 0) with both terms stacked in one
                   // 128-row A tile: 64 output rows per tile, N = 256 MMAs
                   // (chosen by gemm_launch for EPI_DUAL requests)
};

// One GEMM request: A (u8 codes, rows of `lda` bytes, K valid) against the
// device weight w (N rows of w->ld bytes).
struct GemmRequest {
  int epi = EPI_LINEAR;
  int M = 0;
  const uint8_t* a = nullptr;
  int lda = 0;
  const float* sx = nullptr;
  const int32_t* zp = nullptr;
  const uint8_t* a2 = nullptr;  // EPI_DUAL
  const float* sx2 = nullptr;
  const int32_t* zp2 = nullptr;
  const IroInt8DevWeight* w = nullptr;
  const float* bias = nullptr;  // per weight row; GATED uses w->bias
  float* y = nullptr;
  int ldy = 0;
  int32_t* work = nullptr;
  int ldw = 0;
  int accumulate = 0;
  float* outs[4] = {nullptr, nullptr, nullptr, nullptr};
  int nout = 0, seg = 0;
  float* hidden = nullptr;  // GATED: [M, w->hidden], row pitch ldh
  int ldh = 0;
  // EPI_LINEAR / EPI_DUAL: y += rgate[row / rgate_rows][n] * result (the
  // DiT's gated residual, dit.c:1013-1020, in its order: the result rounded,
  // times the gate, then added); `accumulate` must be 0.
  const float* rgate = nullptr;
  int rgate_rows = 0;
  // EPI_QKV: head RMSNorm weights of q and k ([seg], head dim 64, 16-byte
  // aligned), the RoPE tables in groups of four pairs ([8][tokens][4] cos /
  // sin: element ((pair / 4) * tokens + token) * 4 + pair % 4, so a warp's 32
  // rows read 32 consecutive tokens' groups) and the norm epsilon.  The
  // attention operands go out in fp16 (range-checked, IRO_ERR_RANGE): q and
  // k to hq / hk ([rows, seg], 16-byte aligned), v transposed to hvt
  // ([rows / tokens] x heads x 64 rows of vt_ld halves, vt_ld a multiple of
  // 8; columns tokens..vt_ld-1 are zeroed); the gate to outs[3] in fp32.
  // Row r is token r % tokens of sequence r / tokens.
  const float* hn_q = nullptr;
  const float* hn_k = nullptr;
  const float* rcos = nullptr;
  const float* rsin = nullptr;
  __half* hq = nullptr;
  __half* hk = nullptr;
  __half* hvt = nullptr;
  int vt_ld = 0;
  int tokens = 0;
  float eps = 0.0f;
  int force_bn = 0;         // 0 = heuristic
  int no_alloc = 0;         // never allocate (skips the IRO_GEMM_TRACE buffer)
};

int gemm_launch(Ctx* c, const GemmRequest& r, cudaStream_t s);

// IRO_GEMM_PROFILE (gemm_profile.cu): per-shape device time of gemm_launch.
bool gemm_profile_on();
void* gemm_profile_begin(const GemmRequest& r, cudaStream_t s);
void gemm_profile_end(void* token, const GemmRequest& r, cudaStream_t s);

// iro_int8_swiglu_dev with an optional gated residual in the W2 epilogue:
// out += rgate[row / rgate_rows] * swiglu(x) when rgate is set (out then
// holds the residual stream), out = swiglu(x) otherwise.  With qx set, x is
// already quantised (codes qx [M, K], row scale sx and zero point zx) and
// x itself is not read.
// residual_w13: the two-term activation path for W1/W3 too (dit.c:923-947
// with IRO_INT8_RESIDUAL bit 4): x quantised with its residual term, both
// terms through W1|W3, then silu(w1) * w3; needs x (not qx).
int swiglu_run(Ctx* c, const float* x, int M, const IroInt8DevWeight* w13,
               const IroInt8DevWeight* w2, const float* b2, float* out, int residual_w2,
               void* workspace, cudaStream_t s, const float* rgate, int rgate_rows,
               const uint8_t* qx = nullptr, const float* sx = nullptr,
               const int32_t* zx = nullptr, int residual_w13 = 0, int stats_layer = -1);

// Workspace of swiglu_run (iro_int8_swiglu_workspace_bytes plus the two-term
// W1/W3 buffers when residual_w13 is set).
size_t swiglu_workspace_bytes_ex(int M, int D, int H, int residual_w2, int residual_w13);


}  // namespace iro
