// dit_block.cuh — the DiT block split into its AdaLN parameters and its body,
// so that a caller whose blocks share one conditioning vector (every layer
// of a sampler step) computes all layers' parameters in one batch.
#pragma once

#include "runtime.cuh"

namespace iro {

// Scratch for dit_adaln_params over `sets` = 2 * n_blocks matrix sets.
size_t dit_adaln_scratch_bytes(int sets, int rows, int D, int R);

// AdaLN parameters (dit.c:543-593) of n_blocks blocks (both halves each,
// 2 * n_blocks <= 2 * IRO_DIT_MAX_LAYERS) for cond [rows, 3D]: params gets
// [n_blocks][2 halves][3: shift, scale, gate][rows][D].
int dit_adaln_params(const IroDiTBlockDev* const* blks, int n_blocks, const float* cond,
                     int rows, float* params, void* scratch, cudaStream_t s);

// Argument check shared by the block entry points (IRO_OK or IRO_ERR_*).
int dit_block_check(const IroDiTBlockDev* blk, const float* x, int cond_rows, const float* ctx_k,
                    const float* ctx_v, const uint8_t* ctx_mask, int context_batch, int B, int S,
                    int C, const float* rope_cos, const float* rope_sin);

// Workspace of dit_block_run.
size_t dit_block_body_bytes(const IroDiTBlockDev* blk, int B, int S, int C, int context_batch);

// The block (dit.c:983-1051) on x [B*S, D] with precomputed AdaLN
// parameters: ada[half * 3 + branch] -> [cond_rows][D] (shift, scale, gate).
int dit_block_run(Ctx* c, const IroDiTBlockDev* blk, float* x, const float* const* ada,
                  int cond_rows, const float* ctx_k, const float* ctx_v,
                  const uint8_t* ctx_mask, int context_batch, int B, int S, int C,
                  const float* rcos, const float* rsin, void* workspace, cudaStream_t s,
                  int stats_layer = -1, const float* rope_t = nullptr);

}  // namespace iro
