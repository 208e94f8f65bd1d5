// diag.cuh — the int8 activation diagnostics of the DiT (dit.c:340-412):
// IRO_INT8_STATS per (layer, group) row statistics and IRO_INT8_DUMP raw
// activation files, recorded on the device path at the reference's four
// points (Q/K/V/gate input, Wo input, W1/W3 input, W2 input).
#pragma once

#include "runtime.cuh"

namespace iro {

constexpr int kStatGroups = 4;     // qkvg, wo, w13, w2
constexpr int kStatChannels = 8192;  // argmax histogram length (K above it is not recorded)

// True when IRO_INT8_STATS (not "0") or IRO_INT8_DUMP is set.
bool diag_enabled();

// Record rows x [M, K] (device) as activation group `group` of `layer`
// (layer < 0: nothing).  Stream-ordered; the dump copies synchronise.
int diag_record(int layer, int group, const float* x, int M, int K, cudaStream_t s);

}  // namespace iro
