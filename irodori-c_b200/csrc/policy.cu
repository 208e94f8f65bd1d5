// policy.cu — the reference's int8 policy switches (environment variables,
// parsing and defaults as dit.c:429-436 and dacvae.c:27-71), so an engine on
// the device path can configure each projection and convolution the way the
// reference's own code would.  Host-only; read on every call.
#include <stdlib.h>

#include "irodori_b200.h"

namespace {

int env_mask(const char* name, int fallback) {
  const char* e = getenv(name);
  return (e && *e) ? (int)strtol(e, nullptr, 0) & 15 : fallback;
}

}  // namespace

extern "C" {

int iro_policy_dit_residual_mask(void) { return env_mask("IRO_INT8_RESIDUAL", 8); }

// dit.c:284-291: IRO_INT8_MASK, default 15 (every group in int8); the block
// takes the complement, the groups left in fp32.
int iro_policy_dit_fp32_groups(void) { return 15 & ~env_mask("IRO_INT8_MASK", 15); }

// dit.c:297-304: IRO_INT8_EMULATE, strtol base 0 without a mask, default 0.
int iro_policy_dit_emulate(void) {
  const char* e = getenv("IRO_INT8_EMULATE");
  return (e && *e) ? (int)strtol(e, nullptr, 0) : 0;
}

int iro_policy_codec_int8_mask(void) { return env_mask("IRO_CODEC_INT8_MASK", 15); }

int iro_policy_codec_residual_mask(void) {
  return env_mask("IRO_CODEC_INT8_RESIDUAL", 4 | 8);
}

int iro_policy_codec_residual_stages(void) {
  return env_mask("IRO_CODEC_INT8_RESIDUAL_STAGES", 8);
}

// dacvae.c:748, 957-959, 985-986, 1228: the initial Conv7 (1) and the
// upsample (2) follow their residual bit alone; the residual units' Conv7 (4)
// and Conv1 (8) also need their stage's bit.
int iro_policy_codec_residual(int stage, int group) {
  if (group != 1 && group != 2 && group != 4 && group != 8) return 0;
  if (!(iro_policy_codec_residual_mask() & group)) return 0;
  if (group == 4 || group == 8)
    return stage >= 0 && stage < 31 && ((iro_policy_codec_residual_stages() >> stage) & 1);
  return 1;
}

}  // extern "C"
