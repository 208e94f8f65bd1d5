// containers.cu — device mirrors of the reference's int8 model containers
// (IroDiTInt8, dit.h:47-58 / dit.c:235-262; IroDACVAEInt8, dacvae.h:47-67 /
// dacvae.c:230-275) with the same payload accounting in `bytes`.
#include <string.h>

#include "runtime.cuh"

using namespace iro;

extern "C" {

size_t iro_int8_dev_weight_bytes(const IroInt8DevWeight* w) {
  if (!w || !w->data) return 0;
  return (size_t)w->N * (size_t)w->ld + (size_t)w->N * (sizeof(float) + sizeof(int32_t)) +
         (w->bias ? (size_t)w->N * sizeof(float) : 0);
}

void iro_dit_int8_dev_free(IroDiTInt8Dev* q) {
  if (!q) return;
  for (int l = 0; l < 16; l++) {
    iro_int8_dev_weight_free(&q->layer[l].qkvg);
    iro_int8_dev_weight_free(&q->layer[l].wo);
    iro_int8_dev_weight_free(&q->layer[l].w13);
    iro_int8_dev_weight_free(&q->layer[l].w2);
  }
  memset(q, 0, sizeof(*q));
}

int iro_dit_int8_dev_upload(IroDiTInt8Dev* dst, const IroDiTInt8HostLayer* layers,
                            int n_layers) {
  if (!dst || !layers || n_layers <= 0 || n_layers > 16) return IRO_ERR_INVALID;
  memset(dst, 0, sizeof(*dst));
  for (int l = 0; l < n_layers; l++) {
    const IroDiTInt8HostLayer& h = layers[l];
    IroDiTInt8DevLayer& d = dst->layer[l];
    const IroInt8Weight* qkvg[4] = {&h.wq, &h.wk, &h.wv, &h.gate};
    int st = iro_int8_dev_weight_concat(&d.qkvg, qkvg, nullptr, 4);
    if (!st) st = iro_int8_dev_weight_upload(&d.wo, &h.wo, nullptr);
    if (!st) st = iro_int8_dev_weight_gated_pair(&d.w13, &h.w1, &h.w3, nullptr, nullptr);
    if (!st) st = iro_int8_dev_weight_upload(&d.w2, &h.w2, nullptr);
    if (st) {
      iro_dit_int8_dev_free(dst);
      return st;
    }
    dst->bytes += iro_int8_dev_weight_bytes(&d.qkvg) + iro_int8_dev_weight_bytes(&d.wo) +
                  iro_int8_dev_weight_bytes(&d.w13) + iro_int8_dev_weight_bytes(&d.w2);
  }
  dst->layers = n_layers;
  return IRO_OK;
}

void iro_dacvae_int8_dev_free(IroDACVAEInt8Dev* q) {
  if (!q) return;
  iro_int8_dev_weight_free(&q->initial);
  for (int s = 0; s < IRO_B200_DACVAE_STAGES; s++) {
    iro_int8_dev_weight_free(&q->stage[s].upsample);
    for (int r = 0; r < IRO_B200_DACVAE_RESIDUALS; r++) {
      iro_int8_dev_weight_free(&q->stage[s].residual[r].conv0);
      iro_int8_dev_weight_free(&q->stage[s].residual[r].conv1);
    }
  }
  memset(q, 0, sizeof(*q));
}

int iro_dacvae_int8_dev_upload(IroDACVAEInt8Dev* dst, const IroDACVAEInt8Host* src) {
  if (!dst || !src) return IRO_ERR_INVALID;
  memset(dst, 0, sizeof(*dst));
  auto up = [&](IroInt8DevWeight* d, const IroInt8Weight* h) {
    const int st = iro_int8_dev_weight_upload(d, h, nullptr);
    if (!st) dst->bytes += iro_int8_dev_weight_bytes(d);
    return st;
  };
  int st = up(&dst->initial, &src->initial);
  for (int s = 0; !st && s < IRO_B200_DACVAE_STAGES; s++) {
    st = up(&dst->stage[s].upsample, &src->stage[s].upsample);
    for (int r = 0; !st && r < IRO_B200_DACVAE_RESIDUALS; r++) {
      st = up(&dst->stage[s].residual[r].conv0, &src->stage[s].residual[r].conv0);
      if (!st) st = up(&dst->stage[s].residual[r].conv1, &src->stage[s].residual[r].conv1);
    }
  }
  if (st) iro_dacvae_int8_dev_free(dst);
  return st;
}

}  // extern "C"
