/* ref_dit_shim.c — TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference DiT source (dit.c, included from the reference tree
 * on the compiler's include path, never copied) and exports a wrapper around
 * its file-static int8 SwiGLU block, dit.c:913-976, at the reference's fixed
 * dimensions (model 1280, hidden 3680).  IRO_INT8_RESIDUAL in the process
 * environment selects the W2 two-term policy exactly as in the reference.
 */
#include "dit.c"

int ref_dit_dims(int *model_dim, int *mlp_dim) {
    *model_dim = MODEL_DIM;
    *mlp_dim = MLP_DIM;
    return 0;
}

static IroInt8Weight ref_weight(const int8_t *d, const float *s,
                                const int32_t *c, int N, int K) {
    IroInt8Weight w;
    w.data = (int8_t *)d;
    w.scale = (float *)s;
    w.colsum = (int32_t *)c;
    w.N = N;
    w.K = K;
    return w;
}

int ref_dit_swiglu_int8(const float *x, int rows,
                        const int8_t *w1, const float *s1, const int32_t *c1,
                        const int8_t *w3, const float *s3, const int32_t *c3,
                        const int8_t *w2, const float *s2, const int32_t *c2,
                        float *out) {
    IroSwiGLU mlp;
    memset(&mlp, 0, sizeof(mlp));
    IroDiTInt8Layer layer;
    memset(&layer, 0, sizeof(layer));
    layer.w1 = ref_weight(w1, s1, c1, MLP_DIM, MODEL_DIM);
    layer.w3 = ref_weight(w3, s3, c3, MLP_DIM, MODEL_DIM);
    layer.w2 = ref_weight(w2, s2, c2, MODEL_DIM, MLP_DIM);
    return dit_swiglu(&mlp, x, 1, rows, out, -1, NULL, &layer);
}

/* The reference's whole transformer block, dit.c:983-1051, at layer 0 with
   the int8 projections (the engine's default int8 path: IRO_INT8_MASK 15,
   residual policy from IRO_INT8_RESIDUAL, W2 two-term by default).
   adaln: 18 fp32 pointers, attention then MLP AdaLN, each in IroAdaLN order;
   wq, wk, wv, gate, wo, w1, w3, w2: int8 weights quantised by the caller with
   iro_int8_weight_quantize.  x [B*S, 1280] is updated in place. */
int ref_dit_block_w(float *x, const float *cond, const float *ctx_k,
                    const float *ctx_v, const uint8_t *ctx_mask,
                    int context_batch, int B, int S, int C,
                    const float *const *adaln, const float *q_norm,
                    const float *k_norm, const int8_t *const *wdata,
                    const float *const *wscale, const int32_t *const *wcolsum,
                    const float *const *w_fp32);

int ref_dit_block_int8(float *x, const float *cond, const float *ctx_k,
                       const float *ctx_v, const uint8_t *ctx_mask,
                       int context_batch, int B, int S, int C,
                       const float *const *adaln, const float *q_norm,
                       const float *k_norm, const int8_t *const *wdata,
                       const float *const *wscale, const int32_t *const *wcolsum) {
    return ref_dit_block_w(x, cond, ctx_k, ctx_v, ctx_mask, context_batch, B, S, C,
                           adaln, q_norm, k_norm, wdata, wscale, wcolsum, NULL);
}

/* The same block with the fp32 projection weights set as well (w_fp32: wq,
   wk, wv, gate, wo, w1, w3, w2), for the reference's diagnostic switches
   IRO_INT8_MASK and IRO_INT8_EMULATE (dit.c:273-335), which it reads from
   the process environment once. */
int ref_dit_block_w(float *x, const float *cond, const float *ctx_k,
                    const float *ctx_v, const uint8_t *ctx_mask,
                    int context_batch, int B, int S, int C,
                    const float *const *adaln, const float *q_norm,
                    const float *k_norm, const int8_t *const *wdata,
                    const float *const *wscale, const int32_t *const *wcolsum,
                    const float *const *w_fp32) {
    IroDiT *d = calloc(1, sizeof(IroDiT));
    IroDiTInt8 *q = calloc(1, sizeof(IroDiTInt8));
    if (!d || !q) { free(d); free(q); return -1; }
    IroAdaLN *sets[2] = {&d->attention_adaln[0], &d->mlp_adaln[0]};
    for (int i = 0; i < 2; i++) {
        const float *const *a = adaln + 9 * i;
        sets[i]->shift_down = a[0]; sets[i]->shift_up = a[1]; sets[i]->shift_bias = a[2];
        sets[i]->scale_down = a[3]; sets[i]->scale_up = a[4]; sets[i]->scale_bias = a[5];
        sets[i]->gate_down = a[6]; sets[i]->gate_up = a[7]; sets[i]->gate_bias = a[8];
    }
    d->attention[0].q_norm = q_norm;
    d->attention[0].k_norm = k_norm;
    if (w_fp32) {
        d->attention[0].wq = w_fp32[0]; d->attention[0].wk = w_fp32[1];
        d->attention[0].wv = w_fp32[2]; d->attention[0].gate = w_fp32[3];
        d->attention[0].wo = w_fp32[4];
        d->mlp[0].w1 = w_fp32[5]; d->mlp[0].w3 = w_fp32[6]; d->mlp[0].w2 = w_fp32[7];
    }
    d->norm_eps = 1e-5f;
    IroDiTInt8Layer *l = &q->layer[0];
    const int shapes[8][2] = {{MODEL_DIM, MODEL_DIM}, {MODEL_DIM, MODEL_DIM},
                              {MODEL_DIM, MODEL_DIM}, {MODEL_DIM, MODEL_DIM},
                              {MODEL_DIM, MODEL_DIM}, {MLP_DIM, MODEL_DIM},
                              {MLP_DIM, MODEL_DIM}, {MODEL_DIM, MLP_DIM}};
    IroInt8Weight *ws[8] = {&l->wq, &l->wk, &l->wv, &l->gate, &l->wo, &l->w1, &l->w3, &l->w2};
    for (int i = 0; i < 8; i++)
        *ws[i] = ref_weight(wdata[i], wscale[i], wcolsum[i], shapes[i][0], shapes[i][1]);
    d->int8 = q;
    int rc = dit_block(d, 0, x, cond, ctx_k, ctx_v, ctx_mask, context_batch, B, S, C);
    free(d);
    free(q);
    return rc;
}

int ref_dit_block_dims(int *model_dim, int *heads, int *rank, int *mlp_dim) {
    *model_dim = MODEL_DIM;
    *heads = IRO_DIT_HEADS;
    *rank = ADALN_RANK;
    *mlp_dim = MLP_DIM;
    return 0;
}

/* The reference's conditioner, input projection and output head
   (dit.c:488-541, 1070-1090) on caller-owned fp32 weights. */
int ref_dit_condition_w(const float *w0, const float *w1, const float *w2,
                        const float *t, int B, float *cond) {
    IroDiT *d = calloc(1, sizeof(IroDiT));
    if (!d) return -1;
    d->cond_w0 = w0; d->cond_w1 = w1; d->cond_w2 = w2;
    int rc = iro_dit_condition(d, t, B, cond);
    free(d);
    return rc;
}

int ref_dit_input_w(const float *in_w, const float *in_b, const float *x,
                    int B, int S, float *out) {
    IroDiT *d = calloc(1, sizeof(IroDiT));
    if (!d) return -1;
    d->in_w = in_w; d->in_b = in_b;
    int rc = iro_dit_input(d, x, B, S, out);
    free(d);
    return rc;
}

int ref_dit_output_w(const float *out_norm, const float *out_w, const float *out_b,
                     const float *x, int B, int S, float *velocity) {
    IroDiT *d = calloc(1, sizeof(IroDiT));
    if (!d) return -1;
    d->out_norm = out_norm; d->out_w = out_w; d->out_b = out_b;
    d->norm_eps = 1e-5f;
    int rc = iro_dit_output(d, x, B, S, velocity);
    free(d);
    return rc;
}

/* The reference's residual-policy switch as it reads it (dit.c:429-436);
   cached per process by the reference. */
int ref_dit_residual_mask(void) { return dit_int8_residual_mask(); }

/* The reference's diagnostic switches IRO_INT8_MASK and IRO_INT8_EMULATE as
   its own readers parse them (dit.c:284-304). */
int ref_dit_int8_mask(void) { return dit_int8_mask(); }
int ref_dit_int8_emulate(void) { return dit_int8_emulate(); }
