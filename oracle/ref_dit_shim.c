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
