/* ref_vnni_shim.c — TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference's VNNI prototype benchmark (tests/bench_vnni_linear.c,
 * included from the reference tree, never copied) and exports its file-static
 * symmetric activation quantiser (bench_vnni_linear.c:82-101), the BASELINE
 * "absmax/127, stored u8 = s8 + 128" mode, so fixtures can pin it.  The
 * benchmark's main() is renamed away and its BLAS hooks are stubbed: only the
 * quantiser is ever called.
 */
#define main iro_vnni_bench_main_unused
#include "tests/bench_vnni_linear.c"
#undef main

void scipy_cblas_sgemm(int layout, int transa, int transb, int m, int n, int k, float alpha,
                       const float *a, int lda, const float *b, int ldb, float beta, float *c,
                       int ldc) {
    (void)layout; (void)transa; (void)transb; (void)m; (void)n; (void)k; (void)alpha;
    (void)a; (void)lda; (void)b; (void)ldb; (void)beta; (void)c; (void)ldc;
}

void scipy_openblas_set_num_threads(int threads) { (void)threads; }

void ref_quantize_activation_sym(const float *x, uint8_t *qx, float *scale, int m, int k) {
    quantize_activation(x, qx, scale, m, k);
}
