/* iro_oracle.c — CPU restatement of irodori-c's W8A8 int8 path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never the thing
 * measured or shipped.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg load it.
 *
 * Numerics contract: compiled with -O2 -ffp-contract=off (no -ffast-math),
 * every float operation below is one IEEE-754 binary32 operation rounded to
 * nearest-even, in the order the reference writes it.  The integer GEMM is
 * exact, so it may be split over threads freely (the reference's own
 * cross-M determinism test, tests/test_int8_ops.c:87-97, relies on the same
 * fact).  Parity of this file against the reference is pinned by
 * tests/test_oracle.py (against oracle/_ref built from the reference sources,
 * and against the fixtures in tests/golden/).
 */
#include "iro_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <unistd.h>

/* Row-parallel helper: integer sums and per-row float work are independent
   of how rows are split, so the split cannot change any result. */
typedef void (*row_fn)(void *ctx, int begin, int end);
typedef struct { row_fn fn; void *ctx; int begin, end; } row_job;

static void *row_job_run(void *arg) {
    row_job *j = (row_job *)arg;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

static int oracle_threads(void) {
    const char *env = getenv("IRO_ORACLE_THREADS");
    long n = env && *env ? strtol(env, NULL, 10) : sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    return (int)n;
}

static void par_rows(int rows, long long work_per_row, row_fn fn, void *ctx) {
    int nt = oracle_threads();
    if ((long long)rows * work_per_row < (1LL << 20) || rows < 2) nt = 1;
    if (nt > rows) nt = rows;
    if (nt <= 1) {
        fn(ctx, 0, rows);
        return;
    }
    pthread_t tid[64];
    row_job jobs[64];
    int started[64] = {0};
    for (int t = 0; t < nt; t++) {
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].begin = (int)((long long)rows * t / nt);
        jobs[t].end = (int)((long long)rows * (t + 1) / nt);
        started[t] = t > 0 && pthread_create(&tid[t], NULL, row_job_run, &jobs[t]) == 0;
    }
    row_job_run(&jobs[0]);
    for (int t = 1; t < nt; t++) {
        if (started[t]) pthread_join(tid[t], NULL);
        else row_job_run(&jobs[t]);
    }
}

/* float -> int as x86-64 cvttss2si does it for the reference build: NaN and
   out-of-range values give INT32_MIN.  The reference relies on the plain C
   cast; spelling the x86 result out keeps the oracle host-independent. */
static int32_t cast_f2i(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int32_t)v;
}

/* (uint8_t) of a float already clamped to [0,255] (or NaN): x86 truncates
   through a 32-bit conversion, so NaN becomes 0. */
static uint8_t cast_f2u8(float v) { return (uint8_t)(cast_f2i(v) & 0xFF); }

/* ops.c:259-293 — per output row: amax = max |w| (strict '>' update);
   scale = amax/127 (1 for an all-zero row); inv = 1/scale;
   q = clamp(nearbyintf(w*inv), -127, 127); colsum = sum q. */
int oracle_weight_quantize(const float *w, int N, int K,
                           int8_t *data, float *scale, int32_t *colsum) {
    if (!w || !data || !scale || !colsum || N <= 0 || K <= 0) return -1;
    for (int n = 0; n < N; n++) {
        const float *src = w + (size_t)n * K;
        int8_t *dst = data + (size_t)n * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) {
            float mag = fabsf(src[k]);
            if (mag > amax) amax = mag;
        }
        float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        float inv = 1.0f / s;
        int32_t total = 0;
        for (int k = 0; k < K; k++) {
            int32_t v = cast_f2i(nearbyintf(src[k] * inv));
            v = v > 127 ? 127 : v;
            v = v < -127 ? -127 : v;
            dst[k] = (int8_t)v;
            total += v;
        }
        scale[n] = s;
        colsum[n] = total;
    }
    return 0;
}

/* ops.c:295-306 — transpose [K,N] to [N,K], then quantise as above. */
int oracle_weight_quantize_transposed(const float *w, int N, int K,
                                      int8_t *data, float *scale,
                                      int32_t *colsum) {
    if (!w || N <= 0 || K <= 0) return -1;
    float *t = (float *)malloc(sizeof(float) * (size_t)N * K);
    if (!t) return -1;
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) t[(size_t)n * K + k] = w[(size_t)k * N + n];
    int rc = oracle_weight_quantize(t, N, K, data, scale, colsum);
    free(t);
    return rc;
}

/* The per-row parameters of ops.c:329-339 from a row range [lo, hi] that
   already includes 0: s = (hi-lo)/255 (1 when not > 0), inv = 1/s,
   zp = clamp(nearbyintf(-lo*inv), 0, 255). */
static void row_params(float lo, float hi, float *s_out, float *inv_out,
                       int32_t *zp_out) {
    float s = (hi - lo) / 255.0f;
    if (!(s > 0.0f)) s = 1.0f;
    float inv = 1.0f / s;
    int32_t zp = cast_f2i(nearbyintf(-lo * inv));
    zp = zp < 0 ? 0 : zp;
    zp = zp > 255 ? 255 : zp;
    *s_out = s;
    *inv_out = inv;
    *zp_out = zp;
}

/* ops.c:341-345 — one code: clamp(nearbyintf(x*inv + zp), 0, 255). */
static uint8_t quant_code(float x, float inv, float zpf) {
    float v = nearbyintf(x * inv + zpf);
    v = v < 0.0f ? 0.0f : v;
    v = v > 255.0f ? 255.0f : v;
    return cast_f2u8(v);
}

/* ops.c:321-348 — row range forced to include 0 by starting lo = hi = 0 and
   updating with strict comparisons (NaN never replaces the running value). */
typedef struct {
    const float *x;
    int K;
    uint8_t *q;
    float *scale;
    int32_t *zero;
} quant_ctx;

static void quantize_rows_part(void *p, int begin, int end) {
    const quant_ctx *c = (const quant_ctx *)p;
    const int K = c->K;
    for (int m = begin; m < end; m++) {
        const float *src = c->x + (size_t)m * K;
        uint8_t *dst = c->q + (size_t)m * K;
        float lo = 0.0f, hi = 0.0f;
        for (int k = 0; k < K; k++) {
            lo = src[k] < lo ? src[k] : lo;
            hi = src[k] > hi ? src[k] : hi;
        }
        float s, inv;
        int32_t zp;
        row_params(lo, hi, &s, &inv, &zp);
        float zpf = (float)zp;
        for (int k = 0; k < K; k++) dst[k] = quant_code(src[k], inv, zpf);
        c->scale[m] = s;
        c->zero[m] = zp;
    }
}

void oracle_quantize_rows(const float *x, int M, int K,
                          uint8_t *q, float *scale, int32_t *zero) {
    quant_ctx c = {x, K, q, scale, zero};
    par_rows(M, K, quantize_rows_part, &c);
}

/* tests/bench_vnni_linear.c:82-101 — amax/127 scale (1 when amax == 0),
   q = clamp(lrintf(x / s), -127, 127), stored as u8 q + 128.  lrintf under
   the default rounding mode is round-half-even.  zero[m] = 128 makes the
   stored u8 codes valid input for the asymmetric linear, whose epilogue then
   removes 128*colsum (ops.c:468-490; bench_vnni_linear.c:106-108). */
static void quantize_rows_sym_part(void *p, int begin, int end) {
    const quant_ctx *c = (const quant_ctx *)p;
    const int K = c->K;
    for (int m = begin; m < end; m++) {
        const float *src = c->x + (size_t)m * K;
        uint8_t *dst = c->q + (size_t)m * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) {
            float mag = fabsf(src[k]);
            if (mag > amax) amax = mag;
        }
        float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        for (int k = 0; k < K; k++) {
            /* lrintf of NaN / overflow is LONG_MIN on x86-64; (int) keeps the
               low 32 bits, i.e. 0. */
            float r = nearbyintf(src[k] / s);
            int32_t v = (r >= -2147483648.0f && r < 2147483648.0f) ? (int32_t)r : 0;
            v = v > 127 ? 127 : v;
            v = v < -127 ? -127 : v;
            dst[k] = (uint8_t)(v + 128);
        }
        c->scale[m] = s;
        c->zero[m] = 128;
    }
}

void oracle_quantize_rows_sym(const float *x, int M, int K,
                              uint8_t *q, float *scale, int32_t *zero) {
    quant_ctx c = {x, K, q, scale, zero};
    par_rows(M, K, quantize_rows_sym_part, &c);
}

/* ops.c:427-442 — q1 = quant(x); r = x - s1*(q1 - zp1); q2 = quant(r). */
void oracle_quantize_rows_residual(const float *x, int M, int K,
                                   uint8_t *q1, float *scale1, int32_t *zero1,
                                   float *residual,
                                   uint8_t *q2, float *scale2, int32_t *zero2) {
    oracle_quantize_rows(x, M, K, q1, scale1, zero1);
    for (int m = 0; m < M; m++) {
        const float *src = x + (size_t)m * K;
        const uint8_t *code = q1 + (size_t)m * K;
        float *dst = residual + (size_t)m * K;
        const float s = scale1[m];
        const float zpf = (float)zero1[m];
        for (int k = 0; k < K; k++) dst[k] = src[k] - s * ((float)code[k] - zpf);
    }
    oracle_quantize_rows(residual, M, K, q2, scale2, zero2);
}

/* ops.c:351-364 — exact integer sums; threads split rows (exact). */
typedef struct {
    const uint8_t *a;
    const int8_t *b;
    int32_t *c;
    int N, K;
} gemm_ctx;

static void gemm_part(void *p, int begin, int end) {
    const gemm_ctx *g = (const gemm_ctx *)p;
    const int N = g->N, K = g->K;
    for (int m = begin; m < end; m++) {
        const uint8_t *ar = g->a + (size_t)m * K;
        const int8_t *b = g->b;
        int32_t *cr = g->c + (size_t)m * N;
        for (int n = 0; n < N; n++) {
            const int8_t *br = b + (size_t)n * K;
            int32_t acc = 0;
            for (int k = 0; k < K; k++) acc += (int32_t)ar[k] * (int32_t)br[k];
            cr[n] = acc;
        }
    }
}

void oracle_gemm_u8s8(const uint8_t *a, const int8_t *b, int32_t *c,
                      int M, int N, int K) {
    gemm_ctx g = {a, b, c, N, K};
    par_rows(M, (long long)N * K, gemm_part, &g);
}

/* ops.c:468-490 — y = (float)(acc - zp*colsum) * (sx*sw) [+ bias];
   accumulate adds that whole term into y: y = y + (prod [+ bias]). */
typedef struct {
    const int32_t *work;
    const float *scale;
    const int32_t *zero;
    const float *wscale;
    const int32_t *wcolsum;
    int N;
    const float *bias;
    float *y;
    int accumulate;
} epi_ctx;

static void epilogue_part(void *p, int begin, int end) {
    const epi_ctx *e = (const epi_ctx *)p;
    const int N = e->N, accumulate = e->accumulate;
    const int32_t *work = e->work, *zero = e->zero, *wcolsum = e->wcolsum;
    const float *scale = e->scale, *wscale = e->wscale, *bias = e->bias;
    float *y = e->y;
    for (int m = begin; m < end; m++) {
        const int32_t *acc = work + (size_t)m * N;
        float *out = y + (size_t)m * N;
        const float sx = scale[m];
        const int32_t zp = zero[m];
        for (int n = 0; n < N; n++) {
            float term = (float)(acc[n] - zp * wcolsum[n]) * (sx * wscale[n]);
            if (bias) term = term + bias[n];
            out[n] = accumulate ? out[n] + term : term;
        }
    }
}

void oracle_epilogue(const int32_t *work, const float *scale,
                     const int32_t *zero, const float *wscale,
                     const int32_t *wcolsum, int N, const float *bias,
                     float *y, int M, int accumulate) {
    epi_ctx e = {work, scale, zero, wscale, wcolsum, N, bias, y, accumulate};
    par_rows(M, N, epilogue_part, &e);
}

/* ops.c:450-491 (scalar backend, ops.c:466). */
void oracle_linear_ex(const uint8_t *q, const float *scale, const int32_t *zero,
                      const int8_t *wdata, const float *wscale,
                      const int32_t *wcolsum, int N, int K,
                      const float *bias, float *y, int M, int32_t *work,
                      int accumulate) {
    oracle_gemm_u8s8(q, wdata, work, M, N, K);
    oracle_epilogue(work, scale, zero, wscale, wcolsum, N, bias, y, M,
                    accumulate);
}

/* ops.c:781-784. */
void oracle_silu_mul(float *x, const float *gate, size_t count) {
    for (size_t i = 0; i < count; i++)
        x[i] = (x[i] / (1.0f + expf(-x[i]))) * gate[i];
}

/* dacvae.c:340-348. */
int oracle_conv1d_out_len(int T_in, int kernel, int stride, int dilation,
                          int padding) {
    if (T_in <= 0 || stride <= 0 || kernel <= 0 || dilation <= 0) return -1;
    long long span = (long long)dilation * (kernel - 1) + 1;
    long long num = (long long)T_in + 2LL * padding - span;
    long long out = num < 0 ? -1 : num / stride + 1;
    return out <= 0 || out > 0x7fffffff ? -1 : (int)out;
}

/* dacvae.c:543-688 without snake.  For output row t the taps read input rows
   it = t*stride - padding + tap*dilation.  The row range is the min/max over
   the valid taps' rows with 0 included (dacvae.c:607-627); the parameters
   follow row_params; padding taps are the zero point (dacvae.c:651-655).
   With residual, a second term codes the remainder with scale s/255 and
   zero point 128 (dacvae.c:637-663) and is accumulated without bias
   (dacvae.c:679-681).  The reference processes rows in blocks of rows_cap;
   every output row's codes and sums depend only on that row, so the
   unblocked loop below gives identical results.  cols_out/scale_out/
   zero_out, when not NULL, receive the first-term im2col codes
   [T_out, k*C] and row parameters for byte-level comparison. */
int oracle_conv1d_int8(const float *input, int T_in, int C,
                       const int8_t *wdata, const float *wscale,
                       const int32_t *wcolsum, int N, int kernel, int stride,
                       int dilation, int padding, const float *bias,
                       int residual, float *output,
                       uint8_t *cols_out, float *scale_out, int32_t *zero_out) {
    int T_out = oracle_conv1d_out_len(T_in, kernel, stride, dilation, padding);
    if (T_out <= 0 || !input || !wdata || !output || C <= 0 || N <= 0) return -1;
    const int inner = kernel * C;
    float *rlo = (float *)malloc(sizeof(float) * (size_t)T_in);
    float *rhi = (float *)malloc(sizeof(float) * (size_t)T_in);
    const int block = 1024;
    uint8_t *cols = (uint8_t *)malloc((size_t)block * inner);
    uint8_t *cols2 = residual ? (uint8_t *)malloc((size_t)block * inner) : NULL;
    float *sc = (float *)malloc(sizeof(float) * block);
    int32_t *zr = (int32_t *)malloc(sizeof(int32_t) * block);
    float *sc2 = (float *)malloc(sizeof(float) * block);
    int32_t *zr2 = (int32_t *)malloc(sizeof(int32_t) * block);
    int32_t *work = (int32_t *)malloc(sizeof(int32_t) * (size_t)block * N);
    if (!rlo || !rhi || !cols || (residual && !cols2) || !sc || !zr || !sc2 ||
        !zr2 || !work) {
        free(rlo); free(rhi); free(cols); free(cols2); free(sc); free(zr);
        free(sc2); free(zr2); free(work);
        return -1;
    }
    /* dacvae.c:607-617 — per input row range with 0 included. */
    for (int r = 0; r < T_in; r++) {
        const float *row = input + (size_t)r * C;
        float lo = 0.0f, hi = 0.0f;
        for (int c = 0; c < C; c++) {
            lo = row[c] < lo ? row[c] : lo;
            hi = row[c] > hi ? row[c] : hi;
        }
        rlo[r] = lo;
        rhi[r] = hi;
    }
    for (int start = 0; start < T_out; start += block) {
        int rows = T_out - start < block ? T_out - start : block;
        for (int r = 0; r < rows; r++) {
            int t = start + r;
            float lo = 0.0f, hi = 0.0f;
            for (int tap = 0; tap < kernel; tap++) {
                long long it = (long long)t * stride - padding + (long long)tap * dilation;
                if (it < 0 || it >= T_in) continue;
                lo = rlo[it] < lo ? rlo[it] : lo;
                hi = rhi[it] > hi ? rhi[it] : hi;
            }
            float s, inv;
            int32_t zp;
            row_params(lo, hi, &s, &inv, &zp);
            const float zpf = (float)zp;
            const float inv2 = 255.0f / s;
            sc[r] = s;
            zr[r] = zp;
            sc2[r] = s / 255.0f;
            zr2[r] = 128;
            uint8_t *dst = cols + (size_t)r * inner;
            uint8_t *dst2 = residual ? cols2 + (size_t)r * inner : NULL;
            for (int tap = 0; tap < kernel; tap++) {
                long long it = (long long)t * stride - padding + (long long)tap * dilation;
                uint8_t *td = dst + (size_t)tap * C;
                if (it < 0 || it >= T_in) {
                    memset(td, zp, (size_t)C);
                    if (residual) memset(dst2 + (size_t)tap * C, 128, (size_t)C);
                    continue;
                }
                const float *row = input + (size_t)it * C;
                for (int c = 0; c < C; c++) {
                    float v = nearbyintf(row[c] * inv + zpf);
                    v = v < 0.0f ? 0.0f : v;
                    v = v > 255.0f ? 255.0f : v;
                    td[c] = cast_f2u8(v);
                    if (residual) {
                        float rem = row[c] - s * (v - zpf);
                        float v2 = nearbyintf(rem * inv2 + 128.0f);
                        v2 = v2 < 0.0f ? 0.0f : v2;
                        v2 = v2 > 255.0f ? 255.0f : v2;
                        dst2[(size_t)tap * C + c] = cast_f2u8(v2);
                    }
                }
            }
        }
        if (cols_out) memcpy(cols_out + (size_t)start * inner, cols, (size_t)rows * inner);
        if (scale_out) memcpy(scale_out + start, sc, sizeof(float) * rows);
        if (zero_out) memcpy(zero_out + start, zr, sizeof(int32_t) * rows);
        float *out = output + (size_t)start * N;
        oracle_linear_ex(cols, sc, zr, wdata, wscale, wcolsum, N, inner, bias,
                         out, rows, work, 0);
        if (residual)
            oracle_linear_ex(cols2, sc2, zr2, wdata, wscale, wcolsum, N, inner,
                             NULL, out, rows, work, 1);
    }
    free(rlo); free(rhi); free(cols); free(cols2); free(sc); free(zr);
    free(sc2); free(zr2); free(work);
    return T_out;
}

/* dit.c:913-969 through ops.c, with optional biases (the BASELINE SwiGLU
   configuration seeds one per projection; dit.c passes NULL):
   quantise x once (dit.c:944), W1 and W3 linears (dit.c:945-946),
   h = silu(W1x) * W3x (dit.c:956, ops.c:781-784), quantise h (two-term
   when residual_w2, dit.c:963-966 / dit.c:479-486), W2 linear(s). */
int oracle_swiglu(const float *x, int M, int D, int H,
                  const int8_t *w1, const float *s1, const int32_t *c1,
                  const float *b1,
                  const int8_t *w3, const float *s3, const int32_t *c3,
                  const float *b3,
                  const int8_t *w2, const float *s2, const int32_t *c2,
                  const float *b2,
                  int residual_w2, float *out, float *hidden_out) {
    size_t mh = (size_t)M * H;
    uint8_t *qx = (uint8_t *)malloc((size_t)M * D);
    float *sx = (float *)malloc(sizeof(float) * M);
    int32_t *zx = (int32_t *)malloc(sizeof(int32_t) * M);
    float *h1 = (float *)malloc(sizeof(float) * mh);
    float *h3 = (float *)malloc(sizeof(float) * mh);
    int32_t *work = (int32_t *)malloc(sizeof(int32_t) * mh);
    uint8_t *qh = (uint8_t *)malloc(mh);
    uint8_t *qh2 = (uint8_t *)malloc(mh);
    float *rem = residual_w2 ? (float *)malloc(sizeof(float) * mh) : NULL;
    float *sh = (float *)malloc(sizeof(float) * M), *sh2 = (float *)malloc(sizeof(float) * M);
    int32_t *zh = (int32_t *)malloc(sizeof(int32_t) * M), *zh2 = (int32_t *)malloc(sizeof(int32_t) * M);
    int ok = qx && sx && zx && h1 && h3 && work && qh && qh2 && sh && sh2 && zh && zh2 &&
             (!residual_w2 || rem);
    if (ok) {
        oracle_quantize_rows(x, M, D, qx, sx, zx);
        oracle_linear_ex(qx, sx, zx, w1, s1, c1, H, D, b1, h1, M, work, 0);
        oracle_linear_ex(qx, sx, zx, w3, s3, c3, H, D, b3, h3, M, work, 0);
        oracle_silu_mul(h1, h3, mh);
        if (hidden_out) memcpy(hidden_out, h1, sizeof(float) * mh);
        if (residual_w2) {
            oracle_quantize_rows_residual(h1, M, H, qh, sh, zh, rem, qh2, sh2, zh2);
            oracle_linear_ex(qh, sh, zh, w2, s2, c2, D, H, b2, out, M, work, 0);
            oracle_linear_ex(qh2, sh2, zh2, w2, s2, c2, D, H, NULL, out, M, work, 1);
        } else {
            oracle_quantize_rows(h1, M, H, qh, sh, zh);
            oracle_linear_ex(qh, sh, zh, w2, s2, c2, D, H, b2, out, M, work, 0);
        }
    }
    free(qx); free(sx); free(zx); free(h1); free(h3); free(work); free(qh);
    free(qh2); free(rem); free(sh); free(sh2); free(zh); free(zh2);
    return ok ? 0 : -1;
}

/* dacvae.c:350-358. */
int oracle_convtranspose1d_out_len(int T_in, int kernel, int stride,
                                   int padding, int output_padding) {
    if (T_in <= 0 || stride <= 0 || kernel <= 0) return -1;
    long long out = (long long)(T_in - 1) * stride - 2LL * padding + kernel +
                    output_padding;
    return out <= 0 || out > 0x7fffffff ? -1 : (int)out;
}

/* The codec's W8A8 transposed convolution, dacvae.c:696-790 with the int8
   weight and no snake (alpha = NULL):
   - every output row starts as the bias (dacvae.c:707-709);
   - the input rows [T_in, C_in] are quantised per row (asymmetric, or the
     two-term residual form when `residual`, dacvae.c:748-772);
   - expanded[r, tap*C_out + c] = linear(q, W) without bias, plus the second
     term accumulated (dacvae.c:766-767);
   - expanded row r, tap t is added onto output row r*stride - padding + t
     when that row exists (dacvae.c:776-787).
   The reference walks the input in blocks of rows_cap rows; each output
   element receives its additions in increasing input-row order either way,
   so the unblocked loop below gives identical sums.  W is [kernel*C_out,
   C_in] (dacvae.h:47-52).  Returns T_out or -1. */
int oracle_convtranspose1d_int8(const float *input, int T_in, int C_in,
                                int C_out, const int8_t *wdata,
                                const float *wscale, const int32_t *wcolsum,
                                int kernel, int stride, int padding,
                                int output_padding, const float *bias,
                                int residual, float *output) {
    int T_out = oracle_convtranspose1d_out_len(T_in, kernel, stride, padding,
                                               output_padding);
    if (T_out <= 0 || C_in <= 0 || C_out <= 0) return -1;
    const int N = kernel * C_out;
    for (int t = 0; t < T_out; t++)
        for (int c = 0; c < C_out; c++)
            output[(size_t)t * C_out + c] = bias ? bias[c] : 0.0f;
    size_t mk = (size_t)T_in * C_in, mn = (size_t)T_in * N;
    uint8_t *q = (uint8_t *)malloc(mk), *q2 = (uint8_t *)malloc(mk);
    float *s = (float *)malloc(sizeof(float) * T_in);
    float *s2 = (float *)malloc(sizeof(float) * T_in);
    int32_t *z = (int32_t *)malloc(sizeof(int32_t) * T_in);
    int32_t *z2 = (int32_t *)malloc(sizeof(int32_t) * T_in);
    float *rem = residual ? (float *)malloc(sizeof(float) * mk) : NULL;
    float *e = (float *)malloc(sizeof(float) * mn);
    int32_t *work = (int32_t *)malloc(sizeof(int32_t) * mn);
    int ok = q && q2 && s && s2 && z && z2 && e && work && (!residual || rem);
    if (ok) {
        if (residual) {
            oracle_quantize_rows_residual(input, T_in, C_in, q, s, z, rem, q2, s2, z2);
            oracle_linear_ex(q, s, z, wdata, wscale, wcolsum, N, C_in, NULL, e, T_in, work, 0);
            oracle_linear_ex(q2, s2, z2, wdata, wscale, wcolsum, N, C_in, NULL, e, T_in, work, 1);
        } else {
            oracle_quantize_rows(input, T_in, C_in, q, s, z);
            oracle_linear_ex(q, s, z, wdata, wscale, wcolsum, N, C_in, NULL, e, T_in, work, 0);
        }
        for (int r = 0; r < T_in; r++) {
            long long base = (long long)r * stride - padding;
            for (int tap = 0; tap < kernel; tap++) {
                long long ot = base + tap;
                if (ot < 0 || ot >= T_out) continue;
                const float *src = e + (size_t)r * N + (size_t)tap * C_out;
                float *dst = output + (size_t)ot * C_out;
                for (int c = 0; c < C_out; c++) dst[c] += src[c];
            }
        }
    }
    free(q); free(q2); free(s); free(s2); free(z); free(z2); free(rem);
    free(e); free(work);
    return ok ? T_out : -1;
}

/* The residual unit's skip + 1x1 projection, dacvae.c:979-1009: output
   starts as the skip input (dacvae.c:983); the hidden rows are quantised
   (two-term residual form when `residual`) and the projection is
   accumulated onto it, the first term with the bias, the second without
   (dacvae.c:1002-1008). */
int oracle_codec_conv1(const float *hidden, int rows, int C,
                       const int8_t *wdata, const float *wscale,
                       const int32_t *wcolsum, const float *bias,
                       const float *skip, int residual, float *output) {
    if (rows <= 0 || C <= 0) return -1;
    size_t n = (size_t)rows * C;
    memcpy(output, skip, sizeof(float) * n);
    uint8_t *q = (uint8_t *)malloc(n), *q2 = (uint8_t *)malloc(n);
    float *s = (float *)malloc(sizeof(float) * rows);
    float *s2 = (float *)malloc(sizeof(float) * rows);
    int32_t *z = (int32_t *)malloc(sizeof(int32_t) * rows);
    int32_t *z2 = (int32_t *)malloc(sizeof(int32_t) * rows);
    float *rem = residual ? (float *)malloc(sizeof(float) * n) : NULL;
    int32_t *work = (int32_t *)malloc(sizeof(int32_t) * n);
    int ok = q && q2 && s && s2 && z && z2 && work && (!residual || rem);
    if (ok) {
        if (residual) {
            oracle_quantize_rows_residual(hidden, rows, C, q, s, z, rem, q2, s2, z2);
            oracle_linear_ex(q, s, z, wdata, wscale, wcolsum, C, C, bias, output, rows, work, 1);
            oracle_linear_ex(q2, s2, z2, wdata, wscale, wcolsum, C, C, NULL, output, rows, work, 1);
        } else {
            oracle_quantize_rows(hidden, rows, C, q, s, z);
            oracle_linear_ex(q, s, z, wdata, wscale, wcolsum, C, C, bias, output, rows, work, 1);
        }
    }
    free(q); free(q2); free(s); free(s2); free(z); free(z2); free(rem); free(work);
    return ok ? 0 : -1;
}

/* ops.c:375-398 — operands whose 255*127 products overflow int16. */
void oracle_selfcheck_case(uint8_t a[3 * 64], int8_t b[5 * 64],
                           int32_t want[3 * 5]) {
    for (int i = 0; i < 3 * 64; i++)
        a[i] = (uint8_t)(i % 3 == 0 ? 255 : 200 + i % 50);
    for (int i = 0; i < 5 * 64; i++)
        b[i] = (int8_t)(i % 4 == 0 ? 127 : (i % 4 == 1 ? -127 : 90 - i % 60));
    oracle_gemm_u8s8(a, b, want, 3, 5, 64);
}
