/* iro_oracle.h — CPU restatement of irodori-c's W8A8 int8 path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls
 * this code; it is the checker that the CUDA kernels are compared against in
 * tests/, in __graft_entry__.smoke() and in bench.py's cpu_baseline leg.
 *
 * Every function restates one reference routine (cited per function in
 * iro_oracle.c) in plain C with IEEE single-precision semantics: the file is
 * compiled with -O2 -ffp-contract=off and no -ffast-math, which is the build
 * of ops.c whose bytes the GPU kernels must reproduce.
 */
#ifndef IRO_ORACLE_H
#define IRO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-output-channel symmetric s8 weight quantisation (ops.c:259-293). */
int oracle_weight_quantize(const float *w, int N, int K,
                           int8_t *data, float *scale, int32_t *colsum);
/* Same from a [K,N] row-major source (ops.c:295-306). */
int oracle_weight_quantize_transposed(const float *w, int N, int K,
                                      int8_t *data, float *scale,
                                      int32_t *colsum);

/* Per-row asymmetric u8 quantisation with zero point (ops.c:321-348). */
void oracle_quantize_rows(const float *x, int M, int K,
                          uint8_t *q, float *scale, int32_t *zero);

/* Per-row symmetric absmax/127 quantisation stored as u8 = s8 + 128
   (tests/bench_vnni_linear.c:82-101).  zero[m] is set to 128 so the result
   feeds the same linear as the asymmetric form. */
void oracle_quantize_rows_sym(const float *x, int M, int K,
                              uint8_t *q, float *scale, int32_t *zero);

/* Two-term residual quantisation (ops.c:427-442). */
void oracle_quantize_rows_residual(const float *x, int M, int K,
                                   uint8_t *q1, float *scale1, int32_t *zero1,
                                   float *residual,
                                   uint8_t *q2, float *scale2, int32_t *zero2);

/* Exact u8 x s8 -> s32 GEMM, c[M,N] = a[M,K] . b[N,K]^T (ops.c:351-364). */
void oracle_gemm_u8s8(const uint8_t *a, const int8_t *b, int32_t *c,
                      int M, int N, int K);

/* iro_int8_linear_ex (ops.c:450-491): GEMM into work, then the dequant
   epilogue with optional bias and accumulate. */
void oracle_linear_ex(const uint8_t *q, const float *scale, const int32_t *zero,
                      const int8_t *wdata, const float *wscale,
                      const int32_t *wcolsum, int N, int K,
                      const float *bias, float *y, int M, int32_t *work,
                      int accumulate);

/* Dequant epilogue alone, from given s32 sums (ops.c:468-490). */
void oracle_epilogue(const int32_t *work, const float *scale,
                     const int32_t *zero, const float *wscale,
                     const int32_t *wcolsum, int N, const float *bias,
                     float *y, int M, int accumulate);

/* x[i] = (x[i] / (1 + expf(-x[i]))) * gate[i]   (ops.c:781-784). */
void oracle_silu_mul(float *x, const float *gate, size_t count);

/* W8A8 conv1d as the reference codec runs it (dacvae.c:543-688), without the
   snake pre-activation: input time-major [T_in, C], weight rows [N, k*C]
   (tap-major, dacvae.h:11-12), output [T_out, N].  Returns T_out or -1. */
int oracle_conv1d_out_len(int T_in, int kernel, int stride, int dilation,
                          int padding);
int oracle_conv1d_int8(const float *input, int T_in, int C,
                       const int8_t *wdata, const float *wscale,
                       const int32_t *wcolsum, int N, int kernel, int stride,
                       int dilation, int padding, const float *bias,
                       int residual, float *output,
                       uint8_t *cols_out, float *scale_out, int32_t *zero_out);

/* The int8 SwiGLU block as dit.c:913-969 wires it through ops.c:
   quantise x -> W1, W3 (separate linears) -> silu(W1x)*W3x ->
   (residual) quantise h -> W2.  Biases are optional (dit.c passes none).
   hidden_out, when not NULL, receives the gated hidden [M, H]. */
int oracle_swiglu(const float *x, int M, int D, int H,
                  const int8_t *w1, const float *s1, const int32_t *c1,
                  const float *b1,
                  const int8_t *w3, const float *s3, const int32_t *c3,
                  const float *b3,
                  const int8_t *w2, const float *s2, const int32_t *c2,
                  const float *b2,
                  int residual_w2, float *out, float *hidden_out);

/* The codec's W8A8 transposed convolution (dacvae.c:696-790, no snake):
   input [T_in, C_in], W [kernel*C_out, C_in] (tap-major rows), output
   [T_out, C_out] = bias + scatter-add of the per-row linear outputs.
   Returns T_out or -1. */
int oracle_convtranspose1d_out_len(int T_in, int kernel, int stride,
                                   int padding, int output_padding);
int oracle_convtranspose1d_int8(const float *input, int T_in, int C_in,
                                int C_out, const int8_t *wdata,
                                const float *wscale, const int32_t *wcolsum,
                                int kernel, int stride, int padding,
                                int output_padding, const float *bias,
                                int residual, float *output);

/* The residual unit's skip + int8 1x1 projection (dacvae.c:979-1009):
   output = skip + linear(quant(hidden)) [+ second residual term]. */
int oracle_codec_conv1(const float *hidden, int rows, int C,
                       const int8_t *wdata, const float *wscale,
                       const int32_t *wcolsum, const float *bias,
                       const float *skip, int residual, float *output);

/* iro_int8_selfcheck's extreme-value probe (ops.c:375-398): fills the fixed
   3x5x64 operands and the expected sums. */
void oracle_selfcheck_case(uint8_t a[3 * 64], int8_t b[5 * 64],
                           int32_t want[3 * 5]);

#ifdef __cplusplus
}
#endif

#endif
