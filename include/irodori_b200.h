/* irodori_b200.h — C ABI of the B200 (sm_100a) W8A8 int8 linear/GEMM path.
 *
 * Part 1 keeps the reference operator API of irodori-c's ops.h for the int8
 * path, same names, argument meaning and error behaviour, so the C engine's
 * dit.c and dacvae.c link against this library unchanged.  Those calls take
 * HOST pointers (as the reference does); each one stages its operands into
 * device memory, runs the CUDA kernels on the library's stream of the
 * current CUDA device and copies the results back before returning.
 *
 * Part 2 is the stream-ordered DEVICE-pointer family that the fast path
 * uses: quantisers, the tcgen05 GEMM with fused epilogues, the fused QKVG
 * split, the fused SwiGLU block and the kernel-7 codec convolution as an
 * implicit GEMM.  Weights live on the device as IroInt8DevWeight.
 *
 * There is no CPU implementation behind any entry point.  Without a usable
 * sm_100 device every call fails: int-returning calls return a negative
 * IRO_ERR_* code, void calls leave their outputs untouched and record the
 * code for iro_cuda_last_error().
 *
 * Plain C types only; `stream` arguments are cudaStream_t passed as void*
 * (NULL = the library's own stream for the current device).
 */
#ifndef IRODORI_B200_H
#define IRODORI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
    IRO_OK = 0,
    IRO_ERR_INVALID = -1,        /* bad argument / shape (reference's -1)   */
    IRO_ERR_NO_DEVICE = -2,      /* no sm_100 CUDA device                   */
    IRO_ERR_CUDA = -3,           /* a CUDA runtime call failed              */
    IRO_ERR_OOM = -4,            /* device or host allocation failed        */
    IRO_ERR_DEVICE_TIMEOUT = -5, /* a bounded in-kernel wait gave up        */
    IRO_ERR_UNSUPPORTED = -6,    /* shape outside what a kernel supports    */
    IRO_ERR_SELFCHECK = -7,      /* the exact-sum probe failed              */
    IRO_ERR_RANGE = -8           /* a DiT attention operand (q, k, v, context
                                    k/v) beyond the fp16 range (|x| >= 65520)
                                    of the tensor-core attention; the fp32
                                    attention (IRO_DIT_ATTENTION=simt) takes
                                    any finite value                         */
};

/* ======================================================================= */
/* Part 1 — the reference operator API (ops.h), host pointers.             */
/* ======================================================================= */

/* Quantised weight, identical layout to the reference (ops.h:23-28):
   data int8 [N,K] row-major, scale f32 [N], colsum i32 [N] = sum_k data.
   The three buffers are host malloc()s owned by the struct.  The library
   also keeps a device copy per (device, data pointer), made on first use
   and dropped by iro_int8_weight_free (the packed-weight cache). */
typedef struct {
    int8_t *data;
    float *scale;
    int32_t *colsum;
    int N, K;
} IroInt8Weight;

/* ops.h:30 / ops.c:259-293.  Per output channel symmetric s8,
   scale = amax/127.  Computed on the GPU; returns 0, or -1 on NULL, N/K <= 0,
   allocation or device failure (partial state freed). */
int iro_int8_weight_quantize(IroInt8Weight *dst, const float *w, int N, int K);

/* ops.h:33-35 / ops.c:295-306.  Source stored [K,N] row-major. */
int iro_int8_weight_quantize_transposed(IroInt8Weight *dst, const float *w,
                                        int N, int K);

/* ops.h:36 / ops.c:308-314.  Frees, zeroes, drops the device copies. */
void iro_int8_weight_free(IroInt8Weight *w);

/* ops.h:37 / ops.c:316-319. */
size_t iro_int8_weight_bytes(const IroInt8Weight *w);

/* ops.h:39-40 / ops.c:321-348.  Per-row asymmetric u8 with zero point. */
void iro_int8_quantize_rows(const float *x, int M, int K,
                            uint8_t *q, float *scale, int32_t *zero);

/* ops.h:45-47 / ops.c:444-448. */
void iro_int8_linear(const uint8_t *q, const float *scale,
                     const int32_t *zero, const IroInt8Weight *w,
                     const float *bias, float *y, int M, int32_t *work);

/* ops.h:48-51 / ops.c:450-491.  work (M*N int32) receives the raw integer
   sums, as in the reference (its selfcheck reads them back). */
void iro_int8_linear_ex(const uint8_t *q, const float *scale,
                        const int32_t *zero, const IroInt8Weight *w,
                        const float *bias, float *y, int M, int32_t *work,
                        int accumulate);

/* ops.h:57-60 / ops.c:427-442.  residual receives the first-term remainder. */
void iro_int8_quantize_rows_residual(const float *x, int M, int K,
                                     uint8_t *q1, float *scale1, int32_t *zero1,
                                     float *residual,
                                     uint8_t *q2, float *scale2, int32_t *zero2);

/* ops.h:64 / ops.c:367-373.  1 when an sm_100 device is usable. */
int iro_int8_fast_available(void);

/* ops.h:72 / ops.c:400-425.  Initialises the current device's context and
   returns the backend name, or NULL when no device is usable. */
const char *iro_int8_prepare_backend(void);

/* ops.h:78 / ops.c:375-398.  Runs the reference's extreme-value exact-sum
   probe through the tensor-core GEMM; 0 when exact, -1 otherwise. */
int iro_int8_selfcheck(void);

/* ops.h:143 / ops.c:706-716. */
const char *iro_ops_backend_name(void);

/* ======================================================================= */
/* Part 2 — B200 runtime and the device-pointer family.                    */
/* ======================================================================= */

/* Runtime ------------------------------------------------------------------ */

/* Select `device` for this host thread and create its context (stream,
   device error word).  Returns 0 or IRO_ERR_*.  Implicit in every call. */
int iro_cuda_init(int device);
/* Last error recorded on this host thread by a void call (0 = none); reading
   clears it. */
int iro_cuda_last_error(void);
const char *iro_cuda_error_string(int code);
/* Number of sm_100 devices visible (0 when none). */
int iro_cuda_device_count(void);
/* The library stream of the current device (cudaStream_t as void*). */
void *iro_cuda_stream(void);
/* Block until the library stream (or `stream`) is idle; returns status,
   including a pending in-kernel timeout report.  Every entry point's kernels
   report into one error word per device (static device memory); this call
   reads and clears it.  With a non-NULL `stream` it creates no context and
   allocates nothing. */
int iro_cuda_synchronize(void *stream);

/* Device memory helpers for callers without their own allocator. */
void *iro_dev_malloc(size_t bytes);
void iro_dev_free(void *p);
int iro_memcpy_htod(void *dst, const void *src, size_t bytes, void *stream);
int iro_memcpy_dtoh(void *dst, const void *src, size_t bytes, void *stream);
int iro_memcpy_dtod(void *dst, const void *src, size_t bytes, void *stream);
int iro_memset_dev(void *dst, int value, size_t bytes, void *stream);
void *iro_host_alloc_pinned(size_t bytes);
void iro_host_free_pinned(void *p);

/* Device weights -------------------------------------------------------------
   data int8 [N, ld] row-major on the device, ld = K rounded up to 16 bytes
   (zero padded), plus scale/colsum [N] and an optional per-channel bias.
   layout PLAIN is the reference [N,K] order.  layout GATED_PAIR is the
   fused W1|W3 order: for each block of `pair` hidden channels, `pair` W1 rows
   then the matching `pair` W3 rows, so one GEMM tile holds both halves of
   silu(W1 x) * (W3 x) (N = 2 * round_up(H, pair); hidden = H). */
enum { IRO_LAYOUT_PLAIN = 0, IRO_LAYOUT_GATED_PAIR = 1 };

typedef struct {
    int8_t *data;
    float *scale;
    int32_t *colsum;
    float *bias;
    int N, K, ld;
    int layout;
    int pair;    /* GATED_PAIR: channels per half block */
    int hidden;  /* GATED_PAIR: H */
    int device;
    void *priv;  /* library-owned (cached TMA descriptor) */
} IroInt8DevWeight;

/* Upload a host-quantised weight (PLAIN).  bias may be NULL. */
int iro_int8_dev_weight_upload(IroInt8DevWeight *dst, const IroInt8Weight *src,
                               const float *bias);
/* Quantise fp32 device weights [N,K] on the device (same numerics as
   iro_int8_weight_quantize).  bias_dev may be NULL. */
int iro_int8_dev_weight_quantize(IroInt8DevWeight *dst, const float *w_dev,
                                 int N, int K, const float *bias_dev, void *stream);
/* Concatenate host weights along N (fused QKVG: Q|K|V|gate, dit.c:785-792).
   All parts share K; biases (host, per part) may be NULL. */
int iro_int8_dev_weight_concat(IroInt8DevWeight *dst, const IroInt8Weight *const *parts,
                               const float *const *biases, int nparts);
/* Build the GATED_PAIR layout from host W1 and W3 (dit.c:943-947). */
int iro_int8_dev_weight_gated_pair(IroInt8DevWeight *dst, const IroInt8Weight *w1,
                                   const IroInt8Weight *w3, const float *b1,
                                   const float *b3);
void iro_int8_dev_weight_free(IroInt8DevWeight *w);

/* Device bytes of a weight's payload: codes (N x ld), scale, colsum and
   bias.  0 for an empty weight. */
size_t iro_int8_dev_weight_bytes(const IroInt8DevWeight *w);

/* Int8 model containers ----------------------------------------------------
   Device mirrors of the reference's engine-owned int8 copies.  The host-side
   structs below have the member order and types of dit.h:53-55
   (IroDiTInt8Layer) and dacvae.h:52-67 (IroDACVAEInt8*), so an engine can
   pass its own quantised copies (e.g. `(const IroDiTInt8HostLayer *)
   dit_int8.layer`) after iro_dit_int8_quantize / iro_dacvae_int8_quantize.
   `bytes` counts the resident device payload (codes with their 16-byte row
   pitch, scales, colsums, biases, and the W1|W3 pair layout's padding rows),
   as the reference's `bytes` does for its host copies
   (dit.c:253-256, dacvae.c:236-258; reported by generate.h:45-47). */
typedef struct {
    IroInt8Weight wq, wk, wv, gate, wo, w1, w2, w3;
} IroDiTInt8HostLayer;

typedef struct {
    IroInt8DevWeight qkvg;  /* wq|wk|wv|gate concatenated along N */
    IroInt8DevWeight wo;
    IroInt8DevWeight w13;   /* w1, w3 in the GATED_PAIR layout */
    IroInt8DevWeight w2;
} IroDiTInt8DevLayer;

typedef struct {
    IroDiTInt8DevLayer layer[16];
    int layers;
    size_t bytes;
} IroDiTInt8Dev;

/* Upload `n_layers` (1..16) layers.  Returns IRO_OK or IRO_ERR_*; on error
   nothing stays allocated. */
int iro_dit_int8_dev_upload(IroDiTInt8Dev *dst, const IroDiTInt8HostLayer *layers,
                            int n_layers);
void iro_dit_int8_dev_free(IroDiTInt8Dev *q);

#define IRO_B200_DACVAE_STAGES 4     /* dacvae.h:8 */
#define IRO_B200_DACVAE_RESIDUALS 3  /* dacvae.h:9 */

typedef struct {
    IroInt8Weight conv0; /* [C, 7*C] */
    IroInt8Weight conv1; /* [C, C] */
} IroDACVAEInt8HostResidual;

typedef struct {
    IroInt8Weight upsample; /* [kernel*out, in] */
    IroDACVAEInt8HostResidual residual[IRO_B200_DACVAE_RESIDUALS];
} IroDACVAEInt8HostStage;

typedef struct {
    IroInt8Weight initial; /* [1536, 7*1024] */
    IroDACVAEInt8HostStage stage[IRO_B200_DACVAE_STAGES];
    size_t bytes;
} IroDACVAEInt8Host;

typedef struct {
    IroInt8DevWeight conv0, conv1;
} IroDACVAEInt8DevResidual;

typedef struct {
    IroInt8DevWeight upsample;
    IroDACVAEInt8DevResidual residual[IRO_B200_DACVAE_RESIDUALS];
} IroDACVAEInt8DevStage;

typedef struct {
    IroInt8DevWeight initial;
    IroDACVAEInt8DevStage stage[IRO_B200_DACVAE_STAGES];
    size_t bytes;
} IroDACVAEInt8Dev;

/* Upload every weight of a host IroDACVAEInt8 copy (the conv weights as
   [N, kernel*in], the transposed convolutions as [kernel*out, in], as
   iro_int8_conv1d_dev, iro_int8_convtranspose1d_dev and
   iro_int8_codec_conv1_dev take them).  Returns IRO_OK or IRO_ERR_*; on
   error nothing stays allocated. */
int iro_dacvae_int8_dev_upload(IroDACVAEInt8Dev *dst, const IroDACVAEInt8Host *src);
void iro_dacvae_int8_dev_free(IroDACVAEInt8Dev *q);

/* Quantisers (device pointers, stream ordered) ------------------------------ */

/* ops.c:321-348 on the device: q u8 [M,K], scale [M], zero [M]. */
int iro_int8_quantize_rows_dev(const float *x, int M, int K, uint8_t *q,
                               float *scale, int32_t *zero, void *stream);
/* Symmetric absmax/127 (tests/bench_vnni_linear.c:82-101), stored u8 = s8+128
   with zero[m] = 128, so it feeds the same linear. */
int iro_int8_quantize_rows_sym_dev(const float *x, int M, int K, uint8_t *q,
                                   float *scale, int32_t *zero, void *stream);
/* ops.c:427-442; residual may be NULL (not stored). */
int iro_int8_quantize_rows_residual_dev(const float *x, int M, int K,
                                        uint8_t *q1, float *scale1, int32_t *zero1,
                                        float *residual,
                                        uint8_t *q2, float *scale2, int32_t *zero2,
                                        void *stream);

/* GEMM + fused epilogues ------------------------------------------------------ */

/* ops.c:450-491 on the device: y[M,N] (=|+=) (acc - zero*colsum)*(scale*wscale)
   (+ bias).  work (M*N int32) is optional (NULL = not stored).  q rows are
   K bytes apart; K % 16 != 0 is supported through an internal repack. */
int iro_int8_linear_dev(const uint8_t *q, const float *scale, const int32_t *zero,
                        const IroInt8DevWeight *w, const float *bias, float *y,
                        int M, int32_t *work, int accumulate, void *stream);

/* Two-term residual linear in one pass (dit.c:479-486): y = linear(q1) [+bias]
   then += linear(q2), with both accumulators in TMEM. */
int iro_int8_linear2_dev(const uint8_t *q1, const float *scale1, const int32_t *zero1,
                         const uint8_t *q2, const float *scale2, const int32_t *zero2,
                         const IroInt8DevWeight *w, const float *bias, float *y,
                         int M, void *stream);

/* Fused QKVG (dit.c:785-792): one GEMM over the concatenated weight, output
   column block g of width `seg` written to outputs[g] ([M, seg] each). */
int iro_int8_linear_split_dev(const uint8_t *q, const float *scale,
                              const int32_t *zero, const IroInt8DevWeight *w,
                              float *const *outputs, int nout, int seg, int M,
                              void *stream);

/* Fused W1|W3 GEMM with the silu gate in the epilogue (dit.c:943-956):
   hidden[M,H] = silu(W1 x + b1) * (W3 x + b3), w13 in GATED_PAIR layout. */
int iro_int8_gated_dev(const uint8_t *q, const float *scale, const int32_t *zero,
                       const IroInt8DevWeight *w13, float *hidden, int M,
                       void *stream);

/* Whole int8 SwiGLU block (dit.c:913-969): quantise x [M,D], fused W1|W3 +
   gate, quantise the hidden (two-term when residual_w2), W2 (+ b2) into
   out [M,D].  workspace of iro_int8_swiglu_workspace_bytes() bytes, or NULL
   for the library's own device arena. */
size_t iro_int8_swiglu_workspace_bytes(int M, int D, int H, int residual_w2);
int iro_int8_swiglu_dev(const float *x, int M, const IroInt8DevWeight *w13,
                        const IroInt8DevWeight *w2, const float *b2, float *out,
                        int residual_w2, void *workspace, void *stream);
/* Host-pointer form of the block: x and out on the host (e2e path). */
int iro_int8_swiglu(const float *x, int M, const IroInt8DevWeight *w13,
                    const IroInt8DevWeight *w2, const float *b2, float *out,
                    int residual_w2);

/* Recorded plans.  A plan records one block's kernel launches, with fixed
   device pointers, as a CUDA graph; iro_plan_launch replays it on `stream`
   with one call.  The plan owns its workspace.  Inputs are read and outputs
   written at launch time, so the caller refills x between launches. */
typedef struct IroPlan IroPlan;
int iro_int8_swiglu_plan(IroPlan **plan, const float *x, int M, const IroInt8DevWeight *w13,
                         const IroInt8DevWeight *w2, const float *b2, float *out,
                         int residual_w2);
int iro_plan_launch(const IroPlan *plan, void *stream);
void iro_plan_free(IroPlan *plan);

/* Host-buffer serving pipeline for the SwiGLU block.  A ring of `depth`
   device slots (input, output, recorded block each); submit() copies x_host
   in, runs the block and copies the result to out_host, all asynchronously,
   so consecutive submissions overlap their host->device copy, compute and
   device->host copy on three streams.  The host buffers must stay valid and
   untouched until wait() returns; they should be page-locked for the copies
   to overlap.  Same numerics as iro_int8_swiglu_dev. */
typedef struct IroSwigluPipe IroSwigluPipe;
int iro_int8_swiglu_pipe_create(IroSwigluPipe **pipe, int M, const IroInt8DevWeight *w13,
                                const IroInt8DevWeight *w2, const float *b2, int residual_w2,
                                int depth);
int iro_int8_swiglu_pipe_submit(IroSwigluPipe *pipe, const float *x_host, float *out_host);
int iro_int8_swiglu_pipe_wait(IroSwigluPipe *pipe);
void iro_int8_swiglu_pipe_free(IroSwigluPipe *pipe);

/* Per-shape GEMM profile (ops.c:14-110, ops.h:126-129, the reference's
   IRO_GEMM_PROFILE): with IRO_GEMM_PROFILE set and not "0", every int8 GEMM
   launch is timed on the device (CUDA events around the kernel) and counted
   per (kind, M, N, K, lda, ldb, ldc, beta), at most 256 shapes.  emit_json
   writes one JSON line in the reference's schema to stderr (backend
   "cuda-sm100a-tcgen05-i8"); iro_dit_sample_euler_dev resets the profile at
   its start and emits it at its end, as sampler.c:142-144, 312-321 do.
   Profiling serialises the launches it brackets. */
int iro_cuda_gemm_profile_enabled(void);
void iro_cuda_gemm_profile_reset(void);
void iro_cuda_gemm_profile_emit_json(const char *status, int steps, int sequence_length,
                                     int context_tokens);

/* The SwiGLU block without allocation.  No counterpart in the reference.
   For callers that cannot allocate device memory where they run the block:
   engines that reserve all device memory at start-up and treat a later
   allocation as a failure, hosts whose device memory belongs to another
   allocator, and latency-critical loops (growing the library arena calls
   cudaFree, which waits for the whole device).  Same arguments and results
   as iro_int8_swiglu_dev without the workspace (bit-identical outputs): the
   scratch is a 64 MiB array inside the library, reserved on every GPU where
   the library's device code is loaded until the process exits.  Calls whose
   scratch (iro_int8_swiglu_workspace_bytes) exceeds 64 MiB are rejected with
   IRO_ERR_UNSUPPORTED and a message on stderr; split the rows (about 4,400
   rows at D 1024 / H 2816, single-term W2).  It calls no cudaMalloc or
   cudaFree and does not touch the library context.  The first call on a
   device resolves the scratch address, so make it before any stream capture.
   Calls share the scratch, which keeps the last call's contents (every byte a
   call reads it writes first): calls that can overlap on the GPU race.  The
   return value covers the launches; a bounded device wait that gave up is
   reported by the next iro_cuda_synchronize(stream) with the same stream.
   `stream` NULL is the legacy default stream. */
int iro_int8_swiglu_noalloc_dev(const float *x, int M, const IroInt8DevWeight *w13,
                                const IroInt8DevWeight *w2, const float *b2, float *out,
                                int residual_w2, void *stream);

/* Codec convolution ------------------------------------------------------------ */

/* dacvae.c:543-688 (no snake): W8A8 conv1d over `batch` independent
   time-major inputs [T_in, C] (contiguous, [batch, T_in, C]) with
   per-output-row quantisation over the union of the kernel taps' rows
   (padding taps = zero point), weight [N, kernel*C] tap-major (dacvae.h:11-12),
   output [batch, T_out, N] (+ bias); residual adds the s/255, zero-point-128
   second term.  Returns T_out (> 0) or IRO_ERR_*. */
int iro_conv1d_out_len(int T_in, int kernel, int stride, int dilation, int padding);
int iro_int8_conv1d_dev(const float *input, int batch, int T_in, int C,
                        const IroInt8DevWeight *w, int kernel, int stride,
                        int dilation, int padding, const float *bias,
                        int residual, float *output, void *stream);

/* dacvae.c:696-790 (int8 weight, no snake): W8A8 transposed (upsampling)
   convolution over `batch` independent time-major inputs [batch, T_in, C_in].
   W is [kernel*C_out, C_in] with row tap*C_out + c (dacvae.h:47-52); output
   [batch, T_out, C_out] = bias (or 0) plus, for every input row r and tap t,
   linear(quant(x_r))[t*C_out .. +C_out] added onto output row
   r*stride - padding + t, each output element's additions in increasing r
   (the reference's order).  residual adds the two-term quantisation's second
   linear (dacvae.c:748-767).  The decoder uses kernel = 2*stride, padding =
   (stride+1)/2, output_padding = stride&1 (dacvae.c:150-160).  C_in must be a
   multiple of 16.  Returns T_out (> 0) or IRO_ERR_*.  The length follows
   iro_convtranspose1d_output_length (dacvae.c:350-358). */
int iro_convtranspose1d_out_len(int T_in, int kernel, int stride, int padding,
                                int output_padding);
int iro_int8_convtranspose1d_dev(const float *input, int batch, int T_in, int C_in,
                                 const IroInt8DevWeight *w, int C_out, int kernel,
                                 int stride, int padding, int output_padding,
                                 const float *bias, int residual, float *output,
                                 void *stream);

/* dacvae.c:979-1009: the residual unit's skip connection plus int8 1x1
   projection, output[rows, C] = skip + (linear(quant(hidden)) + bias)
   [+ linear of the residual term, without bias], each addition rounded in
   the reference's order.  W is [C, C] (w->N == w->K == C, a multiple of 16).
   skip may equal output (in place).  Returns IRO_OK or IRO_ERR_*. */
int iro_int8_codec_conv1_dev(const float *hidden, int rows, const IroInt8DevWeight *w,
                             const float *bias, const float *skip, int residual,
                             float *output, void *stream);

/* DiT block ---------------------------------------------------------------------- */

/* One RF-DiT transformer block (dit.c:983-1051) on the device: AdaLN,
   int8 QKVG, per-head RMSNorm + half RoPE, joint attention over the S latent
   tokens and the valid context tokens with the sigmoid gate, int8 Wo, gated
   residual; AdaLN, int8 SwiGLU, gated residual.  The fp32 tensors are device
   pointers in the reference layouts (dit.h:13-40): adaln[0] is the attention
   AdaLN, adaln[1] the MLP one, each {shift_down [R,D], shift_up [D,R],
   shift_bias [D], scale_down, scale_up, scale_bias, gate_down, gate_up,
   gate_bias}; q_norm, k_norm [D].  qkvg is wq|wk|wv|gate concatenated
   (iro_int8_dev_weight_concat), w13 the gated pair of w1, w3.
   residual_mask follows IRO_INT8_RESIDUAL (dit.c:429-436): the groups whose
   activations are quantised with a second residual term, 1 = Q/K/V/gate,
   2 = Wo, 4 = W1/W3, 8 = W2 (the reference default), any combination; other
   bits are IRO_ERR_INVALID.
   fp32_groups and emulate are the reference's error-attribution switches
   (dit.c:273-335, the environment variables IRO_INT8_MASK and
   IRO_INT8_EMULATE), per block; zero (the default) runs every group in int8.
   fp32_groups: the groups (same bits as residual_mask) left out of the int8
   path, i.e. 15 & ~IRO_INT8_MASK: fp32 activations x the fp32 weights.
   emulate: for the int8 groups, 1 = fp32 activations x the dequantised int8
   weights (weight-only error), any other non-zero value = the quantiser's
   codes turned back into fp32 x the fp32 weights (activation-only error).
   w_fp32: the fp32 weights [N, K] on the device, in the order wq, wk, wv,
   gate, wo, w1, w3, w2; needed for the fp32 groups and for emulate != 0, 1.
   A group whose int8 weight is not used may leave it zeroed.  These modes
   are diagnostics: a plain fp32 GEMM, correct rather than fast, with more
   workspace (iro_dit_block_workspace_bytes counts it).  A two-term W1/W3
   (residual_mask bit 4) feeding a non-int8 W2 is IRO_ERR_UNSUPPORTED. */
typedef struct {
    const float *adaln[2][9];
    const float *q_norm;
    const float *k_norm;
    IroInt8DevWeight qkvg, wo, w13, w2;
    int model_dim, heads, head_dim, adaln_rank, mlp_dim;
    float norm_eps;
    int residual_mask;
    int fp32_groups;
    int emulate;
    const float *w_fp32[8];
} IroDiTBlockDev;

/* The reference's int8 policy switches, read from the same environment
   variables with the same parsing (strtol base 0, masked to 4 bits) and
   defaults, for engines that configure the device path as the reference's
   own code would (read on every call, not cached):
     IRO_INT8_RESIDUAL               dit.c:429-436, default 8 (W2)
     IRO_CODEC_INT8_MASK             dacvae.c:43-50, default 15
     IRO_CODEC_INT8_RESIDUAL         dacvae.c:52-60, default 4|8 (Conv7 + Conv1)
     IRO_CODEC_INT8_RESIDUAL_STAGES  dacvae.c:63-71, default 8 (last stage)
   iro_policy_codec_residual(stage, group) is the reference's per-layer
   decision: the group's residual bit and, for the residual-unit convolutions
   (groups 4 and 8), the stage's bit. */
int iro_policy_dit_residual_mask(void);
int iro_policy_codec_int8_mask(void);
int iro_policy_codec_residual_mask(void);
int iro_policy_codec_residual_stages(void);
int iro_policy_codec_residual(int stage, int group);
/* The reference's diagnostic switches for the DiT block's fp32_groups and
   emulate: 15 & ~IRO_INT8_MASK (dit.c:284-291, default mask 15, so 0) and
   IRO_INT8_EMULATE (dit.c:297-304, default 0), parsed the same way. */
int iro_policy_dit_fp32_groups(void);
int iro_policy_dit_emulate(void);

/* Activation diagnostics (dit.c:340-412), recorded by the sampler entry
   points (iro_dit_euler_step_dev, iro_dit_sample_euler_dev: layer index known)
   at the reference's four points, group 0 Q/K/V/gate input, 1 Wo input, 2
   W1/W3 input, 3 W2 input, when IRO_INT8_STATS is set (not "0"):
   per (layer, group) the row count, the sum over rows of max|x| / rms(x) and
   the histogram of each row's first max-|x| channel (8192 channels).
   IRO_INT8_DUMP=dir writes the first three activations per (layer, group) to
   dir/act_L%02d_G%d_%d_M%d_K%d.f32 as the reference does.  Recording takes the
   unfused AdaLN path (h is materialised) and costs a pass per record.
   iro_dit_stats_report prints the reference's summary line per cell to
   stderr (also at process exit once recording has started). */
int iro_dit_stats_read(int layer, int group, double *rows, double *ratio_sum,
                       unsigned int *hist, int hist_len);
void iro_dit_stats_reset(void);
void iro_dit_stats_report(void);

/* dit.c:644-705: RoPE cos/sin tables [S, head_dim/2] as the reference builds
   them (double-precision rotation recurrence, rounded to float); host
   buffers. */
int iro_dit_rope_table(float *cos_out, float *sin_out, int S, int head_dim);
size_t iro_dit_block_workspace_bytes(const IroDiTBlockDev *blk, int B, int S, int C,
                                     int context_batch);
/* x [B*S, D] is updated in place.  cond [cond_rows, 3*D]: cond_rows = B
   (one conditioning row per batch row) or 1 (one row for the whole batch, as
   in a sampler step where every row shares the timestep, sampler.c:246-253).
   ctx_k/ctx_v [context_batch, C, D], context block b / (B / context_batch)
   serving batch row b (1 = shared by the batch, dit.c:903-911; a request's
   CFG rows share its block, sampler.c:219-224); mask [B, C] per batch row
   (dit.c:811-813); rope_cos/sin device [S, 32].  workspace NULL uses the
   library's scratch.  Returns IRO_OK or IRO_ERR_*. */
int iro_dit_block_dev(const IroDiTBlockDev *blk, float *x, const float *cond, int cond_rows,
                      const float *ctx_k, const float *ctx_v, const uint8_t *ctx_mask,
                      int context_batch, int B, int S, int C, const float *rope_cos,
                      const float *rope_sin, void *workspace, void *stream);

/* The blocks and the surrounding fp32 layers of the whole DiT (dit.c:137-
   233): cond_w0 [D, timestep_dim], cond_w1 [D, D], cond_w2 [3D, D], in_w
   [D, latent_dim], in_b [D], out_norm [D], out_w [latent_dim, D], out_b
   [latent_dim]; device pointers. */
#define IRO_DIT_MAX_LAYERS 16
typedef struct {
    IroDiTBlockDev block[IRO_DIT_MAX_LAYERS];
    int layers;
    const float *cond_w0, *cond_w1, *cond_w2;
    const float *in_w, *in_b;
    const float *out_norm, *out_w, *out_b;
    int timestep_dim, latent_dim;
    float norm_eps;
} IroDiTModelDev;

size_t iro_dit_step_workspace_bytes(const IroDiTModelDev *m, int R, int cfg, int S, int C);
/* One Euler step of R requests (sampler.c:238-297): state [R, S, latent_dim]
   on the device is advanced from t to t_next.  Each request runs cfg rows
   (1 = conditional only; row i+1 is the i-th unconditional branch, guided
   with cfg_scales[i], host floats, in the reference's order text, speaker,
   caption of the active branches).  ctx_k[l], ctx_v[l]: host arrays of
   device pointers, layer l's context K/V [R, C, D]; mask [R*cfg, C].
   Returns IRO_OK or IRO_ERR_*. */
int iro_dit_euler_step_dev(const IroDiTModelDev *m, float *state, int R, int cfg, int S,
                           float t, float t_next, const float *cfg_scales,
                           const float *const *ctx_k, const float *const *ctx_v,
                           const uint8_t *mask, int C, void *workspace, void *stream);

/* The reference's public DiT pieces on device buffers (dit.c:502-541,
   1070-1090), stream-ordered; workspace NULL uses the library arena.
   iro_dit_condition_dev: t [B] host floats -> cond [B, 3*model_dim]
   (replaces iro_dit_condition, dit.c:502); workspace is
   iro_dit_stage_workspace_bytes(m, B).  iro_dit_input_dev: x [B*S, latent]
   -> projected [B*S, model_dim] (replaces iro_dit_input, dit.c:532).
   iro_dit_output_dev: RMSNorm + linear -> velocity [B*S, latent] (replaces
   iro_dit_output, dit.c:1070); workspace >= 4*B*S*model_dim bytes.  The fp32
   linears sum each output in the reference's scalar order without fused
   multiply-adds. */
/* The two halves of iro_dit_euler_step_dev, for a step split across GPUs by
   CFG branch (fewer requests than GPUs): iro_dit_velocity_dev runs the model
   (conditioner, input projection, blocks, output head) and writes the raw
   velocity of every row, [R*cfg, S, latent], without touching the state;
   iro_dit_cfg_update_dev then applies sampler.c:283-297's guided Euler update
   to the state from the velocities of all cfg branches per request (rows r*cfg
   .. r*cfg+cfg-1), in the same arithmetic as iro_dit_euler_step_dev.  One GPU
   can run one branch (cfg 1, that branch's mask row), the branches' velocities
   meet by an all-gather, and every GPU then applies the same update.
   Workspace: iro_dit_step_workspace_bytes.  Returns IRO_OK or IRO_ERR_*. */
int iro_dit_velocity_dev(const IroDiTModelDev *m, const float *state, int R, int cfg, int S,
                         float t, const float *const *ctx_k, const float *const *ctx_v,
                         const uint8_t *mask, int C, float *velocity, void *workspace,
                         void *stream);
int iro_dit_cfg_update_dev(const IroDiTModelDev *m, float *state, const float *velocity, int R,
                           int cfg, int S, float t, float t_next, const float *cfg_scales,
                           void *stream);
size_t iro_dit_stage_workspace_bytes(const IroDiTModelDev *m, int rows);
int iro_dit_condition_dev(const IroDiTModelDev *m, const float *t, int B, float *cond,
                          void *workspace, void *stream);
int iro_dit_input_dev(const IroDiTModelDev *m, const float *x, int B, int S, float *projected,
                      void *stream);
int iro_dit_output_dev(const IroDiTModelDev *m, const float *x, int B, int S, float *velocity,
                       void *workspace, void *stream);

/* The Euler sampling loop (sampler.c:241-297) over `steps` steps from
   init_scale down to 0: step i runs at t = (1 - i/steps) * init_scale, with
   all cfg rows while cfg_min_t <= t <= cfg_max_t and the conditional row
   alone outside that window.  Arguments as iro_dit_euler_step_dev; the
   workspace is iro_dit_sample_workspace_bytes(m, R, cfg, S, C, steps).  The
   RoPE tables, and every step's conditioning and AdaLN parameters, are
   computed once per call. */
size_t iro_dit_sample_workspace_bytes(const IroDiTModelDev *m, int R, int cfg, int S, int C,
                                      int steps);
int iro_dit_sample_euler_dev(const IroDiTModelDev *m, float *state, int R, int cfg, int S,
                             int steps, float init_scale, float cfg_min_t, float cfg_max_t,
                             const float *cfg_scales, const float *const *ctx_k,
                             const float *const *ctx_v, const uint8_t *mask, int C,
                             void *workspace, void *stream);

/* Checkpoints: safetensors files mapped read-only --------------------------------- */

/* The reference's loader (safetensors.c, iro_st_load/iro_st_get) mmaps a
   checkpoint and its int8 engine quantises fp32 projections on the host at
   init (dit.c:235-259 -> ops.c:259-293).  These entry points open the same
   files (named iro_st_file_* so they can be linked beside the reference's
   iro_st_* functions) and quantise on the device. */
typedef struct IroStFile IroStFile;
/* Map a .safetensors file read-only and parse its header; every tensor's
   bytes must lie inside the file.  Returns IRO_OK or IRO_ERR_INVALID. */
int iro_st_file_open(IroStFile **file, const char *path);
void iro_st_file_close(IroStFile *file);
int iro_st_file_count(const IroStFile *file);
const char *iro_st_file_name(const IroStFile *file, int index);
/* Geometry of a tensor by name; dtype follows irodori.h's IroDType order
   (0 F32, 1 F16, 2 BF16, 3 I64, 4 I32, 5 I16, 6 I8, 7 U8, 8 BOOL, 9 other);
   shape receives ndims values (at most 8). */
int iro_st_file_tensor(const IroStFile *file, const char *name, int *dtype, int *ndims,
                       uint64_t *shape, uint64_t *nbytes);
/* Pointer into the mapping (valid until iro_st_file_close). */
const void *iro_st_file_data(const IroStFile *file, const char *name);
/* safetensors.c:525-552: release the clean pages of every tensor whose name
   starts with prefix (page-aligned span, clipped to the mapping); pointers
   stay valid and pages fault back in if read.  Returns the bytes released. */
uint64_t iro_st_file_drop_prefix(const IroStFile *file, const char *prefix);
/* ops.c:259-306 on the device: quantise the F32 tensor `name`, [N, K]
   row-major, or [K, N] with transposed = 1, into dst (codes, scales and
   column sums equal iro_int8_weight_quantize's); bias_name (F32 [N]) may be
   NULL.  Synchronous.  Returns IRO_OK or IRO_ERR_*. */
int iro_int8_dev_weight_from_st(IroInt8DevWeight *dst, const IroStFile *file, const char *name,
                                int transposed, const char *bias_name);

/* Failure detection ------------------------------------------------------------- */

/* Launches one block that waits on a device barrier nothing ever completes,
   with an in-kernel limit of `limit_ns`; returns the status the host then
   reads (IRO_ERR_DEVICE_TIMEOUT when the bounded wait gave up as designed). */
int iro_debug_bounded_wait_probe(uint64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* IRODORI_B200_H */
