/* ref_codec_shim.c — TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference codec source (dacvae.c, included from the reference
 * tree given on the compiler's include path, never copied) and exports a thin
 * wrapper around its file-static W8A8 convolution, dacvae.c:543-688, so that
 * tests/golden/make_golden.py can record the reference's own conv7 outputs.
 */
#include "dacvae.c"

int ref_conv1d_int8_forward(const float *input, int input_length, int C,
                            const int8_t *wdata, const float *wscale,
                            const int32_t *wcolsum, int N, int kernel,
                            int stride, int dilation, int padding,
                            const float *bias, int residual, float *output) {
    IroConv1d conv;
    memset(&conv, 0, sizeof(conv));
    conv.in_channels = C;
    conv.out_channels = N;
    conv.kernel = kernel;
    conv.stride = stride;
    conv.dilation = dilation;
    conv.padding = padding;
    IroInt8Weight wq;
    wq.data = (int8_t *)wdata;
    wq.scale = (float *)wscale;
    wq.colsum = (int32_t *)wcolsum;
    wq.N = N;
    wq.K = kernel * C;
    return conv1d_int8_forward(&conv, &wq, input, input_length, output, bias,
                               NULL, residual, NULL, NULL, NULL);
}

int ref_conv1d_output_length(int input_length, int kernel, int stride,
                             int dilation, int padding) {
    IroConv1d conv;
    memset(&conv, 0, sizeof(conv));
    conv.kernel = kernel;
    conv.stride = stride;
    conv.dilation = dilation;
    conv.padding = padding;
    return iro_conv1d_output_length(&conv, input_length);
}

/* The reference's W8A8 transposed convolution, dacvae.c:696-790, with the
   int8 weight and no snake.  Whether it adds the second residual term is
   the reference's own process-wide policy (IRO_CODEC_INT8_RESIDUAL bit 2,
   read once, dacvae.c:54-61); callers that want it set the variable before
   the first call of the process. */
int ref_convtranspose1d_int8_forward(const float *input, int input_length,
                                     int C_in, int C_out, const int8_t *wdata,
                                     const float *wscale,
                                     const int32_t *wcolsum, int kernel,
                                     int stride, int padding,
                                     int output_padding, const float *bias,
                                     float *output) {
    IroConvTranspose1d conv;
    memset(&conv, 0, sizeof(conv));
    conv.bias = bias;
    conv.in_channels = C_in;
    conv.out_channels = C_out;
    conv.kernel = kernel;
    conv.stride = stride;
    conv.padding = padding;
    conv.output_padding = output_padding;
    IroInt8Weight wq;
    wq.data = (int8_t *)wdata;
    wq.scale = (float *)wscale;
    wq.colsum = (int32_t *)wcolsum;
    wq.N = kernel * C_out;
    wq.K = C_in;
    return convtranspose1d_forward_impl(&conv, &wq, input, input_length,
                                        output, NULL, NULL, 0);
}

int ref_convtranspose1d_output_length(int input_length, int kernel,
                                      int stride, int padding,
                                      int output_padding) {
    IroConvTranspose1d conv;
    memset(&conv, 0, sizeof(conv));
    conv.kernel = kernel;
    conv.stride = stride;
    conv.padding = padding;
    conv.output_padding = output_padding;
    return iro_convtranspose1d_output_length(&conv, input_length);
}

/* 1 when the reference's policy adds the second term to the upsample
   (transposed) convolution in this process. */
int ref_codec_upsample_residual(void) {
    return (codec_int8_residual_mask() & IRO_CODEC_GROUP_UPSAMPLE) != 0;
}

/* The reference codec's int8 policy switches as it reads them
   (dacvae.c:43-71); cached per process by the reference. */
void ref_codec_policy(int *mask, int *residual, int *stages) {
    *mask = codec_int8_mask();
    *residual = codec_int8_residual_mask();
    *stages = codec_int8_residual_stages();
}
