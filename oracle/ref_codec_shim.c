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
