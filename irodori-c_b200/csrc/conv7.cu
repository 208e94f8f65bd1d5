// conv7.cu — placeholder while the implicit-GEMM convolution is written.
#include "runtime.cuh"

extern "C" int iro_conv1d_out_len(int T_in, int kernel, int stride, int dilation, int padding) {
  if (T_in <= 0 || stride <= 0 || kernel <= 0 || dilation <= 0) return IRO_ERR_INVALID;
  long long span = (long long)dilation * (kernel - 1) + 1;
  long long num = (long long)T_in + 2LL * padding - span;
  long long out = num < 0 ? -1 : num / stride + 1;
  return out <= 0 || out > 0x7fffffff ? IRO_ERR_INVALID : (int)out;
}

extern "C" int iro_int8_conv1d_dev(const float*, int, int, const IroInt8DevWeight*, int, int, int,
                                   int, const float*, int, float*, void*) {
  return IRO_ERR_UNSUPPORTED;
}
