// conv7.cu — the codec's W8A8 convolution (dacvae.c:543-688) on the GPU.
//
// Semantics (the reference's, not a generic int8 conv): every OUTPUT row t
// quantises its own im2col row.  Its range is the min/max, with 0 included,
// over the input rows its taps read, it = t*stride - padding + tap*dilation
// (dacvae.c:607-627).  Padding taps hold the zero point (dacvae.c:651-655).
// The same input row therefore gets different codes in different output
// rows.  The optional second term codes the remainder with scale s/255 and
// zero point 128 (dacvae.c:637-663) and is accumulated without bias
// (dacvae.c:679-681).
//
// Kernels: conv_row_range (per input row min/max, one warp per row) ->
// conv_pack (per output row: window range, row parameters, tap-major u8
// codes [t, tap*C + c]) -> the tcgen05 GEMM against the [N, kernel*C] weight
// (EPI_LINEAR, or EPI_DUAL for the two-term form).  Rows are processed in
// chunks so the code buffer stays bounded.
#include "conv_igemm.cuh"
#include "gemm_i8.cuh"
#include "quantize.cuh"

namespace iro {

__global__ void __launch_bounds__(256) conv_row_range_kernel(const float* __restrict__ in,
                                                             int rows, int C,
                                                             float* __restrict__ lo_out,
                                                             float* __restrict__ hi_out) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* src = in + (size_t)r * C;
  float lo = 0.0f, hi = 0.0f;
  if ((C & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    for (int j = lane; j < C / 4; j += 32) {
      const float4 v = __ldg(s4 + j);
      lo = run_lo(v.x, lo); hi = run_hi(v.x, hi);
      lo = run_lo(v.y, lo); hi = run_hi(v.y, hi);
      lo = run_lo(v.z, lo); hi = run_hi(v.z, hi);
      lo = run_lo(v.w, lo); hi = run_hi(v.w, hi);
    }
  } else {
    for (int c = lane; c < C; c += 32) {
      lo = run_lo(src[c], lo);
      hi = run_hi(src[c], hi);
    }
  }
  warp_minmax(lo, hi);
  if (lane == 0) {
    lo_out[r] = lo;
    hi_out[r] = hi;
  }
}

// Per output row: the window range over its taps' input rows (dacvae.c:
// 618-627) and the row parameters s, 1/s, zero point (ops.c:329-339 form).
__global__ void __launch_bounds__(256) conv_row_params_kernel(
    const float* __restrict__ rlo, const float* __restrict__ rhi, int batch, int T_in,
    int T_out, int kernel, int stride, int dilation, int padding, float* __restrict__ scale,
    int32_t* __restrict__ zero, float* __restrict__ inv_out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= batch * T_out) return;
  const int b = i / T_out;
  const int t = i - b * T_out;
  const size_t base = (size_t)b * T_in;
  float lo = 0.0f, hi = 0.0f;
  for (int tap = 0; tap < kernel; tap++) {
    const long long it = (long long)t * stride - padding + (long long)tap * dilation;
    if (it < 0 || it >= T_in) continue;
    lo = run_lo(rlo[base + it], lo);
    hi = run_hi(rhi[base + it], hi);
  }
  float s, inv;
  int zp;
  row_params(lo, hi, s, inv, zp);
  scale[i] = s;
  zero[i] = zp;
  inv_out[i] = inv;
}

struct PackArgs {
  const float* in;        // [batch, T_in, C]
  const float* rlo;       // [batch * T_in]
  const float* rhi;
  int T_in, C, T_out, kernel, stride, dilation, padding;
  int row0, rows;         // output rows [row0, row0 + rows) of the flattened [batch*T_out]
  uint8_t* cols;          // [rows, ld]
  uint8_t* cols2;         // residual term or nullptr
  int ld;
  float* scale;           // [rows]
  int32_t* zero;
  float* scale2;
  int32_t* zero2;
};

// One warp per output row.
__global__ void __launch_bounds__(256) conv_pack_kernel(PackArgs a) {
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (i >= a.rows) return;
  const int flat = a.row0 + i;
  const int b = flat / a.T_out;
  const int t = flat - b * a.T_out;
  const size_t in_base = (size_t)b * a.T_in;
  // dacvae.c:618-627: window range from the per-input-row ranges.
  float lo = 0.0f, hi = 0.0f;
  for (int tap = 0; tap < a.kernel; tap++) {
    const long long it = (long long)t * a.stride - a.padding + (long long)tap * a.dilation;
    if (it < 0 || it >= a.T_in) continue;
    lo = run_lo(a.rlo[in_base + it], lo);
    hi = run_hi(a.rhi[in_base + it], hi);
  }
  float s, inv;
  int zp;
  row_params(lo, hi, s, inv, zp);
  const float zpf = (float)zp;
  const bool resid = a.cols2 != nullptr;
  const float inv2 = __fdiv_rn(255.0f, s);
  if (lane == 0) {
    a.scale[i] = s;
    a.zero[i] = zp;
    if (resid) {
      a.scale2[i] = __fdiv_rn(s, 255.0f);
      a.zero2[i] = 128;
    }
  }
  uint8_t* dst = a.cols + (size_t)i * a.ld;
  uint8_t* dst2 = resid ? a.cols2 + (size_t)i * a.ld : nullptr;
  const int C = a.C;
  for (int tap = 0; tap < a.kernel; tap++) {
    const long long it = (long long)t * a.stride - a.padding + (long long)tap * a.dilation;
    uint8_t* td = dst + (size_t)tap * C;
    uint8_t* td2 = resid ? dst2 + (size_t)tap * C : nullptr;
    if (it < 0 || it >= a.T_in) {
      for (int c = lane; c < C; c += 32) {
        td[c] = (uint8_t)zp;
        if (resid) td2[c] = 128;
      }
      continue;
    }
    const float* src = a.in + (in_base + it) * (size_t)C;
    for (int c = lane; c < C; c += 32) {
      const float x = __ldg(src + c);
      float v;
      const uint32_t code = quant_code_v(x, inv, zpf, v);
      td[c] = (uint8_t)code;
      if (resid) {
        // dacvae.c:657-661: remainder against the clamped float code.
        const float rem = __fsub_rn(x, __fmul_rn(s, __fsub_rn(v, zpf)));
        td2[c] = (uint8_t)quant_code(rem, inv2, 128.0f);
      }
    }
  }
  // Zero the pitch padding so TMA tiles past K add nothing.
  for (int k = a.kernel * C + lane; k < a.ld; k += 32) {
    dst[k] = 0;
    if (resid) dst2[k] = 0;
  }
}

}  // namespace iro

using namespace iro;

extern "C" int iro_conv1d_out_len(int T_in, int kernel, int stride, int dilation, int padding) {
  if (T_in <= 0 || stride <= 0 || kernel <= 0 || dilation <= 0) return IRO_ERR_INVALID;
  long long span = (long long)dilation * (kernel - 1) + 1;
  long long num = (long long)T_in + 2LL * padding - span;
  long long out = num < 0 ? -1 : num / stride + 1;
  return out <= 0 || out > 0x7fffffff ? IRO_ERR_INVALID : (int)out;
}

extern "C" int iro_int8_conv1d_dev(const float* input, int batch, int T_in, int C,
                                   const IroInt8DevWeight* w, int kernel, int stride,
                                   int dilation, int padding, const float* bias, int residual,
                                   float* output, void* stream) {
  if (!input || !output || !w || batch <= 0 || C <= 0 || kernel <= 0 ||
      w->layout != IRO_LAYOUT_PLAIN || w->K != kernel * C)
    return IRO_ERR_INVALID;
  const int T_out = iro_conv1d_out_len(T_in, kernel, stride, dilation, padding);
  if (T_out <= 0) return IRO_ERR_INVALID;
  if ((long long)batch * T_out > 0x7fffffffLL) return IRO_ERR_UNSUPPORTED;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  const int K = kernel * C, ld = round_up(K, 16);
  const int total = batch * T_out;
  const int chunk = total < 65536 ? total : 65536;
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t in_rows = (size_t)batch * T_in;
  const size_t bytes = 2 * al(sizeof(float) * in_rows) + al((size_t)chunk * ld) * (residual ? 2 : 1) +
                       4 * al(sizeof(float) * chunk);
  uint8_t* base = static_cast<uint8_t*>(arena_get(c, bytes, &st));
  if (!base) return st;
  size_t off = 0;
  auto take = [&](size_t b) {
    uint8_t* p = base + off;
    off += al(b);
    return p;
  };
  float* rlo = reinterpret_cast<float*>(take(sizeof(float) * in_rows));
  float* rhi = reinterpret_cast<float*>(take(sizeof(float) * in_rows));
  uint8_t* cols = take((size_t)chunk * ld);
  uint8_t* cols2 = residual ? take((size_t)chunk * ld) : nullptr;
  float* sc = reinterpret_cast<float*>(take(sizeof(float) * chunk));
  int32_t* zr = reinterpret_cast<int32_t*>(take(sizeof(float) * chunk));
  float* sc2 = reinterpret_cast<float*>(take(sizeof(float) * chunk));
  int32_t* zr2 = reinterpret_cast<int32_t*>(take(sizeof(float) * chunk));

  conv_row_range_kernel<<<cdiv((int)in_rows, 8), 256, 0, s>>>(input, (int)in_rows, C, rlo, rhi);
  st = check_launch();
  if (st) return st;
  if (conv7_igemm_supported(C, w->N, kernel, stride, dilation, padding, residual, input, output)) {
    // Implicit GEMM: row parameters for all output rows, then one launch.
    float* sc_all = reinterpret_cast<float*>(cols);  // reuse the code buffer area
    int32_t* zr_all = reinterpret_cast<int32_t*>(sc_all + total);
    float* inv_all = reinterpret_cast<float*>(zr_all + total);
    if ((size_t)3 * total * 4 > (size_t)chunk * ld) return IRO_ERR_UNSUPPORTED;
    conv_row_params_kernel<<<cdiv(total, 256), 256, 0, s>>>(rlo, rhi, batch, T_in, T_out, kernel,
                                                             stride, dilation, padding, sc_all,
                                                             zr_all, inv_all);
    st = check_launch();
    if (st) return st;
    st = conv7_igemm_launch(c, input, batch, T_in, C, w, kernel, dilation, padding, bias, sc_all,
                            zr_all, inv_all, output, T_out, s);
    return st ? st : T_out;
  }
  for (int row0 = 0; row0 < total; row0 += chunk) {
    const int rows = total - row0 < chunk ? total - row0 : chunk;
    PackArgs a{input, rlo, rhi, T_in, C, T_out, kernel, stride, dilation, padding, row0, rows,
               cols, cols2, ld, sc, zr, sc2, zr2};
    conv_pack_kernel<<<cdiv(rows, 8), 256, 0, s>>>(a);
    st = check_launch();
    if (st) return st;
    GemmRequest r;
    r.M = rows;
    r.a = cols;
    r.lda = ld;
    r.sx = sc;
    r.zp = zr;
    r.w = w;
    r.bias = bias;
    r.y = output + (size_t)row0 * w->N;
    r.ldy = w->N;
    if (residual) {
      r.epi = EPI_DUAL;
      r.a2 = cols2;
      r.sx2 = sc2;
      r.zp2 = zr2;
    } else {
      r.epi = EPI_LINEAR;
    }
    st = gemm_launch(c, r, s);
    if (st) return st;
  }
  return T_out;
}
