// codec.cu — the codec decoder's other two W8A8 convolutions on the GPU.
//
//  * The transposed (upsampling) convolution, dacvae.c:696-790 with the int8
//    weight.  Every output row starts as the bias (dacvae.c:707-709); the
//    input rows are quantised per row (two-term residual form optional,
//    dacvae.c:748-772); expanded[r, tap*C_out + c] = linear(q, W) without
//    bias, W = [kernel*C_out, C_in] (dacvae.h:47-52); expanded row r, tap t is
//    added onto output row r*stride - padding + t (dacvae.c:776-787).
//    Here: the tcgen05 GEMM writes the expanded rows of a chunk of input rows
//    to a workspace, and a gather kernel adds them onto the output.  Each
//    output element is owned by one thread, which adds its contributions in
//    increasing input-row order, the order of the reference's row loop, so
//    the fp32 sums are the reference's bit for bit.
//
//  * The residual unit's skip + 1x1 projection, dacvae.c:979-1009: output =
//    skip, then the quantised hidden's linear (with bias) accumulated onto
//    it, and the second residual term (without bias) accumulated after that.
//    One GEMM launch does both terms (EPI_DUAL with accumulate keeps the
//    reference's order of additions).
#include "gemm_i8.cuh"
#include "quantize.cuh"

namespace iro {

// out[row, c] = bias[c], or 0 without a bias, for `rows` rows of C floats.
__global__ void fill_rows_kernel(float* __restrict__ out, long long rows, int C,
                                 const float* __restrict__ bias) {
  const long long n = rows * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = bias ? __ldg(bias + (int)(i % C)) : 0.0f;
}

__host__ __device__ inline long long floor_div(long long a, long long b) {
  return a >= 0 ? a / b : -((-a + b - 1) / b);
}

// Output rows [o0, o1) of one sequence take the expanded rows of input rows
// [r0, r0 + n) of that sequence (workspace rows 0 .. n-1, pitch ldE floats).
struct GatherArgs {
  float* out;        // [T_out, C] of this sequence
  const float* e;    // [n, ldE]
  int ldE;
  int r0, n;
  int o0, o1;
  int C, kernel, stride, padding;
};

// One thread per V consecutive channels of one output row.
template <int V>
__global__ void __launch_bounds__(256) convt_gather_kernel(GatherArgs a) {
  const int cv = a.C / V;
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= (long long)(a.o1 - a.o0) * cv) return;
  const int ot = a.o0 + (int)(idx / cv);
  const int c = (int)(idx % cv) * V;
  // Input rows r with r*stride - padding <= ot <= r*stride - padding + kernel - 1.
  long long lo = -floor_div(-(long long)(ot + a.padding - a.kernel + 1), a.stride);
  long long hi = floor_div((long long)ot + a.padding, a.stride);
  if (lo < a.r0) lo = a.r0;
  if (hi > a.r0 + a.n - 1) hi = a.r0 + a.n - 1;
  float* dst = a.out + (size_t)ot * a.C + c;
  if (V == 4) {
    float4 v = *reinterpret_cast<float4*>(dst);
    for (long long r = lo; r <= hi; r++) {
      const int tap = (int)(ot + a.padding - r * a.stride);
      const float4 x = __ldg(reinterpret_cast<const float4*>(
          a.e + (size_t)(r - a.r0) * a.ldE + (size_t)tap * a.C + c));
      v.x = __fadd_rn(v.x, x.x);
      v.y = __fadd_rn(v.y, x.y);
      v.z = __fadd_rn(v.z, x.z);
      v.w = __fadd_rn(v.w, x.w);
    }
    *reinterpret_cast<float4*>(dst) = v;
  } else {
    float v = *dst;
    for (long long r = lo; r <= hi; r++) {
      const int tap = (int)(ot + a.padding - r * a.stride);
      v = __fadd_rn(v, __ldg(a.e + (size_t)(r - a.r0) * a.ldE + (size_t)tap * a.C + c));
    }
    *dst = v;
  }
}

static size_t al256(size_t b) { return (b + 255) / 256 * 256; }

// Workspace of one chunk: codes (and second-term codes), row parameters,
// and optionally the expanded rows.
struct ChunkWs {
  uint8_t* q = nullptr;
  float* s = nullptr;
  int32_t* z = nullptr;
  uint8_t* q2 = nullptr;
  float* s2 = nullptr;
  int32_t* z2 = nullptr;
  float* e = nullptr;
};

static size_t chunk_ws_bytes(int rows, int K, int residual, size_t e_floats) {
  size_t t = al256((size_t)rows * K) + 2 * al256(sizeof(float) * rows);
  if (residual) t += al256((size_t)rows * K) + 2 * al256(sizeof(float) * rows);
  return t + al256(sizeof(float) * e_floats);
}

static ChunkWs chunk_ws_take(uint8_t* base, int rows, int K, int residual, size_t e_floats) {
  ChunkWs w;
  size_t off = 0;
  auto take = [&](size_t b) {
    uint8_t* p = base + off;
    off += al256(b);
    return p;
  };
  w.q = take((size_t)rows * K);
  w.s = reinterpret_cast<float*>(take(sizeof(float) * rows));
  w.z = reinterpret_cast<int32_t*>(take(sizeof(float) * rows));
  if (residual) {
    w.q2 = take((size_t)rows * K);
    w.s2 = reinterpret_cast<float*>(take(sizeof(float) * rows));
    w.z2 = reinterpret_cast<int32_t*>(take(sizeof(float) * rows));
  }
  if (e_floats) w.e = reinterpret_cast<float*>(take(sizeof(float) * e_floats));
  return w;
}

// Quantise `rows` rows of x into the chunk workspace (one or two terms).
static int quantise_chunk(const float* x, int rows, int K, int residual, const ChunkWs& w,
                          cudaStream_t s) {
  if (residual)
    return quantize_rows_residual_launch(x, rows, K, w.q, w.s, w.z, nullptr, w.q2, w.s2, w.z2, s);
  return quantize_rows_launch(x, rows, K, w.q, w.s, w.z, 0, s);
}

// The GEMM of one chunk: y (=|+=) the linear of the chunk's codes.
static int chunk_gemm(Ctx* c, const ChunkWs& w, int rows, const IroInt8DevWeight* wt,
                      const float* bias, float* y, int accumulate, int residual,
                      cudaStream_t s) {
  GemmRequest r;
  r.M = rows;
  r.a = w.q;
  r.lda = wt->K;
  r.sx = w.s;
  r.zp = w.z;
  r.w = wt;
  r.bias = bias;
  r.y = y;
  r.ldy = wt->N;
  r.accumulate = accumulate;
  if (residual) {
    r.epi = EPI_DUAL;
    r.a2 = w.q2;
    r.sx2 = w.s2;
    r.zp2 = w.z2;
  } else {
    r.epi = EPI_LINEAR;
  }
  return gemm_launch(c, r, s);
}

// Workspace budget for the expanded rows of one chunk.
constexpr size_t kExpandedBytes = size_t(256) << 20;

}  // namespace iro

using namespace iro;

extern "C" int iro_convtranspose1d_out_len(int T_in, int kernel, int stride, int padding,
                                           int output_padding) {
  if (T_in <= 0 || stride <= 0 || kernel <= 0) return IRO_ERR_INVALID;
  const long long out =
      (long long)(T_in - 1) * stride - 2LL * padding + kernel + output_padding;
  return out <= 0 || out > 0x7fffffff ? IRO_ERR_INVALID : (int)out;
}

extern "C" int iro_int8_convtranspose1d_dev(const float* input, int batch, int T_in, int C_in,
                                            const IroInt8DevWeight* w, int C_out, int kernel,
                                            int stride, int padding, int output_padding,
                                            const float* bias, int residual, float* output,
                                            void* stream) {
  if (!input || !output || !w || batch <= 0 || C_in <= 0 || C_out <= 0 || kernel <= 0 ||
      stride <= 0 || padding < 0 || output_padding < 0 || w->layout != IRO_LAYOUT_PLAIN ||
      w->K != C_in || (long long)w->N != (long long)kernel * C_out)
    return IRO_ERR_INVALID;
  const int T_out = iro_convtranspose1d_out_len(T_in, kernel, stride, padding, output_padding);
  if (T_out <= 0) return IRO_ERR_INVALID;
  // Codes are written densely (pitch C_in); the GEMM's TMA needs 16-byte rows.
  if (C_in % 16 != 0) return IRO_ERR_UNSUPPORTED;
  if ((long long)batch * T_in > 0x7fffffffLL || (long long)batch * T_out > 0x7fffffffLL)
    return IRO_ERR_UNSUPPORTED;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  const int N = w->N;
  const int total = batch * T_in;
  long long chunk = (long long)(kExpandedBytes / (sizeof(float) * (size_t)N));
  chunk = chunk / 128 * 128;
  if (chunk < 128) chunk = 128;
  if (chunk > total) chunk = total;
  const int rows_max = (int)chunk;
  uint8_t* base = static_cast<uint8_t*>(
      arena_get(c, chunk_ws_bytes(rows_max, C_in, residual, (size_t)rows_max * N), &st));
  if (!base) return st;
  const ChunkWs ws = chunk_ws_take(base, rows_max, C_in, residual, (size_t)rows_max * N);

  const long long out_elems = (long long)batch * T_out * C_out;
  {
    const int blocks = (int)std::min<long long>((out_elems + 255) / 256, 148LL * 16);
    fill_rows_kernel<<<blocks, 256, 0, s>>>(output, (long long)batch * T_out, C_out, bias);
    st = check_launch();
    if (st) return st;
  }
  const bool vec = C_out % 4 == 0 && (reinterpret_cast<uintptr_t>(output) & 15u) == 0;
  for (int f0 = 0; f0 < total; f0 += rows_max) {
    const int rows = std::min(rows_max, total - f0);
    st = quantise_chunk(input + (size_t)f0 * C_in, rows, C_in, residual, ws, s);
    if (st) return st;
    st = chunk_gemm(c, ws, rows, w, nullptr, ws.e, 0, residual, s);
    if (st) return st;
    // Scatter the chunk's expanded rows onto each sequence it covers.
    for (int b = f0 / T_in; b < batch && (long long)b * T_in < f0 + rows; b++) {
      const int rb0 = std::max(f0, b * T_in) - b * T_in;
      const int rb1 = std::min(f0 + rows, (b + 1) * T_in) - b * T_in;
      if (rb1 <= rb0) continue;
      GatherArgs g;
      g.out = output + (size_t)b * T_out * C_out;
      g.e = ws.e + (size_t)(b * T_in + rb0 - f0) * N;
      g.ldE = N;
      g.r0 = rb0;
      g.n = rb1 - rb0;
      g.o0 = (int)std::max(0LL, (long long)rb0 * stride - padding);
      g.o1 = (int)std::min((long long)T_out, (long long)(rb1 - 1) * stride - padding + kernel);
      g.C = C_out;
      g.kernel = kernel;
      g.stride = stride;
      g.padding = padding;
      if (g.o1 <= g.o0) continue;
      const long long threads = (long long)(g.o1 - g.o0) * (vec ? C_out / 4 : C_out);
      const int blocks = (int)((threads + 255) / 256);
      if (vec)
        convt_gather_kernel<4><<<blocks, 256, 0, s>>>(g);
      else
        convt_gather_kernel<1><<<blocks, 256, 0, s>>>(g);
      st = check_launch();
      if (st) return st;
    }
  }
  return T_out;
}

extern "C" int iro_int8_codec_conv1_dev(const float* hidden, int rows,
                                        const IroInt8DevWeight* w, const float* bias,
                                        const float* skip, int residual, float* output,
                                        void* stream) {
  if (!hidden || !skip || !output || !w || rows <= 0 || w->layout != IRO_LAYOUT_PLAIN ||
      w->N != w->K)
    return IRO_ERR_INVALID;
  const int C = w->K;
  if (C % 16 != 0) return IRO_ERR_UNSUPPORTED;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  const int rows_max = (int)std::min<long long>(rows, std::max<long long>(128, (256LL << 20) / C));
  uint8_t* base = static_cast<uint8_t*>(arena_get(c, chunk_ws_bytes(rows_max, C, residual, 0), &st));
  if (!base) return st;
  const ChunkWs ws = chunk_ws_take(base, rows_max, C, residual, 0);
  // dacvae.c:983: the output starts as the skip input.
  if (skip != output) {
    cudaError_t e = cudaMemcpyAsync(output, skip, sizeof(float) * (size_t)rows * C,
                                    cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
  }
  for (int r0 = 0; r0 < rows; r0 += rows_max) {
    const int n = std::min(rows_max, rows - r0);
    st = quantise_chunk(hidden + (size_t)r0 * C, n, C, residual, ws, s);
    if (st) return st;
    st = chunk_gemm(c, ws, n, w, bias, output + (size_t)r0 * C, 1, residual, s);
    if (st) return st;
  }
  return IRO_OK;
}
