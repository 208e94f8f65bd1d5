// noalloc.cu — the int8 SwiGLU block for callers that must not allocate
// device memory.
//
// iro_int8_swiglu_dev() needs about 15 KB of device scratch per row (the
// quantised input, the fp32 hidden and its quantised form).  It takes that
// from a caller workspace or from the library's arena, and the arena grows
// with cudaMalloc.  Some callers cannot allow that on the path that runs the
// block:
//   - engines that reserve all their device memory at start-up and treat any
//     later allocation as a failure (serving processes that share a GPU
//     under a fixed memory budget);
//   - hosts whose device memory belongs to another allocator (a framework's
//     caching pool) and that must not create allocations behind its back;
//   - latency-critical loops, because growing an arena calls cudaFree, which
//     waits for the whole device.
// For them, iro_int8_swiglu_noalloc_dev() runs the same kernels on a scratch
// array compiled into this file.  The CUDA runtime reserves it (64 MiB) on each
// GPU where the library's device code is loaded, and it stays reserved until
// the process exits.
#include <stdio.h>

#include <mutex>

#include "gemm_i8.cuh"
#include "quantize.cuh"

namespace iro {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;

// The scratch.  Host code must not pass this name to a kernel: in host code
// it is a stand-in, not a device address.  The device address comes from
// cudaGetSymbolAddress (noalloc_setup).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

struct NoAllocDevice {
  unsigned char* scratch;  // device address of g_noalloc_scratch
  DevError* err;           // the device's error word (device_error_word)
  int num_sms;
  bool ready;
};

NoAllocDevice g_noalloc_dev[64];
std::mutex g_noalloc_mu;

// Once per device, with that device current: resolve the device addresses
// of the scratch array and of the library's device error word (both static
// device memory).  This is the only set-up; it allocates nothing.
int noalloc_setup(int dev, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    int major = 0, sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
    if (major != 10) return IRO_ERR_NO_DEVICE;
    unsigned char* ptr = nullptr;
    e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
    DevError* err = nullptr;
    const int st = device_error_word(dev, &err);
    if (st != IRO_OK) return st;
    d.scratch = ptr;
    d.err = err;
    d.num_sms = sms;
    d.ready = true;
  }
  *out = &d;
  return IRO_OK;
}

}  // namespace
}  // namespace iro

using namespace iro;

// See include/irodori_b200.h.  The first call on a device resolves the
// scratch address (cudaGetSymbolAddress), which also makes the runtime load
// this library's device code on that device if it has not done so yet; make
// that first call before any stream capture.  Calls share the one scratch
// array, so calls that can overlap on the GPU (different streams without
// ordering between them, or different host threads) race on it.  A bounded
// device wait that gives up inside the kernels records its code in the
// device's error word, which iro_cuda_synchronize() on the call's stream
// reports and clears.
extern "C" int iro_int8_swiglu_noalloc_dev(const float* x, int M, const IroInt8DevWeight* w13,
                                           const IroInt8DevWeight* w2, const float* b2,
                                           float* out, int residual_w2, void* stream) {
  if (!x || !out || !w13 || !w2 || w13->layout != IRO_LAYOUT_GATED_PAIR ||
      w2->layout != IRO_LAYOUT_PLAIN || w2->K != w13->hidden || M < 0)
    return IRO_ERR_INVALID;
  const int D = w13->K, H = w13->hidden;
  if (w2->N != D) return IRO_ERR_INVALID;
  if (D % 16 != 0 || H % 16 != 0) return IRO_ERR_UNSUPPORTED;
  if (M == 0) return IRO_OK;
  const size_t need = iro_int8_swiglu_workspace_bytes(M, D, H, residual_w2);
  if (need > kNoAllocScratchBytes) {
    fprintf(stderr,
            "irodori_b200: iro_int8_swiglu_noalloc_dev: %d rows need %zu bytes of scratch, "
            "more than its fixed %zu; split the rows into smaller calls\n",
            M, need, kNoAllocScratchBytes);
    return IRO_ERR_UNSUPPORTED;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return IRO_ERR_NO_DEVICE;
  }
  NoAllocDevice* nd = nullptr;
  int st = noalloc_setup(dev, &nd);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // Same layout as iro_int8_swiglu_dev's workspace.  Every region is fully
  // written before it is read, so nothing needs clearing between calls.
  unsigned char* ws = nd->scratch;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* p = ws + off;
    off += (bytes + 255) / 256 * 256;
    return p;
  };
  uint8_t* qx = take((size_t)M * D);
  float* sx = reinterpret_cast<float*>(take(sizeof(float) * M));
  int32_t* zx = reinterpret_cast<int32_t*>(take(sizeof(float) * M));
  float* hid = reinterpret_cast<float*>(take(sizeof(float) * (size_t)M * H));
  uint8_t* qh = take((size_t)M * H);
  float* sh = reinterpret_cast<float*>(take(sizeof(float) * M));
  int32_t* zh = reinterpret_cast<int32_t*>(take(sizeof(float) * M));
  uint8_t* qh2 = nullptr;
  float* sh2 = nullptr;
  int32_t* zh2 = nullptr;
  if (residual_w2) {
    qh2 = take((size_t)M * H);
    sh2 = reinterpret_cast<float*>(take(sizeof(float) * M));
    zh2 = reinterpret_cast<int32_t*>(take(sizeof(float) * M));
  }

  // A launch environment that owns nothing: the device, its SM count and
  // the device's error word (the library context, which allocates, is not
  // touched).
  Ctx env;
  env.device = dev;
  env.num_sms = nd->num_sms;
  env.err = nd->err;

  st = quantize_rows_launch(x, M, D, qx, sx, zx, 0, s);
  if (st) return st;
  GemmRequest g;
  g.epi = EPI_GATED;
  g.M = M;
  g.a = qx;
  g.lda = D;
  g.sx = sx;
  g.zp = zx;
  g.w = w13;
  g.hidden = hid;
  g.ldh = H;
  g.no_alloc = 1;
  st = gemm_launch(&env, g, s);
  if (st) return st;
  if (residual_w2)
    st = quantize_rows_residual_launch(hid, M, H, qh, sh, zh, nullptr, qh2, sh2, zh2, s);
  else
    st = quantize_rows_launch(hid, M, H, qh, sh, zh, 0, s);
  if (st) return st;
  GemmRequest r;
  r.M = M;
  r.a = qh;
  r.lda = H;
  r.sx = sh;
  r.zp = zh;
  r.w = w2;
  r.bias = b2 ? b2 : w2->bias;
  r.y = out;
  r.ldy = D;
  r.no_alloc = 1;
  if (residual_w2) {
    r.epi = EPI_DUAL;
    r.a2 = qh2;
    r.sx2 = sh2;
    r.zp2 = zh2;
  } else {
    r.epi = EPI_LINEAR;
  }
  return gemm_launch(&env, r, s);
}
