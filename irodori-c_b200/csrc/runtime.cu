// runtime.cu — device contexts, error reporting, device memory helpers and
// TMA descriptor encoding for the B200 int8 path.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cudaTypedefs.h>

#include "runtime.cuh"

namespace iro {

// The device error word: bounded device waits that give up record their
// code here.  A __device__ variable has one instance per GPU, so every device
// has its own word without an allocation.
__device__ DevError g_device_error;

namespace {

std::mutex g_ctx_mu;
std::mutex g_err_mu;
DevError* g_err_word[64] = {nullptr};
Ctx* g_ctx[64] = {nullptr};
thread_local int t_last_error = 0;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                       &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

}  // namespace

void set_last_error(int code) {
  if (code != IRO_OK && t_last_error == IRO_OK) t_last_error = code;
}

int map_cuda(cudaError_t e) {
  if (e == cudaSuccess) return IRO_OK;
  if (e == cudaErrorMemoryAllocation) return IRO_ERR_OOM;
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ||
      e == cudaErrorInvalidDevice)
    return IRO_ERR_NO_DEVICE;
  return IRO_ERR_CUDA;
}

int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "irodori_b200: kernel launch failed: %s\n", cudaGetErrorString(e));
    return map_cuda(e);
  }
  return IRO_OK;
}

static int create_ctx(int dev, Ctx** out) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) return map_cuda(e);
  if (prop.major != 10) {
    fprintf(stderr, "irodori_b200: device %d is sm_%d%d; this library needs sm_100\n", dev,
            prop.major, prop.minor);
    return IRO_ERR_NO_DEVICE;
  }
  Ctx* c = new Ctx();
  c->device = dev;
  c->num_sms = prop.multiProcessorCount;
  int st = device_error_word(dev, &c->err);
  if (st != IRO_OK) {
    delete c;
    return st;
  }
  e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof(DevError));
  if (e != cudaSuccess) {
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return map_cuda(e);
  }
  *out = c;
  return IRO_OK;
}

Ctx* ctx_existing(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  return g_ctx[dev];
}

Ctx* ctx_current(int* status) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *status = map_cuda(e);
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *status = IRO_ERR_NO_DEVICE;
    return nullptr;
  }
  Ctx* c = g_ctx[dev];
  if (c) {
    *status = IRO_OK;
    return c;
  }
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  if (!g_ctx[dev]) {
    Ctx* nc = nullptr;
    int st = create_ctx(dev, &nc);
    if (st != IRO_OK) {
      *status = st;
      return nullptr;
    }
    g_ctx[dev] = nc;
  }
  *status = IRO_OK;
  return g_ctx[dev];
}

void* arena_get(Ctx* c, size_t bytes, int* status) {
  if (bytes == 0) bytes = 256;
  if (c->arena_bytes < bytes) {
    if (c->arena) {
      cudaStreamSynchronize(c->stream);
      cudaFree(c->arena);
      c->arena = nullptr;
      c->arena_bytes = 0;
    }
    size_t want = bytes + bytes / 4;
    cudaError_t e = cudaMalloc(&c->arena, want);
    if (e != cudaSuccess) {
      cudaGetLastError();
      *status = map_cuda(e);
      return nullptr;
    }
    c->arena_bytes = want;
  }
  *status = IRO_OK;
  return c->arena;
}

int ctx_copy_resources(Ctx* c, int n) {
  cudaError_t e = cudaSuccess;
  if (!c->copy_in) e = cudaStreamCreateWithFlags(&c->copy_in, cudaStreamNonBlocking);
  if (e == cudaSuccess && !c->copy_out)
    e = cudaStreamCreateWithFlags(&c->copy_out, cudaStreamNonBlocking);
  while (e == cudaSuccess && (int)c->events.size() < n) {
    cudaEvent_t ev;
    e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) c->events.push_back(ev);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

int device_error_word(int dev, DevError** out) {
  if (dev < 0 || dev >= 64) return IRO_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_err_mu);
  if (!g_err_word[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_device_error);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
    g_err_word[dev] = static_cast<DevError*>(p);
  }
  *out = g_err_word[dev];
  return IRO_OK;
}

// Synchronous read of the word into host memory on the stack (no pinned
// buffer), then a clear when a code was recorded.
static int take_error_word(DevError* word) {
  DevError h;
  if (cudaMemcpy(&h, word, sizeof(DevError), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return IRO_ERR_CUDA;
  }
  if (h.code != 0) {
    fprintf(stderr, "irodori_b200: device reported error %d (%s; site %d, block %d)\n", h.code,
            iro_cuda_error_string(h.code), h.where, h.block);
    if (cudaMemset(word, 0, sizeof(DevError)) != cudaSuccess) cudaGetLastError();
  }
  return h.code;
}

int take_device_error(Ctx* c) { return take_error_word(c->err); }

int take_device_error_current() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return IRO_ERR_NO_DEVICE;
  }
  DevError* word = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_err_mu);
    if (dev >= 0 && dev < 64) word = g_err_word[dev];
  }
  return word ? take_error_word(word) : IRO_OK;
}

static int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                     uint64_t rows, uint64_t pitch, uint32_t box_inner, uint32_t box_rows,
                     CUtensorMapSwizzle swz) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return IRO_ERR_NO_DEVICE;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (pitch & 15u) != 0)
    return IRO_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fprintf(stderr, "irodori_b200: cuTensorMapEncodeTiled failed (%d)\n", (int)r);
    return IRO_ERR_UNSUPPORTED;
  }
  return IRO_OK;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                CUtensorMapSwizzle swz) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return IRO_ERR_NO_DEVICE;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return IRO_ERR_UNSUPPORTED;
  for (int i = 0; i + 1 < rank; i++)
    if ((strides[i] & 15u) != 0) return IRO_ERR_UNSUPPORTED;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fprintf(stderr, "irodori_b200: cuTensorMapEncodeTiled (rank %d) failed (%d)\n", rank, (int)r);
    return IRO_ERR_UNSUPPORTED;
  }
  return IRO_OK;
}

int make_tmap_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                 uint64_t pitch, uint32_t box_inner, uint32_t box_rows) {
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, inner, rows, pitch, box_inner,
                   box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

int make_tmap_f32_sw128(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                        uint64_t pitch_bytes) {
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, inner, rows, pitch_bytes, 16, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B);
}

int make_tmap_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                  uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_rows) {
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, inner, rows, pitch_bytes,
                   box_inner, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace iro

using namespace iro;

extern "C" {

int iro_cuda_init(int device) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return IRO_ERR_NO_DEVICE;
  }
  if (device < 0 || device >= n) return IRO_ERR_INVALID;
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return map_cuda(e);
  int st;
  ctx_current(&st);
  return st;
}

int iro_cuda_last_error(void) {
  int e = t_last_error;
  t_last_error = 0;
  return e;
}

const char* iro_cuda_error_string(int code) {
  switch (code) {
    case IRO_OK: return "ok";
    case IRO_ERR_INVALID: return "invalid argument";
    case IRO_ERR_NO_DEVICE: return "no usable sm_100 CUDA device";
    case IRO_ERR_CUDA: return "CUDA runtime error";
    case IRO_ERR_OOM: return "out of memory";
    case IRO_ERR_DEVICE_TIMEOUT: return "bounded device wait gave up";
    case IRO_ERR_UNSUPPORTED: return "unsupported shape or alignment";
    case IRO_ERR_SELFCHECK: return "exact-sum selfcheck failed";
    case IRO_ERR_RANGE: return "attention operand beyond the fp16 range";
    default: return "unknown";
  }
}

int iro_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int count = 0;
  for (int d = 0; d < n; d++) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) count++;
  }
  return count;
}

void* iro_cuda_stream(void) {
  int st;
  Ctx* c = ctx_current(&st);
  return c ? static_cast<void*>(c->stream) : nullptr;
}

int iro_cuda_synchronize(void* stream) {
  // With a caller stream no context is needed (nothing is allocated here);
  // without one, the library stream of the current device's context.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!s) {
    int st;
    Ctx* c = ctx_current(&st);
    if (!c) return st;
    s = c->stream;
  }
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  int dev = take_device_error_current();
  return dev ? dev : IRO_OK;
}

void* iro_dev_malloc(size_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
    cudaGetLastError();
    set_last_error(IRO_ERR_OOM);
    return nullptr;
  }
  return p;
}

void iro_dev_free(void* p) {
  if (p) cudaFree(p);
}

static int copy(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, void* stream) {
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, s);
  if (e == cudaSuccess && stream == nullptr) e = cudaStreamSynchronize(s);
  return map_cuda(e);
}

int iro_memcpy_htod(void* dst, const void* src, size_t bytes, void* stream) {
  return copy(dst, src, bytes, cudaMemcpyHostToDevice, stream);
}
int iro_memcpy_dtoh(void* dst, const void* src, size_t bytes, void* stream) {
  return copy(dst, src, bytes, cudaMemcpyDeviceToHost, stream);
}
int iro_memcpy_dtod(void* dst, const void* src, size_t bytes, void* stream) {
  return copy(dst, src, bytes, cudaMemcpyDeviceToDevice, stream);
}

int iro_memset_dev(void* dst, int value, size_t bytes, void* stream) {
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  cudaError_t e = cudaMemsetAsync(dst, value, bytes, s);
  if (e == cudaSuccess && stream == nullptr) e = cudaStreamSynchronize(s);
  return map_cuda(e);
}

void* iro_host_alloc_pinned(size_t bytes) {
  void* p = nullptr;
  if (cudaMallocHost(&p, bytes ? bytes : 1) != cudaSuccess) {
    cudaGetLastError();
    set_last_error(IRO_ERR_OOM);
    return nullptr;
  }
  return p;
}

void iro_host_free_pinned(void* p) {
  if (p) cudaFreeHost(p);
}

}  // extern "C"
