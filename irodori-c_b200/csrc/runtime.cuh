// runtime.cuh — per-device context of the library (stream, device error word,
// device arena, host-weight cache) and host-side helpers shared by the
// entry points.
#pragma once

#include <string.h>

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <unordered_map>
#include <vector>

#include "iro_common.cuh"

namespace iro {

// Device copy of a host IroInt8Weight, kept by the host-pointer API so the
// reference's call pattern (same weight, many linears) uploads once.
struct CachedWeight {
  IroInt8DevWeight dev;
  uint64_t fingerprint;
};

struct Ctx {
  int device = -1;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  DevError* err = nullptr;       // this device's error word (device_error_word)
  void* arena = nullptr;         // device scratch for the host-pointer API
  size_t arena_bytes = 0;
  std::mutex mu;
  std::unordered_map<const void*, CachedWeight> wcache;
  // Copy streams and events for host-pointer calls that overlap their
  // host<->device copies with compute (created on first use).
  cudaStream_t copy_in = nullptr;
  cudaStream_t copy_out = nullptr;
  std::vector<cudaEvent_t> events;
};

// The copy streams and at least `n` events of the context (created lazily).
int ctx_copy_resources(Ctx* c, int n);

// Context of device `dev` if it was already created (no side effects).
Ctx* ctx_existing(int dev);

// Context of the current CUDA device, created on first use.  Sets *status
// (IRO_OK or IRO_ERR_*) and returns nullptr on failure.
Ctx* ctx_current(int* status);

// Record a status for iro_cuda_last_error() on this thread (first error
// sticks until read).
void set_last_error(int code);

// Map a CUDA runtime error to IRO_ERR_* (OOM distinguished).
int map_cuda(cudaError_t e);

// Check the launch just issued; returns IRO_OK or IRO_ERR_CUDA.
int check_launch();

// Device scratch of at least `bytes` from the context arena (grows; the
// previous contents are not kept).  Only for stream-ordered use on the
// context stream.
void* arena_get(Ctx* c, size_t bytes, int* status);

// Device address of the current device's error word: one static
// __device__ word per GPU (no allocation), shared by every entry point,
// resolved once per device with cudaGetSymbolAddress.  `dev` must be the
// current device.
int device_error_word(int dev, DevError** out);

// Read (and clear) the device error word after the stream was synchronised.
int take_device_error(Ctx* c);

// The same for the current device without a context (allocates nothing);
// returns IRO_OK when the word was never resolved on this device.
int take_device_error_current();

// 2-D u8/s8 tensor map for TMA: rows x inner bytes with the given row pitch
// (multiple of 16), box = box_inner x box_rows, 128-byte swizzle.
int make_tmap_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                 uint64_t pitch, uint32_t box_inner, uint32_t box_rows);

// 2-D f32 tensor map for TMA tile stores of 32-row x 16-column boxes with the
// 64-byte swizzle (rows x inner floats, pitch in bytes, multiple of 16).
int make_tmap_f32_sw128(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                        uint64_t pitch_bytes);

// Generic tiled tensor map of rank 1..5: dims and box innermost first,
// strides in bytes for dims 1..rank-1.
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                CUtensorMapSwizzle swz);

// 2-D f32 tensor map without swizzle (for staging fp32 tiles).
int make_tmap_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                  uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_rows);

inline cudaStream_t pick_stream(Ctx* c, void* s) {
  return s ? static_cast<cudaStream_t>(s) : c->stream;
}

// Launch with programmatic stream serialization (see grid_dep_wait): the
// kernel's launch and prologue overlap the previous kernel's tail.  Every
// kernel launched this way calls grid_dep_wait() before its first global
// memory access that depends on earlier work in the stream.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Default in-kernel wait limit (ns) for bounded mbarrier waits.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

inline int round_up(int a, int b) { return (a + b - 1) / b * b; }
inline int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace iro
