// probe.cu — failure-detection probe: a bounded wait that is designed to run
// out, so the host-side error path can be tested without faulting a GPU.
#include "runtime.cuh"

namespace iro {

__global__ void bounded_wait_probe_kernel(DevError* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait gives up after limit_ns and
  // records IRO_ERR_DEVICE_TIMEOUT; the kernel then returns normally.
  if (threadIdx.x == 0) mbar_wait_bounded(&bar, 0, err, 99, nullptr, limit_ns);
}

}  // namespace iro

using namespace iro;

extern "C" int iro_debug_bounded_wait_probe(uint64_t limit_ns) {
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  if (limit_ns > 2000000000ull) limit_ns = 2000000000ull;
  bounded_wait_probe_kernel<<<1, 32, 0, c->stream>>>(c->err, limit_ns);
  st = check_launch();
  if (st) return st;
  return iro_cuda_synchronize(nullptr);
}
