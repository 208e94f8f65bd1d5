// plan.cu — recorded launch plans (CUDA graphs) for repeated blocks.
//
// A serving loop runs the same block with the same buffers every step.  A
// plan records the block's kernel launches once, TMA descriptors included,
// as a CUDA graph; each step then costs one graph launch instead of four
// kernel launches and their descriptor encoding on the host.
#include <stdlib.h>

#include "runtime.cuh"

struct IroPlan {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  void* workspace = nullptr;  // owned
  int device = -1;
};

using namespace iro;

extern "C" {

int iro_int8_swiglu_plan(IroPlan** plan, const float* x, int M, const IroInt8DevWeight* w13,
                         const IroInt8DevWeight* w2, const float* b2, float* out,
                         int residual_w2) {
  if (!plan || !x || !out || !w13 || !w2 || M <= 0) return IRO_ERR_INVALID;
  *plan = nullptr;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  IroPlan* p = new IroPlan();
  p->device = c->device;
  const size_t wsb = iro_int8_swiglu_workspace_bytes(M, w13->K, w13->hidden, residual_w2);
  cudaError_t e = cudaMalloc(&p->workspace, wsb ? wsb : 256);
  cudaStream_t s = nullptr;
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  // One untimed run outside the capture sets the kernels' attributes.
  if (e == cudaSuccess) {
    st = iro_int8_swiglu_dev(x, M, w13, w2, b2, out, residual_w2, p->workspace, s);
    if (st == IRO_OK) e = cudaStreamSynchronize(s);
  }
  if (e == cudaSuccess && st == IRO_OK)
    e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess && st == IRO_OK) {
    st = iro_int8_swiglu_dev(x, M, w13, w2, b2, out, residual_w2, p->workspace, s);
    cudaError_t e2 = cudaStreamEndCapture(s, &p->graph);
    if (e == cudaSuccess) e = e2;
  }
  if (e == cudaSuccess && st == IRO_OK) e = cudaGraphInstantiate(&p->exec, p->graph, 0);
  if (s) cudaStreamDestroy(s);
  if (e != cudaSuccess || st != IRO_OK) {
    if (st == IRO_OK) st = map_cuda(e);
    cudaGetLastError();
    iro_plan_free(p);
    return st;
  }
  *plan = p;
  return IRO_OK;
}

int iro_plan_launch(const IroPlan* plan, void* stream) {
  if (!plan || !plan->exec) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  if (c->device != plan->device) return IRO_ERR_INVALID;
  cudaError_t e = cudaGraphLaunch(plan->exec, pick_stream(c, stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

void iro_plan_free(IroPlan* plan) {
  if (!plan) return;
  if (plan->exec) cudaGraphExecDestroy(plan->exec);
  if (plan->graph) cudaGraphDestroy(plan->graph);
  if (plan->workspace) cudaFree(plan->workspace);
  delete plan;
}

// ---------------------------------------------------------------------------
// Submit/wait pipeline for host-buffer serving: a ring of `depth` device
// slots, each with its own input/output buffers and recorded block, so the
// host->device copy of one step, the compute of the previous one and the
// device->host copy of the one before run at the same time on three streams.

struct Slot {
  float* x = nullptr;
  float* out = nullptr;
  IroPlan* plan = nullptr;
  cudaEvent_t in_done = nullptr, compute_done = nullptr, out_done = nullptr;
  bool used = false;
};

struct IroSwigluPipe {
  int device = -1, M = 0, D = 0, depth = 0, next = 0;
  cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
  Slot* slots = nullptr;
};

void iro_int8_swiglu_pipe_free(IroSwigluPipe* p) {
  if (!p) return;
  if (p->comp) cudaStreamSynchronize(p->comp);
  if (p->d2h) cudaStreamSynchronize(p->d2h);
  if (p->h2d) cudaStreamSynchronize(p->h2d);
  for (int i = 0; p->slots && i < p->depth; i++) {
    Slot& s = p->slots[i];
    iro_plan_free(s.plan);
    if (s.x) cudaFree(s.x);
    if (s.out) cudaFree(s.out);
    if (s.in_done) cudaEventDestroy(s.in_done);
    if (s.compute_done) cudaEventDestroy(s.compute_done);
    if (s.out_done) cudaEventDestroy(s.out_done);
  }
  delete[] p->slots;
  if (p->h2d) cudaStreamDestroy(p->h2d);
  if (p->comp) cudaStreamDestroy(p->comp);
  if (p->d2h) cudaStreamDestroy(p->d2h);
  delete p;
}

int iro_int8_swiglu_pipe_create(IroSwigluPipe** pipe, int M, const IroInt8DevWeight* w13,
                                const IroInt8DevWeight* w2, const float* b2, int residual_w2,
                                int depth) {
  if (!pipe || !w13 || !w2 || M <= 0 || depth < 1 || depth > 8) return IRO_ERR_INVALID;
  *pipe = nullptr;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  IroSwigluPipe* p = new IroSwigluPipe();
  p->device = c->device;
  p->M = M;
  p->D = w13->K;
  p->depth = depth;
  p->slots = new Slot[depth];
  const size_t bytes = sizeof(float) * (size_t)M * p->D;
  cudaError_t e = cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->comp, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking);
  for (int i = 0; e == cudaSuccess && i < depth; i++) {
    Slot& s = p->slots[i];
    e = cudaMalloc(&s.x, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&s.out, bytes);
    if (e == cudaSuccess) e = cudaMemset(s.x, 0, bytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.in_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.compute_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.out_done, cudaEventDisableTiming);
    if (e == cudaSuccess) {
      st = iro_int8_swiglu_plan(&s.plan, s.x, M, w13, w2, b2, s.out, residual_w2);
      if (st != IRO_OK) break;
    }
  }
  if (e != cudaSuccess || st != IRO_OK) {
    if (st == IRO_OK) st = map_cuda(e);
    cudaGetLastError();
    iro_int8_swiglu_pipe_free(p);
    return st;
  }
  *pipe = p;
  return IRO_OK;
}

int iro_int8_swiglu_pipe_submit(IroSwigluPipe* p, const float* x_host, float* out_host) {
  if (!p || !x_host || !out_host) return IRO_ERR_INVALID;
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != p->device) return IRO_ERR_INVALID;
  Slot& s = p->slots[p->next];
  p->next = (p->next + 1) % p->depth;
  const size_t bytes = sizeof(float) * (size_t)p->M * p->D;
  cudaError_t e = cudaSuccess;
  // The slot's buffers are free once its previous result has been copied out.
  if (s.used) e = cudaStreamWaitEvent(p->h2d, s.out_done, 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(s.x, x_host, bytes, cudaMemcpyHostToDevice, p->h2d);
  if (e == cudaSuccess) e = cudaEventRecord(s.in_done, p->h2d);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(p->comp, s.in_done, 0);
  if (e == cudaSuccess) e = cudaGraphLaunch(s.plan->exec, p->comp);
  if (e == cudaSuccess) e = cudaEventRecord(s.compute_done, p->comp);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(p->d2h, s.compute_done, 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out_host, s.out, bytes, cudaMemcpyDeviceToHost, p->d2h);
  if (e == cudaSuccess) e = cudaEventRecord(s.out_done, p->d2h);
  s.used = true;
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

int iro_int8_swiglu_pipe_wait(IroSwigluPipe* p) {
  if (!p) return IRO_ERR_INVALID;
  cudaError_t e = cudaStreamSynchronize(p->d2h);
  if (e == cudaSuccess) e = cudaStreamSynchronize(p->comp);
  if (e == cudaSuccess) e = cudaStreamSynchronize(p->h2d);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  const int dev = take_device_error(c);
  return dev ? dev : IRO_OK;
}

}  // extern "C"
