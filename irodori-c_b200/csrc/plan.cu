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

}  // extern "C"
