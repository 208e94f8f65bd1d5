// abi.cu — the extern "C" entry points of libirodori_b200.so.
//
// Part 1 mirrors irodori-c's ops.h int8 API (host pointers, same argument
// meaning, same 0/-1 and void conventions).  Part 2 is the device-pointer,
// stream-ordered family the fast path uses.  Every entry point runs on the
// GPU; with no usable device they fail (status or iro_cuda_last_error()).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "diag.cuh"
#include "gemm_i8.cuh"
#include "quantize.cuh"

using namespace iro;

namespace {

// RAII lock + context lookup for the host-pointer entry points.
struct HostCall {
  Ctx* c = nullptr;
  int status = IRO_OK;
  std::unique_lock<std::mutex> lock;
  HostCall() {
    c = ctx_current(&status);
    if (c) lock = std::unique_lock<std::mutex>(c->mu);
  }
};

int cuda_st(cudaError_t e) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

// Finish a synchronous host-pointer call: wait for the stream, then fold in
// any error the kernels reported through the device error word.
int finish(Ctx* c, int st) {
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (st == IRO_OK && e != cudaSuccess) st = map_cuda(e);
  int dev = take_device_error(c);
  if (st == IRO_OK && dev != 0) st = dev;
  return st;
}

uint64_t fnv(uint64_t h, const void* p, size_t n) {
  const unsigned char* b = static_cast<const unsigned char*>(p);
  for (size_t i = 0; i < n; i++) {
    h ^= b[i];
    h *= 1099511628211ull;
  }
  return h;
}

uint64_t weight_fingerprint(const IroInt8Weight* w) {
  uint64_t h = 1469598103934665603ull;
  h = fnv(h, &w->N, sizeof(int));
  h = fnv(h, &w->K, sizeof(int));
  h = fnv(h, w->scale, sizeof(float) * (size_t)w->N);
  h = fnv(h, w->colsum, sizeof(int32_t) * (size_t)w->N);
  return h;
}

void dev_weight_release(IroInt8DevWeight* w) {
  if (!w) return;
  if (w->data) cudaFree(w->data);
  if (w->scale) cudaFree(w->scale);
  if (w->colsum) cudaFree(w->colsum);
  if (w->bias) cudaFree(w->bias);
  memset(w, 0, sizeof(*w));
}

// Allocate a device weight of N rows x K, ld = K rounded to 16, zeroed.
int dev_weight_alloc(IroInt8DevWeight* w, int N, int K, bool with_bias) {
  memset(w, 0, sizeof(*w));
  w->N = N;
  w->K = K;
  w->ld = round_up(K, 16);
  cudaGetDevice(&w->device);
  cudaError_t e = cudaMalloc(&w->data, (size_t)N * w->ld);
  if (e == cudaSuccess) e = cudaMemset(w->data, 0, (size_t)N * w->ld);
  if (e == cudaSuccess) e = cudaMalloc(&w->scale, sizeof(float) * (size_t)N);
  if (e == cudaSuccess) e = cudaMalloc(&w->colsum, sizeof(int32_t) * (size_t)N);
  if (e == cudaSuccess && with_bias) e = cudaMalloc(&w->bias, sizeof(float) * (size_t)N);
  if (e != cudaSuccess) {
    int st = cuda_st(e);
    dev_weight_release(w);
    return st;
  }
  return IRO_OK;
}

// Upload host rows [N,K] (pitch K) into the device weight at row `row0`.
int upload_rows(IroInt8DevWeight* w, int row0, const int8_t* data, const float* scale,
                const int32_t* colsum, const float* bias, int N, int K) {
  cudaError_t e = cudaMemcpy2D(w->data + (size_t)row0 * w->ld, (size_t)w->ld, data, (size_t)K,
                               (size_t)K, (size_t)N, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(w->scale + row0, scale, sizeof(float) * (size_t)N, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(w->colsum + row0, colsum, sizeof(int32_t) * (size_t)N,
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess && w->bias) {
    if (bias)
      e = cudaMemcpy(w->bias + row0, bias, sizeof(float) * (size_t)N, cudaMemcpyHostToDevice);
    else
      e = cudaMemset(w->bias + row0, 0, sizeof(float) * (size_t)N);
  }
  return cuda_st(e);
}

// Device copy of a host weight for the host-pointer API (cached).
const IroInt8DevWeight* cached_weight(Ctx* c, const IroInt8Weight* w, int* status) {
  const uint64_t fp = weight_fingerprint(w);
  auto it = c->wcache.find(w->data);
  if (it != c->wcache.end()) {
    if (it->second.fingerprint == fp && it->second.dev.N == w->N && it->second.dev.K == w->K) {
      *status = IRO_OK;
      return &it->second.dev;
    }
    dev_weight_release(&it->second.dev);
    c->wcache.erase(it);
  }
  CachedWeight cw;
  int st = dev_weight_alloc(&cw.dev, w->N, w->K, false);
  if (st == IRO_OK) st = upload_rows(&cw.dev, 0, w->data, w->scale, w->colsum, nullptr, w->N, w->K);
  if (st != IRO_OK) {
    dev_weight_release(&cw.dev);
    *status = st;
    return nullptr;
  }
  cw.fingerprint = fp;
  auto res = c->wcache.emplace(w->data, cw);
  *status = IRO_OK;
  return &res.first->second.dev;
}

void evict_weight(const void* data) {
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  for (int d = 0; d < 64; d++) {
    Ctx* c = ctx_existing(d);
    if (!c) continue;
    std::lock_guard<std::mutex> lock(c->mu);
    auto it = c->wcache.find(data);
    if (it != c->wcache.end()) {
      cudaSetDevice(d);
      dev_weight_release(&it->second.dev);
      c->wcache.erase(it);
    }
  }
  cudaSetDevice(cur);
}

// Device weight quantisation into `dst` (allocated here), from device fp32.
int quantize_into(Ctx* c, IroInt8DevWeight* dst, const float* w_dev, int N, int K,
                  cudaStream_t s) {
  int st = dev_weight_alloc(dst, N, K, false);
  if (st) return st;
  st = weight_quantize_launch(w_dev, N, K, dst->data, dst->ld, dst->scale, dst->colsum, s);
  if (st) dev_weight_release(dst);
  return st;
}

int host_weight_quantize(IroInt8Weight* dst, const float* w, int N, int K, bool transposed) {
  if (!dst || !w || N <= 0 || K <= 0) return -1;
  memset(dst, 0, sizeof(*dst));
  HostCall hc;
  if (!hc.c) {
    set_last_error(hc.status);
    return -1;
  }
  Ctx* c = hc.c;
  const size_t nk = (size_t)N * K;
  dst->data = static_cast<int8_t*>(malloc(nk));
  dst->scale = static_cast<float*>(malloc(sizeof(float) * (size_t)N));
  dst->colsum = static_cast<int32_t*>(malloc(sizeof(int32_t) * (size_t)N));
  if (!dst->data || !dst->scale || !dst->colsum) {
    free(dst->data); free(dst->scale); free(dst->colsum);
    memset(dst, 0, sizeof(*dst));
    set_last_error(IRO_ERR_OOM);
    return -1;
  }
  int st = IRO_OK;
  float* w_dev = static_cast<float*>(arena_get(c, sizeof(float) * nk * (transposed ? 2 : 1), &st));
  CachedWeight cw;
  memset(&cw, 0, sizeof(cw));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(w_dev, w, sizeof(float) * nk, cudaMemcpyHostToDevice, c->stream));
  const float* src = w_dev;
  if (st == IRO_OK && transposed) {
    float* t = w_dev + nk;
    st = transpose_f32_launch(w_dev, K, N, t, c->stream);
    src = t;
  }
  if (st == IRO_OK) st = quantize_into(c, &cw.dev, src, N, K, c->stream);
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpy2DAsync(dst->data, (size_t)K, cw.dev.data, (size_t)cw.dev.ld,
                                   (size_t)K, (size_t)N, cudaMemcpyDeviceToHost, c->stream));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(dst->scale, cw.dev.scale, sizeof(float) * N,
                                 cudaMemcpyDeviceToHost, c->stream));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(dst->colsum, cw.dev.colsum, sizeof(int32_t) * N,
                                 cudaMemcpyDeviceToHost, c->stream));
  st = finish(c, st);
  if (st != IRO_OK) {
    dev_weight_release(&cw.dev);
    free(dst->data); free(dst->scale); free(dst->colsum);
    memset(dst, 0, sizeof(*dst));
    set_last_error(st);
    return -1;
  }
  dst->N = N;
  dst->K = K;
  // The device copy just made is exactly the host result: keep it for the
  // linears that follow.
  auto it = c->wcache.find(dst->data);
  if (it != c->wcache.end()) {
    dev_weight_release(&it->second.dev);
    c->wcache.erase(it);
  }
  cw.fingerprint = weight_fingerprint(dst);
  c->wcache.emplace(dst->data, cw);
  return 0;
}

// Host-pointer linear shared by iro_int8_linear_ex and the selfcheck.
int host_linear(const uint8_t* q, const float* scale, const int32_t* zero,
                const IroInt8Weight* w, const float* bias, float* y, int M, int32_t* work,
                int accumulate) {
  if (!q || !scale || !zero || !w || !w->data || !y || M < 0) return IRO_ERR_INVALID;
  if (M == 0) return IRO_OK;
  HostCall hc;
  if (!hc.c) return hc.status;
  Ctx* c = hc.c;
  const int N = w->N, K = w->K;
  int st = IRO_OK;
  const IroInt8DevWeight* dw = cached_weight(c, w, &st);
  if (!dw) return st;
  const int ldq = round_up(K, 16);
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  const size_t o_q = carve((size_t)M * ldq);
  const size_t o_s = carve(sizeof(float) * M);
  const size_t o_z = carve(sizeof(int32_t) * M);
  const size_t o_b = carve(sizeof(float) * N);
  const size_t o_y = carve(sizeof(float) * (size_t)M * N);
  const size_t o_w = carve(sizeof(int32_t) * (size_t)M * N);
  uint8_t* base = static_cast<uint8_t*>(arena_get(c, off, &st));
  if (!base) return st;
  uint8_t* q_d = base + o_q;
  float* s_d = reinterpret_cast<float*>(base + o_s);
  int32_t* z_d = reinterpret_cast<int32_t*>(base + o_z);
  float* b_d = bias ? reinterpret_cast<float*>(base + o_b) : nullptr;
  float* y_d = reinterpret_cast<float*>(base + o_y);
  int32_t* w_d = reinterpret_cast<int32_t*>(base + o_w);
  cudaStream_t s = c->stream;
  if (ldq != K) st = cuda_st(cudaMemsetAsync(q_d, 0, (size_t)M * ldq, s));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpy2DAsync(q_d, ldq, q, K, K, M, cudaMemcpyHostToDevice, s));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(s_d, scale, sizeof(float) * M, cudaMemcpyHostToDevice, s));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(z_d, zero, sizeof(int32_t) * M, cudaMemcpyHostToDevice, s));
  if (st == IRO_OK && bias)
    st = cuda_st(cudaMemcpyAsync(b_d, bias, sizeof(float) * N, cudaMemcpyHostToDevice, s));
  if (st == IRO_OK && accumulate)
    st = cuda_st(cudaMemcpyAsync(y_d, y, sizeof(float) * (size_t)M * N, cudaMemcpyHostToDevice, s));
  if (st == IRO_OK) {
    GemmRequest r;
    r.epi = EPI_LINEAR;
    r.M = M;
    r.a = q_d;
    r.lda = ldq;
    r.sx = s_d;
    r.zp = z_d;
    r.w = dw;
    r.bias = b_d;
    r.y = y_d;
    r.ldy = N;
    r.work = w_d;
    r.ldw = N;
    r.accumulate = accumulate;
    st = gemm_launch(c, r, s);
  }
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(y, y_d, sizeof(float) * (size_t)M * N, cudaMemcpyDeviceToHost, s));
  if (st == IRO_OK && work)
    st = cuda_st(cudaMemcpyAsync(work, w_d, sizeof(int32_t) * (size_t)M * N,
                                 cudaMemcpyDeviceToHost, s));
  return finish(c, st);
}

int host_quantize(const float* x, int M, int K, uint8_t* q, float* scale, int32_t* zero,
                  float* residual, uint8_t* q2, float* scale2, int32_t* zero2, bool resid) {
  if (!x || !q || !scale || !zero || M < 0 || K <= 0) return IRO_ERR_INVALID;
  if (resid && (!residual || !q2 || !scale2 || !zero2)) return IRO_ERR_INVALID;
  if (M == 0) return IRO_OK;
  HostCall hc;
  if (!hc.c) return hc.status;
  Ctx* c = hc.c;
  const size_t mk = (size_t)M * K;
  const size_t fx = (sizeof(float) * mk + 255) / 256 * 256;
  const size_t fq = (mk + 255) / 256 * 256;
  const size_t fm = (sizeof(float) * M + 255) / 256 * 256;
  size_t total = fx + fq + 2 * fm;
  if (resid) total += fx + fq + 2 * fm;
  int st = IRO_OK;
  uint8_t* base = static_cast<uint8_t*>(arena_get(c, total, &st));
  if (!base) return st;
  float* x_d = reinterpret_cast<float*>(base);
  uint8_t* q_d = base + fx;
  float* s_d = reinterpret_cast<float*>(base + fx + fq);
  int32_t* z_d = reinterpret_cast<int32_t*>(base + fx + fq + fm);
  uint8_t* b2 = base + fx + fq + 2 * fm;
  float* r_d = reinterpret_cast<float*>(b2);
  uint8_t* q2_d = b2 + fx;
  float* s2_d = reinterpret_cast<float*>(b2 + fx + fq);
  int32_t* z2_d = reinterpret_cast<int32_t*>(b2 + fx + fq + fm);
  cudaStream_t s = c->stream;
  st = cuda_st(cudaMemcpyAsync(x_d, x, sizeof(float) * mk, cudaMemcpyHostToDevice, s));
  if (st == IRO_OK)
    st = resid ? quantize_rows_residual_launch(x_d, M, K, q_d, s_d, z_d, r_d, q2_d, s2_d, z2_d, s)
               : quantize_rows_launch(x_d, M, K, q_d, s_d, z_d, 0, s);
  if (st == IRO_OK) st = cuda_st(cudaMemcpyAsync(q, q_d, mk, cudaMemcpyDeviceToHost, s));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(scale, s_d, sizeof(float) * M, cudaMemcpyDeviceToHost, s));
  if (st == IRO_OK)
    st = cuda_st(cudaMemcpyAsync(zero, z_d, sizeof(int32_t) * M, cudaMemcpyDeviceToHost, s));
  if (resid) {
    if (st == IRO_OK)
      st = cuda_st(cudaMemcpyAsync(residual, r_d, sizeof(float) * mk, cudaMemcpyDeviceToHost, s));
    if (st == IRO_OK) st = cuda_st(cudaMemcpyAsync(q2, q2_d, mk, cudaMemcpyDeviceToHost, s));
    if (st == IRO_OK)
      st = cuda_st(cudaMemcpyAsync(scale2, s2_d, sizeof(float) * M, cudaMemcpyDeviceToHost, s));
    if (st == IRO_OK)
      st = cuda_st(cudaMemcpyAsync(zero2, z2_d, sizeof(int32_t) * M, cudaMemcpyDeviceToHost, s));
  }
  return finish(c, st);
}

// Returns a TMA-readable view of q (rows of K bytes): q itself when K is a
// multiple of 16, else a zero-padded copy in the context arena.
const uint8_t* tma_view(Ctx* c, const uint8_t* q, int M, int K, int* ld, cudaStream_t s,
                        size_t arena_off, int* status) {
  if (K % 16 == 0 && (reinterpret_cast<uintptr_t>(q) & 15u) == 0) {
    *ld = K;
    *status = IRO_OK;
    return q;
  }
  const int ldq = round_up(K, 16);
  uint8_t* base = static_cast<uint8_t*>(arena_get(c, arena_off + (size_t)M * ldq, status));
  if (!base) return nullptr;
  uint8_t* dst = base + arena_off;
  *status = repack_rows_launch(q, M, K, dst, ldq, s);
  *ld = ldq;
  return *status == IRO_OK ? dst : nullptr;
}

}  // namespace

extern "C" {

// ============================ Part 1: ops.h ===============================

int iro_int8_weight_quantize(IroInt8Weight* dst, const float* w, int N, int K) {
  return host_weight_quantize(dst, w, N, K, false);
}

int iro_int8_weight_quantize_transposed(IroInt8Weight* dst, const float* w, int N, int K) {
  return host_weight_quantize(dst, w, N, K, true);
}

void iro_int8_weight_free(IroInt8Weight* w) {
  if (!w) return;
  if (w->data) evict_weight(w->data);
  free(w->data);
  free(w->scale);
  free(w->colsum);
  memset(w, 0, sizeof(*w));
}

size_t iro_int8_weight_bytes(const IroInt8Weight* w) {
  if (!w || !w->data) return 0;
  return (size_t)w->N * w->K + (size_t)w->N * (sizeof(float) + sizeof(int32_t));
}

void iro_int8_quantize_rows(const float* x, int M, int K, uint8_t* q, float* scale,
                            int32_t* zero) {
  int st = host_quantize(x, M, K, q, scale, zero, nullptr, nullptr, nullptr, nullptr, false);
  set_last_error(st);
}

void iro_int8_quantize_rows_residual(const float* x, int M, int K, uint8_t* q1, float* scale1,
                                     int32_t* zero1, float* residual, uint8_t* q2,
                                     float* scale2, int32_t* zero2) {
  int st = host_quantize(x, M, K, q1, scale1, zero1, residual, q2, scale2, zero2, true);
  set_last_error(st);
}

void iro_int8_linear(const uint8_t* q, const float* scale, const int32_t* zero,
                     const IroInt8Weight* w, const float* bias, float* y, int M, int32_t* work) {
  set_last_error(host_linear(q, scale, zero, w, bias, y, M, work, 0));
}

void iro_int8_linear_ex(const uint8_t* q, const float* scale, const int32_t* zero,
                        const IroInt8Weight* w, const float* bias, float* y, int M,
                        int32_t* work, int accumulate) {
  set_last_error(host_linear(q, scale, zero, w, bias, y, M, work, accumulate));
}

int iro_int8_fast_available(void) { return iro_cuda_device_count() > 0 ? 1 : 0; }

const char* iro_int8_prepare_backend(void) {
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) {
    set_last_error(st);
    return nullptr;
  }
  return "cuda-sm100a-tcgen05-i8";
}

int iro_int8_selfcheck(void) {
  // ops.c:375-398: 255*127 products overflow int16; the sums must be exact.
  enum { M = 3, N = 5, K = 64 };
  uint8_t a[M * K];
  int8_t b[N * K];
  for (int i = 0; i < M * K; i++) a[i] = (uint8_t)(i % 3 == 0 ? 255 : 200 + i % 50);
  for (int i = 0; i < N * K; i++)
    b[i] = (int8_t)(i % 4 == 0 ? 127 : (i % 4 == 1 ? -127 : 90 - i % 60));
  int32_t want[M * N], got[M * N];
  for (int m = 0; m < M; m++)
    for (int n = 0; n < N; n++) {
      int32_t acc = 0;
      for (int k = 0; k < K; k++) acc += (int32_t)a[m * K + k] * (int32_t)b[n * K + k];
      want[m * N + n] = acc;
    }
  float wscale[N] = {1.0f, 1.0f, 1.0f, 1.0f, 1.0f};
  int32_t colsum[N] = {0, 0, 0, 0, 0};
  IroInt8Weight w = {b, wscale, colsum, N, K};
  float sx[M] = {1.0f, 1.0f, 1.0f}, y[M * N];
  int32_t zero[M] = {0, 0, 0};
  memset(got, 0, sizeof(got));
  int st = host_linear(a, sx, zero, &w, nullptr, y, M, got, 0);
  evict_weight(b);
  if (st != IRO_OK) {
    set_last_error(st);
    return -1;
  }
  return memcmp(got, want, sizeof(got)) == 0 ? 0 : -1;
}

const char* iro_ops_backend_name(void) { return "cuda-sm100a"; }

// ======================= Part 2: device weights ===========================

int iro_int8_dev_weight_upload(IroInt8DevWeight* dst, const IroInt8Weight* src,
                               const float* bias) {
  if (!dst || !src || !src->data || src->N <= 0 || src->K <= 0) return IRO_ERR_INVALID;
  int st;
  if (!ctx_current(&st)) return st;
  st = dev_weight_alloc(dst, src->N, src->K, bias != nullptr);
  if (st) return st;
  st = upload_rows(dst, 0, src->data, src->scale, src->colsum, bias, src->N, src->K);
  if (st) dev_weight_release(dst);
  return st;
}

int iro_int8_dev_weight_quantize(IroInt8DevWeight* dst, const float* w_dev, int N, int K,
                                 const float* bias_dev, void* stream) {
  if (!dst || !w_dev || N <= 0 || K <= 0) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  st = quantize_into(c, dst, w_dev, N, K, s);
  if (st) return st;
  if (bias_dev) {
    cudaError_t e = cudaMalloc(&dst->bias, sizeof(float) * (size_t)N);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dst->bias, bias_dev, sizeof(float) * (size_t)N,
                          cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) {
      dev_weight_release(dst);
      return cuda_st(e);
    }
  }
  if (stream == nullptr) {
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_st(e);
  }
  return IRO_OK;
}

int iro_int8_dev_weight_concat(IroInt8DevWeight* dst, const IroInt8Weight* const* parts,
                               const float* const* biases, int nparts) {
  if (!dst || !parts || nparts <= 0) return IRO_ERR_INVALID;
  int N = 0, K = parts[0] ? parts[0]->K : 0;
  bool any_bias = false;
  for (int i = 0; i < nparts; i++) {
    if (!parts[i] || !parts[i]->data || parts[i]->K != K || parts[i]->N <= 0)
      return IRO_ERR_INVALID;
    N += parts[i]->N;
    if (biases && biases[i]) any_bias = true;
  }
  int st;
  if (!ctx_current(&st)) return st;
  st = dev_weight_alloc(dst, N, K, any_bias);
  if (st) return st;
  int row = 0;
  for (int i = 0; i < nparts && st == IRO_OK; i++) {
    st = upload_rows(dst, row, parts[i]->data, parts[i]->scale, parts[i]->colsum,
                     biases ? biases[i] : nullptr, parts[i]->N, K);
    row += parts[i]->N;
  }
  if (st) dev_weight_release(dst);
  return st;
}

int iro_int8_dev_weight_gated_pair(IroInt8DevWeight* dst, const IroInt8Weight* w1,
                                   const IroInt8Weight* w3, const float* b1, const float* b3) {
  if (!dst || !w1 || !w3 || !w1->data || !w3->data || w1->N != w3->N || w1->K != w3->K ||
      w1->N <= 0 || w1->K <= 0)
    return IRO_ERR_INVALID;
  const int pair = 128, H = w1->N, K = w1->K;
  const int Hp = round_up(H, pair);
  int st;
  if (!ctx_current(&st)) return st;
  st = dev_weight_alloc(dst, 2 * Hp, K, b1 != nullptr || b3 != nullptr);
  if (st) return st;
  // Padding rows (H..Hp) stay zero codes with zero scale: they dequantise
  // to 0 and are never stored.
  cudaError_t e = cudaMemset(dst->scale, 0, sizeof(float) * 2 * (size_t)Hp);
  if (e == cudaSuccess) e = cudaMemset(dst->colsum, 0, sizeof(int32_t) * 2 * (size_t)Hp);
  if (e == cudaSuccess && dst->bias) e = cudaMemset(dst->bias, 0, sizeof(float) * 2 * (size_t)Hp);
  st = cuda_st(e);
  for (int blk = 0; st == IRO_OK && blk < Hp / pair; blk++) {
    const int h0 = blk * pair;
    const int n = std::min(pair, H - h0);
    if (n <= 0) break;
    st = upload_rows(dst, blk * 2 * pair, w1->data + (size_t)h0 * K, w1->scale + h0,
                     w1->colsum + h0, b1 ? b1 + h0 : nullptr, n, K);
    if (st == IRO_OK)
      st = upload_rows(dst, blk * 2 * pair + pair, w3->data + (size_t)h0 * K, w3->scale + h0,
                       w3->colsum + h0, b3 ? b3 + h0 : nullptr, n, K);
  }
  if (st) {
    dev_weight_release(dst);
    return st;
  }
  dst->layout = IRO_LAYOUT_GATED_PAIR;
  dst->pair = pair;
  dst->hidden = H;
  return IRO_OK;
}

void iro_int8_dev_weight_free(IroInt8DevWeight* w) { dev_weight_release(w); }

// ========================= Part 2: quantisers =============================

int iro_int8_quantize_rows_dev(const float* x, int M, int K, uint8_t* q, float* scale,
                               int32_t* zero, void* stream) {
  if (!x || !q || !scale || !zero) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  return quantize_rows_launch(x, M, K, q, scale, zero, 0, pick_stream(c, stream));
}

int iro_int8_quantize_rows_sym_dev(const float* x, int M, int K, uint8_t* q, float* scale,
                                   int32_t* zero, void* stream) {
  if (!x || !q || !scale || !zero) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  return quantize_rows_launch(x, M, K, q, scale, zero, 1, pick_stream(c, stream));
}

int iro_int8_quantize_rows_residual_dev(const float* x, int M, int K, uint8_t* q1,
                                        float* scale1, int32_t* zero1, float* residual,
                                        uint8_t* q2, float* scale2, int32_t* zero2,
                                        void* stream) {
  if (!x || !q1 || !scale1 || !zero1 || !q2 || !scale2 || !zero2) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  return quantize_rows_residual_launch(x, M, K, q1, scale1, zero1, residual, q2, scale2, zero2,
                                       pick_stream(c, stream));
}

// ========================= Part 2: GEMMs ==================================

int iro_int8_linear_dev(const uint8_t* q, const float* scale, const int32_t* zero,
                        const IroInt8DevWeight* w, const float* bias, float* y, int M,
                        int32_t* work, int accumulate, void* stream) {
  if (!w || w->layout != IRO_LAYOUT_PLAIN) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  int lda = 0;
  const uint8_t* a = tma_view(c, q, M, w->K, &lda, s, 0, &st);
  if (!a) return st;
  GemmRequest r;
  r.epi = EPI_LINEAR;
  r.M = M;
  r.a = a;
  r.lda = lda;
  r.sx = scale;
  r.zp = zero;
  r.w = w;
  r.bias = bias;
  r.y = y;
  r.ldy = w->N;
  r.work = work;
  r.ldw = w->N;
  r.accumulate = accumulate;
  return gemm_launch(c, r, s);
}

int iro_int8_linear2_dev(const uint8_t* q1, const float* scale1, const int32_t* zero1,
                         const uint8_t* q2, const float* scale2, const int32_t* zero2,
                         const IroInt8DevWeight* w, const float* bias, float* y, int M,
                         void* stream) {
  if (!w || w->layout != IRO_LAYOUT_PLAIN) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  if (w->K % 16 != 0) return IRO_ERR_UNSUPPORTED;
  GemmRequest r;
  r.epi = EPI_DUAL;
  r.M = M;
  r.a = q1;
  r.lda = w->K;
  r.sx = scale1;
  r.zp = zero1;
  r.a2 = q2;
  r.sx2 = scale2;
  r.zp2 = zero2;
  r.w = w;
  r.bias = bias;
  r.y = y;
  r.ldy = w->N;
  return gemm_launch(c, r, s);
}

int iro_int8_linear_split_dev(const uint8_t* q, const float* scale, const int32_t* zero,
                              const IroInt8DevWeight* w, float* const* outputs, int nout,
                              int seg, int M, void* stream) {
  if (!w || !outputs || w->layout != IRO_LAYOUT_PLAIN) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  int lda = 0;
  const uint8_t* a = tma_view(c, q, M, w->K, &lda, s, 0, &st);
  if (!a) return st;
  GemmRequest r;
  r.epi = EPI_SPLIT;
  r.M = M;
  r.a = a;
  r.lda = lda;
  r.sx = scale;
  r.zp = zero;
  r.w = w;
  r.bias = w->bias;
  r.nout = nout;
  r.seg = seg;
  for (int i = 0; i < nout && i < 4; i++) r.outs[i] = outputs[i];
  return gemm_launch(c, r, s);
}

int iro_int8_gated_dev(const uint8_t* q, const float* scale, const int32_t* zero,
                       const IroInt8DevWeight* w13, float* hidden, int M, void* stream) {
  if (!w13 || w13->layout != IRO_LAYOUT_GATED_PAIR) return IRO_ERR_INVALID;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  cudaStream_t s = pick_stream(c, stream);
  int lda = 0;
  const uint8_t* a = tma_view(c, q, M, w13->K, &lda, s, 0, &st);
  if (!a) return st;
  GemmRequest r;
  r.epi = EPI_GATED;
  r.M = M;
  r.a = a;
  r.lda = lda;
  r.sx = scale;
  r.zp = zero;
  r.w = w13;
  r.hidden = hidden;
  r.ldh = w13->hidden;
  return gemm_launch(c, r, s);
}

// ========================= Part 2: SwiGLU block ============================

size_t iro_int8_swiglu_workspace_bytes(int M, int D, int H, int residual_w2) {
  if (M <= 0 || D <= 0 || H <= 0) return 0;
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  size_t t = al((size_t)M * round_up(D, 16)) + 2 * al(sizeof(float) * M) +  // qx, sx, zx
             al(sizeof(float) * (size_t)M * H) +                           // hidden
             al((size_t)M * round_up(H, 16)) + 2 * al(sizeof(float) * M);   // qh, sh, zh
  if (residual_w2) t += al((size_t)M * round_up(H, 16)) + 2 * al(sizeof(float) * M);
  return t;
}

int iro_int8_swiglu_dev(const float* x, int M, const IroInt8DevWeight* w13,
                        const IroInt8DevWeight* w2, const float* b2, float* out,
                        int residual_w2, void* workspace, void* stream) {
  if (!x || !out || !w13 || !w2 || M < 0) return IRO_ERR_INVALID;
  if (M == 0) return IRO_OK;
  int st;
  Ctx* c = ctx_current(&st);
  if (!c) return st;
  return swiglu_run(c, x, M, w13, w2, b2, out, residual_w2, workspace, pick_stream(c, stream),
                    nullptr, 0);
}

}  // extern "C"

namespace iro {

// silu(w1) * w3 from the W1|W3 pair-block layout (pair W1 columns, then the
// matching pair W3 columns): the reference's iro_silu_mul_inplace
// (ops.c:781-784), x / (1 + expf(-x)) * gate.
__global__ void silu_mul_pairs_kernel(const float* __restrict__ o13, int ld, int pair, int M,
                                      int H, float* __restrict__ hid) {
  const long long n = (long long)M * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / H;
    const int h = (int)(i - m * H);
    const int blk = h / pair, j = h - blk * pair;
    const float* row = o13 + (size_t)m * ld + (size_t)blk * 2 * pair;
    const float a = row[j], g = row[pair + j];
    hid[i] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), g);
  }
}

size_t swiglu_workspace_bytes_ex(int M, int D, int H, int residual_w2, int residual_w13) {
  size_t t = iro_int8_swiglu_workspace_bytes(M, D, H, residual_w2);
  if (t == 0 || !residual_w13) return t;
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  return t + al((size_t)M * round_up(D, 16)) + 2 * al(sizeof(float) * M) +
         al(sizeof(float) * (size_t)M * 2 * round_up(H, 128));
}

int swiglu_run(Ctx* c, const float* x, int M, const IroInt8DevWeight* w13,
               const IroInt8DevWeight* w2, const float* b2, float* out, int residual_w2,
               void* workspace, cudaStream_t s, const float* rgate, int rgate_rows,
               const uint8_t* qx_in, const float* sx_in, const int32_t* zx_in,
               int residual_w13, int stats_layer) {
  if (residual_w13 && !x) return IRO_ERR_INVALID;
  if ((!x && !(qx_in && sx_in && zx_in)) || !out || !w13 || !w2 ||
      w13->layout != IRO_LAYOUT_GATED_PAIR ||
      w2->layout != IRO_LAYOUT_PLAIN || w2->K != w13->hidden || M < 0)
    return IRO_ERR_INVALID;
  const int D = w13->K, H = w13->hidden;
  if (w2->N != D) return IRO_ERR_INVALID;
  if (D % 16 != 0 || H % 16 != 0) return IRO_ERR_UNSUPPORTED;
  if (M == 0) return IRO_OK;
  int st;
  const size_t need = swiglu_workspace_bytes_ex(M, D, H, residual_w2, residual_w13);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!ws) {
    ws = static_cast<uint8_t*>(arena_get(c, need, &st));
    if (!ws) return st;
  }
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = ws + off;
    off += al(bytes);
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
  if (residual_w13) {
    // Two-term W1/W3: both activation terms through the pair-block weight
    // as one two-term linear (y = lin(q1) + lin(q2), dit.c:479-486), then
    // the gate.  The extra buffers follow the single-term workspace.
    const size_t base = iro_int8_swiglu_workspace_bytes(M, D, H, residual_w2);
    size_t off2 = base;
    auto take2 = [&](size_t bytes) {
      uint8_t* p = ws + off2;
      off2 += al(bytes);
      return p;
    };
    uint8_t* qx2 = take2((size_t)M * D);
    float* sx2 = reinterpret_cast<float*>(take2(sizeof(float) * M));
    int32_t* zx2 = reinterpret_cast<int32_t*>(take2(sizeof(float) * M));
    float* o13 = reinterpret_cast<float*>(take2(sizeof(float) * (size_t)M * w13->N));
    st = quantize_rows_residual_launch(x, M, D, qx, sx, zx, nullptr, qx2, sx2, zx2, s);
    if (st) return st;
    GemmRequest r13;
    r13.epi = EPI_DUAL;
    r13.M = M;
    r13.a = qx;
    r13.lda = D;
    r13.sx = sx;
    r13.zp = zx;
    r13.a2 = qx2;
    r13.sx2 = sx2;
    r13.zp2 = zx2;
    r13.w = w13;
    r13.y = o13;
    r13.ldy = w13->N;
    if ((st = gemm_launch(c, r13, s))) return st;
    const long long n = (long long)M * H;
    const int blocks = (int)std::min<long long>((n + 255) / 256, (long long)c->num_sms * 16);
    silu_mul_pairs_kernel<<<blocks, 256, 0, s>>>(o13, w13->N, w13->pair, M, H, hid);
    if ((st = check_launch())) return st;
  } else {
  if (qx_in) {
    qx = const_cast<uint8_t*>(qx_in);
    sx = const_cast<float*>(sx_in);
    zx = const_cast<int32_t*>(zx_in);
  } else {
    st = quantize_rows_launch(x, M, D, qx, sx, zx, 0, s);
    if (st) return st;
  }
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
  st = gemm_launch(c, g, s);
  if (st) return st;
  }
  // W2 input diagnostics (dit.c:964).
  if (stats_layer >= 0 && (st = diag_record(stats_layer, 3, hid, M, H, s))) return st;
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
  r.rgate = rgate;
  r.rgate_rows = rgate_rows;
  if (residual_w2) {
    r.epi = EPI_DUAL;
    r.a2 = qh2;
    r.sx2 = sh2;
    r.zp2 = zh2;
  } else {
    r.epi = EPI_LINEAR;
  }
  return gemm_launch(c, r, s);
}

}  // namespace iro

extern "C" {

// True when `p` is page-locked host memory (async copies can overlap).
static bool is_pinned(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

int iro_int8_swiglu(const float* x, int M, const IroInt8DevWeight* w13,
                    const IroInt8DevWeight* w2, const float* b2, float* out, int residual_w2) {
  if (!x || !out || !w13 || !w2 || M < 0) return IRO_ERR_INVALID;
  if (M == 0) return IRO_OK;
  HostCall hc;
  if (!hc.c) return hc.status;
  Ctx* c = hc.c;
  const int D = w13->K;
  const size_t row_bytes = sizeof(float) * (size_t)D;
  // Rows are independent, so the block can run in row chunks: with page-locked
  // host buffers the copy in of chunk i+1, the compute of chunk i and the copy
  // out of chunk i-1 run at once on three streams.  Pageable buffers take one
  // synchronous pass.
  // A chunk must stay large enough that its compute (four kernel launches)
  // is shorter than its copies: ~512 rows, at most 8 chunks.
  const char* env = getenv("IRO_SWIGLU_CHUNK_ROWS");
  const int target = env && *env ? std::max(128, atoi(env)) : 512;
  const bool overlap = M >= 2 * target && is_pinned(x) && is_pinned(out);
  const int nchunk = overlap ? std::min(8, M / target) : 1;
  const int chunk = round_up(cdiv(M, nchunk), 128);
  const size_t xb = (row_bytes * (size_t)M + 255) / 256 * 256;
  const size_t wsb = iro_int8_swiglu_workspace_bytes(std::min(chunk, M), D, w13->hidden, residual_w2);
  int st = IRO_OK;
  uint8_t* base = static_cast<uint8_t*>(arena_get(c, 2 * xb + wsb, &st));
  if (!base) return st;
  float* x_d = reinterpret_cast<float*>(base);
  float* o_d = reinterpret_cast<float*>(base + xb);
  uint8_t* ws = base + 2 * xb;
  cudaStream_t s = c->stream;
  if (!overlap) {
    st = cuda_st(cudaMemcpyAsync(x_d, x, row_bytes * M, cudaMemcpyHostToDevice, s));
    if (st == IRO_OK) st = iro_int8_swiglu_dev(x_d, M, w13, w2, b2, o_d, residual_w2, ws, s);
    if (st == IRO_OK)
      st = cuda_st(cudaMemcpyAsync(out, o_d, row_bytes * M, cudaMemcpyDeviceToHost, s));
    return finish(c, st);
  }
  st = ctx_copy_resources(c, 2 * nchunk + 1);
  if (st) return st;
  cudaEvent_t* ev = c->events.data();
  for (int i = 0, r0 = 0; st == IRO_OK && r0 < M; i++, r0 += chunk) {
    const int rows = std::min(chunk, M - r0);
    const size_t off = (size_t)r0 * D;
    st = cuda_st(cudaMemcpyAsync(x_d + off, x + off, row_bytes * rows, cudaMemcpyHostToDevice,
                                 c->copy_in));
    if (st == IRO_OK) st = cuda_st(cudaEventRecord(ev[2 * i], c->copy_in));
    if (st == IRO_OK) st = cuda_st(cudaStreamWaitEvent(s, ev[2 * i], 0));
    if (st == IRO_OK)
      st = iro_int8_swiglu_dev(x_d + off, rows, w13, w2, b2, o_d + off, residual_w2, ws, s);
    if (st == IRO_OK) st = cuda_st(cudaEventRecord(ev[2 * i + 1], s));
    if (st == IRO_OK) st = cuda_st(cudaStreamWaitEvent(c->copy_out, ev[2 * i + 1], 0));
    if (st == IRO_OK)
      st = cuda_st(cudaMemcpyAsync(out + off, o_d + off, row_bytes * rows, cudaMemcpyDeviceToHost,
                                   c->copy_out));
  }
  cudaError_t e = cudaStreamSynchronize(c->copy_out);
  if (st == IRO_OK && e != cudaSuccess) st = map_cuda(e);
  cudaStreamSynchronize(c->copy_in);
  return finish(c, st);
}

}  // extern "C"
