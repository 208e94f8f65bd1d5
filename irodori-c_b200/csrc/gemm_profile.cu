// gemm_profile.cu — per-shape GEMM profile, the reference's IRO_GEMM_PROFILE
// (ops.c:14-110) for the device GEMMs.
//
// With IRO_GEMM_PROFILE set (and not "0"), every gemm_launch records a CUDA
// event before and after its kernel on the launch stream.  Rows are keyed
// like the reference's (kind, M, N, K, lda, ldb, ldc, beta), at most 256 of
// them (later shapes count as dropped).  Event pairs stay pending until the
// JSON is emitted, or until 4096 are pending; then the host waits for the
// last one and folds the device times in (the reference times its host-side
// GEMM calls; here the time is the kernel's on the device).  The emitted line
// has the reference's schema: {"type":"iro_gemm_profile", "status", "backend",
// "steps", "sequence_length", "context_tokens", "dropped_shapes", "rows":
// [{"kind","M","N","K","lda","ldb","ldc","beta","backend","calls","seconds"}]}.
// Not thread-safe, like the reference's profile state.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "gemm_i8.cuh"

namespace iro {
namespace {

constexpr int kMaxShapes = 256;
constexpr size_t kMaxPending = 4096;

struct Row {
  const char* kind;
  int m, n, k, lda, ldb, ldc;
  float beta;
  unsigned long long calls;
  double seconds;
};

struct Pending {
  int row;  // index into rows, -1 when the shape was dropped
  cudaEvent_t start, stop;
};

int g_state = -1;
Row g_rows[kMaxShapes];
int g_count = 0;
unsigned long long g_dropped = 0;
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_free;

cudaEvent_t take_event() {
  if (!g_free.empty()) {
    cudaEvent_t e = g_free.back();
    g_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

// Fold every pending pair's device time into its row.
void resolve() {
  if (g_pending.empty()) return;
  cudaEventSynchronize(g_pending.back().stop);
  for (const Pending& p : g_pending) {
    float ms = 0.0f;
    if (p.row >= 0 && cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess) {
      g_rows[p.row].calls++;
      g_rows[p.row].seconds += 1e-3 * (double)ms;
    }
    g_free.push_back(p.start);
    g_free.push_back(p.stop);
  }
  cudaGetLastError();
  g_pending.clear();
}

int find_row(const char* kind, int m, int n, int k, int lda, int ldb, int ldc, float beta) {
  for (int i = 0; i < g_count; i++) {
    const Row& r = g_rows[i];
    if (r.kind == kind && r.m == m && r.n == n && r.k == k && r.lda == lda && r.ldb == ldb &&
        r.ldc == ldc && r.beta == beta)
      return i;
  }
  if (g_count >= kMaxShapes) {
    g_dropped++;
    return -1;
  }
  g_rows[g_count] = Row{kind, m, n, k, lda, ldb, ldc, beta, 0, 0.0};
  return g_count++;
}

const char* kind_of(const GemmRequest& r) {
  switch (r.epi) {
    case EPI_LINEAR: return r.rgate ? "linear_int8_gated_residual" : "linear_int8";
    case EPI_SPLIT: return "linear_int8_split";
    case EPI_GATED: return "gated_int8";
    case EPI_DUAL: return r.nout > 0 ? "linear2_int8_split" : "linear2_int8";
    case EPI_QKV: return "qkvg_int8";
    default: return "gemm_int8";
  }
}

}  // namespace

bool gemm_profile_on() {
  if (g_state < 0) {
    const char* e = getenv("IRO_GEMM_PROFILE");
    g_state = (e && strcmp(e, "0") != 0) ? 1 : 0;
  }
  return g_state == 1;
}

void* gemm_profile_begin(const GemmRequest& r, cudaStream_t s) {
  if (!gemm_profile_on() || r.no_alloc) return nullptr;
  cudaEvent_t a = take_event(), b = take_event();
  if (!a || !b) return nullptr;
  cudaEventRecord(a, s);
  Pending* p = new Pending{-1, a, b};
  return p;
}

void gemm_profile_end(void* token, const GemmRequest& r, cudaStream_t s) {
  if (!token) return;
  Pending* p = static_cast<Pending*>(token);
  cudaEventRecord(p->stop, s);
  const IroInt8DevWeight* w = r.w;
  const int ldc = r.epi == EPI_GATED ? r.ldh : (r.nout > 0 ? r.seg : r.ldy);
  const float beta = (r.accumulate || r.rgate) ? 1.0f : 0.0f;
  p->row = find_row(kind_of(r), r.M, w->N, w->K, r.lda, w->ld, ldc, beta);
  g_pending.push_back(*p);
  delete p;
  if (g_pending.size() >= kMaxPending) resolve();
}

}  // namespace iro

using namespace iro;

extern "C" {

int iro_cuda_gemm_profile_enabled(void) { return gemm_profile_on() ? 1 : 0; }

void iro_cuda_gemm_profile_reset(void) {
  if (!gemm_profile_on()) return;
  resolve();
  memset(g_rows, 0, sizeof(g_rows));
  g_count = 0;
  g_dropped = 0;
}

void iro_cuda_gemm_profile_emit_json(const char* status, int steps, int sequence_length,
                                     int context_tokens) {
  if (!gemm_profile_on()) return;
  resolve();
  const char* backend = "cuda-sm100a-tcgen05-i8";
  fprintf(stderr,
          "{\"type\":\"iro_gemm_profile\",\"status\":\"%s\",\"backend\":\"%s\",\"steps\":%d,"
          "\"sequence_length\":%d,\"context_tokens\":%d,\"dropped_shapes\":%llu,\"rows\":[",
          status ? status : "unknown", backend, steps, sequence_length, context_tokens,
          g_dropped);
  for (int i = 0; i < g_count; i++) {
    const Row& r = g_rows[i];
    if (i) fputc(',', stderr);
    fprintf(stderr,
            "{\"kind\":\"%s\",\"M\":%d,\"N\":%d,\"K\":%d,\"lda\":%d,\"ldb\":%d,\"ldc\":%d,"
            "\"beta\":%.1f,\"backend\":\"%s\",\"calls\":%llu,\"seconds\":%.9f}",
            r.kind, r.m, r.n, r.k, r.lda, r.ldb, r.ldc, r.beta, backend, r.calls, r.seconds);
  }
  fputs("]}\n", stderr);
  fflush(stderr);
}

}  // extern "C"
