// diag.cu — IRO_INT8_STATS / IRO_INT8_DUMP on the device path (dit.c:340-412).
//
// Stats: per (layer, group), the number of rows, the sum over rows of
// max|x| / rms(x) (rms from a double sum of squares) and the histogram of
// the channel holding each row's first maximum of |x|, accumulated on the
// device; iro_dit_stats_report() prints the reference's summary line per
// cell (also at exit when IRO_INT8_STATS is set, as the reference does).
// Dump: IRO_INT8_DUMP=dir writes the first three activations per (layer,
// group) as raw fp32 files named as the reference names them.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "diag.cuh"

namespace iro {
namespace {

struct StatCell {
  double ratio_sum;
  unsigned long long rows;
  unsigned int hist[kStatChannels];
};

constexpr int kCells = IRO_DIT_MAX_LAYERS * kStatGroups;

std::mutex g_mu;
StatCell* g_table = nullptr;  // device, kCells cells
int g_device = -1;
int g_dump_counts[IRO_DIT_MAX_LAYERS][kStatGroups];
bool g_atexit = false;

bool stats_on() {
  const char* e = getenv("IRO_INT8_STATS");
  return e && strcmp(e, "0") != 0;
}

const char* dump_dir() {
  const char* d = getenv("IRO_INT8_DUMP");
  return (d && *d) ? d : nullptr;
}

// One warp per row: double sum of squares, max |x| and its first channel.
__global__ void __launch_bounds__(256) row_stats_kernel(const float* __restrict__ x, int M, int K,
                                                        StatCell* __restrict__ cell) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float* r = x + (size_t)row * K;
  double ss = 0.0;
  float amax = 0.0f;
  int arg = 0;
  for (int k = lane; k < K; k += 32) {
    const float v = r[k];
    ss += (double)v * v;
    const float a = fabsf(v);
    if (a > amax) {  // first maximum of this lane's channels
      amax = a;
      arg = k;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
    const int oarg = __shfl_xor_sync(0xffffffffu, arg, o);
    if (oa > amax || (oa == amax && oarg < arg)) {
      amax = oa;
      arg = oarg;
    }
  }
  if (lane == 0) {
    const double rms = sqrt(ss / K);
    atomicAdd(&cell->ratio_sum, rms > 0 ? (double)amax / rms : 0.0);
    atomicAdd(&cell->rows, 1ull);
    if (arg < kStatChannels) atomicAdd(&cell->hist[arg], 1u);
  }
}

int ensure_table() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (g_table && g_device == dev) return IRO_OK;
  if (g_table) cudaFree(g_table);
  g_table = nullptr;
  cudaError_t e = cudaMalloc(&g_table, sizeof(StatCell) * kCells);
  if (e == cudaSuccess) e = cudaMemset(g_table, 0, sizeof(StatCell) * kCells);
  if (e != cudaSuccess) {
    cudaGetLastError();
    g_table = nullptr;
    return map_cuda(e);
  }
  g_device = dev;
  return IRO_OK;
}

void report_at_exit() { iro_dit_stats_report(); }

}  // namespace

bool diag_enabled() { return stats_on() || dump_dir() != nullptr; }

int diag_record(int layer, int group, const float* x, int M, int K, cudaStream_t s) {
  if (layer < 0 || layer >= IRO_DIT_MAX_LAYERS || group < 0 || group >= kStatGroups || M <= 0)
    return IRO_OK;
  std::lock_guard<std::mutex> lock(g_mu);
  if (const char* dir = dump_dir()) {
    if (g_dump_counts[layer][group] < 3) {
      std::vector<float> h((size_t)M * K);
      cudaError_t e =
          cudaMemcpyAsync(h.data(), x, sizeof(float) * h.size(), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) {
        cudaGetLastError();
        return map_cuda(e);
      }
      char path[512];
      snprintf(path, sizeof(path), "%s/act_L%02d_G%d_%d_M%d_K%d.f32", dir, layer, group,
               g_dump_counts[layer][group], M, K);
      if (FILE* f = fopen(path, "wb")) {
        fwrite(h.data(), sizeof(float), h.size(), f);
        fclose(f);
      }
      g_dump_counts[layer][group]++;
    }
  }
  if (!stats_on()) return IRO_OK;
  int st = ensure_table();
  if (st) return st;
  if (!g_atexit) {
    atexit(report_at_exit);
    g_atexit = true;
  }
  row_stats_kernel<<<cdiv(M, 8), 256, 0, s>>>(x, M, K, g_table + layer * kStatGroups + group);
  return check_launch();
}

}  // namespace iro

using namespace iro;

extern "C" {

int iro_dit_stats_read(int layer, int group, double* rows, double* ratio_sum,
                       unsigned int* hist, int hist_len) {
  if (layer < 0 || layer >= IRO_DIT_MAX_LAYERS || group < 0 || group >= kStatGroups || !rows ||
      !ratio_sum)
    return IRO_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_mu);
  *rows = 0;
  *ratio_sum = 0;
  if (!g_table) return IRO_OK;
  StatCell cell;
  cudaError_t e = cudaMemcpy(&cell, g_table + layer * kStatGroups + group, sizeof(cell),
                             cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  *rows = (double)cell.rows;
  *ratio_sum = cell.ratio_sum;
  if (hist)
    memcpy(hist, cell.hist, sizeof(unsigned int) * (size_t)std::min(hist_len, kStatChannels));
  return IRO_OK;
}

void iro_dit_stats_reset(void) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_table) cudaMemset(g_table, 0, sizeof(StatCell) * kCells);
  memset(g_dump_counts, 0, sizeof(g_dump_counts));
}

// dit.c:354-376: one line per recorded (layer, group).
void iro_dit_stats_report(void) {
  static const char* const names[kStatGroups] = {"qkvg", "wo", "w13", "w2"};
  std::vector<unsigned int> hist(kStatChannels);
  for (int layer = 0; layer < IRO_DIT_MAX_LAYERS; layer++) {
    for (int g = 0; g < kStatGroups; g++) {
      double rows = 0, ratio = 0;
      if (iro_dit_stats_read(layer, g, &rows, &ratio, hist.data(), kStatChannels) || rows <= 0)
        continue;
      unsigned int best = 0;
      int best_ch = -1, frequent = 0;
      for (int k = 0; k < kStatChannels; k++) {
        if (hist[k] > best) {
          best = hist[k];
          best_ch = k;
        }
        if ((double)hist[k] >= 0.05 * rows) frequent++;
      }
      fprintf(stderr,
              "int8-stats layer=%2d group=%-4s rows=%.0f mean_max/rms=%.2f "
              "top_channel=%d share=%.2f channels>=5%%=%d\n",
              layer, names[g], rows, ratio / rows, best_ch, (double)best / rows, frequent);
    }
  }
}

}  // extern "C"
