// gemm_splitk.cu — the plain int8 linear (EPI_LINEAR) for GEMMs with few
// tiles and long K, split over K across a two-CTA thread-block cluster.
//
// W2 of the config-2 block (M=2048, N=1024, K=2816) has 128 tiles of 128x128
// in the one-CTA kernel: each CTA streams 720 KB of operands for one tile,
// which the L2-to-SM feed caps at about 6.4 us, and 20 SMs sit idle.  Here a
// cluster of two CTAs owns one 128x256 tile; CTA r runs the MMAs of K blocks
// [r*h, r*h + h) into its own TMEM (half the operand bytes per CTA per output
// element of a 128x128 tile, so the MMAs set the pace).  Then the two
// exchange partial sums through distributed shared memory: CTA r sends the
// int32 partials of the other CTA's column half and keeps its own, adds the
// received ones (integer addition, exact), and runs the reference epilogue
// (ops.c:468-490) on its 128 x 128 half.
//
// Measured on B200 for W2 of config 2: mainloop 4.0 us (from 6.4), but
// staging and the 64 KB bulk copy to the peer take ~2.6 us and the half-tile
// epilogue ~2.4 us, so one launch ends at ~10.5 us, the same as the one-CTA
// kernel; it is therefore opt-in (IRO_GEMM_SPLITK=1).
//
// Roles as in gemm_i8.cu: warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2..17 epilogue.  Both cluster barriers are reached by every
// thread on every path, so an aborted CTA cannot strand its peer.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "epi_math.cuh"
#include "gemm_i8.cuh"

namespace iro {
namespace {

constexpr int SBM = 128;
constexpr int SBN = 256;          // tile columns (two 128-column halves)
constexpr int SHALF = SBN / 2;
constexpr int SBK = 128;          // K bytes per stage
constexpr int kSEpiWarps = 16;
constexpr int kSThreads = 64 + 32 * kSEpiWarps;
constexpr int kSStgBytes = 32 * kChunk * 4;
constexpr int kSStgBufs = 2;
constexpr int kSSmemMax = 232448;

struct SCfg {
  static constexpr int A_BYTES = SBM * SBK;
  static constexpr int B_BYTES = SBN * SBK;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STG = kSEpiWarps * kSStgBufs * kSStgBytes;
  static constexpr int PARAMS = 3 * SHALF * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int FIXED = STG + PARAMS + BAR_BYTES + 1024;
  static constexpr int STAGES_RAW = (kSSmemMax - FIXED) / STAGE;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = STAGES * STAGE + FIXED;
  // Peer partials in, own partials out: both in the ring once it is idle.
  static constexpr int RECV = SBM * SHALF * 4;
  static constexpr uint32_t IDESC = idesc_i8(SBM, SBN, 0);
  static_assert(STAGES >= 2, "pipeline needs two stages");
  static_assert(2 * RECV <= STAGES * STAGE, "exchange buffers fit the ring");
  static_assert(SMEM <= kSSmemMax, "shared memory budget");
};

struct SplitParams {
  int M, N, num_kb, tiles_m;
  const float* sx;
  const int32_t* zp;
  const float* wscale;
  const int32_t* wcolsum;
  const float* bias;
  float* y;
  int ldy;
  int accumulate;
  DevError* err;
  uint64_t limit_ns;
  unsigned long long* trace;  // optional per-CTA timestamps (IRO_SPLITK_TRACE)
};

enum { ST_ENTRY = 0, ST_TMA0, ST_FULL0, ST_TFULL, ST_SYNC1, ST_SENT, ST_SYNC2, ST_END,
       ST_SLOTS = 8 };
const char* const kStNames[ST_SLOTS] = {"entry", "tma0", "full0", "tfull",
                                        "sync1", "sent", "sync2", "end"};

__device__ __forceinline__ void strace(const SplitParams& p, int slot) {
  if (p.trace) p.trace[blockIdx.x * ST_SLOTS + slot] = globaltimer_ns();
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Cluster-wide barrier (every thread of both CTAs): release of the
// arriving thread's prior writes, acquire for what follows the wait.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_peer(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// Bulk copy of `bytes` from this CTA's shared memory to a peer CTA's, which
// completes as transactions on the peer's mbarrier (both addresses in the
// cluster window).
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta,
                                                  uint32_t bytes, uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes"
      " [%0], [%1], %2, [%3];" ::"r"(dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(mbar_cluster)
      : "memory");
}

// Receive-buffer slot of (row, 16-byte chunk q of the 128-column half): rows
// of 512 bytes, chunks XOR-swizzled by the row so a warp's 32 rows spread
// over all banks.
__device__ __forceinline__ uint32_t recv_off(int row, int q) {
  return (uint32_t)(row * (SHALF * 4) + ((q ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kSThreads, 1)
    gemm_i8_splitk_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmO, const SplitParams p) {
  using C = SCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stg_base = smem + C::STAGES * C::STAGE;
  float* prm = reinterpret_cast<float*>(stg_base + C::STG);  // colsum, scale, bias [SHALF]
  uint64_t* full = reinterpret_cast<uint64_t*>(stg_base + C::STG + C::PARAMS);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* recv_bar = tfull + 1;  // the peer's partials have arrived
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int tile = blockIdx.x >> 1;
  const int mb = tile % p.tiles_m, nb = tile / p.tiles_m;
  const int half = (p.num_kb + 1) / 2;
  const int kb0 = (int)rank * half;
  const int kb1 = min(p.num_kb, kb0 + half);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(recv_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, SBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_wait();
  if (threadIdx.x == 0) strace(p, ST_ENTRY);

  bool got = false;  // epilogue: this CTA's partial sums are complete
  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int kb = kb0; kb < kb1; kb++) {
        if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 21, abort_flag, p.limit_ns)) break;
        uint8_t* sa = smem + s * C::STAGE;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        tma_load_2d(sa, &tmA, &full[s], kb * SBK, mb * SBM);
        tma_load_2d(sa + C::A_BYTES, &tmB, &full[s], kb * SBK, nb * SBN);
        if (kb == kb0) strace(p, ST_TMA0);
        if (++s == C::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; kb++) {
        if (!mbar_wait_bounded(&full[s], ph, p.err, 22, abort_flag, p.limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (kb == kb0) strace(p, ST_FULL0);
        const uint32_t a_addr = smem_u32(smem + s * C::STAGE);
        const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
        for (int j = 0; j < SBK / 32; j++)
          mma_i8(tmem_base, sw128_desc(a_addr + 32 * j), sw128_desc(b_addr + 32 * j), C::IDESC,
                 (kb > kb0 || j > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
        if (++s == C::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (ok) mma_commit(tfull);
    }
    __syncwarp();
  } else {
    got = mbar_wait_bounded(tfull, 0, p.err, 23, abort_flag, p.limit_ns);
    tc_fence_after();
    if (warp == 2 && lane == 0) {
      strace(p, ST_TFULL);
      // Armed before the cluster barrier, so before the peer can send.
      mbar_arrive_expect_tx(recv_bar, C::RECV);
    }
  }
  // Both CTAs' MMAs are complete (or abandoned): the rings are free.
  cluster_sync_all();
  if (warp == 2 && lane == 0) strace(p, ST_SYNC1);

  const int e = warp - 2;
  const int quad = warp & 3;
  const int part = e >> 2;
  const int et = threadIdx.x - 64;
  const int row_l = quad * 32 + lane;  // tile row of this thread
  const uint32_t tlane = (uint32_t)(quad * 32) << 16;
  uint8_t* sendbuf = smem + C::RECV;
  if (warp >= 2 && got) {
    // Stage the partials of the peer's column half, then one thread pushes
    // them to the peer in a single bulk copy.
    const uint32_t other = rank ^ 1u;
#pragma unroll
    for (int c = 0; c < 2; c++) {
      const int col = part * 32 + c * kChunk;  // within the half
      uint32_t r[kChunk];
      tmem_ld_32x32b_x16(tmem_base + tlane + other * SHALF + col, r);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 4; q++)
        *reinterpret_cast<uint4*>(sendbuf + recv_off(row_l, col / 4 + q)) =
            make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
    }
    fence_async_shared();
  }
  if (warp >= 2) {
    if (named_bar_or(1, 32 * kSEpiWarps, !got)) got = false;
    if (et == 0 && got)
      bulk_copy_to_peer(map_peer(smem_u32(smem), rank ^ 1u), smem_u32(sendbuf), C::RECV,
                        map_peer(smem_u32(recv_bar), rank ^ 1u));
  }
  if (warp >= 2 && et < SHALF) {
    const int n = nb * SBN + (int)rank * SHALF + et;
    const bool ok = n < p.N;
    reinterpret_cast<int*>(prm)[et] = ok ? __ldg(p.wcolsum + n) : 0;
    prm[SHALF + et] = ok ? __ldg(p.wscale + n) : 0.0f;
    prm[2 * SHALF + et] = (ok && p.bias) ? __ldg(p.bias + n) : 0.0f;
  }
  if (warp == 2 && lane == 0) strace(p, ST_SENT);
  if (warp >= 2) {
    // The peer's partials have landed; the parameters are staged.
    if (got) got = mbar_wait_bounded(recv_bar, 0, p.err, 24, abort_flag, p.limit_ns);
    named_bar(1, 32 * kSEpiWarps);
    if (warp == 2 && lane == 0) strace(p, ST_SYNC2);
  }

  if (warp >= 2) {
    const int row = mb * SBM + row_l;
    const bool row_ok = row < p.M;
    const float sx = row_ok ? __ldg(p.sx + row) : 0.0f;
    const int zp = row_ok ? __ldg(p.zp + row) : 0;
    const int* p_cs = reinterpret_cast<const int*>(prm);
    uint8_t* stg_mine = stg_base + e * kSStgBufs * kSStgBytes;
    const uint8_t* recv = smem;
    int sbuf = 0;
    for (int c = 0; c < 2 && got; c++) {
      const int col = part * 32 + c * kChunk;
      const int n0 = nb * SBN + (int)rank * SHALF + col;
      if (n0 >= p.N) break;  // warp-uniform
      uint32_t r[kChunk];
      tmem_ld_32x32b_x16(tmem_base + tlane + rank * SHALF + col, r);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint4 o = *reinterpret_cast<const uint4*>(recv + recv_off(row_l, col / 4 + q));
        r[4 * q] = (uint32_t)((int)r[4 * q] + (int)o.x);
        r[4 * q + 1] = (uint32_t)((int)r[4 * q + 1] + (int)o.y);
        r[4 * q + 2] = (uint32_t)((int)r[4 * q + 2] + (int)o.z);
        r[4 * q + 3] = (uint32_t)((int)r[4 * q + 3] + (int)o.w);
      }
      float v[kChunk];
      linear_bias_chunk(r, col, p_cs, prm + SHALF, prm + 2 * SHALF, zp, sx, v);
      if (p.accumulate) {
        // ops.c:473-481: y += dequant + bias.
        const float* yrow = p.y + (size_t)row * p.ldy + n0;
#pragma unroll
        for (int j = 0; j < kChunk; j++)
          v[j] = __fadd_rn((row_ok && n0 + j < p.N) ? yrow[j] : 0.0f, v[j]);
      }
      uint8_t* stg = stg_mine + sbuf * kSStgBytes;
      sbuf ^= 1;
      if (lane == 0) bulk_wait_read<kSStgBufs - 1>();
      __syncwarp();
      stage_row16(stg, lane, v);
      fence_async_shared();
      __syncwarp();
      if (lane == 0 && mb * SBM + quad * 32 < p.M) {
        tma_store_2d(&tmO, stg, n0, mb * SBM + quad * 32);
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
    if (warp == 2 && lane == 0) strace(p, ST_END);
  }
  // The peer has received this CTA's bulk copy (it waited for it before
  // arriving), so the send buffer may go away with the CTA.
  cluster_sync_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, SBN);
  }
}

}  // namespace

bool splitk_eligible(const GemmRequest& r, int num_sms) {
  if (r.epi != EPI_LINEAR || r.work || r.force_bn || r.rgate) return false;
  const IroInt8DevWeight* w = r.w;
  const int num_kb = cdiv(w->K, SBK);
  const int tiles = cdiv(r.M, SBM) * cdiv(w->N, SBN);
  // Worth it when the one-CTA kernel would leave SMs idle on long tiles.
  const int tiles128 = cdiv(r.M, SBM) * cdiv(w->N, 128);
  return num_kb >= 8 && tiles128 <= num_sms && 2 * tiles <= num_sms &&
         (reinterpret_cast<uintptr_t>(r.y) & 15u) == 0 && (r.ldy & 3) == 0;
}

int splitk_launch(Ctx* c, const GemmRequest& r, cudaStream_t s) {
  using C = SCfg;
  static bool attr_done[64] = {false};
  if (!attr_done[c->device]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_splitk_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return map_cuda(e);
    attr_done[c->device] = true;
  }
  const IroInt8DevWeight* w = r.w;
  CUtensorMap ta, tb, to;
  int st = make_tmap_u8(&ta, r.a, (uint64_t)w->K, (uint64_t)r.M, (uint64_t)r.lda, SBK, SBM);
  if (!st) st = make_tmap_u8(&tb, w->data, (uint64_t)w->K, (uint64_t)w->N, (uint64_t)w->ld, SBK, SBN);
  if (!st) st = make_tmap_f32_sw128(&to, r.y, (uint64_t)w->N, (uint64_t)r.M, (uint64_t)r.ldy * 4);
  if (st) return st;
  SplitParams p;
  memset(&p, 0, sizeof(p));
  p.M = r.M;
  p.N = w->N;
  p.num_kb = cdiv(w->K, SBK);
  p.tiles_m = cdiv(r.M, SBM);
  p.sx = r.sx;
  p.zp = r.zp;
  p.wscale = w->scale;
  p.wcolsum = w->colsum;
  p.bias = r.bias;
  p.y = r.y;
  p.ldy = r.ldy;
  p.accumulate = r.accumulate;
  p.err = c->err;
  p.limit_ns = kWaitLimitNs;
  const int tiles = p.tiles_m * cdiv(w->N, SBN);

  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(2 * tiles);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // IRO_SPLITK_TRACE=1: per-CTA timeline on stderr (diagnostic; synchronises).
  static int trace_on = -1;
  if (trace_on < 0) {
    const char* t = getenv("IRO_SPLITK_TRACE");
    trace_on = (t && *t && *t != '0') ? 1 : 0;
  }
  const int grid = 2 * tiles;
  unsigned long long* tr = nullptr;
  // The trace buffer is an allocation: never on the no-allocation path.
  if (trace_on && !r.no_alloc &&
      cudaMalloc(&tr, sizeof(unsigned long long) * ST_SLOTS * grid) == cudaSuccess)
    cudaMemsetAsync(tr, 0, sizeof(unsigned long long) * ST_SLOTS * grid, s);
  else
    cudaGetLastError();
  p.trace = tr;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_i8_splitk_kernel, ta, tb, to, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (tr) cudaFree(tr);
    return map_cuda(e);
  }
  if (tr) {
    std::vector<unsigned long long> h((size_t)ST_SLOTS * grid);
    cudaStreamSynchronize(s);
    cudaMemcpy(h.data(), tr, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(tr);
    unsigned long long t0 = ~0ull;
    for (int i = 0; i < grid; i++)
      if (h[(size_t)i * ST_SLOTS]) t0 = std::min(t0, h[(size_t)i * ST_SLOTS]);
    fprintf(stderr, "[splitk trace] M=%d N=%d K=%d grid=%d\n", r.M, w->N, w->K, grid);
    for (int k = 0; k < ST_SLOTS; k++) {
      std::vector<double> v;
      for (int i = 0; i < grid; i++) {
        const unsigned long long t = h[(size_t)i * ST_SLOTS + k];
        if (t >= t0) v.push_back((t - t0) * 1e-3);
      }
      if (v.empty()) continue;
      std::sort(v.begin(), v.end());
      fprintf(stderr, "  %-6s n=%3zu min %8.2f  med %8.2f  max %8.2f us\n", kStNames[k], v.size(),
              v.front(), v[v.size() / 2], v.back());
    }
  }
  return check_launch();
}

}  // namespace iro
