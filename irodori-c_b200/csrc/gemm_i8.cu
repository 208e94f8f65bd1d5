// gemm_i8.cu — persistent, warp-specialised u8 x s8 -> s32 GEMM on the
// sm_100a tensor cores (tcgen05.mma kind::i8, accumulators in TMEM), fed by
// TMA through a shared-memory ring, with the dequantisation epilogues of the
// reference's int8 linear fused in.
//
// Roles (576 threads, one CTA per SM):
//   warp 0       TMA producer: A tile [128 x 128 B] (+ second A for the dual
//                term) and B tile [BN x 128 B] per stage, 128-byte swizzle.
//   warp 1       TMEM allocator + MMA issuer: 4 MMAs of K=32 per stage into
//                one of two TMEM accumulator buffers; commits release the
//                stage and, after the last K block, hand the buffer over.
//   warps 2..17  epilogue, four warps per TMEM lane quadrant, each a quarter
//                of the tile's columns: tcgen05.ld 16 columns at a time, the
//                exact reference float arithmetic (ops.c:468-490), 64-byte
//                swizzled staging and TMA tile stores; runs while the MMA
//                warp fills the other accumulator.  Epilogues that read the
//                old output (accumulate, gated residual) TMA-load it into
//                the same staging buffers, one chunk ahead.
//
// Epilogue kinds: LINEAR, SPLIT (column blocks to separate outputs), GATED
// (silu(W1) * W3 from the pair-interleaved weight), DUAL (two activation
// terms, two accumulators), DUAL2 (two terms stacked in one A tile: rows
// 0-63 term 1, rows 64-127 term 2 of the same 64 output rows; quadrants 2-3
// hand their dequantised term to quadrants 0-1 through shared memory), QKV
// (the DiT's QKVG split with head RMSNorm, RoPE and the V^T store).
//
// Parity: the integer sums are exact.  The epilogue uses explicitly rounded
// intrinsics in the reference's order, so fp32 outputs are bit-identical to
// the IEEE build of ops.c.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "epi_math.cuh"
#include "gemm_i8.cuh"

namespace iro {

constexpr int BM = 128;
constexpr int kHalfM = 64;  // output rows per EPI_DUAL2 tile
constexpr int BKB = 128;  // K bytes per pipeline stage (one swizzle row)
constexpr int kEpiWarps = 16;      // 4 per TMEM lane quadrant / per scheduler
constexpr int kParts = kEpiWarps / 4;  // column parts per quadrant
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemMax = 232448;  // 227 KB opt-in per CTA
constexpr int kStgBytes = 32 * kChunk * 4;  // one staging tile: 32 rows x 16 fp32
constexpr int kStgBufs = 2;                 // staging tiles per epilogue warp

// PAIR: a two-CTA cluster shares one tcgen05.mma.cta_group::2 of M = 256
// (each CTA's 128 A rows) x N = BN; each CTA stages only half of B (BN/2
// rows), so a CTA's operand bytes per output drop by a third at BN = 256.
template <int BN, int EPI, bool PAIR = false>
struct Cfg {
  static constexpr int NA = (EPI == EPI_DUAL) ? 2 : 1;
  static constexpr int A_BYTES = BM * BKB;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // B rows this CTA stages
  static constexpr int B_BYTES = B_ROWS * BKB;
  static constexpr int STAGE = NA * A_BYTES + B_BYTES;
  static constexpr int STG = kEpiWarps * kStgBufs * kStgBytes;
  static constexpr int PARAMS = 2 * 3 * BN * 4;  // double-buffered colsum/scale/bias
  static constexpr int BAR_BYTES = 512;  // pipeline barriers, then 2 per epilogue warp
  static constexpr int FIXED = STG + PARAMS + BAR_BYTES + 1024;
  static constexpr int STAGES_RAW = (kSmemMax - FIXED) / STAGE;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int ACC_COLS = (EPI == EPI_DUAL) ? 2 * BN : BN;
  static constexpr int TMEM_COLS = (2 * ACC_COLS) <= 32    ? 32
                                   : (2 * ACC_COLS) <= 64  ? 64
                                   : (2 * ACC_COLS) <= 128 ? 128
                                   : (2 * ACC_COLS) <= 256 ? 256
                                                           : 512;
  static constexpr int SMEM = STAGES * STAGE + FIXED;
  static constexpr uint32_t IDESC = idesc_i8(PAIR ? 2 * BM : BM, BN, 0);
  static_assert(!PAIR || EPI != EPI_DUAL, "the two-accumulator form runs on one CTA");
  static_assert(2 * ACC_COLS <= 512, "TMEM holds 512 columns");
  static_assert(STAGES >= 2, "pipeline needs two stages");
  static_assert(SMEM <= kSmemMax, "shared memory budget");
};

struct GemmParams {
  int M, N, K, num_kb, tiles_m, tiles_n, num_tiles;
  int n_fast;  // tile order: N blocks fastest (A reused through L2) or M blocks fastest
  const float* sx;
  const int32_t* zp;
  const float* sx2;
  const int32_t* zp2;
  const float* wscale;
  const int32_t* wcolsum;
  const float* bias;
  float* y;
  int ldy;
  int32_t* work;
  int ldw;
  int accumulate;
  const float* rgate;
  int rgate_rows;
  int tma_out;  // outputs written by TMA tile stores (else direct stores)
  float* outs[4];
  int seg;
  float* hidden;
  int ldh;
  int H;
  const float* hn_q;  // EPI_QKV
  const float* hn_k;
  const float* rcos;
  const float* rsin;
  __half* hq;
  __half* hk;
  __half* hvt;
  int vt_ld, tokens, heads;
  float eps;
  DevError* err;
  uint64_t limit_ns;
  unsigned long long* trace;  // optional per-CTA timestamps (IRO_GEMM_TRACE)
};

// Trace slots per CTA (globaltimer ns): entry, first TMA issue, first stage
// landed at the MMA warp, last MMA commit of the first tile, first
// accumulator handed to the epilogue, end of the first tile's epilogue,
// exit, tiles processed.
enum { TR_ENTRY = 0, TR_TMA0, TR_FULL0, TR_MMA_END0, TR_EPI0, TR_EPI_END0, TR_EXIT, TR_TILES,
       TR_SLOTS = 8 };

// Tile -> (row block, column block).  N-fastest when the activation operand
// is the larger one: the CTAs in flight then share a few row blocks of A
// (read once from DRAM, the rest from L2) instead of streaming all of A once
// per column block.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& mb, int& nb) {
  if (p.n_fast) {
    mb = t / p.tiles_n;
    nb = t - mb * p.tiles_n;
  } else {
    nb = t / p.tiles_m;
    mb = t - nb * p.tiles_m;
  }
}

__device__ __forceinline__ void trace_mark(const GemmParams& p, int slot) {
  if (p.trace) p.trace[blockIdx.x * TR_SLOTS + slot] = globaltimer_ns();
}

// ---- CTA pairs (two-CTA clusters, tcgen05 cta_group::2), no multicast loads.

__device__ __forceinline__ uint32_t pair_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void pair_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t pair_addr(const void* ptr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(ptr)), "r"(rank));
  return r;
}

// Bounded wait with cluster-scope acquire, for phases completed by the peer
// CTA's arrivals (its TMEM reads must be ordered before the next MMAs).
__device__ __forceinline__ bool pair_wait(uint64_t* bar, uint32_t parity, DevError* err,
                                          int where, volatile int* abort_flag,
                                          uint64_t limit_ns) {
  auto poll = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
  };
  if (poll()) return true;
  const long long t0 = clock64();
  const long long limit_cycles = (long long)(limit_ns * 2ull);
  while (!poll()) {
    if (abort_flag != nullptr && *abort_flag) return false;
    if (clock64() - t0 > limit_cycles) {
      report_error(err, IRO_ERR_DEVICE_TIMEOUT, where);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void pair_arrive(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// TMA tile load into this CTA's shared memory, completion counted on an
// mbarrier of either CTA of the pair (`cluster_bar`, a shared::cluster
// address).  Not a multicast load.
__device__ __forceinline__ void pair_tma_load_2d(void* dst, const CUtensorMap* map,
                                                 uint32_t cluster_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}

// D[tmem of both CTAs] (+)= A[smem, 128 rows per CTA] . B[smem, BN/2 rows per
// CTA]^T, kind::i8, M = 256, issued by the leader CTA.
__device__ __forceinline__ void pair_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (same offset) in both CTAs of the pair once the pair MMAs
// issued so far have completed.  The multicast here is the completion
// signal's, not a load's.
__device__ __forceinline__ void pair_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

// The same on this (the leader) CTA's barrier only.
__device__ __forceinline__ void pair_commit_local(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Output tensor maps (row-major fp32, box 32 rows x 16 columns, 64-byte swizzle).
struct OutMaps {
  CUtensorMap m[4];
};

template <int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ OutMaps tmO, const GemmParams p) {
  using C = Cfg<BN, EPI, PAIR>;
  // PAIR: CTAs 2k and 2k+1 form a cluster that works through pair tiles
  // (2 x 128 rows); rank r owns row block 2 * mb + r of pair tile mb.  The
  // leader (rank 0) issues the MMAs and holds the stage and accumulator
  // barriers they wait on.
  const uint32_t rank = PAIR ? pair_rank() : 0u;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stg_base = smem + C::STAGES * C::STAGE;             // 1024-aligned
  float* prm = reinterpret_cast<float*>(stg_base + C::STG);    // [2][3][BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(stg_base + C::STG + C::PARAMS);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Completion of every MMA issued, waited for before TMEM is freed when a
  // bounded wait gave up mid-tile.
  uint64_t* drain = tempty + 3;
  // Per epilogue warp and staging buffer: completion of the TMA load of the
  // old output values (accumulate / gated residual epilogues).
  uint64_t* xbar = reinterpret_cast<uint64_t*>(stg_base + C::STG + C::PARAMS + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    for (int i = 0; i < 2 * kEpiWarps; i++) mbar_init(&xbar[i], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI == EPI_DUAL || EPI == EPI_DUAL2) tma_prefetch_desc(&tmA2);
  }
  if (warp == 1) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(C::TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) pair_sync();  // the leader's barriers exist before the peer signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above overlaps the previous kernel's tail under a
  // programmatic launch; everything below may read its outputs.
  grid_dep_wait();
  if (threadIdx.x == 0) trace_mark(p, TR_ENTRY);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      long long armed = 0;  // stages armed so far (loads issued)
      for (int tile = tile0; ok && tile < p.num_tiles; tile += tstep) {
        int mb, nb;
        tile_coords(p, tile, mb, nb);
        if (PAIR) mb = 2 * mb + (int)rank;
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 1, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          armed++;
          uint8_t* sa = smem + s * C::STAGE;
          uint8_t* sb = sa + C::NA * C::A_BYTES;
          if (PAIR) {
            // Both CTAs' A rows and B halves complete on the leader's full[s],
            // which the leader arms with the pair's bytes.
            const uint32_t fb = pair_addr(&full[s], 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::STAGE);
            if (EPI == EPI_DUAL2) {
              pair_tma_load_2d(sa, &tmA, fb, kb * BKB, mb * kHalfM);
              pair_tma_load_2d(sa + kHalfM * BKB, &tmA2, fb, kb * BKB, mb * kHalfM);
            } else {
              pair_tma_load_2d(sa, &tmA, fb, kb * BKB, mb * BM);
            }
            pair_tma_load_2d(sb, &tmB, fb, kb * BKB, nb * BN + (int)rank * C::B_ROWS);
            if (tile == tile0 && kb == 0) trace_mark(p, TR_TMA0);
            if (++s == C::STAGES) {
              s = 0;
              ph ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          if (EPI == EPI_DUAL2) {
            // Rows 0-63 of the A tile: term 1 of output rows mb*64..; rows
            // 64-127: term 2 of the same rows (two 64-row boxes).
            tma_load_2d(sa, &tmA, &full[s], kb * BKB, mb * kHalfM);
            tma_load_2d(sa + kHalfM * BKB, &tmA2, &full[s], kb * BKB, mb * kHalfM);
          } else {
            tma_load_2d(sa, &tmA, &full[s], kb * BKB, mb * BM);
          }
          if (EPI == EPI_DUAL) tma_load_2d(sa + C::A_BYTES, &tmA2, &full[s], kb * BKB, mb * BM);
          tma_load_2d(sb, &tmB, &full[s], kb * BKB, nb * BN);
          if (tile == tile0 && kb == 0) trace_mark(p, TR_TMA0);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        // A wait gave up: no load may still be landing in shared memory when
        // the CTA exits.  Wait (bounded, regardless of the abort flag) for
        // the last armed phase of every stage; in the normal path the MMA
        // warp has consumed them all.  (A pair's phases, counted on the
        // leader, include the peer's loads; the peer leaves only after the
        // closing cluster barrier.)
        for (int st = 0; st < C::STAGES && st < armed; st++) {
          const long long uses = (armed - 1 - st) / C::STAGES + 1;
          mbar_wait_bounded(&full[st], (uint32_t)((uses - 1) & 1), p.err, 13, nullptr,
                            p.limit_ns);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && rank == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int tile = tile0; ok && tile < p.num_tiles; tile += tstep) {
        const bool free_acc =
            PAIR ? pair_wait(&tempty[acc], aph ^ 1u, p.err, 2, abort_flag, p.limit_ns)
                 : mbar_wait_bounded(&tempty[acc], aph ^ 1u, p.err, 2, abort_flag, p.limit_ns);
        if (!free_acc) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * C::ACC_COLS);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait_bounded(&full[s], ph, p.err, 3, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (tile == tile0 && kb == 0) trace_mark(p, TR_FULL0);
          const uint32_t a_addr = smem_u32(smem + s * C::STAGE);
          const uint32_t b_addr = a_addr + C::NA * C::A_BYTES;
#pragma unroll
          for (int j = 0; j < BKB / 32; j++) {
            const uint64_t bd = sw128_desc(b_addr + 32 * j);
            const uint32_t accum = (kb > 0 || j > 0) ? 1u : 0u;
            if (PAIR) {
              pair_mma_i8(d, sw128_desc(a_addr + 32 * j), bd, C::IDESC, accum);
            } else {
              mma_i8(d, sw128_desc(a_addr + 32 * j), bd, C::IDESC, accum);
              if (EPI == EPI_DUAL)
                mma_i8(d + BN, sw128_desc(a_addr + C::A_BYTES + 32 * j), bd, C::IDESC, accum);
            }
          }
          if (PAIR) pair_commit_both(&empty[s]);
          else mma_commit(&empty[s]);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR) pair_commit_both(&tfull[acc]);
        else mma_commit(&tfull[acc]);
        if (tile == tile0) trace_mark(p, TR_MMA_END0);
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
      if (!ok) {
        // MMAs of an unfinished tile may still run: wait (bounded) for all of
        // them before TMEM is freed.
        if (PAIR) pair_commit_local(drain);
        else mma_commit(drain);
        mbar_wait_bounded(drain, 0, p.err, 14, nullptr, p.limit_ns);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (16 warps) ----------------
    const int e = warp - 2;          // 0..15
    const int quad = warp & 3;       // TMEM lanes 32*quad .. 32*quad+31
    const int part = e >> 2;         // which quarter of the tile's columns
    const int et = threadIdx.x - 64; // 0..511
    uint8_t* stg_mine = stg_base + e * kStgBufs * kStgBytes;
    int sbuf = 0;  // next staging tile of this warp
    bool head_pending = false;  // EPI_QKV: a whole-head store may still read both buffers
    int acc = 0;
    uint32_t aph = 0;
    int pbuf = 0;
    // Per-tile parameters: one output column per thread (colsum, scale,
    // bias) and one row per lane (scale, zero point).  They are fetched into
    // registers one tile ahead, so their global-load latency overlaps the
    // previous tile's epilogue instead of delaying this one.
    static_assert(BN <= 32 * kEpiWarps, "one staged column per epilogue thread");
    struct Prefetch {
      int cs;
      float sw, b, sx, sx2;
      int zp, zp2;
    } pf;
    auto fetch = [&](int t) {
      int mb, nb;
      tile_coords(p, t, mb, nb);
      if (PAIR) mb = 2 * mb + (int)rank;
      const int n = nb * BN + et;
      const bool ok = et < BN && n < p.N;
      pf.cs = ok ? __ldg(p.wcolsum + n) : 0;
      pf.sw = ok ? __ldg(p.wscale + n) : 0.0f;
      if (EPI == EPI_QKV) {
        // The bias slot carries the head-norm weight of q / k columns (the
        // QKVG projection has no bias).
        const int gq = ok ? n / p.seg : 2;
        pf.b = gq == 0 ? __ldg(p.hn_q + n) : gq == 1 ? __ldg(p.hn_k + (n - p.seg)) : 0.0f;
      } else {
        pf.b = (ok && p.bias) ? __ldg(p.bias + n) : 0.0f;
      }
      const int r = (EPI == EPI_DUAL2 ? mb * kHalfM + (quad & 1) * 32 : mb * BM + quad * 32) + lane;
      const bool rok = r < p.M;
      // EPI_DUAL2: quadrants 2 and 3 hold the second term (its row scales).
      const bool term2 = EPI == EPI_DUAL2 && quad >= 2;
      pf.sx = rok ? __ldg((term2 ? p.sx2 : p.sx) + r) : 0.0f;
      pf.zp = rok ? __ldg((term2 ? p.zp2 : p.zp) + r) : 0;
      pf.sx2 = (EPI == EPI_DUAL && rok) ? __ldg(p.sx2 + r) : 0.0f;
      pf.zp2 = (EPI == EPI_DUAL && rok) ? __ldg(p.zp2 + r) : 0;
    };
    if (tile0 < p.num_tiles) fetch(tile0);
    // Old output values (y += ..., or the gated residual) come in by TMA
    // tile loads into the staging buffer that the chunk's result then goes
    // out from: one bulk copy per 32 x 16 chunk instead of per-lane row
    // loads, and the next chunk's load is in flight while this one computes.
    constexpr bool kMayLoadOld = (EPI == EPI_LINEAR || EPI == EPI_DUAL || EPI == EPI_DUAL2);
    static_assert(kStgBufs == 2, "old-value loads alternate between two staging buffers");
    // EPI_DUAL2: quadrants 2 and 3 only pass their dequantised second term
    // to quadrants 0 and 1 (through their own staging buffers), which finish
    // and store the rows.
    const bool writer2 = EPI == EPI_DUAL2 && quad >= 2;
    const bool xload = kMayLoadOld && !writer2 && p.tma_out && (p.accumulate || p.rgate != nullptr);
    uint32_t xc = 0;  // EPI_DUAL2 hand-over buffer counter (same sequence in both warps)
    uint32_t xph = 0;  // parity of each staging buffer's load barrier
    // An old-value load whose wait gave up: this warp issues no further loads
    // and stores nothing more (it still joins every barrier, so no partner
    // warp is left waiting); the abort flag winds the CTA down.
    bool xfail = false;
    auto x_issue = [&](int buf, int col, int r0) {
      // Lane 0: the buffer's previous store has finished reading it.
      if (lane == 0 && !xfail) {
        bulk_wait_read<0>();
        uint64_t* bar = &xbar[2 * e + buf];
        mbar_arrive_expect_tx(bar, kStgBytes);
        tma_load_2d(stg_mine + buf * kStgBytes, &tmO.m[0], bar, col, r0);
      }
    };
    // `drain`: wait for the load to land even when the CTA is aborting.
    auto x_wait = [&](int buf, bool drain) -> bool {
      const bool ok = xfail ? false
                            : mbar_wait_bounded(&xbar[2 * e + buf], (xph >> buf) & 1u, p.err,
                                                12, drain ? nullptr : abort_flag, p.limit_ns);
      xph ^= 1u << buf;
      xfail = __any_sync(0xffffffffu, !ok);
      return !xfail;
    };
    // The leader's accumulator-free barrier (the MMA warp waits on it).
    const uint32_t tempty_leader0 = PAIR ? pair_addr(&tempty[0], 0) : 0u;
    for (int tile = tile0; tile < p.num_tiles; tile += tstep) {
      int mb, nb;
      tile_coords(p, tile, mb, nb);
      if (PAIR) mb = 2 * mb + (int)rank;
      // Stage this tile's per-column parameters (the buffer was last read by
      // the tile before the previous one, which every warp has finished).
      float* pc = prm + pbuf * 3 * BN;
      int* p_cs = reinterpret_cast<int*>(pc);
      float* p_sw = pc + BN;
      float* p_b = pc + 2 * BN;
      if (et < BN) {
        p_cs[et] = pf.cs;
        p_sw[et] = pf.sw;
        p_b[et] = pf.b;
      }
      const int row0 = EPI == EPI_DUAL2 ? mb * kHalfM + (quad & 1) * 32 : mb * BM + quad * 32;
      const int row = row0 + lane;
      const bool row_ok = row < p.M;
      const float sx = pf.sx;
      const int zp = pf.zp;
      const float sx2 = pf.sx2;
      const int zp2 = pf.zp2;
      if (tile + tstep < p.num_tiles) fetch(tile + tstep);
      // The first chunk's old values load while the accumulator fills.
      // Quadrants wholly below the last row load nothing (and store nothing).
      const bool xrow = xload && row0 < p.M;
      const bool x_first = xrow && nb * BN + part * (BN / kParts) < p.N;
      if (x_first) x_issue(sbuf, nb * BN + part * (BN / kParts), row0);
      // The vote doubles as the barrier that publishes the staged parameters;
      // if any warp's bounded wait gave up, all epilogue warps stop together.
      const bool got = mbar_wait_bounded(&tfull[acc], aph, p.err, 4, abort_flag, p.limit_ns);
      if (named_bar_or(1, 32 * kEpiWarps, !got)) {
        if (x_first) x_wait(sbuf, true);  // no load may still be landing at exit
        break;
      }
      tc_fence_after();
      if (e == 0 && lane == 0 && tile == tile0) trace_mark(p, TR_EPI0);
      const uint32_t tbase =
          tmem_base + (uint32_t)(acc * C::ACC_COLS) + ((uint32_t)(quad * 32) << 16);

      // One 16-column chunk: values v for (row, out_col0 .. +15) of output
      // map `om` / pointer `dst_row` (direct fallback).
      auto emit = [&](const float (&v)[kChunk], const CUtensorMap* om, int out_col0, int out_cols,
                      float* dst_row) {
        if (p.tma_out) {
          // The store issued kStgBufs chunks ago read this tile; wait only
          // for that one (at most kStgBufs - 1 stores stay in flight).
          uint8_t* stg = stg_mine + sbuf * kStgBytes;
          sbuf = sbuf + 1 == kStgBufs ? 0 : sbuf + 1;
          if (lane == 0) {
            if (EPI == EPI_QKV && head_pending) bulk_wait_read<0>();
            else bulk_wait_read<kStgBufs - 1>();
          }
          head_pending = false;
          __syncwarp();
          stage_row16(stg, lane, v);
          fence_async_shared();
          __syncwarp();
          if (lane == 0 && row0 < p.M && out_col0 < out_cols) {
            tma_store_2d(om, stg, out_col0, row0);
            bulk_commit();
          }
        } else if (row_ok) {
          store_row16(dst_row, v, out_cols - out_col0);
        }
      };

      if (EPI == EPI_GATED) {
        // Columns [0, BN/2) hold W1 rows, [BN/2, BN) the matching W3 rows.
        constexpr int HALF = BN / 2;
        constexpr int PER = HALF / kParts;  // hidden columns per epilogue warp
        for (int c0 = part * PER; c0 < (part + 1) * PER; c0 += kChunk) {
          const int h0 = nb * HALF + c0;
          if (h0 >= p.H) break;  // warp-uniform
          uint32_t r1[kChunk], r3[kChunk];
          tmem_ld_32x32b_x16(tbase + c0, r1);
          tmem_ld_32x32b_x16(tbase + HALF + c0, r3);
          tmem_ld_wait();
          float v[kChunk];
          gated_chunk(r1, r3, c0, HALF + c0, p_cs, p_sw, p_b, zp, sx, v);
          emit(v, &tmO.m[0], h0, p.H, p.hidden + (size_t)row * p.ldh + h0);
        }
      } else if constexpr (EPI == EPI_QKV) {
        // One head (64 columns) per warp.  q and k: the head RMSNorm in the
        // reference's order (sequential mean square, then x * (inv * w);
        // dit.c:638-690) and, on the first half of the heads, the rotation
        // of each (even, odd) pair by the token's RoPE angle.  v: stored
        // transposed per head (the attention kernel's V^T rows; for a fixed
        // dimension the warp's 32 rows are 32 consecutive tokens, so each
        // store instruction writes 128 contiguous bytes).  gate: as is.
        static_assert(BN / kParts == 64, "one head per epilogue warp");
        const int c0 = part * 64;
        const int n0 = nb * BN + c0;
        if (n0 < p.N) {  // warp-uniform
          const int g = n0 / p.seg;
          const int col0 = n0 - g * p.seg;
          const int head = col0 >> 6;
          const int seq = row_ok ? row / p.tokens : 0;
          const int tok = row_ok ? row - seq * p.tokens : 0;
          auto deq = [&](int c, float (&v)[kChunk]) {
            uint32_t r[kChunk];
            tmem_ld_32x32b_x16(tbase + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < kChunk / 4; i++) {
              const int4 cs = *reinterpret_cast<const int4*>(p_cs + c + 4 * i);
              const float4 sw = *reinterpret_cast<const float4*>(p_sw + c + 4 * i);
              float2 lo = dequant2(r[4 * i], r[4 * i + 1], zp, cs.x, cs.y, sx, sw.x, sw.y);
              float2 hi = dequant2(r[4 * i + 2], r[4 * i + 3], zp, cs.z, cs.w, sx, sw.z, sw.w);
              if (p.bias) {
                const float4 b = *reinterpret_cast<const float4*>(p_b + c + 4 * i);
                lo = add2_rn(lo, make_float2(b.x, b.y));
                hi = add2_rn(hi, make_float2(b.z, b.w));
              }
              v[4 * i] = lo.x;
              v[4 * i + 1] = lo.y;
              v[4 * i + 2] = hi.x;
              v[4 * i + 3] = hi.y;
            }
          };
          if (g < 2) {
            // Pass 1: the mean square; each dequantised chunk goes back over
            // its accumulator in TMEM (this tile's columns, this warp's lanes),
            // so pass 2 reads it instead of dequantising again.
            float ms = 0.0f;
            for (int ch = 0; ch < 64; ch += kChunk) {
              float v[kChunk];
              deq(c0 + ch, v);
#pragma unroll
              for (int j = 0; j < kChunk; j++) ms = __fadd_rn(ms, __fmul_rn(v[j], v[j]));
              tmem_st_32x32b_x16(tbase + c0 + ch, reinterpret_cast<const uint32_t(&)[kChunk]>(v));
            }
            tmem_st_wait();
            const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ms, 64.0f), p.eps)));
            const bool rope = head < p.heads / 2;
            // RoPE tables in groups of four pairs, [8][tokens][4]: one vector
            // load gives a lane the four (cos, sin) of its token, and the
            // warp's 32 consecutive tokens read 512 contiguous bytes.
            const float4* rc4 = reinterpret_cast<const float4*>(p.rcos) + tok;
            const float4* rs4 = reinterpret_cast<const float4*>(p.rsin) + tok;
            __half* hrow = (g == 0 ? p.hq : p.hk) + (size_t)row * p.seg + col0;
            if (p.tma_out) {
              // The warp's 32 rows x 64 halves go out as one tile store from
              // both staging buffers (4 KB, rows of 128 bytes in the 128-byte
              // swizzle); every earlier store of this warp has read them.
              if (lane == 0) bulk_wait_read<0>();
              __syncwarp();
            }
            for (int ch = 0; ch < 64; ch += kChunk) {
              // This chunk's RoPE groups load before the TMEM read, which
              // then covers their latency.
              float4 c4[2], s4[2];
              if (rope) {
#pragma unroll
                for (int q2 = 0; q2 < 2; q2++) {
                  const size_t gi = (size_t)((ch >> 3) + q2) * p.tokens;
                  c4[q2] = __ldg(rc4 + gi);
                  s4[q2] = __ldg(rs4 + gi);
                }
              }
              float v[kChunk];
              tmem_ld_32x32b_x16(tbase + c0 + ch, reinterpret_cast<uint32_t(&)[kChunk]>(v));
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < kChunk; j += 4) {
                // Norm weights staged with the tile's column parameters.
                const float4 w4 = *reinterpret_cast<const float4*>(p_b + c0 + ch + j);
                v[j] = __fmul_rn(v[j], __fmul_rn(inv, w4.x));
                v[j + 1] = __fmul_rn(v[j + 1], __fmul_rn(inv, w4.y));
                v[j + 2] = __fmul_rn(v[j + 2], __fmul_rn(inv, w4.z));
                v[j + 3] = __fmul_rn(v[j + 3], __fmul_rn(inv, w4.w));
              }
              if (rope) {
#pragma unroll
                for (int j = 0; j < kChunk; j += 8) {
                  // Pairs (ch + j) / 2 .. + 3 form group (ch + j) / 8.
                  const float4 cg = c4[j >> 3], sg = s4[j >> 3];
                  const float cr[4] = {cg.x, cg.y, cg.z, cg.w};
                  const float sr[4] = {sg.x, sg.y, sg.z, sg.w};
#pragma unroll
                  for (int t = 0; t < 4; t++) {
                    const float x0 = v[j + 2 * t], x1 = v[j + 2 * t + 1];
                    v[j + 2 * t] = __fsub_rn(__fmul_rn(x0, cr[t]), __fmul_rn(x1, sr[t]));
                    v[j + 2 * t + 1] = __fadd_rn(__fmul_rn(x0, sr[t]), __fmul_rn(x1, cr[t]));
                  }
                }
              }
              uint32_t hw[kChunk / 2];
#pragma unroll
              for (int j = 0; j < kChunk / 2; j++) hw[j] = pack_half2_rn(v[2 * j], v[2 * j + 1]);
              check_half_range(v, p.err, 102 + g);
              if (p.tma_out) {
                // 16-byte chunks c, c + 1 of this lane's row, swizzled.
                uint8_t* srow = stg_mine + lane * 128;
                const int c = ch >> 3;
                *reinterpret_cast<uint4*>(srow + ((c ^ (lane & 7)) << 4)) =
                    make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(srow + (((c + 1) ^ (lane & 7)) << 4)) =
                    make_uint4(hw[4], hw[5], hw[6], hw[7]);
              } else if (row_ok) {
                uint4* dst = reinterpret_cast<uint4*>(hrow + ch);
                dst[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                dst[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
              }
            }
            if (p.tma_out) {
              fence_async_shared();
              __syncwarp();
              if (lane == 0 && row0 < p.M) {
                tma_store_2d(&tmO.m[g], stg_mine, col0, row0);
                bulk_commit();
              }
              __syncwarp();
              sbuf = 0;
              head_pending = true;  // the next staging write waits for this read
            }
          } else if (g == 2) {
            __half* vrow = p.hvt + (size_t)(seq * p.heads + head) * 64 * p.vt_ld + tok;
            const int pad = (row_ok && tok == p.tokens - 1) ? p.vt_ld - p.tokens : 0;
            for (int ch = 0; ch < 64; ch += kChunk) {
              float v[kChunk];
              deq(c0 + ch, v);
              if (row_ok) {
                check_half_range(v, p.err, 104);
#pragma unroll
                for (int j = 0; j < kChunk; j++) {
                  __half* dst = vrow + (size_t)(ch + j) * p.vt_ld;
                  dst[0] = __float2half_rn(v[j]);
                  for (int t = 1; t <= pad; t++) dst[t] = __float2half_rn(0.0f);
                }
              }
            }
          } else {
            float* drow = p.outs[3] + (size_t)row * p.seg + col0;
            for (int ch = 0; ch < 64; ch += kChunk) {
              float v[kChunk];
              deq(c0 + ch, v);
              emit(v, &tmO.m[3], col0 + ch, p.seg, drow + ch);
            }
          }
        }
      } else if (writer2) {
        // EPI_DUAL2 second term: dequantise (no bias) and hand over.
        constexpr int PER = BN / kParts;
        const int bar_id = 2 + part * 2 + (quad & 1);
        for (int c0 = part * PER; c0 < (part + 1) * PER; c0 += kChunk) {
          const int n0 = nb * BN + c0;
          if (n0 >= p.N) break;  // warp-uniform, the same in the partner warp
          uint32_t r[kChunk];
          tmem_ld_32x32b_x16(tbase + c0, r);
          tmem_ld_wait();
          float v[kChunk];
#pragma unroll
          for (int i = 0; i < kChunk / 4; i++) {
            const int c = c0 + 4 * i;
            const int4 cs = *reinterpret_cast<const int4*>(p_cs + c);
            const float4 sw = *reinterpret_cast<const float4*>(p_sw + c);
            const float2 lo = dequant2(r[4 * i], r[4 * i + 1], zp, cs.x, cs.y, sx, sw.x, sw.y);
            const float2 hi = dequant2(r[4 * i + 2], r[4 * i + 3], zp, cs.z, cs.w, sx, sw.z, sw.w);
            v[4 * i] = lo.x;
            v[4 * i + 1] = lo.y;
            v[4 * i + 2] = hi.x;
            v[4 * i + 3] = hi.y;
          }
          // Buffers alternate, so this write never meets the partner's read
          // of the previous chunk (which it finished before the last barrier).
          stage_row16(stg_mine + (xc & 1) * kStgBytes, lane, v);
          named_bar(bar_id, 64);
          xc++;
        }
      } else {
        constexpr int PER = BN / kParts;
        for (int c0 = part * PER; c0 < (part + 1) * PER; c0 += kChunk) {
          const int n0 = nb * BN + c0;
          if (n0 >= p.N) break;  // warp-uniform
          uint32_t r[kChunk];
          tmem_ld_32x32b_x16(tbase + c0, r);
          uint32_t r2[kChunk];
          if (EPI == EPI_DUAL) tmem_ld_32x32b_x16(tbase + BN + c0, r2);
          tmem_ld_wait();
          int g = 0, col0 = n0, ncols = p.N, ld = p.ldy;
          float* base = p.y;
          if (EPI == EPI_SPLIT || (EPI == EPI_DUAL && p.seg > 0)) {
            g = n0 / p.seg;
            col0 = n0 - g * p.seg;
            ncols = p.seg;
            ld = p.seg;
            base = g == 0 ? p.outs[0] : g == 1 ? p.outs[1] : g == 2 ? p.outs[2] : p.outs[3];
          }
          float* drow = base + (size_t)row * ld + col0;
          const int valid = ncols - col0;
          float v[kChunk];
          const bool gated_res =
              (EPI == EPI_LINEAR || EPI == EPI_DUAL || EPI == EPI_DUAL2) && p.rgate != nullptr;
          if (xload) {
            // Next chunk's old values into the other buffer, then this one's.
            const int c1 = c0 + kChunk;
            if (xrow && c1 < (part + 1) * PER && nb * BN + c1 < p.N)
              x_issue(sbuf ^ 1, nb * BN + c1, row0);
            if (xrow) x_wait(sbuf, false);  // a give-up sets xfail (no store below)
            if (EPI == EPI_LINEAR) {
              // All four groups now (fewer registers live than reading them
              // group by group in this variant); the two-term variants read
              // them group by group below.
              const uint8_t* xr = stg_mine + sbuf * kStgBytes + lane * 64;
#pragma unroll
              for (int i = 0; i < 4; i++) {
                const float4 o4 = *reinterpret_cast<const float4*>(xr + ((i ^ ((lane >> 1) & 3)) << 4));
                v[4 * i] = o4.x;
                v[4 * i + 1] = o4.y;
                v[4 * i + 2] = o4.z;
                v[4 * i + 3] = o4.w;
              }
            }
          } else if ((EPI == EPI_LINEAR || EPI == EPI_DUAL || EPI == EPI_DUAL2) &&
                     (p.accumulate || gated_res)) {
            if (p.tma_out && valid >= kChunk) {
              // 16-byte aligned rows (the TMA store path requires it): four
              // vector loads per lane instead of sixteen scalar ones.
#pragma unroll
              for (int j = 0; j < kChunk / 4; j++) {
                const float4 o4 = row_ok ? reinterpret_cast<const float4*>(drow)[j]
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                v[4 * j] = o4.x;
                v[4 * j + 1] = o4.y;
                v[4 * j + 2] = o4.z;
                v[4 * j + 3] = o4.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < kChunk; j++) v[j] = (row_ok && j < valid) ? drow[j] : 0.0f;
            }
          }
          const float* grow =
              (gated_res && row_ok) ? p.rgate + (size_t)(row / p.rgate_rows) * p.N + n0 : nullptr;
          const uint8_t* xs = stg_mine + sbuf * kStgBytes + lane * 64;
          // EPI_DUAL2: the partner warp (two quadrants up, e - 2) has staged
          // this chunk's second term.
          const uint8_t* t2 =
              EPI == EPI_DUAL2
                  ? stg_base + (e - 2) * kStgBufs * kStgBytes + (xc & 1) * kStgBytes + lane * 64
                  : nullptr;
          if (EPI == EPI_DUAL2) {
            named_bar(2 + part * 2 + (quad & 1), 64);
            xc++;
          }
#pragma unroll
          for (int i = 0; i < kChunk / 4; i++) {
            if (xload && EPI != EPI_LINEAR) {
              // 16-byte group i of this lane's row (64-byte swizzle).
              const float4 o4 = *reinterpret_cast<const float4*>(xs + ((i ^ ((lane >> 1) & 3)) << 4));
              v[4 * i] = o4.x;
              v[4 * i + 1] = o4.y;
              v[4 * i + 2] = o4.z;
              v[4 * i + 3] = o4.w;
            }
            const int c = c0 + 4 * i;
            const int4 cs = *reinterpret_cast<const int4*>(p_cs + c);
            const float4 sw = *reinterpret_cast<const float4*>(p_sw + c);
            float2 lo = dequant2(r[4 * i], r[4 * i + 1], zp, cs.x, cs.y, sx, sw.x, sw.y);
            float2 hi = dequant2(r[4 * i + 2], r[4 * i + 3], zp, cs.z, cs.w, sx, sw.z, sw.w);
            if (p.bias) {
              const float4 b = *reinterpret_cast<const float4*>(p_b + c);
              lo = add2_rn(lo, make_float2(b.x, b.y));
              hi = add2_rn(hi, make_float2(b.z, b.w));
            }
            if (EPI == EPI_DUAL) {
              // Two accumulating linears in the reference's order:
              // y = (y + (d1 + bias)) + d2 (ops.c:473-481 applied twice).
              if (p.accumulate) {
                lo = add2_rn(make_float2(v[4 * i], v[4 * i + 1]), lo);
                hi = add2_rn(make_float2(v[4 * i + 2], v[4 * i + 3]), hi);
              }
              lo = add2_rn(lo, dequant2(r2[4 * i], r2[4 * i + 1], zp2, cs.x, cs.y, sx2, sw.x, sw.y));
              hi = add2_rn(hi, dequant2(r2[4 * i + 2], r2[4 * i + 3], zp2, cs.z, cs.w, sx2, sw.z, sw.w));
            }
            if (EPI == EPI_DUAL2) {
              if (p.accumulate) {
                lo = add2_rn(make_float2(v[4 * i], v[4 * i + 1]), lo);
                hi = add2_rn(make_float2(v[4 * i + 2], v[4 * i + 3]), hi);
              }
              const float4 d2 =
                  *reinterpret_cast<const float4*>(t2 + ((i ^ ((lane >> 1) & 3)) << 4));
              lo = add2_rn(lo, make_float2(d2.x, d2.y));
              hi = add2_rn(hi, make_float2(d2.z, d2.w));
            }
            if (EPI == EPI_LINEAR && p.accumulate) {
              lo = add2_rn(make_float2(v[4 * i], v[4 * i + 1]), lo);
              hi = add2_rn(make_float2(v[4 * i + 2], v[4 * i + 3]), hi);
            }
            if (gated_res) {
              const float4 gv = grow ? *reinterpret_cast<const float4*>(grow + 4 * i)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
              lo = make_float2(__fadd_rn(v[4 * i], __fmul_rn(gv.x, lo.x)),
                               __fadd_rn(v[4 * i + 1], __fmul_rn(gv.y, lo.y)));
              hi = make_float2(__fadd_rn(v[4 * i + 2], __fmul_rn(gv.z, hi.x)),
                               __fadd_rn(v[4 * i + 3], __fmul_rn(gv.w, hi.y)));
            }
            v[4 * i] = lo.x;
            v[4 * i + 1] = lo.y;
            v[4 * i + 2] = hi.x;
            v[4 * i + 3] = hi.y;
          }
          if (xload) {
            // The result goes out from the buffer its old values came in by
            // (each lane rewrites only its own row).
            uint8_t* stg = stg_mine + sbuf * kStgBytes;
            stage_row16(stg, lane, v);
            fence_async_shared();
            __syncwarp();
            if (lane == 0 && row0 < p.M && !xfail) {
              tma_store_2d(&tmO.m[0], stg, n0, row0);
              bulk_commit();
            }
            sbuf ^= 1;
          } else {
            emit(v, &tmO.m[g], col0, ncols, drow);
          }
          if (EPI == EPI_LINEAR && p.work != nullptr && row_ok) {
            int32_t* wrow = p.work + (size_t)row * p.ldw + n0;
#pragma unroll
            for (int j = 0; j < kChunk; j++)
              if (j < valid) wrow[j] = (int)r[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) pair_arrive(tempty_leader0 + 8u * (uint32_t)acc);
        else mbar_arrive(&tempty[acc]);
      }
      if (e == 0 && lane == 0 && tile == tile0) trace_mark(p, TR_EPI_END0);
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
      pbuf ^= 1;
    }
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
  }

  __syncthreads();
  // A pair: the leader's MMAs no longer read this CTA's shared memory, and
  // every remote arrival has landed, before either CTA frees anything.
  if (PAIR) pair_sync();
  if (threadIdx.x == 0 && p.trace) {
    trace_mark(p, TR_EXIT);
    p.trace[blockIdx.x * TR_SLOTS + TR_TILES] =
        (unsigned long long)((p.num_tiles - tile0 + tstep - 1) / tstep);
  }
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(C::TMEM_COLS)
                   : "memory");
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// IRO_GEMM_TRACE=1: print a per-role timeline of each GEMM launch (median and
// max over CTAs, microseconds from the earliest CTA entry).  Diagnostic only;
// synchronises the stream after every launch.
static int trace_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("IRO_GEMM_TRACE");
    on = (e && *e && *e != '0') ? 1 : 0;
  }
  return on;
}

static void trace_report(const char* name, int M, int N, int K, const unsigned long long* dev,
                         int grid, cudaStream_t s) {
  std::vector<unsigned long long> h((size_t)grid * TR_SLOTS);
  cudaStreamSynchronize(s);
  cudaMemcpy(h.data(), dev, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  unsigned long long t0 = ~0ull;
  for (int b = 0; b < grid; b++) t0 = std::min(t0, h[(size_t)b * TR_SLOTS + TR_ENTRY]);
  const char* names[7] = {"entry", "tma0", "full0", "mma_end0", "epi0", "epi_end0", "exit"};
  fprintf(stderr, "[gemm trace] %s M=%d N=%d K=%d grid=%d tiles/cta=%llu..%llu\n", name, M, N, K,
          grid, h[(size_t)(grid - 1) * TR_SLOTS + TR_TILES], h[TR_TILES]);
  for (int k = 0; k < 7; k++) {
    std::vector<double> v;
    for (int b = 0; b < grid; b++) {
      unsigned long long t = h[(size_t)b * TR_SLOTS + k];
      if (t >= t0) v.push_back((t - t0) * 1e-3);
    }
    std::sort(v.begin(), v.end());
    if (v.empty()) continue;
    fprintf(stderr, "  %-9s min %8.2f  med %8.2f  max %8.2f us\n", names[k], v.front(),
            v[v.size() / 2], v.back());
  }
}

static bool out_tma_ok(const float* base, int ld) {
  return base != nullptr && (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && (ld & 3) == 0;
}

template <int BN, int EPI, bool PAIR = false>
static int launch_t(Ctx* c, const GemmRequest& r, const GemmParams& p0, cudaStream_t s) {
  using C = Cfg<BN, EPI, PAIR>;
  static bool attr_done[64] = {false};
  if (!attr_done[c->device]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<BN, EPI, PAIR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return map_cuda(e);
    attr_done[c->device] = true;
  }
  const IroInt8DevWeight* w = r.w;
  CUtensorMap ta, tb, ta2;
  constexpr int ABOX = EPI == EPI_DUAL2 ? kHalfM : BM;  // A rows per TMA box
  int st = make_tmap_u8(&ta, r.a, (uint64_t)w->K, (uint64_t)r.M, (uint64_t)r.lda, BKB, ABOX);
  if (st) return st;
  st = make_tmap_u8(&tb, w->data, (uint64_t)w->K, (uint64_t)w->N, (uint64_t)w->ld, BKB,
                    C::B_ROWS);
  if (st) return st;
  if (EPI == EPI_DUAL || EPI == EPI_DUAL2) {
    st = make_tmap_u8(&ta2, r.a2, (uint64_t)w->K, (uint64_t)r.M, (uint64_t)r.lda, BKB, ABOX);
    if (st) return st;
  } else {
    ta2 = ta;
  }
  GemmParams p = p0;
  OutMaps om;
  memset(&om, 0, sizeof(om));
  // Output tiles go out through TMA stores when every output is 16-byte
  // aligned with a 16-byte multiple pitch; otherwise direct stores.
  bool tma = true;
  if (EPI == EPI_GATED) {
    tma = out_tma_ok(r.hidden, r.ldh);
    if (tma)
      st = make_tmap_f32_sw128(&om.m[0], r.hidden, (uint64_t)w->hidden, (uint64_t)r.M,
                               (uint64_t)r.ldh * 4);
  } else if (EPI == EPI_QKV) {
    // The gate and the fp16 q, k through tile stores (q, k: one 32-row x
    // 64-half head per warp, 128-byte swizzle); V^T by direct stores.
    tma = out_tma_ok(r.outs[3], r.seg);
    if (tma)
      st = make_tmap_f32_sw128(&om.m[3], r.outs[3], (uint64_t)r.seg, (uint64_t)r.M,
                               (uint64_t)r.seg * 4);
    for (int i = 0; i < 2 && tma && st == IRO_OK; i++) {
      const cuuint64_t dims[2] = {(cuuint64_t)r.seg, (cuuint64_t)r.M};
      const cuuint64_t strides[1] = {(cuuint64_t)r.seg * 2};
      const cuuint32_t box[2] = {64, 32};
      st = encode_tmap(&om.m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, i == 0 ? r.hq : r.hk, dims,
                       strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
  } else if (EPI == EPI_SPLIT || (EPI == EPI_DUAL && r.nout > 0)) {
    for (int i = 0; i < r.nout && tma; i++) tma = out_tma_ok(r.outs[i], r.seg);
    for (int i = 0; tma && i < r.nout && st == IRO_OK; i++)
      st = make_tmap_f32_sw128(&om.m[i], r.outs[i], (uint64_t)r.seg, (uint64_t)r.M,
                               (uint64_t)r.seg * 4);
  } else {
    tma = out_tma_ok(r.y, r.ldy);
    if (tma)
      st = make_tmap_f32_sw128(&om.m[0], r.y, (uint64_t)w->N, (uint64_t)r.M,
                               (uint64_t)r.ldy * 4);
  }
  if (st) return st;
  p.tma_out = tma ? 1 : 0;
  // Output rows per tile: 128 (64 for the stacked two-term form), twice that
  // for a pair tile.
  p.tiles_m = cdiv(r.M, (EPI == EPI_DUAL2 ? kHalfM : BM) * (PAIR ? 2 : 1));
  p.tiles_n = cdiv(w->N, BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  {
    const size_t a_bytes = (size_t)r.M * w->K * (r.epi == EPI_DUAL ? 2 : 1);
    const size_t b_bytes = (size_t)w->N * w->K;
    p.n_fast = a_bytes > b_bytes ? 1 : 0;
  }
  // Persistent grid: one CTA per SM, or as many co-resident pairs as the
  // GPCs hold (a GPC with an odd count of free SMs leaves one idle).
  int slots = c->num_sms;
  if (PAIR) {
    static int pairs[64] = {0};
    if (!pairs[c->device]) {
      cudaLaunchConfig_t oc;
      memset(&oc, 0, sizeof(oc));
      oc.gridDim = dim3(c->num_sms);
      oc.blockDim = dim3(kThreads);
      oc.dynamicSmemBytes = (size_t)C::SMEM;
      cudaLaunchAttribute ca[1];
      ca[0].id = cudaLaunchAttributeClusterDimension;
      ca[0].val.clusterDim.x = 2;
      ca[0].val.clusterDim.y = 1;
      ca[0].val.clusterDim.z = 1;
      oc.attrs = ca;
      oc.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_i8_kernel<BN, EPI, PAIR>, &oc) != cudaSuccess ||
          n <= 0) {
        cudaGetLastError();
        n = c->num_sms / 2;
      }
      pairs[c->device] = n < c->num_sms / 2 ? n : c->num_sms / 2;
    }
    slots = pairs[c->device];
  }
  const int grid = (p.num_tiles < slots ? p.num_tiles : slots) * (PAIR ? 2 : 1);
  unsigned long long* tr = nullptr;
  if (trace_enabled() && !r.no_alloc) {
    cudaMalloc(&tr, sizeof(unsigned long long) * TR_SLOTS * (size_t)grid);
    cudaMemsetAsync(tr, 0, sizeof(unsigned long long) * TR_SLOTS * (size_t)grid, s);
    p.trace = tr;
  }
  cudaError_t le;
  if (PAIR) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)C::SMEM;
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
    le = cudaLaunchKernelEx(&cfg, gemm_i8_kernel<BN, EPI, PAIR>, ta, tb, ta2, om, p);
  } else {
    le = launch_pdl(gemm_i8_kernel<BN, EPI, PAIR>, dim3(grid), dim3(kThreads), (size_t)C::SMEM,
                    s, ta, tb, ta2, om, p);
  }
  st = le == cudaSuccess ? check_launch() : (cudaGetLastError(), map_cuda(le));
  if (tr) {
    char name[48];
    snprintf(name, sizeof(name), "bn%d/epi%d%s", BN, EPI, PAIR ? "/pair" : "");
    trace_report(name, r.M, w->N, w->K, tr, grid, s);
    cudaFree(tr);
  }
  return st;
}

// Tile width: the fewest waves of the persistent grid, with a per-tile cost
// that grows with BN plus a fixed part for the epilogue hand-off.
static int pick_bn(int M, int N, int sms, int dual) {
  const int cands[3] = {256, 128, 64};
  int best = 128;
  double best_cost = 1e30;
  for (int i = dual ? 1 : 0; i < 3; i++) {
    const int bn = cands[i];
    const long tiles = (long)cdiv(M, BM) * cdiv(N, bn);
    const long waves = (tiles + sms - 1) / sms;
    const double cost = (double)waves * (bn + 48);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// CTA-pair tiles (tcgen05 cta_group::2, two-CTA clusters, 256 x 256 per
// pair): the pair MMA runs at the full tensor rate (measured ~137 cycles per
// 256x256x32 int8 MMA, against ~200 for the one-CTA 128x256x32), but each
// CTA's epilogue of a tile measured 25-45% slower in a pair, so pairs pay
// only where the mainloop dominates: the stacked two-term linear (EPI_DUAL2,
// K = 2816) over several waves (the DiT's W2 at 24,000 rows: 115 us against
// 127).  Elsewhere (gated, QKVG, plain linears) they measured slower.
static bool pair_pays(const GemmRequest& r, int num_sms) {
  const long pair_tiles = (long)cdiv(r.M, 2 * kHalfM) * cdiv(r.w->N, 256);
  return r.w->K >= 2048 && pair_tiles >= 2L * (num_sms / 2);
}

static int gemm_launch_impl(Ctx* c, const GemmRequest& r, cudaStream_t s);

int gemm_launch(Ctx* c, const GemmRequest& r, cudaStream_t s) {
  // IRO_GEMM_PROFILE: device time of the launch per shape (gemm_profile.cu).
  void* tok = (r.M > 0 && r.w) ? gemm_profile_begin(r, s) : nullptr;
  const int st = gemm_launch_impl(c, r, s);
  if (tok) gemm_profile_end(tok, r, s);
  return st;
}

static int gemm_launch_impl(Ctx* c, const GemmRequest& r, cudaStream_t s) {
  const IroInt8DevWeight* w = r.w;
  if (r.M == 0) return IRO_OK;
  if (r.M < 0 || !w || !w->data || !r.a || !r.sx || !r.zp) return IRO_ERR_INVALID;
  if ((r.lda & 15) != 0 || r.lda < w->K) return IRO_ERR_UNSUPPORTED;
  if (r.rgate && ((r.epi != EPI_LINEAR && r.epi != EPI_DUAL) || r.accumulate || !r.y ||
                  r.rgate_rows <= 0 || (w->N & 15) != 0 ||
                  (reinterpret_cast<uintptr_t>(r.rgate) & 15u) != 0))
    return IRO_ERR_INVALID;
  GemmParams p{};
  p.M = r.M;
  p.N = w->N;
  p.K = w->K;
  p.num_kb = cdiv(w->K, BKB);
  p.sx = r.sx;
  p.zp = r.zp;
  p.sx2 = r.sx2;
  p.zp2 = r.zp2;
  p.wscale = w->scale;
  p.wcolsum = w->colsum;
  p.bias = (r.epi == EPI_GATED) ? w->bias : r.bias;
  p.y = r.y;
  p.ldy = r.ldy;
  p.work = r.work;
  p.ldw = r.ldw;
  p.accumulate = r.accumulate;
  p.rgate = r.rgate;
  p.rgate_rows = r.rgate_rows;
  for (int i = 0; i < 4; i++) p.outs[i] = r.outs[i];
  p.seg = r.seg;
  p.hidden = r.hidden;
  p.ldh = r.ldh;
  p.H = w->hidden;
  p.hn_q = r.hn_q;
  p.hn_k = r.hn_k;
  p.rcos = r.rcos;
  p.rsin = r.rsin;
  p.hq = r.hq;
  p.hk = r.hk;
  p.hvt = r.hvt;
  p.vt_ld = r.vt_ld;
  p.tokens = r.tokens;
  p.heads = r.seg / 64;
  p.eps = r.eps;
  p.err = c->err;
  p.limit_ns = kWaitLimitNs;
  switch (r.epi) {
    case EPI_LINEAR: {
      if (!r.y) return IRO_ERR_INVALID;
      const int bn = r.force_bn ? r.force_bn : pick_bn(r.M, w->N, c->num_sms, 0);
      if (bn == 256) return launch_t<256, EPI_LINEAR>(c, r, p, s);
      if (bn == 128) return launch_t<128, EPI_LINEAR>(c, r, p, s);
      return launch_t<64, EPI_LINEAR>(c, r, p, s);
    }
    case EPI_SPLIT: {
      if (r.nout < 1 || r.nout > 4 || r.seg <= 0 || r.seg % 32 != 0 ||
          r.seg * r.nout != w->N)
        return IRO_ERR_UNSUPPORTED;
      for (int i = 0; i < r.nout; i++)
        if (!r.outs[i]) return IRO_ERR_INVALID;
      const int bn = r.force_bn ? r.force_bn : pick_bn(r.M, w->N, c->num_sms, 0);
      if (bn == 256) return launch_t<256, EPI_SPLIT>(c, r, p, s);
      if (bn == 128) return launch_t<128, EPI_SPLIT>(c, r, p, s);
      return launch_t<64, EPI_SPLIT>(c, r, p, s);
    }
    case EPI_QKV: {
      // Four segments of whole 64-column heads; one head per epilogue warp
      // needs 256-column tiles.
      if (r.nout != 4 || r.seg <= 0 || r.seg % 64 != 0 || r.seg * 4 != w->N || r.accumulate ||
          r.bias ||  // the bias slot carries the norm weights
          r.work || r.tokens <= 0 || r.M % r.tokens != 0 || r.vt_ld < r.tokens ||
          r.vt_ld - r.tokens > 7 || r.vt_ld % 8 != 0)
        return IRO_ERR_UNSUPPORTED;
      if (!r.hq || !r.hk || !r.outs[3] || !r.hvt || !r.hn_q || !r.hn_k || !r.rcos || !r.rsin)
        return IRO_ERR_INVALID;
      // Vector loads of the norm weights and the grouped RoPE tables, vector
      // stores of the fp16 q and k rows.
      for (const void* q : {(const void*)r.hn_q, (const void*)r.hn_k, (const void*)r.rcos,
                            (const void*)r.rsin, (const void*)r.hq, (const void*)r.hk})
        if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0) return IRO_ERR_UNSUPPORTED;
      return launch_t<256, EPI_QKV>(c, r, p, s);
    }
    case EPI_GATED:
      // The tile holds one pair block: `pair` W1 rows then the matching W3 rows.
      if (w->layout != IRO_LAYOUT_GATED_PAIR || !r.hidden) return IRO_ERR_UNSUPPORTED;
      if (w->pair == 128) return launch_t<256, EPI_GATED>(c, r, p, s);
      if (w->pair == 64) return launch_t<128, EPI_GATED>(c, r, p, s);
      return IRO_ERR_UNSUPPORTED;
    case EPI_DUAL: {
      // With nout > 0 the columns go to nout buffers of `seg` columns each
      // (the QKVG split, for the two-term QKVG policy); y is then unused.
      if (!r.a2 || !r.sx2 || !r.zp2) return IRO_ERR_INVALID;
      if (r.nout > 0) {
        if (r.nout > 4 || r.seg <= 0 || r.seg % 128 != 0 || r.seg * r.nout != w->N ||
            r.accumulate || r.rgate)
          return IRO_ERR_UNSUPPORTED;
        for (int i = 0; i < r.nout; i++)
          if (!r.outs[i]) return IRO_ERR_INVALID;
      } else if (!r.y) {
        return IRO_ERR_INVALID;
      }
      // Into y: both terms stacked in one A tile, N = 256 MMAs.
      if (r.nout == 0 && !r.force_bn && pair_pays(r, c->num_sms))
        return launch_t<256, EPI_DUAL2, true>(c, r, p, s);
      if (r.nout == 0 && !r.force_bn) return launch_t<256, EPI_DUAL2>(c, r, p, s);
      const int bn = r.force_bn ? r.force_bn : pick_bn(r.M, w->N, c->num_sms, 1);
      if (bn == 128) return launch_t<128, EPI_DUAL>(c, r, p, s);
      return launch_t<64, EPI_DUAL>(c, r, p, s);
    }
    default:
      return IRO_ERR_INVALID;
  }
}

}  // namespace iro
