// dit_attention.cu — the DiT block's joint attention (dit.c:806-862) on the
// 5th-generation tensor cores.
//
// One CTA per (128-query tile, head, batch row).  Keys are the row's S self
// tokens followed by its context block (C tokens, invalid ones masked out),
// in tiles of 64 keys; two CTAs share an SM (99 KB of shared memory and 256
// TMEM columns each), so each SM sub-partition runs two softmax warps:
//
//   transpose   V (and the context V) to per-head V^T rows [64 dims x keys]
//               in the workspace, so that both products take K-major
//               operands (v_transpose_kernel)
//   TMA warp    Q tile once, then K and V^T tiles through a two-stage ring,
//               fp32 with the 128-byte swizzle (128 B rows of 32 floats)
//   MMA warp    S_j = Q K_j^T    (tcgen05 kind::tf32, 128 x 64, K = 64,
//                                 accumulator in TMEM, three S/P buffers)
//               O  += P_j V_j    (A = P_j straight from TMEM, B = V_j^T
//                                 K-major in shared memory, 128 x 64 in TMEM)
//   4 warps     one query row per thread: scores from TMEM, scale 1/8, mask,
//               online softmax, P_j written back over S_j in TMEM; at the
//               end O / l times the sigmoid gate (ops.c:786-789) to `mix`.
//
// Softmax runs in the log2 domain (t = s / 8 * log2 e, p = 2^(t - m) with
// ex2.approx, one FFMA and one MUFU op per score).  The running maximum is
// only raised (and O rescaled in TMEM) when a tile's maximum exceeds it by
// more than log2(e^8), so p <= e^8 and O is rescaled a handful of times per
// row rather than once per tile.  Since p / sum p does not depend on m, this
// changes rounding only.  The products run in tf32 (operands rounded to a
// 10-bit mantissa, fp32 accumulation): about 1e-3 relative error on the
// attention output, against exact fp32 products in attention_kernel
// (dit_block.cu), which IRO_DIT_ATTENTION=simt selects.
//
// Every wait is bounded (DevError + abort flag); on give-up each role drains
// what it issued before the TMEM is freed.
#include <math.h>
#include <string.h>

#include "dit_attention.cuh"

namespace iro {
namespace {

constexpr int kQ = 128;                 // queries per CTA (MMA M)
constexpr int kKT = 64;                 // keys per tile
constexpr int kDH = 64;                 // head dimension
constexpr int kThreads = 192;           // TMA warp, MMA warp, 4 softmax warps
constexpr int kQHalf = kQ * 128;        // 128 query rows x 32 floats
constexpr int kQBytes = 2 * kQHalf;
constexpr int kKHalf = kKT * 128;       // 64 key rows x 32 floats
constexpr int kKBytes = 2 * kKHalf;
constexpr int kVtChunk = kDH * 128;     // V^T tile chunk: 64 dim rows x 32 keys
constexpr int kVBytes = (kKT / 32) * kVtChunk;
constexpr int kBarOff = kQBytes + 2 * kKBytes + 2 * kVBytes;  // 96 KB of tiles
constexpr int kMaxCtxWords = 256;       // context mask bits in shared memory (C <= 8192)
constexpr int kSmem = 1024 + kBarOff + 256 + 4 * kMaxCtxWords;
// Two CTAs per SM: 2 x 99 KB of shared memory, 2 x 256 TMEM columns.
constexpr uint32_t kTmemCols = 256;
constexpr int kSBufs = 3;               // S/P buffers in TMEM
constexpr int kPvLag = 1;               // PVs issued between PV_j and S_{j+3}
constexpr uint32_t kColO = kSBufs * kKT;  // S/P buffers at columns 0, 64, 128; O at 192
// Scores are kept in the log2 domain: t = s_raw * (1/8) * log2(e), p = 2^(t - m).
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
constexpr float kRescaleGap = 8.0f * 1.4426950408889634f;  // e^8 in the log2 domain

// vt[((b * heads + h) * 64 + d) * ld + s] = v[(b * S + s) * D + h * 64 + d],
// zero for s in [S, ld).  One block per (32 tokens, head, row block).
__global__ void __launch_bounds__(256) v_transpose_kernel(const float* __restrict__ v,
                                                          float* __restrict__ vt, int S, int D,
                                                          int heads, int ld) {
  __shared__ float tile[kDH][33];
  const int s0 = blockIdx.x * 32, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x;
  for (int i = t; i < 32 * kDH; i += 256) {
    const int ss = i / kDH, d = i % kDH;
    const int s = s0 + ss;
    tile[d][ss] = s < S ? v[((size_t)b * S + s) * D + (size_t)h * kDH + d] : 0.0f;
  }
  __syncthreads();
  for (int i = t; i < 32 * kDH; i += 256) {
    const int d = i / 32, ss = i % 32;
    const int s = s0 + ss;
    if (s < ld) vt[(((size_t)b * heads + h) * kDH + d) * ld + s] = tile[d][ss];
  }
}

struct Args {
  int S, C, ctx_group, n_self, n_ctx, D, heads;
  const uint8_t* mask;  // [B, C]
  const float* g;       // gate projection [B*S, D]
  float* mix;           // output [B*S, D]
  DevError* err;
  uint64_t limit_ns;
  // Diagnostic dump of CTA (0, 0, 0), null in the library: raw scores of the
  // first key tile [128][128], then per row O [128][64], l [128], m [128].
  float* dbg;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// CTA pairs (a two-CTA cluster sharing one tcgen05 MMA of M = 256).
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Bounded wait with cluster-scope acquire: for phases completed by arrivals
// from the peer CTA's threads (their TMEM writes must be visible here).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, DevError* err,
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

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr)
               : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t mbar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar_cluster)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_ss_pair(uint32_t d, uint64_t a, uint64_t b,
                                                 uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_ts_pair(uint32_t d, uint32_t a, uint64_t b,
                                                 uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive on the same barrier in both CTAs of the pair once the pair's MMAs
// issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

template <int N>
__device__ __forceinline__ uint32_t (&sub32(uint32_t (&r)[N], int c))[32] {
  return *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]);
}

// PAIR: a two-CTA cluster computes 256 query rows with M = 256 MMAs issued
// by the leader (rank 0); each CTA loads its own Q rows, half of each K tile
// (32 of 64 keys) and half of each V^T tile (32 of 64 dimensions), and the
// TMA completions, P hand-offs and MMA commits meet on the leader's barriers
// (commits multicast to both CTAs).  Otherwise one CTA runs M = 128.
template <bool PAIR>
__global__ void __launch_bounds__(kThreads, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmCK,
                        const __grid_constant__ CUtensorMap tmCV, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kQBytes;         // two stages
  uint8_t* sV = sK + 2 * kKBytes;       // two stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* q_full = bars;         // 1
  uint64_t* k_full = bars + 1;     // 2 stages
  uint64_t* v_full = bars + 3;     // 2 stages
  uint64_t* k_empty = bars + 5;    // 2 stages (after S)
  uint64_t* v_empty = bars + 7;    // 2 stages (after PV)
  uint64_t* s_full = bars + 9;     // 3 S/P buffers
  uint64_t* p_full = bars + 12;    // 3
  uint64_t* pv_done = bars + 15;   // 3
  uint64_t* drain = bars + 18;     // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* ctx_bits = reinterpret_cast<uint32_t*>(smem + kBarOff + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, hd = blockIdx.y, q0 = blockIdx.x * kQ;
  const int T = a.n_self + a.n_ctx;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  // Per-CTA shares of the K and V^T tiles (bytes of one 32-wide slice).
  constexpr int KH = (PAIR ? kKT / 2 : kKT) * 128;   // K rows x 128 B
  constexpr int VC = (PAIR ? kDH / 2 : kDH) * 128;   // V^T rows x 128 B
  constexpr uint32_t IDS = idesc_tf32(PAIR ? 2 * kQ : kQ, kKT, 0);
  constexpr uint32_t IDPV = idesc_tf32(PAIR ? 2 * kQ : kQ, kDH, 0);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < kSBufs; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], PAIR ? 256 : 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmCK);
    tma_prefetch_desc(&tmCV);
  }
  if (warp == 1) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // the leader's barriers exist before the peer uses them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();

  if (warp == 0) {
    // ---------------- TMA producers: lane 0 Q and K, lane 1 V^T ----------------
    if (lane < 2) {
      const int cb = b / a.ctx_group;
      int issued = 0;
      if (lane == 0) {
        const int qrow0 = b * a.S + q0;
        if (PAIR) {
          // The leader's MMAs read both CTAs' Q rows: both loads count on the
          // leader's q_full.
          const uint32_t qb = cluster_addr(q_full, 0);
          if (leader) mbar_arrive_expect_tx(q_full, 2 * kQBytes);
          tma_load_2d_pair(sQ, &tmQ, qb, hd * kDH, qrow0);
          tma_load_2d_pair(sQ + kQHalf, &tmQ, qb, hd * kDH + 32, qrow0);
        } else {
          mbar_arrive_expect_tx(q_full, kQBytes);
          tma_load_2d(sQ, &tmQ, q_full, hd * kDH, qrow0);
          tma_load_2d(sQ + kQHalf, &tmQ, q_full, hd * kDH + 32, qrow0);
        }
      }
      uint64_t* full = lane == 0 ? k_full : v_full;
      uint64_t* empty = lane == 0 ? k_empty : v_empty;
      for (int j = 0; j < T; j++) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait_bounded(&empty[st], ((j - 2) >> 1) & 1, a.err, 1, abort_flag,
                                         a.limit_ns))
          break;
        const bool self = j < a.n_self;
        const uint32_t fb = PAIR ? cluster_addr(&full[st], 0) : 0u;
        if (lane == 0) {
          // This CTA's key rows of tile j.
          const CUtensorMap* mk = self ? &tmK : &tmCK;
          const int y = (self ? b * a.S + j * kKT : cb * a.C + (j - a.n_self) * kKT) +
                        (int)rank * (KH / 128);
          uint8_t* dk = sK + st * kKBytes;
          if (PAIR) {
            // Both CTAs' halves complete on the leader's barrier, which
            // expects the pair's bytes (one CTA's full-tile total).
            if (leader) mbar_arrive_expect_tx(&full[st], kKBytes);
            tma_load_2d_pair(dk, mk, fb, hd * kDH, y);
            tma_load_2d_pair(dk + KH, mk, fb, hd * kDH + 32, y);
          } else {
            mbar_arrive_expect_tx(&full[st], kKBytes);
            tma_load_2d(dk, mk, &full[st], hd * kDH, y);
            tma_load_2d(dk + KH, mk, &full[st], hd * kDH + 32, y);
          }
        } else {
          // This CTA's V^T rows (head dimensions) of tile j.
          const CUtensorMap* mv = self ? &tmV : &tmCV;
          const int x0 = (self ? j : j - a.n_self) * kKT;
          const int vrow = ((self ? b : cb) * a.heads + hd) * kDH + (int)rank * (VC / 128);
          uint8_t* dv = sV + st * kVBytes;
          if (PAIR) {
            if (leader) mbar_arrive_expect_tx(&full[st], kVBytes);
#pragma unroll
            for (int c = 0; c < kKT / 32; c++) tma_load_2d_pair(dv + c * VC, mv, fb, x0 + 32 * c, vrow);
          } else {
            mbar_arrive_expect_tx(&full[st], kVBytes);
#pragma unroll
            for (int c = 0; c < kKT / 32; c++)
              tma_load_2d(dv + c * VC, mv, &full[st], x0 + 32 * c, vrow);
          }
        }
        issued = j + 1;
      }
      // Drain: every load issued has landed before the CTA may exit (on the
      // normal path these phases completed long ago).
      if (leader && lane == 0) mbar_wait_bounded(q_full, 0, a.err, 9, nullptr, a.limit_ns);
      for (int j = issued - 1; leader && j >= 0 && j >= issued - 2; j--)
        mbar_wait_bounded(&full[j & 1], (j >> 1) & 1, a.err, 9, nullptr, a.limit_ns);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (the leader's, for a pair) ----------------
    // Order (kPvLag = 1): S_0 S_1 S_2 | PV_0 | PV_1 S_3 | PV_2 S_4 | ... |
    // PV_{T-1}.  With three S/P buffers S_{j+3} needs PV_j complete; issued
    // after PV_{j+1}, its wait overlaps PV_{j+1} in the tensor pipe instead of
    // draining it.  (Measured at config 3 it runs at the same speed as
    // kPvLag = 0, S_{j+3} right after PV_j.)
    if (lane == 0 && leader) {
      const uint32_t q_addr = smem_u32(sQ);
      auto commit = [&](uint64_t* bar) {
        if (PAIR) mma_commit_pair(bar);
        else mma_commit(bar);
      };
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1, sb = j % kSBufs;
        if (!mbar_wait_bounded(&k_full[st], (j >> 1) & 1, a.err, 3, abort_flag, a.limit_ns))
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * kKBytes);
        const uint32_t d = tmem + (uint32_t)(sb * kKT);
#pragma unroll
        for (int ks = 0; ks < kDH / 8; ks++) {
          const uint32_t qo = (uint32_t)((ks >> 2) * kQHalf + (ks & 3) * 32);
          const uint32_t ko = (uint32_t)((ks >> 2) * KH + (ks & 3) * 32);
          if (PAIR)
            mma_tf32_ss_pair(d, sw128_desc(q_addr + qo), sw128_desc(k_addr + ko), IDS,
                             ks > 0 ? 1u : 0u);
          else
            mma_tf32_ss(d, sw128_desc(q_addr + qo), sw128_desc(k_addr + ko), IDS,
                        ks > 0 ? 1u : 0u);
        }
        commit(&s_full[sb]);
        commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j & 1, sb = j % kSBufs;
        if (!(PAIR ? mbar_wait_cluster(&p_full[sb], (j / kSBufs) & 1, a.err, 5, abort_flag,
                                       a.limit_ns)
                   : mbar_wait_bounded(&p_full[sb], (j / kSBufs) & 1, a.err, 5, abort_flag,
                                       a.limit_ns)) ||
            !mbar_wait_bounded(&v_full[st], (j >> 1) & 1, a.err, 6, abort_flag, a.limit_ns))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * kVBytes);
        const uint32_t p_tmem = tmem + (uint32_t)(sb * kKT);
#pragma unroll
        for (int ks = 0; ks < kKT / 8; ks++) {
          const uint64_t vd = sw128_desc(v_addr + (uint32_t)((ks >> 2) * VC + (ks & 3) * 32));
          if (PAIR)
            mma_tf32_ts_pair(tmem + kColO, p_tmem + (uint32_t)(ks * 8), vd, IDPV,
                             (j > 0 || ks > 0) ? 1u : 0u);
          else
            mma_tf32_ts(tmem + kColO, p_tmem + (uint32_t)(ks * 8), vd, IDPV,
                        (j > 0 || ks > 0) ? 1u : 0u);
        }
        commit(&pv_done[sb]);
        commit(&v_empty[st]);
        return true;
      };
      bool ok = mbar_wait_bounded(q_full, 0, a.err, 2, abort_flag, a.limit_ns);
      for (int j = 0; ok && j < kSBufs && j < T; j++) ok = issue_s(j);
      for (int j = 0; ok && j < T; j++) {
        ok = issue_pv(j);
        const int i = j - kPvLag;  // buffer i % 3 is free once PV_i has read P_i
        if (ok && i >= 0 && i + kSBufs < T) {
          ok = mbar_wait_bounded(&pv_done[i % kSBufs], (i / kSBufs) & 1, a.err, 4, abort_flag,
                                 a.limit_ns) &&
               issue_s(i + kSBufs);
        }
      }
      // Every S_{i+3} (i + 3 < T) was issued at iteration i + kPvLag < T.
      // Drain: all MMAs issued by this thread have completed.
      if (PAIR)
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                smem_u32(drain))
            : "memory");
      else
        mma_commit(drain);
      mbar_wait_bounded(drain, 0, a.err, 10, nullptr, a.limit_ns);
    }
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue (4 warps) ----------------
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    const int row = quad * 32 + lane;
    const int qrow = q0 + row;
    const int st_id = threadIdx.x - 64;  // 0..127
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    // The batch row's context mask as bits (dit.c:828-839).
    {
      const uint8_t* mrow = a.mask + (size_t)b * a.C;
      const int nw = a.n_ctx * (kKT / 32);  // whole tiles; bits past C stay 0
      for (int w = st_id; w < nw; w += 128) {
        uint32_t bits = 0;
        for (int k = 0; k < 32; k++) {
          const int c = w * 32 + k;
          if (c < a.C && mrow[c] != 0) bits |= 1u << k;
        }
        ctx_bits[w] = bits;
      }
      named_bar(1, 128);
    }
    float m = -INFINITY, l = 0.0f;  // running max (log2 domain) and sum
    bool ok = true;
    for (int j = 0; j < T; j++) {
      const int st = j % kSBufs;  // S/P buffer
      ok = mbar_wait_bounded(&s_full[st], (j / kSBufs) & 1, a.err, 7, abort_flag, a.limit_ns);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; c++)
        tmem_ld_32x32b_x32(lane_base + (uint32_t)(st * kKT + 32 * c), sub32(r, c));
      tmem_ld_wait();
      const bool dump = a.dbg != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
      if (dump && j == 0)
        for (int i = 0; i < kKT; i++) a.dbg[row * kKT + i] = __uint_as_float(r[i]);
      // Keys outside the row's set get -inf (their p is exactly 0).
      if (j < a.n_self) {
        const int lim = a.S - j * kKT;
        if (lim < kKT) {
#pragma unroll
          for (int i = 0; i < kKT; i++)
            if (i >= lim) r[i] = __float_as_uint(-INFINITY);
        }
      } else {
        const int w0 = (j - a.n_self) * (kKT / 32);
#pragma unroll
        for (int c = 0; c < kKT / 32; c++) {
          const uint32_t bits = ctx_bits[w0 + c];  // zero past C
#pragma unroll
          for (int i = 0; i < 32; i++)
            if (!((bits >> i) & 1u)) r[32 * c + i] = __float_as_uint(-INFINITY);
        }
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < kKT; i++) mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(r[i]));
      const float rmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      const float mnew = fmaxf(m, rmax * kScaleLog2);
      const bool need = mnew > m + kRescaleGap;
      if (__any_sync(0xffffffffu, need)) {
        const float f = need ? ex2_approx(m - mnew) : 1.0f;
        if (j > 0) {
          // O is quiescent once PV_{j-1} is done (PV_j waits for this tile's P).
          ok = mbar_wait_bounded(&pv_done[(j - 1) % kSBufs], ((j - 1) / kSBufs) & 1, a.err, 8,
                                 abort_flag, a.limit_ns);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < kDH / 32; c++) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(lane_base + kColO + (uint32_t)(32 * c), o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st_32x32b_x32(lane_base + kColO + (uint32_t)(32 * c), o);
          }
        }
        if (need) {
          l *= f;
          m = mnew;
        }
      }
      float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const float neg_m = -m;
#pragma unroll
      for (int i = 0; i < kKT; i++) {
        const float p = ex2_approx(fmaf(__uint_as_float(r[i]), kScaleLog2, neg_m));
        ps[i & 3] += p;
        r[i] = __float_as_uint(p);
      }
      l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
#pragma unroll
      for (int c = 0; c < kKT / 32; c++)
        tmem_st_32x32b_x32(lane_base + (uint32_t)(st * kKT + 32 * c), sub32(r, c));
      tmem_st_wait();
      tc_fence_before();
      if (PAIR) mbar_arrive_cluster(cluster_addr(&p_full[st], 0));
      else mbar_arrive(&p_full[st]);
    }
    if (ok) {
      ok = mbar_wait_bounded(&pv_done[(T - 1) % kSBufs], ((T - 1) / kSBufs) & 1, a.err, 11,
                             abort_flag, a.limit_ns);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      uint32_t o[kDH];
#pragma unroll
      for (int c = 0; c < kDH / 32; c++)
        tmem_ld_32x32b_x32(lane_base + kColO + (uint32_t)(32 * c), sub32(o, c));
      tmem_ld_wait();
      if (a.dbg != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
        for (int i = 0; i < kDH; i++) a.dbg[kQ * kKT + row * kDH + i] = __uint_as_float(o[i]);  // O
        a.dbg[kQ * kKT + kQ * kDH + row] = l;
        a.dbg[kQ * kKT + kQ * kDH + kQ + row] = m;
      }
      if (qrow < a.S) {
        const size_t off = ((size_t)b * a.S + qrow) * a.D + (size_t)hd * kDH;
        const float4* gr = reinterpret_cast<const float4*>(a.g + off);
        float4* out = reinterpret_cast<float4*>(a.mix + off);
        const float inv_l = __fdiv_rn(1.0f, l);
#pragma unroll
        for (int i = 0; i < kDH / 4; i++) {
          const float4 gv = gr[i];
          float4 ov;
          ov.x = __fmul_rn(__fmul_rn(__uint_as_float(o[4 * i]), inv_l),
                           __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv.x))));
          ov.y = __fmul_rn(__fmul_rn(__uint_as_float(o[4 * i + 1]), inv_l),
                           __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv.y))));
          ov.z = __fmul_rn(__fmul_rn(__uint_as_float(o[4 * i + 2]), inv_l),
                           __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv.z))));
          ov.w = __fmul_rn(__fmul_rn(__uint_as_float(o[4 * i + 3]), inv_l),
                           __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv.w))));
          out[i] = ov;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // the leader's MMAs no longer read this CTA
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(kTmemCols)
                   : "memory");
    else
      tmem_dealloc(tmem, kTmemCols);
  }
}

int map2d(CUtensorMap* m, const float* base, int inner, long long rows, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)inner * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

int vt_ld(int n) { return (n + 3) / 4 * 4; }  // 16-byte row pitch

}  // namespace

int attention_tc_vt_ld(int n) { return vt_ld(n); }

namespace {

}  // namespace

size_t attention_tc_workspace_bytes(int B, int S, int C, int context_batch, int D) {
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  return al(sizeof(float) * (size_t)B * D * vt_ld(S)) +
         al(sizeof(float) * (size_t)context_batch * D * vt_ld(C));
}

bool attention_tc_supported(const AttnTcRequest& r) {
  if (cdiv(r.C, kKT) * (kKT / 32) > kMaxCtxWords) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return r.D % 64 == 0 && r.D == r.heads * kDH && al16(r.q) && al16(r.k) && al16(r.v) &&
         al16(r.g) && al16(r.mix) && al16(r.ck) && al16(r.cv) && al16(r.workspace) &&
         r.S > 0 && r.C > 0 && r.B > 0 && r.context_batch > 0 && r.B % r.context_batch == 0;
}

int attention_tc_launch(Ctx* c, const AttnTcRequest& r, cudaStream_t s) {
  if (!attention_tc_supported(r)) return IRO_ERR_UNSUPPORTED;
  const bool pair = !r.single_cta;
  static bool attr_done[64][2] = {{false}};
  if (!attr_done[c->device][pair]) {
    cudaError_t e = pair ? cudaFuncSetAttribute(attention_tc_kernel<true>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem)
                         : cudaFuncSetAttribute(attention_tc_kernel<false>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
    attr_done[c->device][pair] = true;
  }
  // V^T of the self tokens and of the context block.
  const int lds = vt_ld(r.S), ldc = vt_ld(r.C);
  float* vt = static_cast<float*>(r.workspace);
  float* cvt = vt + ((sizeof(float) * (size_t)r.B * r.D * lds + 255) / 256 * 256) / sizeof(float);
  int st;
  if (r.vt_self == nullptr) {
    v_transpose_kernel<<<dim3(cdiv(lds, 32), r.heads, r.B), 256, 0, s>>>(r.v, vt, r.S, r.D,
                                                                          r.heads, lds);
    if ((st = check_launch())) return st;
  } else if (r.vt_self != vt) {
    return IRO_ERR_INVALID;
  }
  v_transpose_kernel<<<dim3(cdiv(ldc, 32), r.heads, r.context_batch), 256, 0, s>>>(
      r.cv, cvt, r.C, r.D, r.heads, ldc);
  if ((st = check_launch())) return st;
  CUtensorMap mq, mk, mv, mck, mcv;
  const long long rows = (long long)r.B * r.S, crows = (long long)r.context_batch * r.C;
  // A CTA of a pair loads half of each K tile (32 keys) and of each V^T tile
  // (32 dimensions).
  const int krows = pair ? kKT / 2 : kKT, vrows = pair ? kDH / 2 : kDH;
  st = map2d(&mq, r.q, r.D, rows, kQ);
  if (!st) st = map2d(&mk, r.k, r.D, rows, krows);
  if (!st) st = map2d(&mv, vt, lds, (long long)r.B * r.D, vrows);
  if (!st) st = map2d(&mck, r.ck, r.D, crows, krows);
  if (!st) st = map2d(&mcv, cvt, ldc, (long long)r.context_batch * r.D, vrows);
  if (st) return st;
  Args a;
  a.S = r.S;
  a.C = r.C;
  a.ctx_group = r.B / r.context_batch;
  a.n_self = cdiv(r.S, kKT);
  a.n_ctx = cdiv(r.C, kKT);
  a.D = r.D;
  a.heads = r.heads;
  a.mask = r.mask;
  a.g = r.g;
  a.mix = r.mix;
  a.err = c->err;
  a.limit_ns = kWaitLimitNs;
  a.dbg = nullptr;
  cudaError_t e;
  if (pair) {
    // Pairs of CTAs (a two-CTA cluster) over 256 query rows.
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(2 * cdiv(r.S, 2 * kQ), r.heads, r.B);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)kSmem;
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
    e = cudaLaunchKernelEx(&cfg, attention_tc_kernel<true>, mq, mk, mv, mck, mcv, a);
  } else {
    const dim3 grid(cdiv(r.S, kQ), r.heads, r.B);
    e = launch_pdl(attention_tc_kernel<false>, grid, dim3(kThreads), (size_t)kSmem, s, mq, mk, mv,
                   mck, mcv, a);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

}  // namespace iro
