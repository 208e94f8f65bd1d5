// dit_attention.cu — the DiT block's joint attention (dit.c:806-862) on the
// 5th-generation tensor cores: fp16 operands, fp32 accumulation.
//
// One CTA per (128-query tile, head, batch row), two CTAs per SM (82 KB of
// shared memory and 256 TMEM columns each).  Keys are the row's S self
// tokens followed by its context block (C tokens, invalid ones masked out),
// in tiles of 128:
//
//   operands    q, k [B*S, D] and the per-head V^T rows [64 dims x keys] in
//               fp16 (written by the QKVG epilogue), the context keys and
//               V^T converted from fp32 by context_prep_kernel
//   TMA warp    Q tile once, then K and V^T tiles through a two-stage ring
//               (128-byte swizzled rows of 64 halves)
//   MMA warp    S_j = Q K_j^T  (kind::f16, 128 x 128, K = 64 in 4 steps)
//               into TMEM columns [0, 128);
//               O += P_j V_j   (A = P_j as fp16 pairs in TMEM columns
//               [128, 192), B = V_j^T K-major in shared memory) into [192, 256)
//   4 warps     one query row per thread: scores from TMEM, scale 1/8, mask,
//               online softmax, P_j packed to fp16 pairs into TMEM; at the
//               end O / l times the sigmoid gate (ops.c:786-789) to `mix`.
//
// The softmax warps release S_j as soon as it sits in registers, so S_{j+1}
// runs on the tensor cores during softmax_j, and PV_j right after it; P_{j+1}
// is stored once PV_j has read P_j.  The other CTA on the SM interleaves its
// own tiles.  A tcgen05 MMA costs by its byte shape (128 rows x N x 32 bytes
// of K): one kind::f16 step does the work of two kind::tf32 steps, and one
// N = 128 step costs 66 cycles against 2 x 50 for two N = 64 steps.
//
// Softmax runs in the log2 domain (t = s / 8 * log2 e, p = 2^(t - m) with
// ex2.approx, one FFMA and one MUFU op per score).  The running maximum is
// only raised (and O rescaled in TMEM) when a tile's maximum exceeds it by
// more than log2(e^8), so p <= e^8 (well inside fp16) and O is rescaled a
// handful of times per row.  Since p / sum p does not depend on m, this
// changes rounding only.  The operands are rounded to fp16 (10-bit
// mantissa) when they are written, against exact fp32 products in
// attention_kernel (dit_block.cu, IRO_DIT_ATTENTION=simt); they must stay
// below 65520 in magnitude, which every producer checks (IRO_ERR_RANGE).
// p below 2^-14 is stored as an fp16 subnormal: an absolute error under
// 2^-25 against l >= 1.
//
// Every wait is bounded (DevError + abort flag); on give-up each role drains
// what it issued before the TMEM is freed.
#include <math.h>
#include <string.h>

#include "dit_attention.cuh"

namespace iro {
namespace {

constexpr int kQ = 128;                      // queries per CTA (MMA M)
constexpr int kKT = 128;                     // keys per tile (S MMA N)
constexpr int kDH = 64;                      // head dimension
constexpr int kThreads = 320;                // TMA warp, MMA warp, 8 softmax warps
constexpr int kRow = 128;                    // bytes per swizzled row: 64 halves
constexpr int kQBytes = kQ * kRow;           // 16 KB
constexpr int kKBytes = kKT * kRow;          // 16 KB
constexpr int kVChunk = kDH * kRow;          // V^T chunk: 64 dim rows x 64 keys
constexpr int kVBytes = (kKT / 64) * kVChunk;  // 16 KB
constexpr int kStages = 2;
constexpr int kBarOff = kQBytes + kStages * (kKBytes + kVBytes);  // 80 KB of tiles
constexpr int kMaxCtxWords = 256;            // context mask bits in shared memory (C <= 8192)
// Barriers, the context mask bits, then the softmax partners' row maxima
// (2 tiles x 2 halves x 128) and sums (2 x 128).
constexpr int kSmem = 1024 + kBarOff + 256 + 4 * kMaxCtxWords + 4 * (4 * kQ + 2 * kQ);
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192;
// Scores are kept in the log2 domain: t = s_raw * (1/8) * log2(e), p = 2^(t - m).
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
constexpr float kRescaleGap = 8.0f * 1.4426950408889634f;  // e^8 in the log2 domain

// Range-check sites (DevError.where) of the fp16 producers.
enum { kSiteCtxK = 100, kSiteCtxV = 101 };

// The context block's keys and V^T in fp16: ck[(cb * C + s) * D + h * 64 + d]
// = ck32[...] and cvt[((cb * heads + h) * 64 + d) * ldc + s] = cv32[(cb * C +
// s) * D + h * 64 + d], zero for s in [C, ldc).  One block per (32 tokens,
// head, context block).
__global__ void __launch_bounds__(256) context_prep_kernel(const float* __restrict__ ck32,
                                                           const float* __restrict__ cv32,
                                                           __half* __restrict__ ck,
                                                           __half* __restrict__ cvt, int C,
                                                           int D, int heads, int ldc,
                                                           DevError* err) {
  __shared__ float tile[kDH][33];
  const int s0 = blockIdx.x * 32, h = blockIdx.y, cb = blockIdx.z;
  const int t = threadIdx.x;
  for (int i = t; i < 32 * kDH; i += 256) {
    const int ss = i / kDH, d = i % kDH;
    const int s = s0 + ss;
    const size_t off = ((size_t)cb * C + s) * D + (size_t)h * kDH + d;
    float v = 0.0f;
    if (s < C) {
      ck[off] = to_half_checked(ck32[off], err, kSiteCtxK);
      v = cv32[off];
    }
    tile[d][ss] = v;
  }
  __syncthreads();
  for (int i = t; i < 32 * kDH; i += 256) {
    const int d = i / 32, ss = i % 32;
    const int s = s0 + ss;
    if (s < ldc)
      cvt[(((size_t)cb * heads + h) * kDH + d) * ldc + s] = to_half_checked(tile[d][ss], err,
                                                                            kSiteCtxV);
  }
}

struct Args {
  int S, C, ctx_group, n_self, n_ctx, D, heads;
  const uint8_t* mask;  // [B, C]
  const float* g;       // gate projection [B*S, D]
  float* mix;           // output [B*S, D]
  DevError* err;
  uint64_t limit_ns;
};

// max(a, b, c) in one instruction (three-input max, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// a * b + c and a + b on packed pairs (fma / add .f32x2, sm_100), each lane
// rounded as its scalar form.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int N>
__device__ __forceinline__ uint32_t (&sub32(uint32_t (&r)[N], int c))[32] {
  return *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]);
}

__global__ void __launch_bounds__(kThreads, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmCK,
                        const __grid_constant__ CUtensorMap tmCV,
                        const __grid_constant__ CUtensorMap tmG, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kQBytes;             // kStages stages
  uint8_t* sV = sK + kStages * kKBytes;     // kStages stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* q_full = bars;         // 1
  uint64_t* k_full = bars + 1;     // 2 stages
  uint64_t* v_full = bars + 3;     // 2 stages
  uint64_t* k_empty = bars + 5;    // 2 stages (after S)
  uint64_t* v_empty = bars + 7;    // 2 stages (after PV)
  uint64_t* s_full = bars + 9;     // S_j in TMEM
  uint64_t* s_free = bars + 10;    // S_j read by the softmax warps (256 arrivals)
  uint64_t* p_full = bars + 11;    // P_j in TMEM (256 arrivals)
  uint64_t* pv_done = bars + 12;   // PV_j complete (P free, O quiescent)
  uint64_t* drain = bars + 13;
  uint64_t* xbar = bars + 14;      // 4: the softmax partners of each TMEM quadrant (64 arrivals)
  uint64_t* g_full = bars + 18;    // the gate tile in the freed K stages
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* ctx_bits = reinterpret_cast<uint32_t*>(smem + kBarOff + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, hd = blockIdx.y, q0 = blockIdx.x * kQ;
  const int T = a.n_self + a.n_ctx;
  constexpr uint32_t IDS = idesc_f16(kQ, kKT);
  constexpr uint32_t IDPV = idesc_f16(kQ, kDH);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(p_full, 256);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 4; i++) mbar_init(&xbar[i], 64);
    mbar_init(g_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmCK);
    tma_prefetch_desc(&tmCV);
    tma_prefetch_desc(&tmG);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();

  if (warp == 0) {
    // ---------------- TMA producers: lane 0 Q and K, lane 1 V^T ----------------
    if (lane < 2) {
      const int cb = b / a.ctx_group;
      int issued = 0;
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_2d(sQ, &tmQ, q_full, hd * kDH, b * a.S + q0);
      }
      uint64_t* full = lane == 0 ? k_full : v_full;
      uint64_t* empty = lane == 0 ? k_empty : v_empty;
      for (int j = 0; j < T; j++) {
        const int st = j & 1;
        if (j >= kStages && !mbar_wait_bounded(&empty[st], ((j - kStages) >> 1) & 1, a.err, 1,
                                               abort_flag, a.limit_ns))
          break;
        const bool self = j < a.n_self;
        if (lane == 0) {
          const CUtensorMap* mk = self ? &tmK : &tmCK;
          const int y = self ? b * a.S + j * kKT : cb * a.C + (j - a.n_self) * kKT;
          mbar_arrive_expect_tx(&full[st], kKBytes);
          tma_load_2d(sK + st * kKBytes, mk, &full[st], hd * kDH, y);
        } else {
          // V^T rows (head dimensions) of tile j, in two chunks of 64 keys.
          const CUtensorMap* mv = self ? &tmV : &tmCV;
          const int x0 = (self ? j : j - a.n_self) * kKT;
          const int vrow = ((self ? b : cb) * a.heads + hd) * kDH;
          uint8_t* dv = sV + st * kVBytes;
          mbar_arrive_expect_tx(&full[st], kVBytes);
#pragma unroll
          for (int c = 0; c < kKT / 64; c++)
            tma_load_2d(dv + c * kVChunk, mv, &full[st], x0 + 64 * c, vrow);
        }
        issued = j + 1;
      }
      // The gate tile [128 rows x 64 dims] fp32, for the epilogue, into the
      // two K stages once the last S products have read them (dims 32 c ..
      // 32 c + 31 into stage c, 128-byte swizzled rows).
      bool g_issued = false;
      if (lane == 0 && issued == T) {
        bool ok = true;
        for (int j = T - 1; ok && j >= 0 && j >= T - kStages; j--)
          ok = mbar_wait_bounded(&k_empty[j & 1], (j >> 1) & 1, a.err, 15, abort_flag,
                                 a.limit_ns);
        if (ok) {
          mbar_arrive_expect_tx(g_full, kStages * kKBytes);
#pragma unroll
          for (int c = 0; c < 2; c++)
            tma_load_2d(sK + c * kKBytes, &tmG, g_full, hd * kDH + 32 * c, b * a.S + q0);
          g_issued = true;
        }
      }
      // Drain: every load issued has landed before the CTA may exit (on the
      // normal path these phases completed long ago).
      if (lane == 0) mbar_wait_bounded(q_full, 0, a.err, 9, nullptr, a.limit_ns);
      if (g_issued) mbar_wait_bounded(g_full, 0, a.err, 9, nullptr, a.limit_ns);
      for (int j = issued - 1; j >= 0 && j >= issued - kStages; j--)
        mbar_wait_bounded(&full[j & 1], (j >> 1) & 1, a.err, 9, nullptr, a.limit_ns);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // Order: S_0 | S_1 PV_0 | S_2 PV_1 | ... | PV_{T-1}.  S_{j+1} waits for
    // the softmax warps to have read S_j; PV_j for P_j.
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait_bounded(&k_full[st], (j >> 1) & 1, a.err, 3, abort_flag, a.limit_ns))
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * kKBytes);
#pragma unroll
        for (int ks = 0; ks < kDH / 16; ks++)
          mma_f16_ss(tmem + kColS, sw128_desc(q_addr + ks * 32), sw128_desc(k_addr + ks * 32),
                     IDS, ks > 0 ? 1u : 0u);
        mma_commit(s_full);
        mma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait_bounded(p_full, j & 1, a.err, 5, abort_flag, a.limit_ns) ||
            !mbar_wait_bounded(&v_full[st], (j >> 1) & 1, a.err, 6, abort_flag, a.limit_ns))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * kVBytes);
#pragma unroll
        for (int ks = 0; ks < kKT / 16; ks++) {
          // Keys 16 ks .. 16 ks + 15: chunk ks / 4 of the V^T tile, 32-byte
          // step ks % 4 inside its rows; P columns 8 ks .. 8 ks + 7.
          const uint64_t vd = sw128_desc(v_addr + (uint32_t)((ks >> 2) * kVChunk + (ks & 3) * 32));
          mma_f16_ts(tmem + kColO, tmem + kColP + (uint32_t)(ks * 8), vd, IDPV,
                     (j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(pv_done);
        mma_commit(&v_empty[st]);
        return true;
      };
      bool ok = mbar_wait_bounded(q_full, 0, a.err, 2, abort_flag, a.limit_ns) && issue_s(0);
      for (int j = 0; ok && j < T; j++) {
        if (j + 1 < T)
          ok = mbar_wait_bounded(s_free, j & 1, a.err, 4, abort_flag, a.limit_ns) &&
               issue_s(j + 1);
        ok = ok && issue_pv(j);
      }
      // Drain: all MMAs issued by this thread have completed.
      mma_commit(drain);
      mbar_wait_bounded(drain, 0, a.err, 10, nullptr, a.limit_ns);
    }
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue (8 warps) ----------------
    // Two threads per query row: warps 2-5 take keys 0-63 of each tile,
    // warps 6-9 keys 64-127 (a warp reads the TMEM lanes of quadrant warp % 4).
    // The partners meet once per tile on their quadrant's mbarrier (phase j
    // for tile j, phase T for the final sums) to share the row maximum; l is
    // summed per half and added at the end.  The meeting is a bounded wait
    // like every other one, so a partner that gave up cannot strand the
    // other (a hardware named barrier would wait for it forever).
    const int quad = warp & 3;          // TMEM lanes 32*quad .. 32*quad+31
    const int hf = (warp - 2) >> 2;     // key half of each tile
    const int row = quad * 32 + lane;
    const int qrow = q0 + row;
    const int st_id = threadIdx.x - 64;  // 0..255
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t colS = kColS + 64u * hf, colP = kColP + 32u * hf, colO = kColO + 32u * hf;
    float* xmax = reinterpret_cast<float*>(ctx_bits + kMaxCtxWords);  // [2 tiles][2 halves][128]
    float* xl = xmax + 2 * 2 * kQ;                                   // [2 halves][128]
    // The batch row's context mask as bits (dit.c:828-839): word w from one
    // coalesced 32-byte load and a ballot, words spread over the 8 warps.
    {
      const uint8_t* mrow = a.mask + (size_t)b * a.C;
      const int nw = a.n_ctx * (kKT / 32);  // whole tiles; bits past C stay 0
      for (int w = (warp - 2); w < nw; w += 8) {
        const int c = w * 32 + lane;
        const uint32_t bits = __ballot_sync(0xffffffffu, c < a.C && mrow[c] != 0);
        if (lane == 0) ctx_bits[w] = bits;
      }
      named_bar(1, 256);
    }
    float m = -INFINITY, l = 0.0f;  // running max (log2 domain) and this half's sum
    bool ok = true;
    for (int j = 0; j < T; j++) {
      ok = mbar_wait_bounded(s_full, j & 1, a.err, 7, abort_flag, a.limit_ns);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[64];
      tmem_ld_32x32b_x32(lane_base + colS, sub32(r, 0));
      tmem_ld_32x32b_x32(lane_base + colS + 32u, sub32(r, 1));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(s_free);  // the MMA warp may overwrite S with S_{j+1}
      // Keys outside the row's set get -inf (their p is exactly 0).
      if (j < a.n_self) {
        const int lim = a.S - j * kKT - 64 * hf;
        if (lim < 64) {
#pragma unroll
          for (int i = 0; i < 64; i++)
            if (i >= lim) r[i] = __float_as_uint(-INFINITY);
        }
      } else {
        const int w0 = (j - a.n_self) * (kKT / 32) + 2 * hf;
#pragma unroll
        for (int c = 0; c < 2; c++) {
          const uint32_t bits = ctx_bits[w0 + c];  // zero past C
          if (bits != 0xffffffffu) {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (!((bits >> i) & 1u)) r[32 * c + i] = __float_as_uint(-INFINITY);
          }
        }
      }
      // Eight running maxima, two scores per three-input max.
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; i++) mx[i] = __uint_as_float(r[i]);
#pragma unroll
      for (int i = 8; i < 64; i += 16)
#pragma unroll
        for (int c = 0; c < 8; c++)
          mx[c] = fmax3(mx[c], __uint_as_float(r[i + c]),
                        i + 8 + c < 64 ? __uint_as_float(r[i + 8 + c]) : mx[c]);
      const float hmax = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]),
                               fmaxf(mx[6], mx[7]));
      // The row maximum over both halves (double-buffered by tile parity: a
      // partner past this tile's barrier has read the previous tile's slot).
      xmax[((j & 1) * 2 + hf) * kQ + row] = hmax;
      mbar_arrive(&xbar[quad]);
      ok = mbar_wait_bounded(&xbar[quad], j & 1, a.err, 13, abort_flag, a.limit_ns);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      const float rmax = fmaxf(hmax, xmax[((j & 1) * 2 + (hf ^ 1)) * kQ + row]);
      const float mnew = fmaxf(m, rmax * kScaleLog2);
      const bool need = mnew > m + kRescaleGap;
      bool pv_waited = false;
      if (__any_sync(0xffffffffu, need)) {
        const float f = need ? ex2_approx(m - mnew) : 1.0f;
        if (j > 0) {
          // O is quiescent once PV_{j-1} is done (PV_j waits for this tile's P).
          ok = mbar_wait_bounded(pv_done, (j - 1) & 1, a.err, 8, abort_flag, a.limit_ns);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          pv_waited = true;
          tc_fence_after();
          // This thread's 32 columns of the row's O, in 16-column pieces.
#pragma unroll 1
          for (int c = 0; c < 2; c++) {
            uint32_t o[16];
            tmem_ld_32x32b_x16(lane_base + colO + (uint32_t)(16 * c), o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st_32x32b_x16(lane_base + colO + (uint32_t)(16 * c), o);
          }
        }
        if (need) {
          l *= f;
          m = mnew;
        }
      }
      // Pairs of keys through the packed f32x2 FMA and add: t = s * c - m,
      // p = 2^t, per-lane sums in two pairs of accumulators.
      float2 ps[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
      const float2 scale2 = make_float2(kScaleLog2, kScaleLog2), negm2 = make_float2(-m, -m);
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const float2 t = ffma2(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
                               scale2, negm2);
        const float2 pp = make_float2(ex2_approx(t.x), ex2_approx(t.y));
        ps[i & 1] = fadd2(ps[i & 1], pp);
        r[i] = pack_half2_rn(pp.x, pp.y);  // fp16 pair of the A operand: key 2i low, 2i + 1 high
      }
      l += (ps[0].x + ps[0].y) + (ps[1].x + ps[1].y);
      // P_j goes over P_{j-1} once PV_{j-1} has read it.
      if (j > 0 && !pv_waited) {
        ok = mbar_wait_bounded(pv_done, (j - 1) & 1, a.err, 12, abort_flag, a.limit_ns);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      tmem_st_32x32b_x32(lane_base + colP, sub32(r, 0));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // The row's l: both halves summed with the same maxima.
    if (ok) {
      xl[hf * kQ + row] = l;
      mbar_arrive(&xbar[quad]);
      ok = mbar_wait_bounded(&xbar[quad], T & 1, a.err, 14, abort_flag, a.limit_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        l += xl[(hf ^ 1) * kQ + row];
        ok = mbar_wait_bounded(pv_done, (T - 1) & 1, a.err, 11, abort_flag, a.limit_ns);
        ok = __all_sync(0xffffffffu, ok);
      }
    }
    if (ok) {
      tc_fence_after();
      uint32_t o[32];
      tmem_ld_32x32b_x32(lane_base + colO, o);
      tmem_ld_wait();
      ok = mbar_wait_bounded(g_full, 0, a.err, 16, abort_flag, a.limit_ns);
      if (ok && qrow < a.S) {
        // Dimensions 32 hf .. 32 hf + 31 of the head; the gate from K stage
        // hf (16-byte chunk i of the row at i ^ (row & 7)).  The sigmoid in
        // fast single-precision form (ex2.approx-based exp and division,
        // relative error ~1e-6, far under the fp16 operands' rounding).
        const size_t off = ((size_t)b * a.S + qrow) * a.D + (size_t)hd * kDH + 32 * hf;
        const uint8_t* grow = sK + hf * kKBytes + row * kRow;
        float4* out = reinterpret_cast<float4*>(a.mix + off);
        const float inv_l = __fdiv_rn(1.0f, l);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 gv = *reinterpret_cast<const float4*>(grow + ((i ^ (row & 7)) << 4));
          float4 ov;
          ov.x = __uint_as_float(o[4 * i]) * inv_l * __fdividef(1.0f, 1.0f + __expf(-gv.x));
          ov.y = __uint_as_float(o[4 * i + 1]) * inv_l * __fdividef(1.0f, 1.0f + __expf(-gv.y));
          ov.z = __uint_as_float(o[4 * i + 2]) * inv_l * __fdividef(1.0f, 1.0f + __expf(-gv.z));
          ov.w = __uint_as_float(o[4 * i + 3]) * inv_l * __fdividef(1.0f, 1.0f + __expf(-gv.w));
          out[i] = ov;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// 2-D fp16 tensor map: rows x inner halves (pitch = inner halves), box of
// 64 halves (one 128-byte swizzled row) x box_rows.
int map2d_h(CUtensorMap* m, const __half* base, int inner, long long rows, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

int vt_ld(int n) { return (n + 7) / 8 * 8; }  // 16-byte row pitch

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

int attention_tc_vt_ld(int n) { return vt_ld(n); }

size_t attention_tc_workspace_bytes(int B, int S, int C, int context_batch, int D) {
  const size_t h = sizeof(__half);
  return al256(h * (size_t)B * D * vt_ld(S)) + 2 * al256(h * (size_t)B * S * D) +
         al256(h * (size_t)context_batch * C * D) +
         al256(h * (size_t)context_batch * D * vt_ld(C));
}

AttnTcOperands attention_tc_operands(const AttnTcRequest& r) {
  const size_t h = sizeof(__half);
  uint8_t* p = static_cast<uint8_t*>(r.workspace);
  AttnTcOperands o;
  o.ldv = vt_ld(r.S);
  o.ldc = vt_ld(r.C);
  o.vt = reinterpret_cast<__half*>(p);
  p += al256(h * (size_t)r.B * r.D * o.ldv);
  o.q = reinterpret_cast<__half*>(p);
  p += al256(h * (size_t)r.B * r.S * r.D);
  o.k = reinterpret_cast<__half*>(p);
  p += al256(h * (size_t)r.B * r.S * r.D);
  o.ck = reinterpret_cast<__half*>(p);
  p += al256(h * (size_t)r.context_batch * r.C * r.D);
  o.cvt = reinterpret_cast<__half*>(p);
  return o;
}

bool attention_tc_supported(const AttnTcRequest& r) {
  if (cdiv(r.C, kKT) * (kKT / 32) > kMaxCtxWords) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  auto al256p = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 255u) == 0; };
  return r.D % 64 == 0 && r.D == r.heads * kDH && al16(r.g) && al16(r.mix) && al16(r.ck) &&
         al16(r.cv) && al256p(r.workspace) && r.S > 0 && r.C > 0 && r.B > 0 &&
         r.context_batch > 0 && r.B % r.context_batch == 0;
}

int attention_tc_launch(Ctx* c, const AttnTcRequest& r, cudaStream_t s) {
  if (!attention_tc_supported(r)) return IRO_ERR_UNSUPPORTED;
  static bool attr_done[64] = {false};
  if (!attr_done[c->device]) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return map_cuda(e);
    }
    attr_done[c->device] = true;
  }
  const AttnTcOperands o = attention_tc_operands(r);
  context_prep_kernel<<<dim3(cdiv(o.ldc, 32), r.heads, r.context_batch), 256, 0, s>>>(
      r.ck, r.cv, o.ck, o.cvt, r.C, r.D, r.heads, o.ldc, c->err);
  int st = check_launch();
  if (st) return st;
  CUtensorMap mq, mk, mv, mck, mcv;
  const long long rows = (long long)r.B * r.S, crows = (long long)r.context_batch * r.C;
  st = map2d_h(&mq, o.q, r.D, rows, kQ);
  if (!st) st = map2d_h(&mk, o.k, r.D, rows, kKT);
  if (!st) st = map2d_h(&mv, o.vt, o.ldv, (long long)r.B * r.D, kDH);
  if (!st) st = map2d_h(&mck, o.ck, r.D, crows, kKT);
  if (!st) st = map2d_h(&mcv, o.cvt, o.ldc, (long long)r.context_batch * r.D, kDH);
  CUtensorMap mg;
  if (!st) {
    // The gate: fp32 [B*S, D], boxes of 32 floats (128 bytes) x 128 rows.
    const cuuint64_t dims[2] = {(cuuint64_t)r.D, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)r.D * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)kQ};
    st = encode_tmap(&mg, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, r.g, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  }
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
  const dim3 grid(cdiv(r.S, kQ), r.heads, r.B);
  cudaError_t e = launch_pdl(attention_tc_kernel, grid, dim3(kThreads), (size_t)kSmem, s, mq, mk,
                             mv, mck, mcv, mg, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  return IRO_OK;
}

}  // namespace iro
