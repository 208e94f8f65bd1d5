// dit_attention.cu — the DiT block's joint attention (dit.c:806-862) on the
// 5th-generation tensor cores: fp16 operands, fp32 accumulation.
//
// One CTA per (128-query tile, head, batch row), two CTAs per SM (83 KB of
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
//   8 warps     16 query rows each, four threads per row (16-lane TMEM
//               loads): scores, scale 1/8, mask, online softmax with the
//               row maximum and sum by shuffles, P_j packed to fp16 pairs
//               into TMEM; at the end O / l times the sigmoid gate
//               (ops.c:786-789) to `mix`.
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
// Barriers, then the context mask bits.
constexpr int kSmem = 1024 + kBarOff + 256 + 4 * kMaxCtxWords;
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
  grid_dep_wait();  // launched with programmatic stream serialization
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

// 16-lane TMEM shapes (a warp reads 16 lanes from its lane base, four
// threads per lane; thread t holds lanes base + t / 4 and base + t / 4 + 8):
//   16x256b: per 8-column repetition c, the registers 4c .. 4c + 3 are
//            (lane t/4, columns 8c + 2(t%4) and + 1), then (lane t/4 + 8,
//            the same two columns);
//   16x128b: per 4-column repetition c, registers 2c, 2c + 1 are lane t/4 and
//            lane t/4 + 8 at column 4c + t%4.
__device__ __forceinline__ void tmem_ld_16x256b_x16(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_16x128b_x16(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.16x128b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
}

__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
               : "memory");
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
  uint64_t* g_full = bars + 14;    // the gate tile in the freed K stages
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
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
    // Each warp owns 16 query rows (TMEM lanes 32 * (warp % 4) + 16 * sub ..
    // + 15) with four threads per row, through the 16-lane TMEM shapes:
    // thread t holds rows t / 4 and t / 4 + 8 of the warp's 16, and of each
    // 8-key group the two keys 2(t%4), 2(t%4) + 1.  The four threads of a row
    // share its maximum and sum by shuffles.
    const int quad = warp & 3;
    const int sub = (warp - 2) >> 2;
    const int jj = lane & 3;             // key pair within each 8-key group
    const int lbase = quad * 32 + sub * 16;
    const int rr0 = lbase + (lane >> 2), rr1 = rr0 + 8;  // this thread's two rows
    const uint32_t lane_addr = tmem + ((uint32_t)lbase << 16);
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
    float m0 = -INFINITY, m1 = -INFINITY;  // running maxima (log2 domain) of the two rows
    float l0 = 0.0f, l1 = 0.0f;            // this thread's share of their sums
    bool ok = true;
    for (int j = 0; j < T; j++) {
      ok = mbar_wait_bounded(s_full, j & 1, a.err, 7, abort_flag, a.limit_ns);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[64];
      tmem_ld_16x256b_x16(lane_addr + kColS, r);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(s_free);  // the MMA warp may overwrite S with S_{j+1}
      // Keys outside the row's set get -inf (their p is exactly 0); key
      // 8c + 2jj + e sits in registers 4c + e (row 0) and 4c + 2 + e (row 1).
      if (j < a.n_self) {
        const int lim = a.S - j * kKT - 2 * jj;
        if (lim < kKT) {
#pragma unroll
          for (int c = 0; c < 16; c++)
#pragma unroll
            for (int e = 0; e < 2; e++)
              if (8 * c + e >= lim) {
                r[4 * c + e] = __float_as_uint(-INFINITY);
                r[4 * c + 2 + e] = __float_as_uint(-INFINITY);
              }
        }
      } else {
        const int w0 = (j - a.n_self) * (kKT / 32);
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) {
          const uint32_t bits = ctx_bits[w0 + q4] >> (2 * jj);  // zero past C
          if ((bits & 0x03030303u) != 0x03030303u) {
#pragma unroll
            for (int cc = 0; cc < 4; cc++)
#pragma unroll
              for (int e = 0; e < 2; e++)
                if (!((bits >> (8 * cc + e)) & 1u)) {
                  r[4 * (4 * q4 + cc) + e] = __float_as_uint(-INFINITY);
                  r[4 * (4 * q4 + cc) + 2 + e] = __float_as_uint(-INFINITY);
                }
          }
        }
      }
      // Row maxima: this thread's 32 scores of each row, then the row's four
      // threads.
      float x0 = fmaxf(__uint_as_float(r[0]), __uint_as_float(r[1]));
      float x1 = fmaxf(__uint_as_float(r[2]), __uint_as_float(r[3]));
      float y0 = fmaxf(__uint_as_float(r[4]), __uint_as_float(r[5]));
      float y1 = fmaxf(__uint_as_float(r[6]), __uint_as_float(r[7]));
#pragma unroll
      for (int c = 2; c < 16; c += 2) {
        x0 = fmax3(x0, __uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]));
        x1 = fmax3(x1, __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]));
        y0 = fmax3(y0, __uint_as_float(r[4 * c + 4]), __uint_as_float(r[4 * c + 5]));
        y1 = fmax3(y1, __uint_as_float(r[4 * c + 6]), __uint_as_float(r[4 * c + 7]));
      }
      float rmax0 = fmaxf(x0, y0), rmax1 = fmaxf(x1, y1);
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        rmax0 = fmaxf(rmax0, __shfl_xor_sync(0xffffffffu, rmax0, o));
        rmax1 = fmaxf(rmax1, __shfl_xor_sync(0xffffffffu, rmax1, o));
      }
      const float mn0 = fmaxf(m0, rmax0 * kScaleLog2), mn1 = fmaxf(m1, rmax1 * kScaleLog2);
      const bool need0 = mn0 > m0 + kRescaleGap, need1 = mn1 > m1 + kRescaleGap;
      bool pv_waited = false;
      if (__any_sync(0xffffffffu, need0 || need1)) {
        const float f0 = need0 ? ex2_approx(m0 - mn0) : 1.0f;
        const float f1 = need1 ? ex2_approx(m1 - mn1) : 1.0f;
        if (j > 0) {
          // O is quiescent once PV_{j-1} is done (PV_j waits for this tile's P).
          ok = mbar_wait_bounded(pv_done, (j - 1) & 1, a.err, 8, abort_flag, a.limit_ns);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          pv_waited = true;
          tc_fence_after();
          // In two 32-column pieces: the 64 scores are live here.
#pragma unroll 1
          for (int hh = 0; hh < 2; hh++) {
            uint32_t o[16];
            tmem_ld_16x256b_x4(lane_addr + kColO + 32u * hh, o);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 4; c++) {
              o[4 * c] = __float_as_uint(__uint_as_float(o[4 * c]) * f0);
              o[4 * c + 1] = __float_as_uint(__uint_as_float(o[4 * c + 1]) * f0);
              o[4 * c + 2] = __float_as_uint(__uint_as_float(o[4 * c + 2]) * f1);
              o[4 * c + 3] = __float_as_uint(__uint_as_float(o[4 * c + 3]) * f1);
            }
            tmem_st_16x256b_x4(lane_addr + kColO + 32u * hh, o);
          }
        }
        if (need0) {
          l0 *= f0;
          m0 = mn0;
        }
        if (need1) {
          l1 *= f1;
          m1 = mn1;
        }
      }
      // p = 2^(s * c - m) per key pair (packed f32x2 FMA and add); the pair
      // of row 0 and the pair of row 1 of each group become the two fp16
      // columns this thread stores (16x128b: registers 2c, 2c + 1).
      float2 ps0 = make_float2(0.0f, 0.0f), ps1 = make_float2(0.0f, 0.0f);
      const float2 scale2 = make_float2(kScaleLog2, kScaleLog2);
      const float2 negm0 = make_float2(-m0, -m0), negm1 = make_float2(-m1, -m1);
#pragma unroll
      for (int c = 0; c < 16; c++) {
        const float2 t0 = ffma2(make_float2(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1])),
                                scale2, negm0);
        const float2 t1 = ffma2(make_float2(__uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3])),
                                scale2, negm1);
        const float2 p0 = make_float2(ex2_approx(t0.x), ex2_approx(t0.y));
        const float2 p1 = make_float2(ex2_approx(t1.x), ex2_approx(t1.y));
        ps0 = fadd2(ps0, p0);
        ps1 = fadd2(ps1, p1);
        r[2 * c] = pack_half2_rn(p0.x, p0.y);  // registers 2c, 2c + 1 were read at group c / 2
        r[2 * c + 1] = pack_half2_rn(p1.x, p1.y);
      }
      l0 += ps0.x + ps0.y;
      l1 += ps1.x + ps1.y;
      // P_j goes over P_{j-1} once PV_{j-1} has read it.
      if (j > 0 && !pv_waited) {
        ok = mbar_wait_bounded(pv_done, (j - 1) & 1, a.err, 12, abort_flag, a.limit_ns);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      tmem_st_16x128b_x16(lane_addr + kColP, reinterpret_cast<const uint32_t(&)[32]>(r));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) {
      // The rows' sums over their four threads.
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
      }
      ok = mbar_wait_bounded(pv_done, (T - 1) & 1, a.err, 11, abort_flag, a.limit_ns);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      uint32_t o[32];
      tmem_ld_16x256b_x8(lane_addr + kColO, o);
      tmem_ld_wait();
      ok = mbar_wait_bounded(g_full, 0, a.err, 16, abort_flag, a.limit_ns);
      if (ok) {
        // Dimensions 8c + 2jj, + 1 of the head for the two rows; the gate
        // from K stage d / 32 (16-byte chunk (d % 32) / 4 of the row at
        // chunk ^ (row & 7)).  The sigmoid in fast single-precision form
        // (ex2.approx-based exp and division, relative error ~1e-6, far
        // under the fp16 operands' rounding).
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int rr = h ? rr1 : rr0;
          const int qrow = q0 + rr;
          if (qrow >= a.S) continue;
          const float inv_l = __fdiv_rn(1.0f, h ? l1 : l0);
          float* orow = a.mix + ((size_t)b * a.S + qrow) * a.D + (size_t)hd * kDH;
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const int d = 8 * c + 2 * jj;
            const uint8_t* gch = sK + (d >> 5) * kKBytes + rr * kRow +
                                 ((((d & 31) >> 2) ^ (rr & 7)) << 4) + (d & 3) * 4;
            const float2 gv = *reinterpret_cast<const float2*>(gch);
            float2 ov;
            ov.x = __uint_as_float(o[4 * c + 2 * h]) * inv_l * __fdividef(1.0f, 1.0f + __expf(-gv.x));
            ov.y = __uint_as_float(o[4 * c + 2 * h + 1]) * inv_l *
                   __fdividef(1.0f, 1.0f + __expf(-gv.y));
            *reinterpret_cast<float2*>(orow + d) = ov;
          }
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
  cudaError_t pe = launch_pdl(context_prep_kernel, dim3(cdiv(o.ldc, 32), r.heads, r.context_batch),
                              dim3(256), 0, s, r.ck, r.cv, o.ck, o.cvt, r.C, r.D, r.heads, o.ldc,
                              c->err);
  if (pe != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(pe);
  }
  int st = IRO_OK;
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
