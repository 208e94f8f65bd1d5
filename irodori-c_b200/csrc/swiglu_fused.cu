// swiglu_fused.cu — the whole int8 SwiGLU MLP block (dit.c:913-969 through
// ops.c) as ONE persistent cooperative kernel:
//
//   A  quantise x rows (ops.c:321-348)              -> qx, sx, zx
//   B  W1|W3 GEMM + dequant + silu gate (tcgen05)   -> hidden (fp32), and
//      the per-row range of the hidden, folded in with integer atomics
//   C  quantise hidden rows with those ranges       -> qh, sh, zh
//   D  W2 GEMM + dequant + bias (tcgen05)           -> out
//
// The separate-kernel path (quantiser, GEMM, quantiser, GEMM) leaves SMs idle
// at every kernel boundary and in every GEMM's last partial wave; here the
// phases are linked per 128-row block by counters in global memory, so an SM
// that has finished its share of one phase starts on the next phase's work as
// soon as the rows it needs are complete.  Work is assigned statically:
//   B  gated tile t (row block t / tiles_n1, pair block t % tiles_n1) on CTA
//      t % G; CTAs [c0, G) get one tile fewer (c0 = tiles % G),
//   C  hidden rows on the warps of the lighter CTAs, in row order,
//   D  W2 tile j on CTA (c0 + j) % G, in row-block order.
// Every cross-CTA wait is a bounded poll; a poll that runs out records
// IRO_ERR_DEVICE_TIMEOUT and raises a global abort flag that every other
// wait also checks, so a failed launch ends quickly with an error status.
// The launch is cooperative (all CTAs co-resident, one per SM).
//
// Roles (576 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2..17 quantisers and epilogues.  Arithmetic is the
// separate-kernel path's: the same quantiser, dequantisation and silu code,
// so the outputs are identical to it.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "epi_math.cuh"
#include "gemm_i8.cuh"
#include "swiglu_fused.cuh"

namespace iro {
namespace {

constexpr int FBM = 128;
constexpr int FBK = 128;           // K bytes per pipeline stage
constexpr int FBN1 = 256;          // W1|W3 tile: 128 hidden channels
constexpr int kFEpiWarps = 16;
constexpr int kFThreads = 64 + 32 * kFEpiWarps;
constexpr int kFStgBytes = 32 * kChunk * 4;
constexpr int kFStgBufs = 2;
constexpr int kFSmemMax = 232448;

struct FCfg {
  static constexpr int A_BYTES = FBM * FBK;
  static constexpr int B_BYTES = FBN1 * FBK;  // W2 tiles use the first BN2 rows
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STG = kFEpiWarps * kFStgBufs * kFStgBytes;
  static constexpr int PARAMS = 2 * 3 * FBN1 * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int FIXED = STG + PARAMS + BAR_BYTES + 1024;
  static constexpr int STAGES_RAW = (kFSmemMax - FIXED) / STAGE;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = STAGES * STAGE + FIXED;
  static constexpr int ACC_COLS = FBN1;
  static constexpr int TMEM_COLS = 512;
  static_assert(STAGES >= 2, "pipeline needs two stages");
  static_assert(SMEM <= kFSmemMax, "shared memory budget");
};

// Counter block (int32, zeroed before each launch), one counter per 128-byte
// line so that polls of one counter do not slow increments of another: the
// abort flag, the number of quantised x rows, then per 128-row block the
// gated-tile completions (one count per epilogue warp and tile) and the
// quantised hidden rows.
constexpr int kCtLine = 32;
enum { CT_ABORT = 0, CT_XROWS = kCtLine, CT_HEAD = 2 * kCtLine };
inline size_t ctr_ints(int tiles_m) { return (size_t)kCtLine * (2 + 2 * (size_t)tiles_m); }

struct FusedParams {
  int M, D, H, N2;
  int tiles_m, tiles_n1, tiles_g, tiles_n2, tiles_2;
  int kb1, kb2;
  int c0;        // CTAs [0, c0) hold one more gated tile
  int qh_first;  // first CTA of the hidden-quantiser group
  const float* x;
  uint8_t* qx;
  float* sx;
  int32_t* zx;
  float* hidden;
  int* hlo;      // per-row hidden range, order-preserving integer encoding
  int* hhi;
  uint8_t* qh;
  float* sh;
  int32_t* zh;
  const float* w13_scale;
  const int32_t* w13_colsum;
  const float* w13_bias;
  const float* w2_scale;
  const int32_t* w2_colsum;
  const float* b2;
  int* ctr;      // ctr_ints(tiles_m) counters, see CT_*
  DevError* err;
  uint64_t limit_ns;
  unsigned long long* trace;  // optional per-CTA timestamps (IRO_FUSED_TRACE)
};

// Trace slots per CTA (globaltimer ns).
enum { FT_ENTRY = 0, FT_A_END, FT_P_TMA0, FT_M_FULL0, FT_M_END0, FT_M_END1, FT_B_TFULL0,
       FT_B_TILE0, FT_B_TFULL1, FT_B_TILE1, FT_B_END, FT_C_END, FT_P_W2READY, FT_D_TFULL0,
       FT_D_END, FT_EXIT, FT_SLOTS = 16 };
const char* const kFtNames[FT_SLOTS] = {"entry",    "A_end",   "P_tma0",   "M_full0",
                                        "M_end0",   "M_end1",  "B_tfull0", "B_tile0",
                                        "B_tfull1", "B_tile1", "B_end",    "C_end",
                                        "P_w2ready", "D_tfull0", "D_end",  "exit"};

__device__ __forceinline__ void ftrace(const FusedParams& p, int slot) {
  if (p.trace) p.trace[blockIdx.x * FT_SLOTS + slot] = globaltimer_ns();
}

// Float <-> int encoding whose signed-integer order is the float order
// (for non-NaN values), so atomicMin/atomicMax compute float min/max.
// +0.0 encodes to 0.
__device__ __forceinline__ int ord_enc(float f) {
  const int b = __float_as_int(f);
  return b ^ ((b >> 31) & 0x7fffffff);
}
__device__ __forceinline__ float ord_dec(int i) { return __int_as_float(i ^ ((i >> 31) & 0x7fffffff)); }

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Count increment with release semantics at GPU scope.  Release is
// cumulative: writes of other threads ordered before it by a warp or CTA
// barrier become visible to whoever acquires the count, so only the
// incrementing thread pays for the ordering.
__device__ __forceinline__ void add_release(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded poll until *ctr >= target (acquire).  On running out, records the
// error and raises the global abort flag; returns false on abort.
__device__ bool wait_count(const FusedParams& p, const int* ctr, int target, int where,
                           volatile int* cta_abort) {
  if (ld_acquire(ctr) >= target) return true;
  volatile int* gabort = p.ctr + CT_ABORT;
  const long long t0 = clock64();
  const long long limit_cycles = (long long)(p.limit_ns * 2ull);
  unsigned ns = 64;
  while (true) {
    __nanosleep(ns);
    ns = ns < 256 ? 2 * ns : 256;
    if (ld_acquire(ctr) >= target) return true;
    if (*gabort) {
      if (cta_abort) *cta_abort = 1;
      return false;
    }
    if (clock64() - t0 > limit_cycles) {
      report_error(p.err, IRO_ERR_DEVICE_TIMEOUT, where);
      atomicExch(p.ctr + CT_ABORT, 1);
      if (cta_abort) *cta_abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ int rows_in(const FusedParams& p, int mb) {
  return min(FBM, p.M - mb * FBM);
}

// Quantise one fp32 row of K (a multiple of 4) with one warp, the
// reference's asymmetric scheme (ops.c:321-348): two passes over the row
// (range, then codes), codes stored four at a time.  Each lane loads up to
// kQU float4 before using any, so a pass costs one memory latency per
// 128*kQU floats rather than one per float4.
constexpr int kQU = 8;

__device__ __forceinline__ void load_group(const float4* s4, int n4, int base, int lane,
                                           float4 (&v)[kQU]) {
#pragma unroll
  for (int u = 0; u < kQU; u++) {
    const int j = base + u * 32 + lane;
    v[u] = j < n4 ? __ldcg(s4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

__device__ __forceinline__ void code_group(const float4 (&v)[kQU], int n4, int base, int lane,
                                           float inv, float zpf, uint32_t* d4) {
#pragma unroll
  for (int u = 0; u < kQU; u++) {
    const int j = base + u * 32 + lane;
    if (j < n4)
      d4[j] = quant_code(v[u].x, inv, zpf) | (quant_code(v[u].y, inv, zpf) << 8) |
              (quant_code(v[u].z, inv, zpf) << 16) | (quant_code(v[u].w, inv, zpf) << 24);
  }
}

__device__ void quant_row_warp(const float* src, int K, uint8_t* dst, float* s_out,
                               int32_t* z_out, int lane) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  const int n4 = K / 4;
  float lo = 0.0f, hi = 0.0f;
  float4 v[kQU];
  for (int base = 0; base < n4; base += 32 * kQU) {
    load_group(s4, n4, base, lane, v);
#pragma unroll
    for (int u = 0; u < kQU; u++) {
      // Padding lanes hold zeros, which the range includes anyway.
      lo = run_lo(v[u].x, lo); hi = run_hi(v[u].x, hi);
      lo = run_lo(v[u].y, lo); hi = run_hi(v[u].y, hi);
      lo = run_lo(v[u].z, lo); hi = run_hi(v[u].z, hi);
      lo = run_lo(v[u].w, lo); hi = run_hi(v[u].w, hi);
    }
  }
  warp_minmax(lo, hi);
  float s, inv;
  int zp;
  row_params(lo, hi, s, inv, zp);
  uint32_t* d4 = reinterpret_cast<uint32_t*>(dst);
  if (n4 <= 32 * kQU) {
    code_group(v, n4, 0, lane, inv, (float)zp, d4);  // the row is still in registers
  } else {
    for (int base = 0; base < n4; base += 32 * kQU) {
      load_group(s4, n4, base, lane, v);
      code_group(v, n4, base, lane, inv, (float)zp, d4);
    }
  }
  if (lane == 0) {
    *s_out = s;
    *z_out = zp;
  }
}

__global__ void __launch_bounds__(kFThreads, 1)
    swiglu_fused_kernel(const __grid_constant__ CUtensorMap tmQx,
                        const __grid_constant__ CUtensorMap tmW13,
                        const __grid_constant__ CUtensorMap tmHid,
                        const __grid_constant__ CUtensorMap tmQh,
                        const __grid_constant__ CUtensorMap tmW2,
                        const __grid_constant__ CUtensorMap tmY, const FusedParams p,
                        const int BN2) {
  using C = FCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stg_base = smem + C::STAGES * C::STAGE;
  float* prm = reinterpret_cast<float*>(stg_base + C::STG);
  uint64_t* full = reinterpret_cast<uint64_t*>(stg_base + C::STG + C::PARAMS);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  int* xrows = p.ctr + CT_XROWS;
  int* done_g = p.ctr + CT_HEAD;                        // + mb * kCtLine
  int* ready_h = p.ctr + CT_HEAD + p.tiles_m * kCtLine;  // + mb * kCtLine

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kFEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQx);
    tma_prefetch_desc(&tmW13);
    tma_prefetch_desc(&tmQh);
    tma_prefetch_desc(&tmW2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) ftrace(p, FT_ENTRY);

  // Static schedules (every role derives the same sequence).
  const int n_gated = cta < p.tiles_g ? (p.tiles_g - cta + G - 1) / G : 0;
  const int j0 = (cta - p.c0 + G) % G;  // first W2 tile of this CTA
  const int n_w2 = j0 < p.tiles_2 ? (p.tiles_2 - j0 + G - 1) / G : 0;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      // Every gated tile reads quantised x rows from all CTAs: wait for all.
      if (n_gated > 0) {
        ok = wait_count(p, xrows, p.M, 10, abort_flag);
        fence_proxy_async_global();
      }
      int have = -1;
      for (int i = 0; ok && i < n_gated; i++) {
        const int t = cta + i * G;
        const int mb = t / p.tiles_n1, nb = t % p.tiles_n1;
        for (int kb = 0; kb < p.kb1; kb++) {
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 1, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], C::A_BYTES + FBN1 * FBK);
          tma_load_2d(sa, &tmQx, &full[s], kb * FBK, mb * FBM);
          tma_load_2d(sa + C::A_BYTES, &tmW13, &full[s], kb * FBK, nb * FBN1);
          if (i == 0 && kb == 0) ftrace(p, FT_P_TMA0);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      have = -1;
      for (int i = 0; ok && i < n_w2; i++) {
        const int j = j0 + i * G;
        const int mb = j / p.tiles_n2, nb = j % p.tiles_n2;
        if (mb != have) {
          if (!wait_count(p, ready_h + mb * kCtLine, rows_in(p, mb), 11, abort_flag)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
          if (i == 0) ftrace(p, FT_P_W2READY);
          have = mb;
        }
        for (int kb = 0; kb < p.kb2; kb++) {
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 1, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], C::A_BYTES + BN2 * FBK);
          tma_load_2d(sa, &tmQh, &full[s], kb * FBK, mb * FBM);
          tma_load_2d(sa + C::A_BYTES, &tmW2, &full[s], kb * FBK, nb * BN2);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.ctr + CT_ABORT, 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      const uint32_t idesc1 = idesc_i8(FBM, FBN1, 0);
      const uint32_t idesc2 = idesc_i8(FBM, BN2, 0);
      for (int i = 0; ok && i < n_gated + n_w2; i++) {
        const bool g = i < n_gated;
        const uint32_t idesc = g ? idesc1 : idesc2;
        const int nkb = g ? p.kb1 : p.kb2;
        if (!mbar_wait_bounded(&tempty[acc], aph ^ 1u, p.err, 2, abort_flag, p.limit_ns)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * C::ACC_COLS);
        for (int kb = 0; kb < nkb; kb++) {
          if (!mbar_wait_bounded(&full[s], ph, p.err, 3, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (i == 0 && kb == 0) ftrace(p, FT_M_FULL0);
          const uint32_t a_addr = smem_u32(smem + s * C::STAGE);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < FBK / 32; k++)
            mma_i8(d, sw128_desc(a_addr + 32 * k), sw128_desc(b_addr + 32 * k), idesc,
                   (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (i < 2) ftrace(p, i == 0 ? FT_M_END0 : FT_M_END1);
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
    }
    __syncwarp();
  } else {
    // ---------------- quantisers and epilogues (16 warps) ----------------
    const int e = warp - 2;
    const int quad = warp & 3;        // TMEM lanes 32*quad .. +31
    const int part = e >> 2;          // column quarter of a tile
    const int et = threadIdx.x - 64;  // 0..511
    uint8_t* stg_mine = stg_base + e * kFStgBufs * kFStgBytes;
    int sbuf = 0;
    int acc = 0;
    uint32_t aph = 0;
    int pbuf = 0;
    bool dead = false;

    // ---- A: quantise x; reset the hidden ranges of the same rows ----
    // One count per CTA once all its rows are written; then every CTA
    // waits for all rows (its gated tiles read rows from everywhere).
    {
      const int gw = cta * kFEpiWarps + e, nw = G * kFEpiWarps;
      for (int row = gw; row < p.M; row += nw) {
        quant_row_warp(p.x + (size_t)row * p.D, p.D, p.qx + (size_t)row * p.D, p.sx + row,
                       p.zx + row, lane);
        if (lane == 0) {
          p.hlo[row] = 0;  // ord_enc(+0.0f): the range always includes 0
          p.hhi[row] = 0;
        }
      }
      named_bar(2, 32 * kFEpiWarps);
      bool ok = true;
      if (et == 0) {
        int mine = 0;
        for (int w = 0; w < kFEpiWarps; w++) {
          const int r0 = cta * kFEpiWarps + w;
          if (r0 < p.M) mine += (p.M - r0 + nw - 1) / nw;
        }
        if (mine) add_release(xrows, mine);
        ftrace(p, FT_A_END);
        ok = wait_count(p, xrows, p.M, 13, abort_flag);
      }
      dead = named_bar_or(2, 32 * kFEpiWarps, !ok);
      (void)ld_acquire(xrows);
    }

    // One 16-column chunk out through the warp's staging tile and a TMA store.
    auto emit = [&](const float (&v)[kChunk], const CUtensorMap* om, int col0, int ncols,
                    int row0) {
      uint8_t* stg = stg_mine + sbuf * kFStgBytes;
      sbuf = sbuf + 1 == kFStgBufs ? 0 : sbuf + 1;
      if (lane == 0) bulk_wait_read<kFStgBufs - 1>();
      __syncwarp();
      stage_row16(stg, lane, v);
      fence_async_shared();
      __syncwarp();
      if (lane == 0 && row0 < p.M && col0 < ncols) {
        tma_store_2d(om, stg, col0, row0);
        bulk_commit();
      }
    };
    // Stage one tile's column parameters (published by the vote barrier).
    auto stage_params = [&](const int32_t* cs, const float* sw, const float* b, int n0, int bn,
                            int N) {
      float* pc = prm + pbuf * 3 * FBN1;
      int* p_cs = reinterpret_cast<int*>(pc);
      if (et < bn) {
        const int n = n0 + et;
        const bool ok = n < N;
        p_cs[et] = ok ? __ldg(cs + n) : 0;
        pc[FBN1 + et] = ok ? __ldg(sw + n) : 0.0f;
        pc[2 * FBN1 + et] = (ok && b) ? __ldg(b + n) : 0.0f;
      }
    };
    // Completion of a gated tile for the hidden quantisers: this warp's
    // stores and range atomics are visible before its count goes up.
    int pending = -1;
    // Called right after this tile's first chunk store: every bulk group but
    // the newest one belongs to the previous tile.
    auto flush_pending = [&]() {
      if (pending < 0) return;
      __syncwarp();
      if (lane == 0) {
        bulk_wait_all<1>();          // the previous tile's hidden stores are done
        fence_proxy_async_global();  // ... and ordered before the release
        add_release(done_g + pending * kCtLine, 1);
      }
      __syncwarp();
      pending = -1;
    };
    // After the last gated tile: all groups.
    auto flush_last = [&]() {
      if (pending < 0) return;
      __syncwarp();
      if (lane == 0) {
        bulk_wait_all<0>();
        fence_proxy_async_global();
        add_release(done_g + pending * kCtLine, 1);
      }
      __syncwarp();
      pending = -1;
    };

    // ---- B: gated tiles ----
    // Column parameters and row parameters are fetched into registers one
    // tile ahead, so their load latency overlaps the previous tile.
    constexpr int HALF = FBN1 / 2;
    constexpr int PER = HALF / 4;  // hidden columns per warp per tile
    struct Prefetch {
      int cs;
      float sw, b, sx;
      int zp;
    } pf;
    auto fetch_gated = [&](int i) {
      const int t = cta + i * G;
      const int mb = t / p.tiles_n1, nb = t % p.tiles_n1;
      const int n = nb * FBN1 + et;
      const bool ok = et < FBN1;  // the pair layout pads W1|W3 to whole tiles
      pf.cs = ok ? __ldg(p.w13_colsum + n) : 0;
      pf.sw = ok ? __ldg(p.w13_scale + n) : 0.0f;
      pf.b = (ok && p.w13_bias) ? __ldg(p.w13_bias + n) : 0.0f;
      const int r = mb * FBM + quad * 32 + lane;
      pf.sx = r < p.M ? __ldcg(p.sx + r) : 0.0f;
      pf.zp = r < p.M ? __ldcg(p.zx + r) : 0;
    };
    if (n_gated > 0) fetch_gated(0);
    for (int i = 0; i < n_gated; i++) {
      const int t = cta + i * G;
      const int mb = t / p.tiles_n1, nb = t % p.tiles_n1;
      float* pcw = prm + pbuf * 3 * FBN1;
      if (et < FBN1) {
        reinterpret_cast<int*>(pcw)[et] = pf.cs;
        pcw[FBN1 + et] = pf.sw;
        pcw[2 * FBN1 + et] = pf.b;
      }
      const float sx = pf.sx;
      const int zp = pf.zp;
      if (i + 1 < n_gated) fetch_gated(i + 1);
      const bool got =
          !dead && mbar_wait_bounded(&tfull[acc], aph, p.err, 4, abort_flag, p.limit_ns);
      if (named_bar_or(1, 32 * kFEpiWarps, !got)) {
        dead = true;
        break;
      }
      if (i < 2 && e == 0 && lane == 0) ftrace(p, i == 0 ? FT_B_TFULL0 : FT_B_TFULL1);
      tc_fence_after();
      const float* pc = prm + pbuf * 3 * FBN1;
      const int* p_cs = reinterpret_cast<const int*>(pc);
      const int row0 = mb * FBM + quad * 32;
      const int row = row0 + lane;
      const bool row_ok = row < p.M;
      const uint32_t tbase =
          tmem_base + (uint32_t)(acc * C::ACC_COLS) + ((uint32_t)(quad * 32) << 16);
      float lo = 0.0f, hi = 0.0f;
      for (int c0 = part * PER; c0 < (part + 1) * PER; c0 += kChunk) {
        const int h0 = nb * HALF + c0;
        if (h0 >= p.H) break;  // warp-uniform
        uint32_t r1[kChunk], r3[kChunk];
        tmem_ld_32x32b_x16(tbase + c0, r1);
        tmem_ld_32x32b_x16(tbase + HALF + c0, r3);
        tmem_ld_wait();
        float v[kChunk];
        gated_chunk(r1, r3, c0, HALF + c0, p_cs, pc + FBN1, pc + 2 * FBN1, zp, sx, v);
#pragma unroll
        for (int j = 0; j < kChunk; j++) {
          lo = run_lo(v[j], lo);
          hi = run_hi(v[j], hi);
        }
        emit(v, &tmHid, h0, p.H, row0);
        flush_pending();  // the previous tile's stores are long done here
      }
      if (row_ok) {
        atomicMin(p.hlo + row, ord_enc(lo));
        atomicMax(p.hhi + row, ord_enc(hi));
      }
      pending = mb;
      if (i < 2 && e == 0 && lane == 0) ftrace(p, i == 0 ? FT_B_TILE0 : FT_B_TILE1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
      pbuf ^= 1;
    }
    flush_last();
    if (e == 0 && lane == 0) ftrace(p, FT_B_END);

    // ---- C: quantise hidden rows (lighter CTAs) ----
    // Items of 16 rows of one row block, one row per warp; one thread per
    // CTA polls the block's gated-tile count, one count per item after.
    if (!dead && cta >= p.qh_first) {
      const int nq = G - p.qh_first;
      const int items = p.tiles_m * (FBM / kFEpiWarps);
      for (int it = cta - p.qh_first; it < items; it += nq) {
        const int mb = it / (FBM / kFEpiWarps);
        const int r0 = mb * FBM + (it % (FBM / kFEpiWarps)) * kFEpiWarps;
        if (r0 >= p.M) break;  // CTA-uniform
        bool ok = true;
        if (et == 0) ok = wait_count(p, done_g + mb * kCtLine, kFEpiWarps * p.tiles_n1, 12, nullptr);
        if (named_bar_or(2, 32 * kFEpiWarps, !ok)) {
          dead = true;
          break;
        }
        (void)ld_acquire(done_g + mb * kCtLine);
        const int row = r0 + e;
        if (row < p.M) {
          float s, inv;
          int zp;
          row_params(ord_dec(__ldcg(p.hlo + row)), ord_dec(__ldcg(p.hhi + row)), s, inv, zp);
          const float4* s4 = reinterpret_cast<const float4*>(p.hidden + (size_t)row * p.H);
          uint32_t* d4 = reinterpret_cast<uint32_t*>(p.qh + (size_t)row * p.H);
          float4 v[kQU];
          for (int base = 0; base < p.H / 4; base += 32 * kQU) {
            load_group(s4, p.H / 4, base, lane, v);
            code_group(v, p.H / 4, base, lane, inv, (float)zp, d4);
          }
          if (lane == 0) {
            p.sh[row] = s;
            p.zh[row] = zp;
          }
        }
        named_bar(2, 32 * kFEpiWarps);
        if (et == 0) add_release(ready_h + mb * kCtLine, min(kFEpiWarps, p.M - r0));
      }
    }
    if (e == 0 && lane == 0) ftrace(p, FT_C_END);

    // ---- D: W2 tiles ----
    const int per2 = BN2 / 4;
    for (int i = 0; i < n_w2; i++) {
      const int j = j0 + i * G;
      const int mb = j / p.tiles_n2, nb = j % p.tiles_n2;
      stage_params(p.w2_colsum, p.w2_scale, p.b2, nb * BN2, BN2, p.N2);
      const bool got =
          !dead && mbar_wait_bounded(&tfull[acc], aph, p.err, 5, abort_flag, p.limit_ns);
      if (named_bar_or(1, 32 * kFEpiWarps, !got)) {
        dead = true;
        break;
      }
      if (i == 0 && e == 0 && lane == 0) ftrace(p, FT_D_TFULL0);
      tc_fence_after();
      (void)ld_acquire(ready_h + mb * kCtLine);
      const float* pc = prm + pbuf * 3 * FBN1;
      const int* p_cs = reinterpret_cast<const int*>(pc);
      const int row0 = mb * FBM + quad * 32;
      const int row = row0 + lane;
      const bool row_ok = row < p.M;
      const float sx = row_ok ? __ldcg(p.sh + row) : 0.0f;
      const int zp = row_ok ? __ldcg(p.zh + row) : 0;
      const uint32_t tbase =
          tmem_base + (uint32_t)(acc * C::ACC_COLS) + ((uint32_t)(quad * 32) << 16);
      for (int c0 = part * per2; c0 < (part + 1) * per2; c0 += kChunk) {
        const int n0 = nb * BN2 + c0;
        if (n0 >= p.N2) break;  // warp-uniform
        uint32_t r[kChunk];
        tmem_ld_32x32b_x16(tbase + c0, r);
        tmem_ld_wait();
        float v[kChunk];
        linear_bias_chunk(r, c0, p_cs, pc + FBN1, pc + 2 * FBN1, zp, sx, v);
        emit(v, &tmY, n0, p.N2, row0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
      pbuf ^= 1;
    }
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
    if (e == 0 && lane == 0) ftrace(p, FT_D_END);
  }
  __syncthreads();
  if (threadIdx.x == 0) ftrace(p, FT_EXIT);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

size_t swiglu_fused_extra_bytes(int M) {
  const int tiles_m = cdiv(M, FBM);
  return 2 * al256(sizeof(int) * (size_t)M) + al256(sizeof(int) * ctr_ints(tiles_m));
}

bool swiglu_fused_supported(Ctx* c, const float* x, int M, const IroInt8DevWeight* w13,
                            const IroInt8DevWeight* w2, const float* out, int residual_w2) {
  if (residual_w2 || M <= 0 || !c || c->num_sms <= 0) return false;
  // x is read as float4; the output goes out through TMA tile stores.
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u))
    return false;
  if (w13->layout != IRO_LAYOUT_GATED_PAIR || w13->pair != 128) return false;
  const int D = w13->K, H = w13->hidden;
  if (D % 16 != 0 || H % 16 != 0 || w2->N != D || w2->K != H) return false;
  if (w13->ld != D || w2->ld != H) return false;
  // Opt-in: on the config-2 block (M=2048, D=1024, H=2816) the phases'
  // serial tail (last row blocks -> hidden quantisation -> W2) still makes
  // this slower than the separate kernels.
  const char* env = getenv("IRO_SWIGLU_FUSED");
  return env && *env == '1';
}

int swiglu_fused_launch(Ctx* c, const float* x, int M, const IroInt8DevWeight* w13,
                        const IroInt8DevWeight* w2, const float* b2, float* out,
                        const SwigluBuffers& b, cudaStream_t s) {
  using C = FCfg;
  static bool attr_done[64] = {false};
  if (!attr_done[c->device]) {
    cudaError_t e = cudaFuncSetAttribute(swiglu_fused_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return map_cuda(e);
    attr_done[c->device] = true;
  }
  const int D = w13->K, H = w13->hidden, N2 = w2->N;
  const int BN2 = 128;
  FusedParams p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.D = D;
  p.H = H;
  p.N2 = N2;
  p.tiles_m = cdiv(M, FBM);
  p.tiles_n1 = cdiv(H, FBN1 / 2);
  p.tiles_g = p.tiles_m * p.tiles_n1;
  p.tiles_n2 = cdiv(N2, BN2);
  p.tiles_2 = p.tiles_m * p.tiles_n2;
  p.kb1 = cdiv(D, FBK);
  p.kb2 = cdiv(H, FBK);
  const int G = c->num_sms;
  p.c0 = p.tiles_g % G;
  // Hidden rows go to the CTAs with one gated tile fewer, when there are
  // enough of them to keep that phase short; otherwise to every CTA.
  p.qh_first = (p.c0 != 0 && G - p.c0 >= G / 4) ? p.c0 : 0;
  p.x = x;
  p.qx = b.qx;
  p.sx = b.sx;
  p.zx = b.zx;
  p.hidden = b.hidden;
  p.hlo = b.hlo;
  p.hhi = b.hhi;
  p.qh = b.qh;
  p.sh = b.sh;
  p.zh = b.zh;
  p.w13_scale = w13->scale;
  p.w13_colsum = w13->colsum;
  p.w13_bias = w13->bias;
  p.w2_scale = w2->scale;
  p.w2_colsum = w2->colsum;
  p.b2 = b2;
  p.ctr = b.ctr;
  p.err = c->err;
  p.limit_ns = kWaitLimitNs;

  CUtensorMap tmQx, tmW13, tmHid, tmQh, tmW2, tmY;
  int st = make_tmap_u8(&tmQx, b.qx, (uint64_t)D, (uint64_t)M, (uint64_t)D, FBK, FBM);
  if (!st) st = make_tmap_u8(&tmW13, w13->data, (uint64_t)D, (uint64_t)w13->N, (uint64_t)w13->ld,
                             FBK, FBN1);
  if (!st) st = make_tmap_f32_sw128(&tmHid, b.hidden, (uint64_t)H, (uint64_t)M, (uint64_t)H * 4);
  if (!st) st = make_tmap_u8(&tmQh, b.qh, (uint64_t)H, (uint64_t)M, (uint64_t)H, FBK, FBM);
  if (!st) st = make_tmap_u8(&tmW2, w2->data, (uint64_t)H, (uint64_t)N2, (uint64_t)w2->ld, FBK,
                             BN2);
  if (!st) st = make_tmap_f32_sw128(&tmY, out, (uint64_t)N2, (uint64_t)M, (uint64_t)N2 * 4);
  if (st) return st;

  cudaError_t e = cudaMemsetAsync(b.ctr, 0, sizeof(int) * ctr_ints(p.tiles_m), s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_cuda(e);
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // IRO_FUSED_TRACE=1: per-CTA phase timeline on stderr (diagnostic only;
  // synchronises the stream, so not for use under stream capture).
  static int trace_on = -1;
  if (trace_on < 0) {
    const char* t = getenv("IRO_FUSED_TRACE");
    trace_on = (t && *t && *t != '0') ? 1 : 0;
  }
  unsigned long long* tr = nullptr;
  if (trace_on) {
    if (cudaMalloc(&tr, sizeof(unsigned long long) * FT_SLOTS * G) != cudaSuccess) {
      cudaGetLastError();
      tr = nullptr;
    } else {
      cudaMemsetAsync(tr, 0, sizeof(unsigned long long) * FT_SLOTS * G, s);
    }
  }
  p.trace = tr;
  e = cudaLaunchKernelEx(&cfg, swiglu_fused_kernel, tmQx, tmW13, tmHid, tmQh, tmW2, tmY, p, BN2);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (tr) cudaFree(tr);
    return map_cuda(e);
  }
  if (tr) {
    std::vector<unsigned long long> h((size_t)FT_SLOTS * G);
    cudaStreamSynchronize(s);
    cudaMemcpy(h.data(), tr, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(tr);
    unsigned long long t0 = ~0ull;
    for (int i = 0; i < G; i++) t0 = std::min(t0, h[(size_t)i * FT_SLOTS]);
    fprintf(stderr, "[fused trace] M=%d D=%d H=%d grid=%d gated tiles=%d (c0=%d) w2 tiles=%d\n",
            M, D, H, G, p.tiles_g, p.c0, p.tiles_2);
    for (int k = 0; k < FT_SLOTS; k++) {
      std::vector<double> v;
      for (int i = 0; i < G; i++) {
        const unsigned long long t = h[(size_t)i * FT_SLOTS + k];
        if (t >= t0) v.push_back((t - t0) * 1e-3);
      }
      if (v.empty()) continue;
      std::sort(v.begin(), v.end());
      fprintf(stderr, "  %-10s n=%3zu min %8.2f  med %8.2f  max %8.2f us\n", kFtNames[k], v.size(),
              v.front(), v[v.size() / 2], v.back());
    }
  }
  return IRO_OK;
}

}  // namespace iro
