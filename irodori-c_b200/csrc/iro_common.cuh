// iro_common.cuh — shared device helpers for the sm_100a int8 path:
// IEEE-exact quantisation arithmetic, bounded mbarrier waits, TMA loads and
// the tcgen05 (5th-gen tensor core / TMEM) primitives, all as inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "irodori_b200.h"

namespace iro {

// ---------------------------------------------------------------------------
// Device error word.  Bounded waits that run out record a code here (the
// first one wins) instead of trapping, so the context stays usable and the
// host reports a status.
struct DevError {
  int code;      // IRO_ERR_* (0 = none)
  int where;     // which wait gave up
  int block;     // blockIdx.x of the reporter
  int pad;
};

__device__ __forceinline__ void report_error(DevError* e, int code, int where) {
  if (e == nullptr) return;
  if (atomicCAS(&e->code, 0, code) == 0) {
    e->where = where;
    e->block = blockIdx.x;
  }
}

// fp32 -> fp16 for the DiT attention operands, with their range check:
// finite values whose magnitude rounds past the largest half (|x| >= 65520)
// are reported as IRO_ERR_RANGE (`where` names the producer); NaN and inf
// pass through as in fp32.
__device__ __forceinline__ __half to_half_checked(float x, DevError* err, int where) {
  if (fabsf(x) >= 65520.0f && fabsf(x) != __int_as_float(0x7f800000)) {
    report_error(err, IRO_ERR_RANGE, where);
  }
  return __float2half_rn(x);
}

// Two floats as packed halves (lo in the low 16 bits), round to nearest.
__device__ __forceinline__ uint32_t pack_half2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// to_half_checked's range check for a chunk of values at once: the largest
// finite magnitude against 65520 (a chunk holding an inf is not reported;
// the inf passes through as in fp32).
template <int N>
__device__ __forceinline__ void check_half_range(const float (&v)[N], DevError* err, int where) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < N; i++) amax = fmaxf(amax, fabsf(v[i]));
  if (amax >= 65520.0f && amax != __int_as_float(0x7f800000)) report_error(err, IRO_ERR_RANGE, where);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Quantisation arithmetic.  Every operation is an explicit round-to-nearest
// intrinsic so that nvcc cannot contract a multiply-add into an FMA: the CPU
// reference computes each product and sum as a separately rounded binary32
// operation.

// float -> int32 with the x86-64 cvttss2si result for NaN / out of range
// (INT32_MIN), which is what the reference's plain C casts produce on its
// host.  `v` is integral here (already rounded), so truncation is exact.
__device__ __forceinline__ int f2i_x86(float v) {
  return (v >= -2147483648.0f && v < 2147483648.0f) ? __float2int_rz(v)
                                                     : (int)0x80000000;
}

// Row parameters from a range [lo, hi] that includes 0:
// s = (hi-lo)/255 (1 if not > 0); inv = 1/s; zp = clamp(rint(-lo*inv),0,255).
__device__ __forceinline__ void row_params(float lo, float hi, float& s,
                                           float& inv, int& zp) {
  s = __fdiv_rn(__fsub_rn(hi, lo), 255.0f);
  if (!(s > 0.0f)) s = 1.0f;
  inv = __fdiv_rn(1.0f, s);
  int z = f2i_x86(rintf(__fmul_rn(-lo, inv)));
  z = z < 0 ? 0 : z;
  z = z > 255 ? 255 : z;
  zp = z;
}

// One asymmetric code: clamp(rint(x*inv + zp), 0, 255); NaN -> 0 as the
// reference's (uint8_t) cast gives on x86-64.  t = x*inv + zp is rounded as
// the reference rounds it; clamping t to [0, 255] before rounding gives the
// same code (rint is monotone and keeps 0 and 255; fmaxf sends a NaN to 0),
// and the rounding is one add of 1.5 * 2^23: for t in [0, 255] the sum is
// exactly 1.5 * 2^23 + rint(t) (ties to even, as nearbyintf), so the code is
// the low byte of its bits and the rounded value is the sum minus 1.5 * 2^23.
// No float<->int conversions (which issue at half rate).
constexpr float kRintMagic = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t kRintMagicBits = 0x4B400000u;

__device__ __forceinline__ float quant_round(float x, float inv, float zpf) {
  const float t = fminf(fmaxf(__fadd_rn(__fmul_rn(x, inv), zpf), 0.0f), 255.0f);
  return __fadd_rn(t, kRintMagic);
}

__device__ __forceinline__ uint32_t quant_code(float x, float inv, float zpf) {
  return __float_as_uint(quant_round(x, inv, zpf)) - kRintMagicBits;
}

// The same code, also returning the clamped float value (the conv's
// remainder term uses it).  For a NaN input the reference keeps v = NaN while
// this gives 0; the remainder is NaN either way (it subtracts from x).
__device__ __forceinline__ uint32_t quant_code_v(float x, float inv, float zpf,
                                                 float& vout) {
  const float m = quant_round(x, inv, zpf);
  vout = __fsub_rn(m, kRintMagic);
  return __float_as_uint(m) - kRintMagicBits;
}

// Four codes packed little-endian (x in the low byte), with the rounded
// values (for the two-term residual) in r.
__device__ __forceinline__ uint32_t quant_code4(float4 x, float inv, float zpf, float4& r) {
  const float m0 = quant_round(x.x, inv, zpf), m1 = quant_round(x.y, inv, zpf);
  const float m2 = quant_round(x.z, inv, zpf), m3 = quant_round(x.w, inv, zpf);
  r = make_float4(__fsub_rn(m0, kRintMagic), __fsub_rn(m1, kRintMagic),
                  __fsub_rn(m2, kRintMagic), __fsub_rn(m3, kRintMagic));
  const uint32_t lo = __byte_perm(__float_as_uint(m0), __float_as_uint(m1), 0x0040);
  const uint32_t hi = __byte_perm(__float_as_uint(m2), __float_as_uint(m3), 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

__device__ __forceinline__ uint32_t quant_code4(float4 x, float inv, float zpf) {
  float4 r;
  return quant_code4(x, inv, zpf, r);
}

// Running min/max of a row.  The reference updates with strict comparisons
// (a NaN never replaces the running value, -0.0 never replaces +0.0).
// fminf/fmaxf agree on NaN; they may keep -0.0 where the reference keeps
// +0.0, which changes no output: the range enters only as hi - lo (equal for
// either zero) and rint(-lo * inv) (a zero either way).
__device__ __forceinline__ float run_lo(float v, float lo) { return fminf(v, lo); }
__device__ __forceinline__ float run_hi(float v, float hi) { return fmaxf(v, hi); }

__device__ __forceinline__ void warp_minmax(float& lo, float& hi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float l2 = __shfl_xor_sync(0xffffffffu, lo, o);
    float h2 = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = run_lo(l2, lo);
    hi = run_hi(h2, hi);
  }
}

__device__ __forceinline__ float warp_max(float a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float b = __shfl_xor_sync(0xffffffffu, a, o);
    a = b > a ? b : a;
  }
  return a;
}

// Dequantised output of one accumulator:
// (float)(acc - zp*colsum) * (sx*sw) [+ bias], each step rounded.
__device__ __forceinline__ float dequant(int acc, int zp, int colsum, float sx,
                                         float sw) {
  return __fmul_rn(__int2float_rn(acc - zp * colsum), __fmul_rn(sx, sw));
}

// Two dequantised outputs (the reference's scalar formula twice).  Packed
// f32x2 arithmetic is not used here: ptxas may contract a packed product
// and a packed sum into one FFMA2 even with explicit .rn, which changes the
// rounding; the scalar __fmul_rn / __fadd_rn are never contracted.
__device__ __forceinline__ float2 dequant2(uint32_t acc0, uint32_t acc1, int zp, int cs0,
                                           int cs1, float sx, float sw0, float sw1) {
  return make_float2(dequant((int)acc0, zp, cs0, sx, sw0), dequant((int)acc1, zp, cs1, sx, sw1));
}

__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
}

// silu(a) * g as the reference writes it, (a / (1 + expf(-a))) * g
// (ops.c:781-784), for the N outputs one lane holds in an epilogue chunk.
// expf is the CUDA math library's (a faster hardware-ex2 exponential was
// tried and moved the hidden up to 5 ulp from the host libm, enough to flip
// requantisation codes).
//
// The quotient a / d (d = 1 + expf(-a) >= 1) uses Markstein's method: an
// approximate reciprocal r, q0 = a*r, the exact residual a - q0*d from one
// FMA, and one correction q0 + residual*r.  That lands within half an ulp of
// a/d except when a/d lies within ~2^-23 ulp of a rounding boundary, and it
// needs d < 2^126 (the flushed reciprocal vanishes above) and a != +inf.
// One warp vote per chunk sends the rare chunks outside that range
// (a <= -87 or a = +inf) to the exactly rounded division, so the common path
// has no per-output branch or select and the chunk's outputs schedule
// together.  NaN inputs take the fast path and stay NaN.
template <int N>
__device__ __forceinline__ void silu_gate_chunk(const float (&a)[N], const float (&g)[N],
                                                float (&out)[N]) {
  float d[N];
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < N; j++) {
    d[j] = __fadd_rn(1.0f, expf(-a[j]));
    m = fmaxf(m, fmaxf(d[j], a[j]));
  }
  if (__any_sync(0xffffffffu, m >= 8.5070592e37f)) {  // 2^126
#pragma unroll
    for (int j = 0; j < N; j++) out[j] = __fmul_rn(__fdiv_rn(a[j], d[j]), g[j]);
  } else {
#pragma unroll
    for (int j = 0; j < N; j++) {
      float r;
      asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d[j]));
      const float q0 = __fmul_rn(a[j], r);
      const float e = __fmaf_rn(-q0, d[j], a[j]);
      out[j] = __fmul_rn(__fmaf_rn(e, r, q0), g[j]);
    }
  }
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel in the stream drains.
// It must call grid_dep_wait() before it reads or writes global memory that
// kernel touches; without that launch attribute the call returns at once.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory addresses and mbarriers.

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One bounded poll of the phase with the given parity.  The suspend-time
// hint lets the hardware park the thread until the phase completes (or the
// hint expires) instead of spinning on shared memory, which would compete
// with the tensor cores' operand reads.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after
// about `limit_ns` (or when `abort` is raised by another role).  The bound
// uses the SM cycle counter, converted at 2 cycles per ns, so a slower clock
// only lengthens the wait.  Returns false on give-up, after recording the
// error.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  DevError* err, int where,
                                                  volatile int* abort_flag,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  const long long limit_cycles = (long long)(limit_ns * 2ull);
  while (!mbar_try_wait(bar, parity)) {
    if (abort_flag != nullptr && *abort_flag) return false;
    if (clock64() - t0 > limit_cycles) {
      report_error(err, IRO_ERR_DEVICE_TIMEOUT, where);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) loads, no multicast.

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// TMA tile store from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x,
                                             int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(smem_u32(smem_src))
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (TMA).
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier over `count` threads (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier over `count` threads that also ORs a predicate across them:
// every participant learns whether any of them passed `pred` = true.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA issue, commit, loads and fences.

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, kind::i8, one CTA.  `accumulate` = 0
// overwrites D.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM into 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 columns of 32-bit TMEM into 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored as rows
// of 128 bytes with the 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B): 8-row core groups 1024 bytes apart, version 1,
// layout type 2 (SWIZZLE_128B).  The tile base must be 1024-byte aligned;
// K steps inside the 128-byte row advance the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused)
  d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset
  d |= (uint64_t)1 << 46;                          // descriptor version
  d |= (uint64_t)2 << 61;                          // SWIZZLE_128B
  return d;
}

// Shared-memory descriptor for an MN-major operand (B of D = A.B^T with B's
// N index contiguous) stored as 128-byte rows of 32 fp32 along N, one row per
// K index, with the 128-byte swizzle: consecutive K rows 128 bytes apart,
// 8-row K groups 1024 bytes apart (stride byte offset), and the next 32 N
// elements `mn_stride` bytes further (leading byte offset).
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t smem_addr, uint32_t mn_stride) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((mn_stride >> 4) & 0x3FFFu) << 16;  // leading byte offset
  d |= (uint64_t)(1024 >> 4) << 32;                   // stride byte offset
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f16 operands: D = f32, A = B =
// f16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16 (K = 16 per instruction).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16, A = 128 lanes x K halves
// packed two per 32-bit column (K / 2 columns).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 registers per thread into 32 lanes x 32 columns of 32-bit TMEM.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 16 registers per thread into 32 lanes x 16 columns of 32-bit TMEM.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Instruction descriptor for kind::i8: D = s32, A = u8 (0) or s8 (1),
// B = s8, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, int a_signed) {
  return (2u << 4) | ((uint32_t)a_signed << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

}  // namespace iro
