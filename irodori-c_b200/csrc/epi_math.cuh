// epi_math.cuh — per-chunk epilogue arithmetic of the GEMM kernel
// (gemm_i8.cu).
//
// A chunk is 16 consecutive accumulator columns of one TMEM lane (one output
// row per thread, tcgen05.ld 32x32b).  Column parameters (colsum, weight
// scale, bias) are staged in shared memory and read as broadcast vectors.
#pragma once

#include "iro_common.cuh"

namespace iro {

constexpr int kChunk = 16;  // columns per tcgen05.ld / staging tile

// Staging layout for one warp's 32 x 16 fp32 tile in the 64-byte swizzle the
// TMA store expects: 16-byte chunk c of row r lives at chunk c ^ ((r >> 1) & 3).
__device__ __forceinline__ void stage_row16(uint8_t* stg, int r, const float (&v)[kChunk]) {
#pragma unroll
  for (int c = 0; c < 4; c++) {
    float4* d = reinterpret_cast<float4*>(stg + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    *d = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
}

// Direct stores of one row's chunk (fallback for unaligned outputs).
__device__ __forceinline__ void store_row16(float* dst, const float (&v)[kChunk], int valid) {
#pragma unroll
  for (int j = 0; j < kChunk; j++)
    if (j < valid) dst[j] = v[j];
}

// The gated hidden for one chunk: r1 holds W1 sums for columns c0.., r3 the
// matching W3 sums for columns c3.. of the same tile (dit.c:940-956:
// a = dequant(W1) + b1, g = dequant(W3) + b3, h = silu(a) * g).  Without a
// bias the staged bias is +0, and x + 0 == x here: a dequantised value is
// never -0 (an int converts to +0 and the scales are positive), so the bias
// needs no branch.
__device__ __forceinline__ void gated_chunk(const uint32_t (&r1)[kChunk],
                                            const uint32_t (&r3)[kChunk], int c0, int c3,
                                            const int* p_cs, const float* p_sw,
                                            const float* p_b, int zp, float sx,
                                            float (&v)[kChunk]) {
  float a1[kChunk], a3[kChunk];
#pragma unroll
  for (int i = 0; i < kChunk / 4; i++) {
    const int c1 = c0 + 4 * i, c3i = c3 + 4 * i;
    const int4 cs1 = *reinterpret_cast<const int4*>(p_cs + c1);
    const float4 sw1 = *reinterpret_cast<const float4*>(p_sw + c1);
    const int4 cs3 = *reinterpret_cast<const int4*>(p_cs + c3i);
    const float4 sw3 = *reinterpret_cast<const float4*>(p_sw + c3i);
    float2 a1lo = dequant2(r1[4 * i], r1[4 * i + 1], zp, cs1.x, cs1.y, sx, sw1.x, sw1.y);
    float2 a1hi = dequant2(r1[4 * i + 2], r1[4 * i + 3], zp, cs1.z, cs1.w, sx, sw1.z, sw1.w);
    float2 a3lo = dequant2(r3[4 * i], r3[4 * i + 1], zp, cs3.x, cs3.y, sx, sw3.x, sw3.y);
    float2 a3hi = dequant2(r3[4 * i + 2], r3[4 * i + 3], zp, cs3.z, cs3.w, sx, sw3.z, sw3.w);
    const float4 b1 = *reinterpret_cast<const float4*>(p_b + c1);
    const float4 b3 = *reinterpret_cast<const float4*>(p_b + c3i);
    a1lo = add2_rn(a1lo, make_float2(b1.x, b1.y));
    a1hi = add2_rn(a1hi, make_float2(b1.z, b1.w));
    a3lo = add2_rn(a3lo, make_float2(b3.x, b3.y));
    a3hi = add2_rn(a3hi, make_float2(b3.z, b3.w));
    a1[4 * i] = a1lo.x;
    a1[4 * i + 1] = a1lo.y;
    a1[4 * i + 2] = a1hi.x;
    a1[4 * i + 3] = a1hi.y;
    a3[4 * i] = a3lo.x;
    a3[4 * i + 1] = a3lo.y;
    a3[4 * i + 2] = a3hi.x;
    a3[4 * i + 3] = a3hi.y;
  }
  silu_gate_chunk(a1, a3, v);
}

// One chunk of the plain linear with bias: y = dequant(acc) + bias
// (ops.c:482-485).  The bias is +0 when absent, as above.
__device__ __forceinline__ void linear_bias_chunk(const uint32_t (&r)[kChunk], int c0,
                                                  const int* p_cs, const float* p_sw,
                                                  const float* p_b, int zp, float sx,
                                                  float (&v)[kChunk]) {
#pragma unroll
  for (int i = 0; i < kChunk / 4; i++) {
    const int c = c0 + 4 * i;
    const int4 cs = *reinterpret_cast<const int4*>(p_cs + c);
    const float4 sw = *reinterpret_cast<const float4*>(p_sw + c);
    const float4 b = *reinterpret_cast<const float4*>(p_b + c);
    const float2 lo = add2_rn(dequant2(r[4 * i], r[4 * i + 1], zp, cs.x, cs.y, sx, sw.x, sw.y),
                              make_float2(b.x, b.y));
    const float2 hi = add2_rn(dequant2(r[4 * i + 2], r[4 * i + 3], zp, cs.z, cs.w, sx, sw.z, sw.w),
                              make_float2(b.z, b.w));
    v[4 * i] = lo.x;
    v[4 * i + 1] = lo.y;
    v[4 * i + 2] = hi.x;
    v[4 * i + 3] = hi.y;
  }
}

}  // namespace iro
