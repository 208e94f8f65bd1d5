// gemm_i8.cu — persistent, warp-specialised u8 x s8 -> s32 GEMM on the
// sm_100a tensor cores (tcgen05.mma kind::i8, accumulators in TMEM), fed by
// TMA through a shared-memory ring, with the dequantisation epilogues of the
// reference's int8 linear fused in.
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: A tile [128 x 128 B] (+ second A for the dual
//               term) and B tile [BN x 128 B] per stage, 128-byte swizzle.
//   warp 1      TMEM allocator + MMA issuer: 4 MMAs of K=32 per stage into
//               one of two TMEM accumulator buffers; commits release the
//               stage and, after the last K block, hand the buffer over.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, the exact
//               reference float arithmetic (ops.c:468-490), global stores;
//               runs while the MMA warp fills the other accumulator.
//
// Parity: the integer sums are exact.  The epilogue uses explicitly rounded
// intrinsics in the reference's order, so fp32 outputs are bit-identical to
// the IEEE build of ops.c.
#include "gemm_i8.cuh"

namespace iro {

constexpr int BM = 128;
constexpr int BKB = 128;  // K bytes per pipeline stage (one swizzle row)
constexpr int kThreads = 192;
constexpr int kStageBudget = 196 * 1024;

template <int BN, int EPI>
struct Cfg {
  static constexpr int NA = (EPI == EPI_DUAL) ? 2 : 1;
  static constexpr int A_BYTES = BM * BKB;
  static constexpr int B_BYTES = BN * BKB;
  static constexpr int STAGE = NA * A_BYTES + B_BYTES;
  static constexpr int STAGES = (kStageBudget / STAGE) > 8 ? 8 : (kStageBudget / STAGE);
  static constexpr int ACC_COLS = (EPI == EPI_DUAL) ? 2 * BN : BN;
  static constexpr int TMEM_COLS = (2 * ACC_COLS) <= 32    ? 32
                                   : (2 * ACC_COLS) <= 64  ? 64
                                   : (2 * ACC_COLS) <= 128 ? 128
                                   : (2 * ACC_COLS) <= 256 ? 256
                                                           : 512;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE + BAR_BYTES + 1024;
  static constexpr uint32_t IDESC = idesc_i8(BM, BN, 0);
  static_assert(2 * ACC_COLS <= 512, "TMEM holds 512 columns");
  static_assert(STAGES >= 2, "pipeline needs two stages");
};

struct GemmParams {
  int M, N, K, num_kb, tiles_m, tiles_n, num_tiles;
  const float* sx;
  const int32_t* zp;
  const float* sx2;
  const int32_t* zp2;
  const float* wscale;
  const int32_t* wcolsum;
  const float* bias;
  int bias_vec;  // bias 16-byte aligned
  float* y;
  int ldy;
  int32_t* work;
  int ldw;
  int accumulate;
  float* outs[4];
  int seg;
  float* hidden;
  int ldh;
  int H;
  DevError* err;
  uint64_t limit_ns;
};

// Per-column parameters of 4 consecutive weight rows n..n+3 (colsum, weight
// scale, bias), guarded against n >= N.  `vec` = the 4 rows are in range and
// 16-byte aligned in every array.
struct Col4 {
  int4 cs;
  float4 sw;
  float4 b;
};

__device__ __forceinline__ Col4 load_col4(const int32_t* __restrict__ colsum,
                                          const float* __restrict__ wscale,
                                          const float* __restrict__ bias, int bias_vec, int n,
                                          int N) {
  Col4 c;
  if (n + 4 <= N) {
    c.cs = __ldg(reinterpret_cast<const int4*>(colsum + n));
    c.sw = __ldg(reinterpret_cast<const float4*>(wscale + n));
    if (bias && bias_vec) {
      c.b = __ldg(reinterpret_cast<const float4*>(bias + n));
    } else if (bias) {
      c.b = make_float4(__ldg(bias + n), __ldg(bias + n + 1), __ldg(bias + n + 2),
                        __ldg(bias + n + 3));
    } else {
      c.b = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {
    int cs[4];
    float sw[4], b[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const bool ok = n + j < N;
      cs[j] = ok ? __ldg(colsum + n + j) : 0;
      sw[j] = ok ? __ldg(wscale + n + j) : 0.0f;
      b[j] = (ok && bias) ? __ldg(bias + n + j) : 0.0f;
    }
    c.cs = make_int4(cs[0], cs[1], cs[2], cs[3]);
    c.sw = make_float4(sw[0], sw[1], sw[2], sw[3]);
    c.b = make_float4(b[0], b[1], b[2], b[3]);
  }
  return c;
}

__device__ __forceinline__ float get4(const float4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}
__device__ __forceinline__ int get4(const int4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// Store 4 floats at dst (valid of them in range; vec = 16-byte aligned).
__device__ __forceinline__ void store4(float* dst, const float (&v)[4], int valid, bool vec) {
  if (valid >= 4 && vec) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int j = 0; j < 4; j++)
      if (j < valid) dst[j] = v[j];
  }
}

__device__ __forceinline__ void load4(const float* src, float (&v)[4], int valid, bool vec) {
  if (valid >= 4 && vec) {
    const float4 t = *reinterpret_cast<const float4*>(src);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
#pragma unroll
    for (int j = 0; j < 4; j++) v[j] = j < valid ? src[j] : 0.0f;
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2, const GemmParams p) {
  using C = Cfg<BN, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI == EPI_DUAL) tma_prefetch_desc(&tmA2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int mb = tile % p.tiles_m, nb = tile / p.tiles_m;
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 1, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE;
          uint8_t* sb = sa + C::NA * C::A_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          tma_load_2d(sa, &tmA, &full[s], kb * BKB, mb * BM);
          if (EPI == EPI_DUAL) tma_load_2d(sa + C::A_BYTES, &tmA2, &full[s], kb * BKB, mb * BM);
          tma_load_2d(sb, &tmB, &full[s], kb * BKB, nb * BN);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
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
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        if (!mbar_wait_bounded(&tempty[acc], aph ^ 1u, p.err, 2, abort_flag, p.limit_ns)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * C::ACC_COLS);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait_bounded(&full[s], ph, p.err, 3, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * C::STAGE);
          const uint32_t b_addr = a_addr + C::NA * C::A_BYTES;
#pragma unroll
          for (int j = 0; j < BKB / 32; j++) {
            const uint64_t bd = sw128_desc(b_addr + 32 * j);
            const uint32_t accum = (kb > 0 || j > 0) ? 1u : 0u;
            mma_i8(d, sw128_desc(a_addr + 32 * j), bd, C::IDESC, accum);
            if (EPI == EPI_DUAL)
              mma_i8(d + BN, sw128_desc(a_addr + C::A_BYTES + 32 * j), bd, C::IDESC, accum);
          }
          mma_commit(&empty[s]);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    int acc = 0;
    uint32_t aph = 0;
    const bool y_vec = ((p.ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 15u) == 0);
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int mb = tile % p.tiles_m, nb = tile / p.tiles_m;
      bool got = mbar_wait_bounded(&tfull[acc], aph, p.err, 4, abort_flag, p.limit_ns);
      got = __all_sync(0xffffffffu, got);
      if (!got) break;
      tc_fence_after();
      const int row = mb * BM + quad * 32 + lane;
      const bool row_ok = row < p.M;
      const float sx = row_ok ? __ldg(p.sx + row) : 0.0f;
      const int zp = row_ok ? __ldg(p.zp + row) : 0;
      const uint32_t tbase =
          tmem_base + (uint32_t)(acc * C::ACC_COLS) + ((uint32_t)(quad * 32) << 16);

      if (EPI == EPI_GATED) {
        // Columns [0, BN/2) hold W1 rows, [BN/2, BN) the matching W3 rows.
        constexpr int HALF = BN / 2;
        const bool hv = ((p.ldh & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.hidden) & 15u) == 0);
        for (int c0 = 0; c0 < HALF; c0 += 32) {
          const int h0 = nb * HALF + c0;
          if (h0 >= p.H) break;  // warp-uniform
          uint32_t r1[32], r3[32];
          tmem_ld_32x32b_x32(tbase + c0, r1);
          tmem_ld_32x32b_x32(tbase + HALF + c0, r3);
          tmem_ld_wait();
          float* hrow = p.hidden + (size_t)row * p.ldh + h0;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const int n1 = nb * BN + c0 + 4 * i;
            const Col4 k1 = load_col4(p.wcolsum, p.wscale, p.bias, 1, n1, p.N);
            const Col4 k3 = load_col4(p.wcolsum, p.wscale, p.bias, 1, n1 + HALF, p.N);
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              float a1 = dequant((int)r1[4 * i + j], zp, get4(k1.cs, j), sx, get4(k1.sw, j));
              float a3 = dequant((int)r3[4 * i + j], zp, get4(k3.cs, j), sx, get4(k3.sw, j));
              if (p.bias) {
                a1 = __fadd_rn(a1, get4(k1.b, j));
                a3 = __fadd_rn(a3, get4(k3.b, j));
              }
              // ops.c:781-784: (x / (1 + expf(-x))) * g
              v[j] = __fmul_rn(__fdiv_rn(a1, __fadd_rn(1.0f, expf(-a1))), a3);
            }
            if (row_ok) store4(hrow + 4 * i, v, p.H - h0 - 4 * i, hv);
          }
        }
      } else {
        const bool vec_out = (EPI == EPI_SPLIT) ? ((p.seg & 3) == 0) : y_vec;
        for (int c0 = 0; c0 < BN; c0 += 32) {
          const int n0 = nb * BN + c0;
          if (n0 >= p.N) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c0, r);
          uint32_t r2[32];
          if (EPI == EPI_DUAL) tmem_ld_32x32b_x32(tbase + BN + c0, r2);
          tmem_ld_wait();
          float sx2 = 0.0f;
          int zp2 = 0;
          if (EPI == EPI_DUAL && row_ok) {
            sx2 = __ldg(p.sx2 + row);
            zp2 = __ldg(p.zp2 + row);
          }
          float* dst;
          int ld;
          if (EPI == EPI_SPLIT) {
            const int g = n0 / p.seg;
            float* base = g == 0 ? p.outs[0] : g == 1 ? p.outs[1] : g == 2 ? p.outs[2] : p.outs[3];
            dst = base + (n0 - g * p.seg);
            ld = p.seg;
          } else {
            dst = p.y + n0;
            ld = p.ldy;
          }
          float* drow = dst + (size_t)row * ld;
          int32_t* wrow = (EPI == EPI_LINEAR && p.work) ? p.work + (size_t)row * p.ldw + n0 : nullptr;
          const bool w_vec = (p.ldw & 3) == 0;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const int n = n0 + 4 * i;
            const int valid = p.N - n;
            const Col4 k = load_col4(p.wcolsum, p.wscale, p.bias, p.bias_vec, n, p.N);
            float old[4] = {0.f, 0.f, 0.f, 0.f};
            if (EPI == EPI_LINEAR && p.accumulate && row_ok && valid > 0)
              load4(drow + 4 * i, old, valid, vec_out);
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              float t = dequant((int)r[4 * i + j], zp, get4(k.cs, j), sx, get4(k.sw, j));
              if (p.bias) t = __fadd_rn(t, get4(k.b, j));
              if (EPI == EPI_DUAL)
                t = __fadd_rn(t, dequant((int)r2[4 * i + j], zp2, get4(k.cs, j), sx2, get4(k.sw, j)));
              if (EPI == EPI_LINEAR && p.accumulate) t = __fadd_rn(old[j], t);
              v[j] = t;
            }
            if (row_ok && valid > 0) {
              store4(drow + 4 * i, v, valid, vec_out);
              if (wrow) {
                if (valid >= 4 && w_vec) {
                  *reinterpret_cast<int4*>(wrow + 4 * i) =
                      make_int4((int)r[4 * i], (int)r[4 * i + 1], (int)r[4 * i + 2], (int)r[4 * i + 3]);
                } else {
#pragma unroll
                  for (int j = 0; j < 4; j++)
                    if (j < valid) wrow[4 * i + j] = (int)r[4 * i + j];
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN, int EPI>
static int launch_t(Ctx* c, const GemmRequest& r, const GemmParams& p0, cudaStream_t s) {
  using C = Cfg<BN, EPI>;
  static bool attr_done[64] = {false};
  if (!attr_done[c->device]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<BN, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return map_cuda(e);
    attr_done[c->device] = true;
  }
  const IroInt8DevWeight* w = r.w;
  CUtensorMap ta, tb, ta2;
  int st = make_tmap_u8(&ta, r.a, (uint64_t)w->K, (uint64_t)r.M, (uint64_t)r.lda, BKB, BM);
  if (st) return st;
  st = make_tmap_u8(&tb, w->data, (uint64_t)w->K, (uint64_t)w->N, (uint64_t)w->ld, BKB, BN);
  if (st) return st;
  if (EPI == EPI_DUAL) {
    st = make_tmap_u8(&ta2, r.a2, (uint64_t)w->K, (uint64_t)r.M, (uint64_t)r.lda, BKB, BM);
    if (st) return st;
  } else {
    ta2 = ta;
  }
  GemmParams p = p0;
  p.tiles_m = cdiv(r.M, BM);
  p.tiles_n = cdiv(w->N, BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  const int grid = p.num_tiles < c->num_sms ? p.num_tiles : c->num_sms;
  gemm_i8_kernel<BN, EPI><<<grid, kThreads, C::SMEM, s>>>(ta, tb, ta2, p);
  return check_launch();
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

int gemm_launch(Ctx* c, const GemmRequest& r, cudaStream_t s) {
  const IroInt8DevWeight* w = r.w;
  if (r.M == 0) return IRO_OK;
  if (r.M < 0 || !w || !w->data || !r.a || !r.sx || !r.zp) return IRO_ERR_INVALID;
  if ((r.lda & 15) != 0 || r.lda < w->K) return IRO_ERR_UNSUPPORTED;
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
  p.bias_vec = p.bias ? ((reinterpret_cast<uintptr_t>(p.bias) & 15u) == 0) : 0;
  p.y = r.y;
  p.ldy = r.ldy;
  p.work = r.work;
  p.ldw = r.ldw;
  p.accumulate = r.accumulate;
  for (int i = 0; i < 4; i++) p.outs[i] = r.outs[i];
  p.seg = r.seg;
  p.hidden = r.hidden;
  p.ldh = r.ldh;
  p.H = w->hidden;
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
    case EPI_GATED:
      if (w->layout != IRO_LAYOUT_GATED_PAIR || w->pair != 128 || !r.hidden)
        return IRO_ERR_UNSUPPORTED;
      return launch_t<256, EPI_GATED>(c, r, p, s);
    case EPI_DUAL: {
      if (!r.a2 || !r.sx2 || !r.zp2 || !r.y) return IRO_ERR_INVALID;
      const int bn = r.force_bn ? r.force_bn : pick_bn(r.M, w->N, c->num_sms, 1);
      if (bn == 128) return launch_t<128, EPI_DUAL>(c, r, p, s);
      return launch_t<64, EPI_DUAL>(c, r, p, s);
    }
    default:
      return IRO_ERR_INVALID;
  }
}

}  // namespace iro
