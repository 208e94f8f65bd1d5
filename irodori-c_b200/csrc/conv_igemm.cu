// conv_igemm.cu — the codec's W8A8 kernel-7 convolution (dacvae.c:543-688)
// as an implicit GEMM on the tcgen05 tensor cores: the u8 im2col operand is
// never written to memory.
//
// Per CTA tile: 128 consecutive output frames of one sequence x all N output
// channels (NT = 512 per tile).  The K loop runs over 64-channel chunks of
// the input and, inside each chunk, over the kernel taps (K index of the
// weight = tap*C + channel, the reference's [out, kernel, in] layout,
// dacvae.h:11-12).
//
// Warp roles (576 threads):
//   warp 0      TMA: the fp32 input window of each channel chunk (rows
//               t0 - pad .. t0 - pad + 127 + (kernel-1)*dilation, 64
//               channels; a 3-D map over [batch, T, C] so rows outside the
//               sequence read as 0 and never reach the next sequence), and
//               the weight tile of each stage (64 K bytes x NT rows).
//   warp 1      TMEM allocation and the MMA issue (two K=32 steps x two
//               N=256 halves per stage).
//   warps 2..9  A producers: per stage, quantise the 128 x 64 fp32 window
//               slice of one tap with each output row's own scale and zero
//               point into the 64-byte-swizzled smem layout the MMA reads.
//               A row outside the sequence is 0 in the window and becomes
//               the zero point, which is what the reference writes for a
//               padding tap; 0 is inside every row range, so the row
//               parameters are unaffected either way.
//   warps 10..17 epilogue: dequantise with the reference's float order
//               (ops.c:468-490), add the bias, TMA tile stores through a 3-D
//               output map (clipped per sequence).
//
// The per-output-row parameters (range over the taps' rows with 0 included,
// dacvae.c:607-627) come from conv_row_range and conv_row_params (conv7.cu)
// before the launch.
#include <string.h>

#include "conv_igemm.cuh"

namespace iro {
namespace {

constexpr int CV_BM = 128;
constexpr int CV_NT = 512;        // output channels per tile
constexpr int CV_BK = 64;         // K bytes (channels of one tap) per stage
constexpr int CV_CH = 64;         // channels per window chunk
constexpr int CV_PROD_WARPS = 8;
constexpr int CV_EPI_WARPS = 8;
constexpr int CV_THREADS = 64 + 32 * (CV_PROD_WARPS + CV_EPI_WARPS);
constexpr int CV_STAGES = 3;       // maximum; p.nstages is 2 or 3
constexpr int CV_A_BYTES = CV_BM * CV_BK;              // 8 KB
constexpr int CV_B_BYTES = CV_NT * CV_BK;              // 32 KB
constexpr int CV_STAGE = CV_A_BYTES + CV_B_BYTES;
constexpr int CV_WIN_ROWS_MAX = 256;  // TMA box rows
constexpr int CV_SMEM_MAX = 232448;
constexpr int CV_STG = 32 * 16 * 4;                    // staging tile per epilogue warp
constexpr uint32_t CV_IDESC = idesc_i8(128, 256, 0);

struct ConvParams {
  int batch, T_in, T_out, C, N, kernel, dilation, padding;
  int tiles_t, num_tiles, n_chunks, stages_per_tile, win_rows, win_bytes, nstages;
  const float* scale;  // per output row [batch*T_out]
  const int32_t* zero;
  const float* inv;
  const int32_t* wcolsum;
  const float* wscale;
  const float* bias;
  DevError* err;
  uint64_t limit_ns;
};

// 64-byte-swizzle K-major descriptor: 8-row core groups 512 bytes apart.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;  // SWIZZLE_64B
  return d;
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int x,
                                             int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(z), "r"(smem_u32(smem_src))
      : "memory");
}

// clamp(rint(x*inv + zp), 0, 255) in one saturating conversion (NaN -> 0).
__device__ __forceinline__ uint32_t code_u8(float x, float inv, float zpf) {
  uint32_t u;
  asm("cvt.rni.sat.u8.f32 %0, %1;" : "=r"(u) : "f"(__fadd_rn(__fmul_rn(x, inv), zpf)));
  return u;
}

__global__ void __launch_bounds__(CV_THREADS, 1)
    conv7_igemm_kernel(const __grid_constant__ CUtensorMap tmIn,
                       const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmOut, const ConvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;                                   // nstages x (A | B)
  float* win = reinterpret_cast<float*>(smem + p.nstages * CV_STAGE);  // 2 x window
  uint8_t* stg = reinterpret_cast<uint8_t*>(win) + 2 * p.win_bytes;   // epilogue staging
  float* prm = reinterpret_cast<float*>(stg + CV_EPI_WARPS * CV_STG);  // colsum|scale|bias [3][NT]
  uint64_t* full = reinterpret_cast<uint64_t*>(prm + 3 * CV_NT);
  uint64_t* empty = full + CV_STAGES;
  uint64_t* wfull = empty + CV_STAGES;   // [2]
  uint64_t* wempty = wfull + 2;          // [2]
  uint64_t* tfull = wempty + 2;
  uint64_t* tempty = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nstages; i++) {
      mbar_init(&full[i], 1 + CV_PROD_WARPS);  // TMA producer + the A producers
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], CV_PROD_WARPS);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, CV_EPI_WARPS);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmIn);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, CV_NT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int kstages = p.stages_per_tile;

  if (warp == 0) {
    // ---------------- TMA: windows and weight tiles ----------------
    if (lane == 0) {
      int s = 0, wb = 0;
      uint32_t ph = 0, wph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int b = tile / p.tiles_t;
        const int t0 = (tile - b * p.tiles_t) * CV_BM;
        for (int cc = 0; ok && cc < p.n_chunks; cc++) {
          // Window of this channel chunk (double-buffered).
          if (!mbar_wait_bounded(&wempty[wb], wph ^ 1u, p.err, 11, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&wfull[wb], (uint32_t)(p.win_rows * CV_CH * 4));
          tma_load_3d(win + (size_t)wb * (p.win_bytes / 4), &tmIn, &wfull[wb], cc * CV_CH,
                      t0 - p.padding, b);
          if (++wb == 2) {
            wb = 0;
            wph ^= 1u;
          }
          for (int tap = 0; tap < p.kernel; tap++) {
            if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 12, abort_flag, p.limit_ns)) {
              ok = false;
              break;
            }
            uint8_t* sb = stages + s * CV_STAGE + CV_A_BYTES;
            mbar_arrive_expect_tx(&full[s], CV_B_BYTES);
            const int kx = tap * p.C + cc * CV_CH;
            tma_load_2d(sb, &tmW, &full[s], kx, 0);
            tma_load_2d(sb + CV_B_BYTES / 2, &tmW, &full[s], kx, 256);
            if (++s == p.nstages) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        if (!mbar_wait_bounded(tempty, aph ^ 1u, p.err, 13, abort_flag, p.limit_ns)) break;
        tc_fence_after();
        for (int ks = 0; ks < kstages; ks++) {
          if (!mbar_wait_bounded(&full[s], ph, p.err, 14, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + s * CV_STAGE);
          const uint32_t b_addr = a_addr + CV_A_BYTES;
#pragma unroll
          for (int j = 0; j < CV_BK / 32; j++) {
            const uint32_t accum = (ks > 0 || j > 0) ? 1u : 0u;
            const uint64_t ad = sw64_desc(a_addr + 32 * j);
            mma_i8(tmem_base, ad, sw64_desc(b_addr + 32 * j), CV_IDESC, accum);
            mma_i8(tmem_base + 256, ad, sw64_desc(b_addr + CV_B_BYTES / 2 + 32 * j), CV_IDESC,
                   accum);
          }
          mma_commit(&empty[s]);
          if (++s == p.nstages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(tfull);
        aph ^= 1u;
      }
    }
    __syncwarp();
  } else if (warp < 2 + CV_PROD_WARPS) {
    // ---------------- A producers ----------------
    const int pt = threadIdx.x - 64;      // 0..255
    const int g = pt & 15;                // channel group: channels 4g..4g+3
    const int rsub = pt >> 4;             // 0..15
    int s = 0, wb = 0;
    uint32_t ph = 0, wph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      const int b = tile / p.tiles_t;
      const int t0 = (tile - b * p.tiles_t) * CV_BM;
      // This thread's 8 rows (rsub + 16 j) and their parameters.
      float inv[8], zpf[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int t = t0 + rsub + 16 * j;
        const bool in = t < p.T_out;
        const size_t gi = (size_t)b * p.T_out + (in ? t : 0);
        inv[j] = in ? __ldg(p.inv + gi) : 0.0f;
        zpf[j] = in ? (float)__ldg(p.zero + gi) : 0.0f;
      }
      for (int cc = 0; ok && cc < p.n_chunks; cc++) {
        if (!mbar_wait_bounded(&wfull[wb], wph, p.err, 15, abort_flag, p.limit_ns)) {
          ok = false;
          break;
        }
        const float* w = win + (size_t)wb * (p.win_bytes / 4);
        for (int tap = 0; tap < p.kernel; tap++) {
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 16, abort_flag, p.limit_ns)) {
            ok = false;
            break;
          }
          uint8_t* sa = stages + s * CV_STAGE;
          const int roff = tap * p.dilation;
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const int r = rsub + 16 * j;
            const float4 x = *reinterpret_cast<const float4*>(w + (size_t)(r + roff) * CV_CH + 4 * g);
            const uint32_t c0 = code_u8(x.x, inv[j], zpf[j]);
            const uint32_t c1 = code_u8(x.y, inv[j], zpf[j]);
            const uint32_t c2 = code_u8(x.z, inv[j], zpf[j]);
            const uint32_t c3 = code_u8(x.w, inv[j], zpf[j]);
            const uint32_t word = __byte_perm(__byte_perm(c0, c1, 0x0040),
                                              __byte_perm(c2, c3, 0x0040), 0x5410);
            // 64-byte swizzle: 16-byte chunk (g >> 2) of row r sits at chunk
            // (g >> 2) ^ ((r >> 1) & 3).
            const int off = r * 64 + ((((g >> 2) ^ ((r >> 1) & 3))) << 4) + ((g & 3) << 2);
            *reinterpret_cast<uint32_t*>(sa + off) = word;
          }
          fence_async_shared();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
          if (++s == p.nstages) {
            s = 0;
            ph ^= 1u;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[wb]);
        if (++wb == 2) {
          wb = 0;
          wph ^= 1u;
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int e = warp - 2 - CV_PROD_WARPS;   // 0..7
    const int quad = warp & 3;
    const int half = e >> 2;                  // output channels [256*half, +256)
    const int et = threadIdx.x - 64 - 32 * CV_PROD_WARPS;  // 0..255
    uint8_t* mystg = stg + e * CV_STG;
    int* p_cs = reinterpret_cast<int*>(prm);
    float* p_sw = prm + CV_NT;
    float* p_b = prm + 2 * CV_NT;
    for (int j = et; j < CV_NT; j += 32 * CV_EPI_WARPS) {
      p_cs[j] = __ldg(p.wcolsum + j);
      p_sw[j] = __ldg(p.wscale + j);
      p_b[j] = p.bias ? __ldg(p.bias + j) : 0.0f;
    }
    named_bar(2, 32 * CV_EPI_WARPS);
    uint32_t aph = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int b = tile / p.tiles_t;
      const int t0 = (tile - b * p.tiles_t) * CV_BM;
      const int trow0 = t0 + quad * 32;
      const int t = trow0 + lane;
      const bool row_ok = t < p.T_out;
      const size_t gi = (size_t)b * p.T_out + (row_ok ? t : 0);
      const float sx = row_ok ? __ldg(p.scale + gi) : 0.0f;
      const int zp = row_ok ? __ldg(p.zero + gi) : 0;
      const bool got = mbar_wait_bounded(tfull, aph, p.err, 17, abort_flag, p.limit_ns);
      if (named_bar_or(3, 32 * CV_EPI_WARPS, !got)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16);
      for (int c0 = half * 256; c0 < half * 256 + 256; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tbase + c0, r);
        tmem_ld_wait();
        float v[16];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int c = c0 + 4 * i;
          const int4 cs = *reinterpret_cast<const int4*>(p_cs + c);
          const float4 sw = *reinterpret_cast<const float4*>(p_sw + c);
          const float4 bb = *reinterpret_cast<const float4*>(p_b + c);
          v[4 * i] = dequant((int)r[4 * i], zp, cs.x, sx, sw.x);
          v[4 * i + 1] = dequant((int)r[4 * i + 1], zp, cs.y, sx, sw.y);
          v[4 * i + 2] = dequant((int)r[4 * i + 2], zp, cs.z, sx, sw.z);
          v[4 * i + 3] = dequant((int)r[4 * i + 3], zp, cs.w, sx, sw.w);
          if (p.bias) {  // no add without a bias: keeps a -0.0 as the reference does
            v[4 * i] = __fadd_rn(v[4 * i], bb.x);
            v[4 * i + 1] = __fadd_rn(v[4 * i + 1], bb.y);
            v[4 * i + 2] = __fadd_rn(v[4 * i + 2], bb.z);
            v[4 * i + 3] = __fadd_rn(v[4 * i + 3], bb.w);
          }
        }
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int cq = 0; cq < 4; cq++) {
          float4* d = reinterpret_cast<float4*>(mystg + lane * 64 + ((cq ^ ((lane >> 1) & 3)) << 4));
          *d = make_float4(v[4 * cq], v[4 * cq + 1], v[4 * cq + 2], v[4 * cq + 3]);
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0 && trow0 < p.T_out) {
          tma_store_3d(&tmOut, mystg, c0, trow0, b);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
      aph ^= 1u;
    }
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, CV_NT);
  }
}

int smem_bytes(int win_bytes, int nstages) {
  return nstages * CV_STAGE + 2 * win_bytes + CV_EPI_WARPS * CV_STG + 3 * CV_NT * 4 + 256 + 1024;
}

int win_bytes_for(int kernel, int dilation) {
  return round_up((CV_BM + (kernel - 1) * dilation) * CV_CH * 4, 1024);
}

}  // namespace

bool conv7_igemm_supported(int C, int N, int kernel, int stride, int dilation, int padding,
                           int residual, const void* input, const void* output) {
  const int win_rows = CV_BM + (kernel - 1) * dilation;
  return stride == 1 && !residual && C % CV_CH == 0 && N == CV_NT && win_rows <= CV_WIN_ROWS_MAX &&
         padding >= 0 && smem_bytes(win_bytes_for(kernel, dilation), 2) <= CV_SMEM_MAX &&
         (reinterpret_cast<uintptr_t>(input) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(output) & 15u) == 0;
}

int conv7_igemm_launch(Ctx* c, const float* input, int batch, int T_in, int C,
                       const IroInt8DevWeight* w, int kernel, int dilation, int padding,
                       const float* bias, const float* scale, const int32_t* zero,
                       const float* inv, float* output, int T_out, cudaStream_t s) {
  const int win_rows = CV_BM + (kernel - 1) * dilation;
  const int wbytes = win_bytes_for(kernel, dilation);
  const int nstages = smem_bytes(wbytes, 3) <= CV_SMEM_MAX ? 3 : 2;
  const int smem = smem_bytes(wbytes, nstages);
  static bool attr_done[64] = {false};
  if (!attr_done[c->device]) {
    cudaError_t e = cudaFuncSetAttribute(conv7_igemm_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, CV_SMEM_MAX);
    if (e != cudaSuccess) return map_cuda(e);
    attr_done[c->device] = true;
  }
  CUtensorMap tin, tw, tout;
  {
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)T_in, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)C * 4, (cuuint64_t)C * 4 * T_in};
    cuuint32_t box[3] = {CV_CH, (cuuint32_t)win_rows, 1};
    int st = encode_tmap(&tin, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, input, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)w->K, (cuuint64_t)w->N};
    cuuint64_t strides[1] = {(cuuint64_t)w->ld};
    cuuint32_t box[2] = {CV_BK, 256};
    int st = encode_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->data, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B);
    if (st) return st;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)w->N, (cuuint64_t)T_out, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)w->N * 4, (cuuint64_t)w->N * 4 * T_out};
    cuuint32_t box[3] = {16, 32, 1};
    int st = encode_tmap(&tout, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, output, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B);
    if (st) return st;
  }
  ConvParams p{};
  p.batch = batch;
  p.T_in = T_in;
  p.T_out = T_out;
  p.C = C;
  p.N = w->N;
  p.kernel = kernel;
  p.dilation = dilation;
  p.padding = padding;
  p.tiles_t = cdiv(T_out, CV_BM);
  p.num_tiles = batch * p.tiles_t;
  p.n_chunks = C / CV_CH;
  p.stages_per_tile = p.n_chunks * kernel;
  p.win_rows = win_rows;
  p.win_bytes = wbytes;
  p.nstages = nstages;
  p.scale = scale;
  p.zero = zero;
  p.inv = inv;
  p.wcolsum = w->colsum;
  p.wscale = w->scale;
  p.bias = bias;
  p.err = c->err;
  p.limit_ns = kWaitLimitNs;
  const int grid = p.num_tiles < c->num_sms ? p.num_tiles : c->num_sms;
  conv7_igemm_kernel<<<grid, CV_THREADS, smem, s>>>(tin, tw, tout, p);
  return check_launch();
}

}  // namespace iro
