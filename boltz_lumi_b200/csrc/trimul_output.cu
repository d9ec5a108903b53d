// Output stage of the triangle multiplication in one kernel:
//
//   o_hat = bf16(LayerNorm_out(O))           O = the per-channel products, bf16 planes [128][n][ld]
//   y = bf16(bf16(o_hat p_out^T) * bf16(sigmoid(bf16(x_hat g_out^T))))
//   z += y  (fp32 residual)  or  out = y  (bf16)
//
// i.e. multiplication.py:124-137 (norm_out over the channel-first product,
// p_out, g_out on the saved input norm, the sigmoid gate) plus the
// Pairformer residual add.  Unfused: a channel-first LayerNorm pass writing
// o_hat, then a GEMM re-reading o_hat, x_hat and z.
//
// One persistent CTA per SM walks tiles of 128 consecutive j of one outer
// index i (tiles never straddle i, so every plane segment is contiguous and
// the 3-D z / x_hat maps clip rows past n).  Warps (14):
//   0     TMA: p_out / g_out weights once (resident), x_hat tiles per tile
//   1     TMEM allocation + MMA: D_p = o_hat p_out^T, D_g = x_hat g_out^T
//         (N = 128 each), double-buffered across tiles (4 x 128 columns)
//   2..5  epilogue: gate, bf16 y, TMA reduce-add into z (or store)
//   6..13 LayerNorm: two threads per pair row, each reading 64 of its 128
//         channels down the planes (16 lanes = 32 contiguous bytes per
//         channel); the halves' sums meet in one shuffle, and each thread
//         writes its 64 normalised channels (one K-block) into the K-major
//         A tile
#include "tc.cuh"

namespace bl {
namespace {

constexpr int kC = 128;
constexpr int kRows = 128;
constexpr int kLnWarps = 8;
constexpr int kThreads = (6 + kLnWarps) * 32;
constexpr int kKBlock = kRows * 64 * 2;  // 16 KB
constexpr int kTile = 2 * kKBlock;       // [128 rows][128 K] bf16 = 32 KB
constexpr int kWOff = 0;                 // W_p, W_g: 2 x 32 KB
constexpr int kAOff = kWOff + 2 * kTile;  // o_hat: 2 x 32 KB
constexpr int kXOff = kAOff + 2 * kTile;  // x_hat: 2 x 32 KB
constexpr int kStageOff = kXOff + 2 * kTile;  // 4 warps x 8 KB
constexpr int kParamOff = kStageOff + 4 * 8192;  // LN weight, bias: 2 x 128 fp32
constexpr int kBarOff = kParamOff + 2 * kC * 4;
constexpr int kSmemBytes = kBarOff + 256;
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct OutArgs {
  const __nv_bfloat16 *prod;
  int64_t plane;  // n * ld
  int64_t ld;
  int n, tiles, tiles_per_i;
  float eps;
  int residual;
  unsigned int *status;
};

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, unsigned int *status, unsigned code) {
  return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, status, code));
}
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float sigmoid_mufu(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    trimul_output_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                         const __grid_constant__ CUtensorMap map_out, const float *ln_w, const float *ln_b,
                         const OutArgs args) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (tc::smem_u32(smem) & 1023u) {  // uniform over the CTA: every thread leaves before any barrier
    if (threadIdx.x == 0) atomicCAS(args.status, 0u, 0x50Fu);
    return;
  }
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *w_full = bars;
  uint64_t *a_full = bars + 1, *a_empty = bars + 3;
  uint64_t *x_full = bars + 5, *x_empty = bars + 7;
  uint64_t *d_full = bars + 9, *d_empty = bars + 11;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 13);
  float *lnw_s = reinterpret_cast<float *>(smem + kParamOff), *lnb_s = lnw_s + kC;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tc::mbar_init(w_full, 1);
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&a_full[b], kLnWarps);
      tc::mbar_init(&a_empty[b], 1);
      tc::mbar_init(&x_full[b], 1);
      tc::mbar_init(&x_empty[b], 1);
      tc::mbar_init(&d_full[b], 1);
      tc::mbar_init(&d_empty[b], 4);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&map_w);
    tc::prefetch_tmap(&map_x);
    tc::prefetch_tmap(&map_out);
  }
  for (int c = threadIdx.x; c < kC; c += kThreads) {
    lnw_s[c] = ln_w ? ln_w[c] : 1.f;
    lnb_s[c] = ln_b ? ln_b[c] : 0.f;
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;  // buffer b: D_p at 256 b, D_g at 256 b + 128

  auto tile_of = [&](int tile, int &i, int &j0, int &valid) {
    i = tile / args.tiles_per_i;
    j0 = (tile - i * args.tiles_per_i) * kRows;
    valid = min(kRows, args.n - j0);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------------- TMA
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(w_full, 2 * kTile);
#pragma unroll
      for (int m = 0; m < 2; ++m)  // m = 0: p_out, 1: g_out (rows 128 m .. of the joint map)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint8_t *dst = smem + kWOff + m * kTile + kb * kKBlock;
          tc::tma_load_2d(dst, &map_w, w_full, kb * 64, 128 * m);
          tc::tma_load_2d(dst + kKBlock / 2, &map_w, w_full, kb * 64, 128 * m + 64);
        }
      int it = 0;
      for (int tile = blockIdx.x; tile < args.tiles; tile += gridDim.x, ++it) {
        int i, j0, valid;
        tile_of(tile, i, j0, valid);
        const int b = it & 1;
        if (!tc::mbar_wait(&x_empty[b], ((it >> 1) & 1) ^ 1, args.status, 0x501)) break;
        tc::mbar_arrive_expect_tx(&x_full[b], kTile);
        uint8_t *dst = smem + kXOff + b * kTile;
        tc::tma_load_3d(dst, &map_x, &x_full[b], 0, j0, i);
        tc::tma_load_3d(dst + kKBlock, &map_x, &x_full[b], 64, j0, i);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(kRows, 128, false, false);
      bool ok = tc::mbar_wait(w_full, 0, args.status, 0x502);
      const uint32_t wp = tc::smem_u32(smem + kWOff), wg = wp + kTile;
      int it = 0;
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++it) {
        const int b = it & 1;
        const uint32_t par = (it >> 1) & 1;
        if (!tc::mbar_wait(&d_empty[b], par ^ 1, args.status, 0x503) ||
            !tc::mbar_wait(&a_full[b], par, args.status, 0x504) ||
            !tc::mbar_wait(&x_full[b], par, args.status, 0x505))
          break;
        tc::tc_fence_after();
        const uint32_t a = tc::smem_u32(smem + kAOff + b * kTile), x = tc::smem_u32(smem + kXOff + b * kTile);
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * kKBlock + (kk & 3) * 32;
          tc::umma_f16_ss(tmem_base + 256 * b, tc::desc_sw128(a + koff, 16), tc::desc_sw128(wp + koff, 16), idesc,
                          kk != 0);
        }
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * kKBlock + (kk & 3) * 32;
          tc::umma_f16_ss(tmem_base + 256 * b + 128, tc::desc_sw128(x + koff, 16), tc::desc_sw128(wg + koff, 16),
                          idesc, kk != 0);
        }
        tc::umma_commit(&a_empty[b]);
        tc::umma_commit(&x_empty[b]);
        tc::umma_commit(&d_full[b]);
      }
    }
  } else if (warp < 6) {
    // ----------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    uint8_t *stage = smem + kStageOff + quarter * 8192;
    int it = 0, count = 0;
    for (int tile = blockIdx.x; tile < args.tiles; tile += gridDim.x, ++it) {
      int i, j0, valid;
      tile_of(tile, i, j0, valid);
      const int b = it & 1;
      if (!warp_wait(&d_full[b], (it >> 1) & 1, args.status, 0x506)) break;
      tc::tc_fence_after();
      const uint32_t tp = tc::tmem_addr(tmem_base, quarter * 32, 256 * b), tg = tp + 128;
      const bool live = quarter * 32 < valid;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {  // 32 output channels per step
        uint32_t p[32], g[32];
        tc::tmem_ld_32x32b_x32(tp + 32 * cc, p);
        tc::tmem_ld_32x32b_x32(tg + 32 * cc, g);
        tc::tmem_ld_wait_regs(p, g);
        if (cc == 3) {
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&d_empty[b]);
        }
        if (!live) continue;
        uint32_t y[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint32_t p2 = cvt_bf16x2(__uint_as_float(p[2 * e]), __uint_as_float(p[2 * e + 1]));
          const uint32_t g2 = cvt_bf16x2(__uint_as_float(g[2 * e]), __uint_as_float(g[2 * e + 1]));
          y[e] = mul_bf16x2(p2, cvt_bf16x2(sigmoid_mufu(bf16_lo(g2)), sigmoid_mufu(bf16_hi(g2))));
        }
        uint8_t *buf = stage + (count & 1) * 4096;
        if (lane == 0) tc::bulk_wait_read<1>();
        __syncwarp();
        if (args.residual) {  // [32 rows][32 fp32] box
#pragma unroll
          for (int e = 0; e < 8; ++e)
            *reinterpret_cast<float4 *>(buf + lane * 128 + ((e ^ (lane & 7)) << 4)) =
                make_float4(bf16_lo(y[2 * e]), bf16_hi(y[2 * e]), bf16_lo(y[2 * e + 1]), bf16_hi(y[2 * e + 1]));
        } else {  // [32 rows][32 bf16] half-row box (64-byte rows, 64-byte swizzle)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            *reinterpret_cast<uint4 *>(buf + lane * 64 + ((e ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(y[4 * e], y[4 * e + 1], y[4 * e + 2], y[4 * e + 3]);
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (args.residual) {
            tc::tma_reduce_add_3d(&map_out, buf, 32 * cc, j0 + 32 * quarter, i);
          } else {
            tc::tma_store_3d(&map_out, buf, 32 * cc, j0 + 32 * quarter, i);
          }
          tc::bulk_commit();
        }
        ++count;
      }
    }
    if (lane == 0) tc::bulk_wait<0>();
  } else {
    // ---------------------------------------------------------------- LayerNorm
    // Two threads per pair row: lanes 0-15 of LayerNorm warp w take rows
    // 16 w .. 16 w + 15 of the tile for channels 0..63, lanes 16-31 the same
    // rows for channels 64..127 (= K-block h of the A tile).  Channel c of
    // row r sits at prod[c * plane + i * ld + j0 + r].
    const int r = (warp - 6) * 16 + (lane & 15);
    const int h = lane >> 4;
    const uint32_t a_row = r * 128, a_sw = r & 7;
    int it = 0;
    for (int tile = blockIdx.x; tile < args.tiles; tile += gridDim.x, ++it) {
      int i, j0, valid;
      tile_of(tile, i, j0, valid);
      const int b = it & 1;
      const bool live = r < valid;
      // The rows of tile + 2 grid go to L2 now (one 256-byte plane segment per channel).
      if (tile + 2 * int(gridDim.x) < args.tiles) {
        int i2, j2, v2;
        tile_of(tile + 2 * gridDim.x, i2, j2, v2);
        const int span = min((v2 * 2 + 15) / 16 * 16, int(args.ld - j2) * 2);  // stays inside the plane row
        for (int c = (warp - 6) * 32 + lane; c < kC; c += kLnWarps * 32)
          tc::prefetch_l2_bulk(args.prod + c * args.plane + int64_t(i2) * args.ld + j2, uint32_t(span));
      }
      uint32_t v[32];  // channels 64 h + 2 q, 64 h + 2 q + 1 packed
      const __nv_bfloat16 *src = args.prod + int64_t(64 * h) * args.plane + int64_t(i) * args.ld + j0 + r;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const uint16_t lo = live ? __ldg(reinterpret_cast<const unsigned short *>(src + (2 * q) * args.plane)) : 0;
        const uint16_t hi = live ? __ldg(reinterpret_cast<const unsigned short *>(src + (2 * q + 1) * args.plane)) : 0;
        v[q] = uint32_t(lo) | (uint32_t(hi) << 16);
      }
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < 32; ++q) sum += bf16_lo(v[q]) + bf16_hi(v[q]);
      sum += __shfl_xor_sync(0xffffffffu, sum, 16);
      const float mean = sum * (1.f / 128.f);
      float sq = 0.f;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const float d0 = bf16_lo(v[q]) - mean, d1 = bf16_hi(v[q]) - mean;
        sq += d0 * d0;
        sq += d1 * d1;
      }
      sq += __shfl_xor_sync(0xffffffffu, sq, 16);
      const float rs = rsqrtf(sq * (1.f / 128.f) + args.eps);
      if (!warp_wait(&a_empty[b], ((it >> 1) & 1) ^ 1, args.status, 0x507)) break;
      uint8_t *abuf = smem + kAOff + b * kTile + h * kKBlock;
#pragma unroll
      for (int c16 = 0; c16 < 8; ++c16) {  // 8 channels per 16-byte chunk
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 64 * h + 8 * c16 + 2 * e;
          const uint32_t x2 = v[4 * c16 + e];
          o[e] = live ? cvt_bf16x2((bf16_lo(x2) - mean) * rs * lnw_s[c] + lnb_s[c],
                                   (bf16_hi(x2) - mean) * rs * lnw_s[c + 1] + lnb_s[c + 1])
                      : 0u;
        }
        *reinterpret_cast<uint4 *>(abuf + a_row + ((c16 ^ a_sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&a_full[b]);
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_trimul_output(const void *prod, int64_t n, int64_t n_outer, int64_t ld, const float *ln_weight,
                                const float *ln_bias, float eps, const void *xn, const void *w_out, float *z,
                                void *out, void *stream) {
  BL_REQUIRE(n >= 0 && n_outer >= 0 && n_outer <= n && n * n < (1ll << 31), "bl_trimul_output: bad n / n_outer");
  if (n == 0 || n_outer == 0) return BL_OK;
  BL_REQUIRE(prod && xn && w_out, "bl_trimul_output: null pointer");
  BL_REQUIRE((z != nullptr) != (out != nullptr), "bl_trimul_output: exactly one of z (residual) and out");
  BL_REQUIRE(ld >= n && ld % 8 == 0 && eps > 0.f, "bl_trimul_output: ld must be >= n and a multiple of 8");
  BL_REQUIRE(aligned_to(prod, 16), "bl_trimul_output: planes must be 16-byte aligned");
  BL_REQUIRE(aligned_to(xn, 16) && aligned_to(w_out, 16) && aligned_to(z ? static_cast<const void *>(z) : out, 16),
             "bl_trimul_output: xn, w_out and the output must be 16-byte aligned");
  CUtensorMap map_w, map_x, map_out;
  {
    uint64_t dims[2] = {uint64_t(kC), 256};
    uint64_t strides[1] = {uint64_t(kC) * 2};
    uint32_t box[2] = {64, 64};
    BL_REQUIRE(encode_tmap(&map_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_out, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_trimul_output: cannot encode the weight map");
  }
  {
    uint64_t dims[3] = {uint64_t(kC), uint64_t(n), uint64_t(n_outer)};
    uint64_t strides[2] = {uint64_t(kC) * 2, uint64_t(n) * kC * 2};
    uint32_t box[3] = {64, 128, 1};
    BL_REQUIRE(encode_tmap(&map_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, xn, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_trimul_output: cannot encode the x_hat map");
  }
  if (z) {
    uint64_t dims[3] = {uint64_t(kC), uint64_t(n), uint64_t(n_outer)};
    uint64_t strides[2] = {uint64_t(kC) * 4, uint64_t(n) * kC * 4};
    uint32_t box[3] = {32, 32, 1};
    BL_REQUIRE(encode_tmap(&map_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, z, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_trimul_output: cannot encode the z map");
  } else {
    uint64_t dims[3] = {uint64_t(kC), uint64_t(n), uint64_t(n_outer)};
    uint64_t strides[2] = {uint64_t(kC) * 2, uint64_t(n) * kC * 2};
    uint32_t box[3] = {32, 32, 1};
    BL_REQUIRE(encode_tmap(&map_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_64B),
               "bl_trimul_output: cannot encode the output map");
  }
  OutArgs a{};
  a.prod = static_cast<const __nv_bfloat16 *>(prod);
  a.plane = n_outer * ld, a.ld = ld, a.n = int(n);
  a.tiles_per_i = int((n + kRows - 1) / kRows);
  a.tiles = int(n_outer) * a.tiles_per_i;
  a.eps = eps;
  a.residual = z != nullptr;
  a.status = device_status_ptr();
  BL_REQUIRE(a.status, "bl_trimul_output: device status word unavailable");
  auto kernel = trimul_output_kernel;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), kSmemBytes));
  const int grid = a.tiles < num_sms() ? a.tiles : num_sms();
  kernel<<<grid, kThreads, kSmemBytes, as_stream(stream)>>>(map_w, map_x, map_out, ln_weight, ln_bias, a);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
