// Pair transition in one kernel on tcgen05 tensor cores:
//
//   x_hat = bf16(LayerNorm(x))                       (fp32 statistics)
//   a = bf16(x_hat fc1^T), b = bf16(x_hat fc2^T)     (128 -> 512 each)
//   u = bf16(bf16(silu(a)) * b)
//   y = bf16(u fc3^T)                                (512 -> 128)
//   z += y   (fp32 residual)   or   out = y   (bf16)
//
// which is upstream Transition.forward under bf16 autocast
// (pair_transition.py:8-28 with the pair_silu_mul kernel of
// kernels/pair_hip.cu:42-64).  Unfused this is four HBM passes over hidden
// tensors of [rows][512] bf16; here the hidden activations never leave the SM.
//
// One persistent CTA per SM walks 128-row tiles.  For every tile the hidden
// dimension is processed in eight chunks of 64 units:
//   MMA1(h):  D1[h % 2] = x_hat . [fc1; fc2](h)^T     N = 128 (64 fc1 | 64 fc2), K = 128
//   SwiGLU:   u(h) = bf16(silu(a)) * b -> shared memory as the K-major A
//             operand of the next MMA (128-byte swizzle)
//   MMA2(h):  D2 += u(h) . fc3(:, h)^T                 N = 128, K = 64
// TMEM: D1 double-buffered (2 x 128 columns) so MMA1(h+1) runs while the
// SwiGLU warps work on chunk h, D2 double-buffered across tiles (2 x 128).
// fc1|fc2 and fc3 chunks stream from L2 through two 2-stage TMA rings (the
// weights are 384 KB, too large to stay resident); the fc1|fc2 loads run one
// chunk ahead of the fc3 loads, so a slot freed by MMA1 is refilled without
// waiting for the later MMA2.  The residual update is a TMA reduce-add of the
// fp32 y tile into z, so z is never loaded by the SM for the residual.
//
// Warps (15): 0 TMA producer, 1 TMEM allocation + MMA1 issue, 2..9 SwiGLU and
// output (TMEM lane quarter = warp % 4; warps 2..5 take hidden units 0..31
// of each chunk and output columns 0..63, warps 6..9 the other halves),
// 10..13 LayerNorm (32 rows each, next rows in flight while normalising),
// 14 MMA2 issue.  With MMA1 and MMA2 on their own issuing threads, MMA1 of
// chunk h + 1 no longer waits behind MMA2 of chunk h - 1 (which waits for the
// SwiGLU of chunk h - 1): measured at N = 512 with z updated in place,
// 156.5 -> 149.4 us, bitwise-identical output.
#include "tc.cuh"

namespace bl {
namespace {

constexpr int kC = 128;       // pair channels
constexpr int kHidden = 512;  // transition hidden width
constexpr int kRows = 128;
constexpr int kChunkUnits = 64;
constexpr int kChunks = kHidden / kChunkUnits;  // 8
constexpr int kEpiWarps = 8;
constexpr int kLnWarps = 4;
constexpr int kFirstEpiWarp = 2;
constexpr int kFirstLnWarp = kFirstEpiWarp + kEpiWarps;
constexpr int kMma2Warp = kFirstLnWarp + kLnWarps;  // fc3 MMA issue
constexpr int kThreads = (kMma2Warp + 1) * 32;

constexpr int kKBlock = kRows * 64 * 2;  // [128 rows][64 K] bf16, 128-byte swizzle: 16 KB
constexpr int kABytes = 2 * kKBlock;     // x_hat tile, K = 128
constexpr int kAOff = 0;                          // 2 x 32 KB
constexpr int kUOff = kAOff + 2 * kABytes;        // 2 x 16 KB  SwiGLU chunk (K = 64)
constexpr int kW12Off = kUOff + 2 * kKBlock;      // 2 x 32 KB  [fc1 rows 64 h..; fc2 rows 64 h..][128 K]
constexpr int kW3Off = kW12Off + 2 * kABytes;     // 2 x 16 KB  fc3[:, 64 h .. 64 h + 64]
constexpr int kStageOff = kW3Off + 2 * kKBlock;   // 8 warps x 4 KB output staging
constexpr int kBarOff = kStageOff + kEpiWarps * 4096;
constexpr int kSmemBytes = kBarOff + 256;
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct TransitionArgs {
  const float *x;
  int64_t rows;
  int tiles;
  const float *ln_w, *ln_b;
  float eps;
  int residual;  // 1: z += y (TMA reduce-add), 0: out = y (bf16 TMA store)
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
// silu(a) = a / (1 + 2^(-a log2 e)) with the MUFU exponent and reciprocal.
// Large negative a gives 2^(+big) = inf, rcp(inf) = 0 and silu = -0.
__device__ __forceinline__ float silu_mufu(float a) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(a * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return a * r;
}

__global__ void __launch_bounds__(kThreads, 1)
    pair_transition_kernel(const __grid_constant__ CUtensorMap map_w12, const __grid_constant__ CUtensorMap map_w3,
                           const __grid_constant__ CUtensorMap map_out, const TransitionArgs args) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (tc::smem_u32(smem) & 1023u) {  // uniform over the CTA: every thread leaves before any barrier
    if (threadIdx.x == 0) atomicCAS(args.status, 0u, 0x40Fu);
    return;
  }
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *a_full = bars + 0, *a_empty = bars + 2;
  uint64_t *w12_full = bars + 4, *w12_empty = bars + 6;
  uint64_t *w3_full = bars + 8, *w3_empty = bars + 10;
  uint64_t *d1_full = bars + 12, *d1_empty = bars + 14;
  uint64_t *u_full = bars + 16, *u_empty = bars + 18;
  uint64_t *d2_full = bars + 20, *d2_empty = bars + 22;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 24);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&a_full[b], kLnWarps);
      tc::mbar_init(&a_empty[b], 1);
      tc::mbar_init(&w12_full[b], 1);
      tc::mbar_init(&w12_empty[b], 1);
      tc::mbar_init(&w3_full[b], 1);
      tc::mbar_init(&w3_empty[b], 1);
      tc::mbar_init(&d1_full[b], 1);
      tc::mbar_init(&d1_empty[b], kEpiWarps);
      tc::mbar_init(&u_full[b], kEpiWarps);
      tc::mbar_init(&u_empty[b], 1);
      tc::mbar_init(&d2_full[b], 1);
      tc::mbar_init(&d2_empty[b], kEpiWarps);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&map_w12);
    tc::prefetch_tmap(&map_w3);
    tc::prefetch_tmap(&map_out);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;  // D1[b] at 128 b, D2[b] at 256 + 128 b

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // fc1|fc2 chunks run one chunk ahead of the fc3 chunks: chunk g + 1's
    // fc1|fc2 slot frees when MMA1(g - 1) completes, well before MMA2(g - 2)
    // frees chunk g's fc3 slot, so its load is not held behind that wait.
    if (lane == 0) {
      const int total = ((args.tiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x)) * kChunks;
      auto load_w12 = [&](int g) -> bool {
        const int b = g & 1, h = g % kChunks;
        if (!tc::mbar_wait(&w12_empty[b], ((g >> 1) & 1) ^ 1, args.status, 0x401)) return false;
        uint8_t *w12 = smem + kW12Off + b * kABytes;
        tc::mbar_arrive_expect_tx(&w12_full[b], kABytes);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          tc::tma_load_2d(w12 + kb * kKBlock, &map_w12, &w12_full[b], kb * 64, kChunkUnits * h);
          tc::tma_load_2d(w12 + kb * kKBlock + kKBlock / 2, &map_w12, &w12_full[b], kb * 64,
                          kHidden + kChunkUnits * h);
        }
        return true;
      };
      auto load_w3 = [&](int g) -> bool {
        const int b = g & 1, h = g % kChunks;
        if (!tc::mbar_wait(&w3_empty[b], ((g >> 1) & 1) ^ 1, args.status, 0x402)) return false;
        tc::mbar_arrive_expect_tx(&w3_full[b], kKBlock);
        tc::tma_load_2d(smem + kW3Off + b * kKBlock, &map_w3, &w3_full[b], kChunkUnits * h, 0);
        return true;
      };
      bool ok = total == 0 || load_w12(0);
      for (int g = 0; ok && g < total; ++g) {
        if (g + 1 < total && !(ok = load_w12(g + 1))) break;
        ok = load_w3(g);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA1 issue (fc1|fc2)
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(kRows, 128, false, false);
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++it) {
        const int ab = it & 1;
        if (!tc::mbar_wait(&a_full[ab], (it >> 1) & 1, args.status, 0x406)) break;
        const uint32_t a_addr = tc::smem_u32(smem + kAOff + ab * kABytes);
        for (int h = 0; h < kChunks && ok; ++h) {
          const int g = it * kChunks + h, b = g & 1;
          const uint32_t par = (g >> 1) & 1;
          if (!tc::mbar_wait(&w12_full[b], par, args.status, 0x407) ||
              !tc::mbar_wait(&d1_empty[b], par ^ 1, args.status, 0x408)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t w_addr = tc::smem_u32(smem + kW12Off + b * kABytes);
#pragma unroll
          for (int kk = 0; kk < kC / 16; ++kk) {
            const uint32_t koff = (kk >> 2) * kKBlock + (kk & 3) * 32;
            tc::umma_f16_ss(tmem_base + 128 * b, tc::desc_sw128(a_addr + koff, 16),
                            tc::desc_sw128(w_addr + koff, 16), idesc, kk != 0);
          }
          tc::umma_commit(&w12_empty[b]);
          tc::umma_commit(&d1_full[b]);
          if (h == kChunks - 1) tc::umma_commit(&a_empty[ab]);
        }
      }
    }
  } else if (warp == kMma2Warp) {
    // ------------------------------------------------------------ MMA2 issue (fc3)
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(kRows, 128, false, false);
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++it) {
        const int db = it & 1;
        if (!tc::mbar_wait(&d2_empty[db], ((it >> 1) & 1) ^ 1, args.status, 0x403)) break;
        for (int h = 0; h < kChunks; ++h) {
          const int g = it * kChunks + h, b = g & 1;
          const uint32_t par = (g >> 1) & 1;
          if (!tc::mbar_wait(&u_full[b], par, args.status, 0x404) ||
              !tc::mbar_wait(&w3_full[b], par, args.status, 0x405)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t u_addr = tc::smem_u32(smem + kUOff + b * kKBlock);
          const uint32_t w_addr = tc::smem_u32(smem + kW3Off + b * kKBlock);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::umma_f16_ss(tmem_base + 256 + 128 * db, tc::desc_sw128(u_addr + kk * 32, 16),
                            tc::desc_sw128(w_addr + kk * 32, 16), idesc, (h | kk) != 0);
          tc::umma_commit(&u_empty[b]);
          tc::umma_commit(&w3_empty[b]);
        }
        if (ok) tc::umma_commit(&d2_full[db]);
      }
    }
  } else if (warp < kFirstLnWarp) {
    // ------------------------------------------------------- SwiGLU and output
    const int quarter = warp & 3, half = (warp - kFirstEpiWarp) >> 2;
    const int row = quarter * 32 + lane;  // TMEM lane = tile row
    uint8_t *stage = smem + kStageOff + (warp - kFirstEpiWarp) * 4096;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++it) {
      const int64_t row0 = int64_t(tile) * kRows;
      for (int h = 0; h < kChunks; ++h) {
        const int g = it * kChunks + h, b = g & 1;
        const uint32_t par = (g >> 1) & 1;
        if (!warp_wait(&d1_full[b], par, args.status, 0x409)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d1 = tc::tmem_addr(tmem_base, quarter * 32, 128 * b + 32 * half);
        uint32_t fa[32], fb[32];
        tc::tmem_ld_32x32b_x32(d1, fa);       // fc1 units 64 h + 32 half + 0..31
        tc::tmem_ld_32x32b_x32(d1 + 64, fb);  // fc2, same units
        tc::tmem_ld_wait_regs(fa, fb);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&d1_empty[b]);
        uint32_t u[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint32_t a2 = cvt_bf16x2(__uint_as_float(fa[2 * e]), __uint_as_float(fa[2 * e + 1]));
          const uint32_t b2 = cvt_bf16x2(__uint_as_float(fb[2 * e]), __uint_as_float(fb[2 * e + 1]));
          u[e] = mul_bf16x2(cvt_bf16x2(silu_mufu(bf16_lo(a2)), silu_mufu(bf16_hi(a2))), b2);
        }
        if (!warp_wait(&u_empty[b], par ^ 1, args.status, 0x40A)) {
          ok = false;
          break;
        }
        // K-major [128 rows][64 K] operand: this warp's 32 units are 16-byte
        // chunks 4 half .. 4 half + 3 of its rows.
        uint8_t *ub = smem + kUOff + b * kKBlock + row * 128;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          *reinterpret_cast<uint4 *>(ub + (((4 * half + e) ^ (row & 7)) << 4)) =
              make_uint4(u[4 * e], u[4 * e + 1], u[4 * e + 2], u[4 * e + 3]);
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&u_full[b]);
      }
      if (!ok) break;
      // Output columns 64 half .. 64 half + 63 of this warp's 32 rows.
      const int db = it & 1;
      if (!warp_wait(&d2_full[db], (it >> 1) & 1, args.status, 0x40B)) break;
      tc::tc_fence_after();
      const uint32_t d2 = tc::tmem_addr(tmem_base, quarter * 32, 256 + 128 * db + 64 * half);
      uint32_t y0[32], y1[32];
      tc::tmem_ld_32x32b_x32(d2, y0);
      tc::tmem_ld_32x32b_x32(d2 + 32, y1);
      tc::tmem_ld_wait_regs(y0, y1);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&d2_empty[db]);
      const bool live = row0 + quarter * 32 < args.rows;
      if (args.residual) {
        // Two [32 rows][32 fp32] boxes; y rounded to bf16 first (fc3's output).
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          const uint32_t *y = bx ? y1 : y0;
          if (lane == 0) tc::bulk_wait_read<0>();
          __syncwarp();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t p0 = cvt_bf16x2(__uint_as_float(y[4 * e]), __uint_as_float(y[4 * e + 1]));
            const uint32_t p1 = cvt_bf16x2(__uint_as_float(y[4 * e + 2]), __uint_as_float(y[4 * e + 3]));
            *reinterpret_cast<float4 *>(stage + lane * 128 + ((e ^ (lane & 7)) << 4)) =
                make_float4(bf16_lo(p0), bf16_hi(p0), bf16_lo(p1), bf16_hi(p1));
          }
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && live) {
            tc::tma_reduce_add_2d(&map_out, stage, 64 * half + 32 * bx, int(row0) + quarter * 32);
            tc::bulk_commit();
          }
        }
      } else {
        // One [32 rows][64 bf16] box.
        if (lane == 0) tc::bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t *y = e < 4 ? y0 + 8 * e : y1 + 8 * (e - 4);
          *reinterpret_cast<uint4 *>(stage + lane * 128 + ((e ^ (lane & 7)) << 4)) =
              make_uint4(cvt_bf16x2(__uint_as_float(y[0]), __uint_as_float(y[1])),
                         cvt_bf16x2(__uint_as_float(y[2]), __uint_as_float(y[3])),
                         cvt_bf16x2(__uint_as_float(y[4]), __uint_as_float(y[5])),
                         cvt_bf16x2(__uint_as_float(y[6]), __uint_as_float(y[7])));
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && live) {
          tc::tma_store_2d(&map_out, stage, 64 * half, int(row0) + quarter * 32);
          tc::bulk_commit();
        }
      }
    }
    if (lane == 0) tc::bulk_wait<0>();
  } else if (warp < kMma2Warp) {
    // --------------------------------------------------------------- LayerNorm
    const int lw = warp - kFirstLnWarp;
    float lnw[4], lnb[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      lnw[e] = args.ln_w ? args.ln_w[lane * 4 + e] : 1.f;
      lnb[e] = args.ln_b ? args.ln_b[lane * 4 + e] : 0.f;
    }
    const uint32_t a_lane_off = (lane >> 4) * kKBlock + (lane & 1) * 8;
    const uint32_t a_chunk = (lane & 15) >> 1;
    const int row_lo = lw * 32;
    auto valid_rows = [&](int tile) -> int {
      const int64_t left = args.rows - int64_t(tile) * kRows;
      return left < kRows ? int(left) : kRows;
    };
    auto load_rows = [&](int tile, int rbase, float4 (&v)[8]) {
      const int valid = valid_rows(tile);
#pragma unroll
      for (int r = 0; r < 8; ++r)
        v[r] = rbase + r < valid
                   ? __ldg(reinterpret_cast<const float4 *>(args.x + (int64_t(tile) * kRows + rbase + r) * kC) + lane)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    // fp32 LayerNorm of 8 rows into the A tile: mean, mean of squared
    // deviations, rstd = rsqrt(var + eps), bf16((x - mean) * rstd * w + b).
    auto normalise = [&](const float4 (&v)[8], int valid, int rbase, uint8_t *abuf) {
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        float mean[4], var[4];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const float4 x = v[4 * g + rr];
          mean[rr] = (x.x + x.y) + (x.z + x.w);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) mean[rr] += __shfl_xor_sync(0xffffffffu, mean[rr], o);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const float4 x = v[4 * g + rr];
          mean[rr] *= 1.f / 128.f;
          const float d0 = x.x - mean[rr], d1 = x.y - mean[rr], d2 = x.z - mean[rr], d3 = x.w - mean[rr];
          float sq = d0 * d0;
          sq += d1 * d1;
          sq += d2 * d2;
          sq += d3 * d3;
          var[rr] = sq;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) var[rr] += __shfl_xor_sync(0xffffffffu, var[rr], o);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const int r = 4 * g + rr, tr = rbase + r;
          const float4 x = v[r];
          const float rs = rsqrtf(var[rr] * (1.f / 128.f) + args.eps);
          const uint2 y = tr < valid ? make_uint2(cvt_bf16x2((x.x - mean[rr]) * rs * lnw[0] + lnb[0],
                                                             (x.y - mean[rr]) * rs * lnw[1] + lnb[1]),
                                                  cvt_bf16x2((x.z - mean[rr]) * rs * lnw[2] + lnb[2],
                                                             (x.w - mean[rr]) * rs * lnw[3] + lnb[3]))
                                     : make_uint2(0u, 0u);
          *reinterpret_cast<uint2 *>(abuf + a_lane_off + tr * 128 + ((a_chunk ^ (tr & 7)) << 4)) = y;
        }
      }
    };
    float4 va[8], vb[8];
    int tile = blockIdx.x, it = 0;
    if (tile < args.tiles) load_rows(tile, row_lo, va);
    for (; tile < args.tiles; tile += gridDim.x, ++it) {
      const int ab = it & 1, valid = valid_rows(tile);
      uint8_t *abuf = smem + kAOff + ab * kABytes;
      const int next = tile + gridDim.x;
      if (lane == 0 && tile + 2 * int(gridDim.x) < args.tiles) {
        const int ahead = tile + 2 * gridDim.x;
        const int rows_ahead = min(32, valid_rows(ahead) - row_lo);
        if (rows_ahead > 0)
          tc::prefetch_l2_bulk(args.x + (int64_t(ahead) * kRows + row_lo) * kC, uint32_t(rows_ahead) * kC * 4);
      }
      load_rows(tile, row_lo + 8, vb);
      if (!warp_wait(&a_empty[ab], ((it >> 1) & 1) ^ 1, args.status, 0x40C)) break;
      normalise(va, valid, row_lo, abuf);
      load_rows(tile, row_lo + 16, va);
      normalise(vb, valid, row_lo + 8, abuf);
      load_rows(tile, row_lo + 24, vb);
      normalise(va, valid, row_lo + 16, abuf);
      if (next < args.tiles) load_rows(next, row_lo, va);
      normalise(vb, valid, row_lo + 24, abuf);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&a_full[ab]);
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

extern "C" int bl_pair_transition(const float *x, int64_t rows, const float *ln_weight, const float *ln_bias,
                                  float eps, const void *w12, const void *w3, float *z, void *out, void *stream) {
  BL_REQUIRE(rows >= 0 && rows < (1ll << 31) - kRows, "bl_pair_transition: bad row count");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(eps > 0.f, "bl_pair_transition: eps must be positive");
  BL_REQUIRE(x && w12 && w3, "bl_pair_transition: null pointer");
  BL_REQUIRE((z != nullptr) != (out != nullptr), "bl_pair_transition: exactly one of z (residual) and out");
  BL_REQUIRE(aligned_to(x, 16) && aligned_to(w12, 16) && aligned_to(w3, 16) &&
                 aligned_to(z ? static_cast<const void *>(z) : out, 16),
             "bl_pair_transition: pointers must be 16-byte aligned");
  CUtensorMap map_w12, map_w3, map_out;
  {
    uint64_t dims[2] = {uint64_t(kC), uint64_t(2 * kHidden)};
    uint64_t strides[1] = {uint64_t(kC) * 2};
    uint32_t box[2] = {64, 64};
    BL_REQUIRE(encode_tmap(&map_w12, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w12, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_pair_transition: cannot encode the fc1|fc2 map");
  }
  {
    uint64_t dims[2] = {uint64_t(kHidden), uint64_t(kC)};
    uint64_t strides[1] = {uint64_t(kHidden) * 2};
    uint32_t box[2] = {64, 128};
    BL_REQUIRE(encode_tmap(&map_w3, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w3, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_pair_transition: cannot encode the fc3 map");
  }
  if (z) {
    uint64_t dims[2] = {uint64_t(kC), uint64_t(rows)};
    uint64_t strides[1] = {uint64_t(kC) * 4};
    uint32_t box[2] = {32, 32};
    BL_REQUIRE(encode_tmap(&map_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, z, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_pair_transition: cannot encode the z map");
  } else {
    uint64_t dims[2] = {uint64_t(kC), uint64_t(rows)};
    uint64_t strides[1] = {uint64_t(kC) * 2};
    uint32_t box[2] = {64, 32};
    BL_REQUIRE(encode_tmap(&map_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_pair_transition: cannot encode the output map");
  }
  TransitionArgs a{};
  a.x = x, a.rows = rows, a.tiles = int((rows + kRows - 1) / kRows);
  a.ln_w = ln_weight, a.ln_b = ln_bias, a.eps = eps;
  a.residual = z != nullptr;
  a.status = device_status_ptr();
  BL_REQUIRE(a.status, "bl_pair_transition: device status word unavailable");
  auto kernel = pair_transition_kernel;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), kSmemBytes));
  const int grid = a.tiles < num_sms() ? a.tiles : num_sms();
  kernel<<<grid, kThreads, kSmemBytes, as_stream(stream)>>>(map_w12, map_w3, map_out, a);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
