// LayerNorm-prologue input projections of the pair ops on tcgen05 tensor cores.
//
// Both triangle ops open with  x_hat = LN(z)  followed by a 128 -> 512 bf16
// projection of x_hat.  Unfused that is three HBM passes (LN writes x_hat,
// the GEMM re-reads it and writes the 512-wide projection, a pack pass
// re-reads that); here one persistent kernel reads the fp32 pair rows once:
//
//   attention (triangle.py:32-104 / upstream TriangleAttention.forward):
//     proj[r] = bf16(x_hat[r] W^T + bias)       W = [linear_q; linear_k; linear_v; linear_g]
//     written as q_s | k | v | s_g with q_s = bf16(q * q_scale) (q / sqrt(d),
//     _prep_qkv) and s_g = bf16(sigmoid(g)) (upstream _wrap_up's gate)
//     tri_bias[h][q][k] = bf16(x_hat[(q, k)] . w_heads[h])   (transposed planes for the ending node)
//   triangle multiplication (multiplication.py:48-120, multiplication_gate_hip.cu:16-20,41-58):
//     a|b[c][i][k] = bf16(bf16(p_c * bf16(sigmoid(g_c))) * mask[i, k])   p = p_in(x_hat), g = g_in(x_hat)
//     x_hat rows stored in bf16 for the output gate g_out(x_hat)
//
// CTA (one per SM, persistent over 128-row tiles), 18 warps (96 registers
// each: some SM sub-partition holds five of them):
//   warp 0       TMA: the [512][128] bf16 weight, once per CTA (resident, 128 KB)
//   warp 1       TMEM allocation (512 columns) + tcgen05.mma issue: four chunks
//                of 128 output columns, chunk j into TMEM columns [128 j, 128 j + 128)
//   warps 2..9   epilogue, two warps per TMEM lane quarter (warp % 4), each
//                taking 64 of a chunk's 128 columns: tcgen05.ld, release the
//                columns, apply the op's epilogue, stage a 32 x 64 block in
//                shared memory and TMA-store it.  Attention computes
//                D = X W^T (lane = pair row, the natural [row][512] output);
//                the triangle multiplication computes D = W X^T (lane =
//                channel, columns = pairs), so each thread's values already
//                run along its channel plane and p / g of a channel share a lane
//   warps 10..17 LayerNorm: each warp normalises 16 rows of the tile in fp32
//                (four batches of 4 rows, the next batch's loads in flight)
//                and writes the bf16 result straight into the 128-byte-swizzled
//                K-major A tile the MMA reads (double-buffered), plus the
//                per-row side outputs (bias heads / x_hat rows); each warp
//                also asks L2 to prefetch its rows two tiles ahead
// The LN of tile t+1, the MMAs of tile t and the epilogue of tile t-1 overlap;
// every wait is bounded.
#include "tc.cuh"

namespace bl {
namespace {

enum ProjectionKind { PROJ_ATTENTION = 0, PROJ_TRIMUL = 1 };

constexpr int kC = 128;         // pair channels (K of the projection)
constexpr int kOut = 512;       // projection width
constexpr int kRows = 128;      // rows per tile (= TMEM lanes)
constexpr int kChunks = 4;      // 128-column output chunks
constexpr int kLnWarps = 8;
constexpr int kLnRowsPerWarp = kRows / kLnWarps;  // 16, in two batches of 8
constexpr int kFirstEpiWarp = 2;
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter: columns 0-63 / 64-127 of every chunk
constexpr int kFirstLnWarp = kFirstEpiWarp + kEpiWarps;
constexpr int kThreads = (kFirstLnWarp + kLnWarps) * 32;  // 18 warps: <= 112 registers per thread

constexpr int kWBytes = kOut * kC * 2;        // 128 KB: chunk j = [128 rows][128 K] as two SW128 K-blocks
constexpr int kWChunkBytes = kRows * kC * 2;  // 32 KB
constexpr int kKBlockBytes = kRows * 64 * 2;  // 16 KB: [128 rows][64 K] bf16, 128-byte swizzle
constexpr int kABytes = kRows * kC * 2;       // 32 KB
constexpr int kStagePerWarp = 4096;  // one staged 32 x 64 block per epilogue warp
constexpr int kWOff = 0;
constexpr int kAOff = kWOff + kWBytes;
constexpr int kStageOff = kAOff + 2 * kABytes;
constexpr int kBiasOff = kStageOff + kEpiWarps * kStagePerWarp;  // fp32 [512] projection bias
constexpr int kBarOff = kBiasOff + kOut * 4;
// The dynamic shared window starts 1024-byte aligned (checked at run time:
// the kernel reports an error instead of running misaligned), so no slack.
constexpr int kSmemBytes = kBarOff + 256;
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct ProjArgs {
  const float *x;  // [rows][128] fp32
  int64_t rows;
  int n;
  int tiles, tiles_per_i;
  const float *ln_w, *ln_b;
  float eps;
  // attention
  const float *bias;  // [512] fp32 or null
  float q_scale;      // applied to columns 0..127 (q)
  const __nv_bfloat16 *w_heads;  // [4][128]
  int transpose;
  __nv_bfloat16 *bias_planes;  // head h at bias_planes + h * bias_hs, rows of bias_ld
  int64_t bias_ld, bias_hs;
  // triangle multiplication
  const float *mask;  // [rows]
  __nv_bfloat16 *xn;  // [rows][128]
  unsigned int *status;
};

struct TileRows {
  int64_t row0;  // first pair row of the tile
  int valid;     // rows of the tile that exist
  int i, k0;     // triangle multiplication: outer index and first inner index
};

// Attention tiles are 128 consecutive pair rows.  Triangle-multiplication
// tiles never straddle an outer index i, so each tile is one contiguous run
// of every channel plane ([c][i][k0 .. k0 + 127]).
template <int KIND> __device__ __forceinline__ TileRows tile_rows(const ProjArgs &a, int tile) {
  TileRows t;
  if constexpr (KIND == PROJ_ATTENTION) {
    t.row0 = int64_t(tile) * kRows;
    const int64_t left = a.rows - t.row0;
    t.valid = left < kRows ? int(left) : kRows;
    t.i = 0, t.k0 = 0;
  } else {
    t.i = tile / a.tiles_per_i;
    t.k0 = (tile - t.i * a.tiles_per_i) * kRows;
    t.row0 = int64_t(t.i) * a.n + t.k0;
    const int left = a.n - t.k0;
    t.valid = left < kRows ? left : kRows;
  }
  return t;
}

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
// sigmoid(x) = 1 / (1 + 2^(-x log2 e)) with the MUFU exponent and reciprocal
// (relative error a few fp32 ulp; the result is rounded to bf16).
__device__ __forceinline__ float sigmoid_mufu(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return r;
}

// One staged row of 64 projection columns (two 32-column TMEM loads) with the
// bias added and rounded to bf16; KIND 1 then scales by q_scale and rounds,
// KIND 2 applies the sigmoid and rounds.
template <int KIND>
__device__ __forceinline__ void stage_row(uint8_t *buf, int lane, const uint32_t (&r0)[32], const uint32_t (&r1)[32],
                                          const float4 *bq, float q_scale) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t *r = e < 4 ? r0 + 8 * e : r1 + 8 * (e - 4);
    const float4 b0 = bq[2 * e], b1 = bq[2 * e + 1];
    uint32_t w[4] = {cvt_bf16x2(__uint_as_float(r[0]) + b0.x, __uint_as_float(r[1]) + b0.y),
                     cvt_bf16x2(__uint_as_float(r[2]) + b0.z, __uint_as_float(r[3]) + b0.w),
                     cvt_bf16x2(__uint_as_float(r[4]) + b1.x, __uint_as_float(r[5]) + b1.y),
                     cvt_bf16x2(__uint_as_float(r[6]) + b1.z, __uint_as_float(r[7]) + b1.w)};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (KIND == 1) w[k] = cvt_bf16x2(bf16_lo(w[k]) * q_scale, bf16_hi(w[k]) * q_scale);
      if constexpr (KIND == 2) w[k] = cvt_bf16x2(sigmoid_mufu(bf16_lo(w[k])), sigmoid_mufu(bf16_hi(w[k])));
    }
    *reinterpret_cast<uint4 *>(buf + lane * 128 + ((e ^ (lane & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Warp-level bf16 MMA (m16n8k16, fp32 accumulate) and its A-fragment load.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&a)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    pair_projection_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_out,
                           const ProjArgs args) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (tc::smem_u32(smem) & 1023u) {  // uniform over the CTA: every thread leaves before any barrier
    if (threadIdx.x == 0) atomicCAS(args.status, 0u, 0x30Fu);
    return;
  }
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *w_full = bars;
  uint64_t *a_full = bars + 1;   // [2] A tile written (8 LN warps arrive)
  uint64_t *a_empty = bars + 3;  // [2] MMAs reading A done
  uint64_t *c_full = bars + 5;   // [4] chunk accumulated in TMEM
  uint64_t *c_empty = bars + 9;  // [4] chunk read out of TMEM (8 epilogue warps arrive)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 13);
  float *bias_s = reinterpret_cast<float *>(smem + kBiasOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tc::mbar_init(w_full, 1);
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&a_full[b], kLnWarps);
      tc::mbar_init(&a_empty[b], 1);
    }
    for (int j = 0; j < kChunks; ++j) {
      tc::mbar_init(&c_full[j], 1);
      tc::mbar_init(&c_empty[j], kEpiWarps);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&map_w);
    tc::prefetch_tmap(&map_out);
  }
  if constexpr (KIND == PROJ_ATTENTION) {
    for (int c = threadIdx.x; c < kOut; c += kThreads) bias_s[c] = args.bias ? args.bias[c] : 0.f;
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // Resident weight, four chunks of 128 W rows.  Attention: W rows in order
    // (q, k, v, g).  Triangle multiplication: p_a, g_a, p_b, g_b, i.e. chunk j
    // = W rows [256 (j % 2) + 128 (j / 2), + 128).
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(w_full, kWBytes);
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint8_t *dst = smem + kWOff + j * kWChunkBytes + kb * kKBlockBytes;
          const int r0 = KIND == PROJ_ATTENTION ? 128 * j : 256 * (j & 1) + 128 * (j >> 1);
          tc::tma_load_2d(dst, &map_w, w_full, kb * 64, r0);
          tc::tma_load_2d(dst + kKBlockBytes / 2, &map_w, w_full, kb * 64, r0 + 64);
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(kRows, 128, false, false);
      bool ok = tc::mbar_wait(w_full, 0, args.status, 0x301);
      const uint32_t w_addr = tc::smem_u32(smem + kWOff);
      int it = 0;
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++it) {
        const int ab = it & 1;
        if (!tc::mbar_wait(&a_full[ab], (it >> 1) & 1, args.status, 0x302)) break;
        tc::tc_fence_after();
        const uint32_t a_addr = tc::smem_u32(smem + kAOff + ab * kABytes);
        for (int j = 0; j < kChunks; ++j) {
          if (!tc::mbar_wait(&c_empty[j], (it & 1) ^ 1, args.status, 0x303)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          // Attention: D[pair][out column] = X W^T (TMEM lane = pair row).
          // Triangle multiplication: D[channel][pair] = W X^T (TMEM lane =
          // channel), so a thread's values run along a channel plane.
#pragma unroll
          for (int kk = 0; kk < kC / 16; ++kk) {
            const uint32_t koff = (kk >> 2) * kKBlockBytes + (kk & 3) * 32;
            const uint64_t x_desc = tc::desc_sw128(a_addr + koff, 16);
            const uint64_t w_desc = tc::desc_sw128(w_addr + j * kWChunkBytes + koff, 16);
            if constexpr (KIND == PROJ_ATTENTION)
              tc::umma_f16_ss(tmem_base + j * 128, x_desc, w_desc, idesc, kk != 0);
            else
              tc::umma_f16_ss(tmem_base + j * 128, w_desc, x_desc, idesc, kk != 0);
          }
          tc::umma_commit(&c_full[j]);
        }
        if (ok) tc::umma_commit(&a_empty[ab]);
      }
    }
  } else if (warp < kFirstLnWarp) {
    // ---------------------------------------------------------------- epilogue
    // TMEM lane quarter = warp % 4; `part` = which 64 of a chunk's 128
    // columns this warp reads.  Each warp stages one 32 x 64 block at a time
    // and waits for its previous TMA store to have read it before the next.
    const int quarter = warp & 3;
    const int part = (warp - kFirstEpiWarp) >> 2;
    uint8_t *stage = smem + kStageOff + (warp - kFirstEpiWarp) * kStagePerWarp;
    int it = 0;
    bool ok = true;
    if constexpr (KIND == PROJ_ATTENTION) {
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++it) {
        const TileRows t = tile_rows<KIND>(args, tile);
        const bool warp_live = quarter * 32 < t.valid;
        for (int j = 0; j < kChunks; ++j) {
          if (!warp_wait(&c_full[j], it & 1, args.status, 0x304)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t taddr = tc::tmem_addr(tmem_base, quarter * 32, j * 128 + part * 64);
          {
            uint32_t r0[32], r1[32];
            tc::tmem_ld_32x32b_x32(taddr, r0);
            tc::tmem_ld_32x32b_x32(taddr + 32, r1);
            tc::tmem_ld_wait_regs(r0, r1);
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&c_empty[j]);
            if (!warp_live) continue;
            const int c0 = j * 128 + part * 64;
            const float4 *bq = reinterpret_cast<const float4 *>(bias_s + c0);  // same address in every lane
            uint8_t *buf = stage;
            if (lane == 0) tc::bulk_wait_read<0>();
            __syncwarp();
            // 16-byte chunk e of the staged row = columns 8 e .. 8 e + 7.  q
            // (chunk 0) leaves scaled, bf16(bf16(q) * q_scale); g (chunk 3)
            // leaves activated, bf16(sigmoid(bf16(g + b))): the flash kernel's
            // operands, with upstream's rounding points.
            if (j == 0)
              stage_row<1>(buf, lane, r0, r1, bq, args.q_scale);
            else if (j == 3)
              stage_row<2>(buf, lane, r0, r1, bq, args.q_scale);
            else
              stage_row<0>(buf, lane, r0, r1, bq, args.q_scale);
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tc::tma_store_2d(&map_out, buf, c0, int(t.row0) + quarter * 32);
              tc::bulk_commit();
            }
          }
        }
      }
    } else {
      // Thread = channel 32 quarter + lane of plane group G (a: G = 0, b: G = 1);
      // TMEM columns = the tile's 128 pairs, of which this warp takes 64
      // (`part`).  p of group G sits in chunk 2 G, g in chunk 2 G + 1.  Per
      // pair: p, g rounded to bf16 (the autocast linears' outputs), s =
      // bf16(sigmoid(g)), bf16(p * s) (exact as mul.rn.bf16x2), then
      // bf16(. * mask).  The staged row of 64 pairs of one channel goes out
      // as one TMA box row.
      float *msk = bias_s + quarter * kRows + part * 64;  // this warp's copy of its 64 pairs' mask
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++it) {
        const TileRows t = tile_rows<KIND>(args, tile);
        float mv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int k = part * 64 + lane * 2 + e;
          mv[e] = k < t.valid ? args.mask[t.row0 + k] : 0.f;
        }
        __syncwarp();
        *reinterpret_cast<float2 *>(msk + lane * 2) = make_float2(mv[0], mv[1]);
        const bool unit = __all_sync(0xffffffffu, mv[0] == 1.f && mv[1] == 1.f);
        __syncwarp();
        for (int G = 0; G < 2; ++G) {
          if (!warp_wait(&c_full[2 * G], it & 1, args.status, 0x304) ||
              !warp_wait(&c_full[2 * G + 1], it & 1, args.status, 0x304)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t tp = tc::tmem_addr(tmem_base, quarter * 32, 256 * G + 64 * part), tg = tp + 128;
          uint32_t pa[16], ga[16], pb[16], gb[16];
          tc::tmem_ld_32x32b_x16(tp, pa);
          tc::tmem_ld_32x32b_x16(tg, ga);
          tc::tmem_ld_wait_regs(pa, ga);
          uint8_t *buf = stage;
          if (lane == 0) tc::bulk_wait_read<0>();  // the previous store has read the staging block
          __syncwarp();
#pragma unroll
          for (int step = 0; step < 4; ++step) {  // 16 pairs per step
            uint32_t(&pc)[16] = (step & 1) ? pb : pa;
            uint32_t(&gc)[16] = (step & 1) ? gb : ga;
            uint32_t(&pn)[16] = (step & 1) ? pa : pb;
            uint32_t(&gn)[16] = (step & 1) ? ga : gb;
            if (step < 3) {  // next 16 pairs in flight while these are processed
              tc::tmem_ld_32x32b_x16(tp + 16 * (step + 1), pn);
              tc::tmem_ld_32x32b_x16(tg + 16 * (step + 1), gn);
            } else {
              tc::tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                tc::mbar_arrive(&c_empty[2 * G]);
                tc::mbar_arrive(&c_empty[2 * G + 1]);
              }
            }
            uint32_t o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const uint32_t p2 = cvt_bf16x2(__uint_as_float(pc[2 * e]), __uint_as_float(pc[2 * e + 1]));
              const uint32_t g2 = cvt_bf16x2(__uint_as_float(gc[2 * e]), __uint_as_float(gc[2 * e + 1]));
              o[e] = mul_bf16x2(p2, cvt_bf16x2(sigmoid_mufu(bf16_lo(g2)), sigmoid_mufu(bf16_hi(g2))));
            }
            if (!unit) {
              const float2 *m2 = reinterpret_cast<const float2 *>(msk + 16 * step);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float2 mm = m2[e];
                o[e] = cvt_bf16x2(bf16_lo(o[e]) * mm.x, bf16_hi(o[e]) * mm.y);
              }
            }
            const int c16 = 2 * step;  // 16-byte chunks of the 128-byte staged row
            *reinterpret_cast<uint4 *>(buf + lane * 128 + ((c16 ^ (lane & 7)) * 16)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4 *>(buf + lane * 128 + (((c16 + 1) ^ (lane & 7)) * 16)) =
                make_uint4(o[4], o[5], o[6], o[7]);
            if (step < 3) tc::tmem_ld_wait_regs(pn, gn);
          }
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && 64 * part < t.valid) {
            tc::tma_store_3d(&map_out, buf, t.k0 + 64 * part, t.i, 128 * G + 32 * quarter);
            tc::bulk_commit();
          }
        }
      }
    }
    if (lane == 0) tc::bulk_wait<0>();
  } else {
    // --------------------------------------------------------------- LayerNorm
    const int lw = warp - kFirstLnWarp;
    float lnw[4], lnb[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      lnw[e] = args.ln_w ? args.ln_w[lane * 4 + e] : 1.f;
      lnb[e] = args.ln_b ? args.ln_b[lane * 4 + e] : 0.f;
    }
    // This lane's 4 channels inside the swizzled A tile: K-block lane / 16,
    // 16-byte chunk (lane % 16) / 2, byte (lane % 2) * 8 within it.
    const uint32_t a_lane_off = (lane >> 4) * kKBlockBytes + (lane & 1) * 8;
    const uint32_t a_chunk = (lane & 15) >> 1;
    const int row_lo = lw * kLnRowsPerWarp;

    // Rows rbase .. rbase + 7 of tile t (zeros past the valid rows).
    auto load_rows = [&](const TileRows &t, int rbase, float4 (&v)[4]) {
#pragma unroll
      for (int r = 0; r < 4; ++r)
        v[r] = rbase + r < t.valid
                   ? __ldg(reinterpret_cast<const float4 *>(args.x + (t.row0 + rbase + r) * kC) + lane)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    };

    // LayerNorm of 4 rows into the A tile (+ side outputs).  Statistics in
    // fp32 as the upstream layer_norm: mean, then the mean of squared
    // deviations, rstd = rsqrt(var + eps), y = bf16((x - mean) * rstd * w + b).
    auto normalise = [&](const float4 (&v)[4], const TileRows &t, int rbase, uint8_t *abuf) {
      {
        constexpr int g = 0;
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
          const int r = 4 * g + rr;
          const int tr = rbase + r;
          const bool live = tr < t.valid;
          const float rs = rsqrtf(var[rr] * (1.f / 128.f) + args.eps);
          const float f0 = (v[r].x - mean[rr]) * rs * lnw[0] + lnb[0];
          const float f1 = (v[r].y - mean[rr]) * rs * lnw[1] + lnb[1];
          const float f2 = (v[r].z - mean[rr]) * rs * lnw[2] + lnb[2];
          const float f3 = (v[r].w - mean[rr]) * rs * lnw[3] + lnb[3];
          const uint2 y = live ? make_uint2(cvt_bf16x2(f0, f1), cvt_bf16x2(f2, f3)) : make_uint2(0u, 0u);
          *reinterpret_cast<uint2 *>(abuf + a_lane_off + tr * 128 + ((a_chunk ^ (tr & 7)) << 4)) = y;
          if constexpr (KIND == PROJ_TRIMUL) {
            if (live) *reinterpret_cast<uint2 *>(args.xn + (t.row0 + tr) * kC + lane * 4) = y;
          }
        }
      }
    };

    // Attention: the four triangle-bias heads of this warp's 16 rows,
    // tri_bias[h][row] = bf16(x_hat[row] . w_heads[h]), read back from the A
    // tile the warp has just written (bf16 x_hat, fp32 accumulation) with
    // eight warp-level m16n8k16 MMAs (heads padded to 8 columns).  TMEM's 512
    // columns hold the q | k | v | g accumulators, so the heads stay on the
    // LayerNorm warp.
    auto bias_heads = [&](const TileRows &t, uint8_t *abuf) {
      const uint32_t a_base = tc::smem_u32(abuf);
      const int mi = lane >> 3;                               // ldmatrix: 8x8 matrix this lane addresses
      const int arow = row_lo + (mi & 1) * 8 + (lane & 7);    // its row
      const int g = lane >> 2, tq = lane & 3;                 // mma fragment: row group, column pair
      const uint32_t *wrow = reinterpret_cast<const uint32_t *>(args.w_heads + (g & 3) * kC);
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < kC / 16; ++ks) {
        const int k = ks * 16 + (mi >> 1) * 8;
        uint32_t a[4];
        ldsm_x4(a_base + (k >> 6) * kKBlockBytes + arow * 128 + ((((k & 63) >> 3) ^ (arow & 7)) << 4), a);
        const uint32_t b0 = g < 4 ? __ldg(wrow + ks * 8 + tq) : 0u;
        const uint32_t b1 = g < 4 ? __ldg(wrow + ks * 8 + 4 + tq) : 0u;
        mma_16816(c, a, b0, b1);
      }
      // c = D[g][2 tq], D[g][2 tq + 1], D[g + 8][2 tq], D[g + 8][2 tq + 1]: heads 2 tq, 2 tq + 1.
      if (tq < 2) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int tr = row_lo + g + 8 * hr;
          if (tr < t.valid) {
            const int row = int(t.row0) + tr;  // n * n < 2^31
            const int q = row / args.n, k = row - q * args.n;
            const int64_t at = args.transpose ? int64_t(k) * args.bias_ld + q : int64_t(q) * args.bias_ld + k;
            args.bias_planes[(2 * tq) * args.bias_hs + at] = __float2bfloat16_rn(c[2 * hr]);
            args.bias_planes[(2 * tq + 1) * args.bias_hs + at] = __float2bfloat16_rn(c[2 * hr + 1]);
          }
        }
      }
    };

    // Software pipeline over 4-row batches (four per tile): the next
    // batch's rows (the rest of this tile, then the first batch of the next
    // tile) are in flight while the current batch is normalised.
    float4 va[4], vb[4];
    int tile = blockIdx.x, it = 0;
    TileRows t{};
    if (tile < args.tiles) {
      t = tile_rows<KIND>(args, tile);
      load_rows(t, row_lo, va);
    }
    for (; tile < args.tiles; tile += gridDim.x, ++it) {
      const int ab = it & 1;
      uint8_t *abuf = smem + kAOff + ab * kABytes;
      load_rows(t, row_lo + 4, vb);
      // This warp's rows two tiles ahead go to L2 now, so the register loads
      // of later batches wait on L2 rather than on HBM.
      if (lane == 0 && tile + 2 * int(gridDim.x) < args.tiles) {
        const TileRows ahead = tile_rows<KIND>(args, tile + 2 * gridDim.x);
        const int rows_ahead = min(kLnRowsPerWarp, ahead.valid - row_lo);
        if (rows_ahead > 0) tc::prefetch_l2_bulk(args.x + (ahead.row0 + row_lo) * kC, uint32_t(rows_ahead) * kC * 4);
      }
      if (!warp_wait(&a_empty[ab], ((it >> 1) & 1) ^ 1, args.status, 0x305)) break;
      normalise(va, t, row_lo, abuf);
      load_rows(t, row_lo + 8, va);
      normalise(vb, t, row_lo + 4, abuf);
      load_rows(t, row_lo + 12, vb);
      normalise(va, t, row_lo + 8, abuf);
      TileRows next = t;
      if (tile + int(gridDim.x) < args.tiles) {
        next = tile_rows<KIND>(args, tile + gridDim.x);
        load_rows(next, row_lo, va);
      }
      normalise(vb, t, row_lo + 12, abuf);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&a_full[ab]);
      if constexpr (KIND == PROJ_ATTENTION) bias_heads(t, abuf);
      t = next;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 512);
  }
}

bool weight_map(CUtensorMap *map, const void *w) {
  uint64_t dims[2] = {uint64_t(kC), uint64_t(kOut)};
  uint64_t strides[1] = {uint64_t(kC) * 2};
  uint32_t box[2] = {64, 64};
  return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int KIND>
int launch_projection(const CUtensorMap &map_w, const CUtensorMap &map_out, const ProjArgs &args,
                      cudaStream_t stream) {
  auto kernel = pair_projection_kernel<KIND>;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), kSmemBytes));
  const int grid = args.tiles < num_sms() ? args.tiles : num_sms();
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(map_w, map_out, args);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

int check_common(const float *x, int64_t n, int64_t n_outer, float eps, const void *w) {
  BL_REQUIRE(n >= 0 && n_outer >= 0 && n_outer <= n && n * n < (1ll << 31), "pair projection: bad n / n_outer");
  BL_REQUIRE(eps > 0.f, "pair projection: eps must be positive");
  BL_REQUIRE(x && w, "pair projection: null pointer");
  BL_REQUIRE(aligned_to(x, 16) && aligned_to(w, 16), "pair projection: x and w must be 16-byte aligned");
  return BL_OK;
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_attention_projection(const float *x, int64_t n, int64_t n_outer, const float *ln_weight,
                                       const float *ln_bias, float eps, const void *w, const float *bias,
                                       float q_scale, const void *w_heads, int transpose, void *proj,
                                       int64_t proj_ld, void *bias_planes, int64_t bias_ld, int64_t bias_hs,
                                       void *stream) {
  if (n == 0 || n_outer == 0) return BL_OK;
  if (int rc = check_common(x, n, n_outer, eps, w)) return rc;
  BL_REQUIRE(w_heads && proj && bias_planes, "bl_attention_projection: null pointer");
  BL_REQUIRE(aligned_to(w_heads, 8), "bl_attention_projection: w_heads must be 8-byte aligned");
  BL_REQUIRE(aligned_to(proj, 16) && proj_ld % 8 == 0 && proj_ld >= kOut,
             "bl_attention_projection: proj rows must be 16-byte aligned and >= 512 wide");
  BL_REQUIRE(transpose ? (bias_ld >= n_outer && bias_hs >= n * bias_ld) : (bias_ld >= n && bias_hs >= n_outer * bias_ld),
             "bl_attention_projection: bias planes too small");
  CUtensorMap map_w, map_out;
  BL_REQUIRE(weight_map(&map_w, w), "bl_attention_projection: cannot encode the weight map");
  {
    uint64_t dims[2] = {uint64_t(kOut), uint64_t(n_outer * n)};
    uint64_t strides[1] = {uint64_t(proj_ld) * 2};
    uint32_t box[2] = {64, 32};
    BL_REQUIRE(encode_tmap(&map_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, proj, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_attention_projection: cannot encode the output map");
  }
  ProjArgs a{};
  a.x = x, a.rows = n_outer * n, a.n = int(n);
  a.tiles = int((a.rows + kRows - 1) / kRows), a.tiles_per_i = 0;
  a.ln_w = ln_weight, a.ln_b = ln_bias, a.eps = eps;
  a.bias = bias, a.q_scale = q_scale;
  a.w_heads = static_cast<const __nv_bfloat16 *>(w_heads), a.transpose = transpose != 0;
  a.bias_planes = static_cast<__nv_bfloat16 *>(bias_planes), a.bias_ld = bias_ld, a.bias_hs = bias_hs;
  a.status = device_status_ptr();
  BL_REQUIRE(a.status, "bl_attention_projection: device status word unavailable");
  return launch_projection<PROJ_ATTENTION>(map_w, map_out, a, as_stream(stream));
}

extern "C" int bl_trimul_projection(const float *x, int64_t n, int64_t n_outer, const float *ln_weight,
                                    const float *ln_bias, float eps, const void *w, const float *mask, void *planes,
                                    int64_t plane_ld, void *xn, void *stream) {
  if (n == 0 || n_outer == 0) return BL_OK;
  if (int rc = check_common(x, n, n_outer, eps, w)) return rc;
  BL_REQUIRE(mask && planes && xn, "bl_trimul_projection: null pointer");
  BL_REQUIRE(aligned_to(planes, 16) && aligned_to(xn, 16) && plane_ld % 8 == 0 && plane_ld >= n,
             "bl_trimul_projection: planes need 16-byte alignment and plane_ld % 8 == 0, >= n");
  CUtensorMap map_w, map_out;
  BL_REQUIRE(weight_map(&map_w, w), "bl_trimul_projection: cannot encode the weight map");
  {
    uint64_t dims[3] = {uint64_t(plane_ld), uint64_t(n_outer), 256};
    uint64_t strides[2] = {uint64_t(plane_ld) * 2, uint64_t(n_outer) * uint64_t(plane_ld) * 2};
    uint32_t box[3] = {64, 1, 32};  // 64 pairs x 32 channels, 128-byte rows
    BL_REQUIRE(encode_tmap(&map_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, planes, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_trimul_projection: cannot encode the plane map");
  }
  ProjArgs a{};
  a.x = x, a.rows = n_outer * n, a.n = int(n);
  a.tiles_per_i = int((n + kRows - 1) / kRows);
  a.tiles = int(n_outer) * a.tiles_per_i;
  a.ln_w = ln_weight, a.ln_b = ln_bias, a.eps = eps;
  a.mask = mask, a.xn = static_cast<__nv_bfloat16 *>(xn);
  a.status = device_status_ptr();
  BL_REQUIRE(a.status, "bl_trimul_projection: device status word unavailable");
  return launch_projection<PROJ_TRIMUL>(map_w, map_out, a, as_stream(stream));
}
