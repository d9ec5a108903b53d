// fp32-accurate linear layers on the bf16 tensor cores:
//
//   Y[m][n] = sum_k X[m][k] * W[n][k]  (+ bias[n])        X, W, Y, bias fp32
//
// The diffusion module and the Pairformer's single track run their linears in
// fp32 with autocast off (upstream AdaLN, ConditionedTransitionBlock,
// AttentionPairBias, transition_s; the reference's diffusion.py:52-68 and
// pair_bias.py:22-36 keep them fp32).  On the CUDA cores those are SIMT
// SGEMMs, and at diffusion sizes (a few hundred tokens, K = 768) they run far
// below peak.  Here every operand is split into three bf16 planes
//
//   x = x1 + x2 + x3,   x1 = bf16(x), x2 = bf16(x - x1), x3 = bf16(x - x1 - x2)
//
// (both subtractions are exact in fp32; |x - x1 - x2 - x3| <= 2^-27 |x|), and
// the product keeps every pair down to 2^-24 relative:
//
//   X W^T = X3 W1 + X2 W2 + X1 W3 + X2 W1 + X1 W2 + X1 W1   (+ terms <= 2^-27)
//
// Each bf16 x bf16 product is exact; what remains is the tensor core's fp32
// accumulation (measured: within 2^-17 of the largest output, a few times an
// fp32 SGEMM's error).  Weights are split once by the caller (cached);
// activations by bl_split3_bf16.
//
// Kernel: persistent, warp-specialised (192 threads): warp 0 TMA-loads the
// three A and three B tiles of each 64-wide K block into a ring, warp 1
// issues the 6 x 4 tcgen05.mma (M = 128, N = BN, K = 16) into a
// double-buffered pair of TMEM accumulators (X1 W1 alone, the five smaller
// products together), warps 2..5 add the two and the bias and TMA-store fp32
// tiles.  Small M gets narrow N tiles (BN = 32 / 64) so the
// grid still covers the SMs without split-K (results stay deterministic).
#include "tc.cuh"

namespace bl {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kStagingBytes = 4096;  // [32 rows][32 fp32], 128-byte swizzled

struct LinArgs {
  int m, n, k;
  int tiles_m, tiles_n;
  int splits, kb_per_split;  // cluster kernel: K blocks [rank * kb_per_split, ...) per CTA
  const float *bias;
  const float *res;  // optional residual added to y (rows of ldr), may alias nothing else
  int64_t ldr;
  float *y;
  int64_t ldy;
  unsigned int *status;
};

template <int BN> struct LinShape {
  static constexpr int kABytes = kBM * kBK * 2;  // one plane
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = 3 * (kABytes + kBBytes);
  static constexpr int kStages = BN <= 32 ? 3 : 2;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kStagingTotal = 4 * 2 * kStagingBytes;
  static constexpr int kBarrierOffset = kRingBytes + kStagingTotal;
  static constexpr int kSmemBytes = kBarrierOffset + 256 + 1024;
  static constexpr uint32_t kTmemCols = 4 * BN;  // 2 buffers x {X1 W1, the five smaller products}
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// (A plane, B plane) of product p, smallest first: (3,1) (2,2) (1,3) (2,1) (1,2) (1,1).
__device__ __forceinline__ int pair_a(int p) { return p == 0 ? 2 : (p == 1 || p == 3) ? 1 : 0; }
__device__ __forceinline__ int pair_b(int p) { return p == 2 ? 2 : (p == 1 || p == 4) ? 1 : 0; }

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    linear_split3_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                         const __grid_constant__ CUtensorMap tma_y, const LinArgs args) {
  using S = LinShape<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::kBarrierOffset);
  uint64_t *empty = full + S::kStages;
  uint64_t *acc_full = empty + S::kStages;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_tiles = args.tiles_m * args.tiles_n;
  const int k_blocks = (args.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 4);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tma_x);
    tc::prefetch_tmap(&tma_w);
    tc::prefetch_tmap(&tma_y);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, S::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / args.tiles_n) * kBM, n0 = (tile % args.tiles_n) * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1u, args.status, 0x601)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * S::kStageBytes;
          uint8_t *sb = sa + 3 * S::kABytes;
          tc::mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
#pragma unroll
          for (int p = 0; p < 3; ++p) {
            tc::tma_load_3d(sa + p * S::kABytes, &tma_x, &full[stage], kb * kBK, m0, p);
            tc::tma_load_3d(sb + p * S::kBBytes, &tma_w, &full[stage], kb * kBK, n0, p);
          }
          if (++stage == S::kStages) stage = 0, phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(kBM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        if (!tc::mbar_wait(&acc_empty[acc], acc_phase ^ 1u, args.status, 0x602)) break;
        tc::tc_fence_after();
        const uint32_t d_hi = tmem_base + uint32_t(acc * 2 * BN), d_lo = d_hi + BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, args.status, 0x603)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + 3 * S::kABytes;
          // The five small products share one accumulator and X1 W1 has its
          // own: the tensor core's fp32 accumulation then never adds a
          // 2^-8-scale term into the full-scale sum (the epilogue adds the two
          // with one fp32 rounding).
#pragma unroll
          for (int p = 0; p < 6; ++p) {
            const uint32_t pa = sa + pair_a(p) * S::kABytes, pb = sb + pair_b(p) * S::kBBytes;
            const uint32_t d = p == 5 ? d_hi : d_lo;
            const bool first = kb == 0 && (p == 0 || p == 5);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              tc::umma_f16_ss(d, tc::desc_sw128(pa + kk * 32, 16), tc::desc_sw128(pb + kk * 32, 16), idesc,
                              !(first && kk == 0));
          }
          tc::umma_commit(&empty[stage]);
          if (++stage == S::kStages) stage = 0, phase ^= 1u;
        }
        tc::umma_commit(&acc_full[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1u;
      }
    }
  } else {
    // Epilogue warps 2..5 own TMEM lane quarters (warp % 4).
    const int quarter = warp & 3;
    uint8_t *staging = smem + S::kRingBytes + quarter * 2 * kStagingBytes;
    int acc = 0;
    uint32_t acc_phase = 0;
    int count = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      const int m0 = (tile / args.tiles_n) * kBM, n0 = (tile % args.tiles_n) * BN;
      const int row0 = m0 + quarter * 32;
      if (!tc::mbar_wait(&acc_full[acc], acc_phase, args.status, 0x604)) break;
      tc::tc_fence_after();
      const uint32_t tbase = tc::tmem_addr(tmem_base, quarter * 32, acc * 2 * BN);
      const bool live = row0 < args.m;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32], rl[32];
        tc::tmem_ld_32x32b_x32(tbase + cc * 32, r);
        tc::tmem_ld_32x32b_x32(tbase + BN + cc * 32, rl);
        tc::tmem_ld_wait_regs(r, rl);
        if (cc + 1 == BN / 32) {  // accumulator read out: the next tile's MMAs may start
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
        }
        const int c0 = n0 + cc * 32;
        if (!live || c0 >= args.n) continue;  // wholly outside Y: no store
        float out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int c = c0 + j;
          out[j] = (__uint_as_float(r[j]) + __uint_as_float(rl[j])) +
                   (args.bias && c < args.n ? __ldg(args.bias + c) : 0.f);
        }
        if (args.res && row0 + lane < args.m) {  // y = x W^T + bias + residual (n % 4 == 0: whole float4s)
          const float *rrow = args.res + int64_t(row0 + lane) * args.ldr + c0;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            if (c0 + j < args.n) {
              const float4 rv = __ldg(reinterpret_cast<const float4 *>(rrow + j));
              out[j] += rv.x, out[j + 1] += rv.y, out[j + 2] += rv.z, out[j + 3] += rv.w;
            }
          }
        }
        uint8_t *buf = staging + (count & 1) * kStagingBytes;
        if (lane == 0) tc::bulk_wait_read<1>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4 *>(buf + lane * 128 + ((j ^ (lane & 7)) * 16)) =
              make_float4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tc::tma_store_2d(&tma_y, buf, c0, row0);
          tc::bulk_commit();
        }
        ++count;
      }
      if (++acc == 2) acc = 0, acc_phase ^= 1u;
    }
    if (lane == 0) tc::bulk_wait<0>();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Problems with few output tiles (skinny m): one cluster of S CTAs per tile,
// CTA rank r accumulating K blocks [r * kbs, (r + 1) * kbs).  Partials meet in
// shared memory: after a cluster barrier CTA r sums rows [r * 128 / S, ...)
// over the S partials in rank order through distributed shared memory
// (deterministic), adds the bias and writes Y.  Every thread reaches both
// cluster barriers on every path (a failed bounded wait only skips work).
// ---------------------------------------------------------------------------
template <int BN> struct ClusterShape {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = 3 * (kABytes + kBBytes);
  static constexpr int kStages = BN <= 32 ? 3 : 2;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kPartLd = BN + 4;  // floats per partial row
  static constexpr int kPartBytes = kBM * kPartLd * 4;
  static constexpr int kBarrierOffset = kRingBytes + kPartBytes;
  static constexpr int kSmemBytes = kBarrierOffset + 256 + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float4 ld_peer_f4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    linear_split3_cluster_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                                 const LinArgs args) {
  using S = ClusterShape<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *part = reinterpret_cast<float *>(smem + S::kRingBytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::kBarrierOffset);
  uint64_t *empty = full + S::kStages;
  uint64_t *acc_full = empty + S::kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int splits = args.splits;
  const int rank = int(cluster_rank());
  const int tile = int(blockIdx.x) / splits;
  const int m0 = (tile / args.tiles_n) * kBM, n0 = (tile % args.tiles_n) * BN;
  const int k_blocks = (args.k + kBK - 1) / kBK;
  const int kb0 = rank * args.kb_per_split, kb1 = min(k_blocks, kb0 + args.kb_per_split);

  if (threadIdx.x == 0) {
    for (int st = 0; st < S::kStages; ++st) {
      tc::mbar_init(&full[st], 1);
      tc::mbar_init(&empty[st], 1);
    }
    tc::mbar_init(acc_full, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tma_x);
    tc::prefetch_tmap(&tma_w);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, S::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait(&empty[stage], phase ^ 1u, args.status, 0x611)) break;
        uint8_t *sa = smem + stage * S::kStageBytes;
        uint8_t *sb = sa + 3 * S::kABytes;
        tc::mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          tc::tma_load_3d(sa + p * S::kABytes, &tma_x, &full[stage], kb * kBK, m0, p);
          tc::tma_load_3d(sb + p * S::kBBytes, &tma_w, &full[stage], kb * kBK, n0, p);
        }
        if (++stage == S::kStages) stage = 0, phase ^= 1u;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(kBM, BN, false, false);
      const uint32_t d_hi = tmem_base, d_lo = tmem_base + BN;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1 && ok; ++kb) {
        if (!(ok = tc::mbar_wait(&full[stage], phase, args.status, 0x612))) break;
        tc::tc_fence_after();
        const uint32_t sa = tc::smem_u32(smem + stage * S::kStageBytes);
        const uint32_t sb = sa + 3 * S::kABytes;
#pragma unroll
        for (int p = 0; p < 6; ++p) {
          const uint32_t pa = sa + pair_a(p) * S::kABytes, pb = sb + pair_b(p) * S::kBBytes;
          const uint32_t d = p == 5 ? d_hi : d_lo;
          const bool first = kb == kb0 && (p == 0 || p == 5);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc::umma_f16_ss(d, tc::desc_sw128(pa + kk * 32, 16), tc::desc_sw128(pb + kk * 32, 16), idesc,
                            !(first && kk == 0));
        }
        tc::umma_commit(&empty[stage]);
        if (++stage == S::kStages) stage = 0, phase ^= 1u;
      }
      if (ok && kb0 < kb1) tc::umma_commit(acc_full);
    }
  } else {
    // This CTA's partial (hi + lo) into shared memory, row = TMEM lane; a
    // rank with no K blocks (k_blocks not a multiple of the split) adds zeros.
    const int quarter = warp & 3;
    if (kb0 >= kb1) {
      float *dst = part + (quarter * 32 + lane) * S::kPartLd;
      for (int j = 0; j < BN; j += 4) *reinterpret_cast<float4 *>(dst + j) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if (tc::mbar_wait(acc_full, 0, args.status, 0x613)) {
      tc::tc_fence_after();
      const uint32_t tbase = tc::tmem_addr(tmem_base, quarter * 32, 0);
      float *dst = part + (quarter * 32 + lane) * S::kPartLd;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32], rl[32];
        tc::tmem_ld_32x32b_x32(tbase + cc * 32, r);
        tc::tmem_ld_32x32b_x32(tbase + BN + cc * 32, rl);
        tc::tmem_ld_wait_regs(r, rl);
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4 *>(dst + cc * 32 + j) =
              make_float4(__uint_as_float(r[j]) + __uint_as_float(rl[j]),
                          __uint_as_float(r[j + 1]) + __uint_as_float(rl[j + 1]),
                          __uint_as_float(r[j + 2]) + __uint_as_float(rl[j + 2]),
                          __uint_as_float(r[j + 3]) + __uint_as_float(rl[j + 3]));
      }
    }
  }
  tc::tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // every partial of the cluster is in shared memory
  {
    const int rows = kBM / splits, r0 = rank * rows;
    constexpr int kCols4 = BN / 4;
    const uint32_t part_addr = tc::smem_u32(part);
    for (int it = threadIdx.x; it < rows * kCols4; it += kThreads) {
      const int r = r0 + it / kCols4, c = 4 * (it % kCols4);
      const uint32_t off = part_addr + uint32_t((r * S::kPartLd + c) * 4);
      float4 v = ld_peer_f4(off, 0);
      for (int p = 1; p < splits; ++p) {
        const float4 w = ld_peer_f4(off, uint32_t(p));
        v.x += w.x, v.y += w.y, v.z += w.z, v.w += w.w;
      }
      const int col = n0 + c, row = m0 + r;
      if (row < args.m && col < args.n) {
        if (args.bias) v.x += args.bias[col], v.y += args.bias[col + 1], v.z += args.bias[col + 2], v.w += args.bias[col + 3];
        if (args.res) {
          const float4 rv = __ldg(reinterpret_cast<const float4 *>(args.res + int64_t(row) * args.ldr + col));
          v.x += rv.x, v.y += rv.y, v.z += rv.z, v.w += rv.w;
        }
        *reinterpret_cast<float4 *>(args.y + int64_t(row) * args.ldy + col) = v;
      }
    }
  }
  __syncwarp();
  cluster_sync_all();  // peers finished reading this CTA's partial
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

template <int BN>
int launch_linear_cluster(const CUtensorMap &tx, const CUtensorMap &tw, LinArgs args, int splits,
                          cudaStream_t stream) {
  using S = ClusterShape<BN>;
  auto kernel = linear_split3_cluster_kernel<BN>;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), S::kSmemBytes));
  const int k_blocks = (args.k + kBK - 1) / kBK;
  args.tiles_n = (args.n + BN - 1) / BN;
  args.kb_per_split = (k_blocks + splits - 1) / splits;
  args.splits = splits;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(unsigned(args.tiles_m * args.tiles_n * splits));
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = S::kSmemBytes;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  BL_CUDA(cudaLaunchKernelEx(&config, kernel, tx, tw, args));
  BL_LAUNCH_CHECK();
  return BL_OK;
}

template <int BN>
int launch_linear(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &ty, LinArgs args,
                  cudaStream_t stream) {
  using S = LinShape<BN>;
  auto kernel = linear_split3_kernel<BN>;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), S::kSmemBytes));
  args.tiles_n = (args.n + BN - 1) / BN;
  const int total = args.tiles_m * args.tiles_n;
  const int grid = total < num_sms() ? total : num_sms();
  kernel<<<grid, kThreads, S::kSmemBytes, stream>>>(tx, tw, ty, args);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

// x = x1 + x2 + x3 in three bf16 planes, four elements per thread.
__global__ void split3_kernel(const float *x, int64_t rows, int64_t cols, int64_t ldx, __nv_bfloat16 *out) {
  const int64_t plane = rows * cols;
  const int64_t quads = plane / 4;
  for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < quads; q += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = 4 * q, r = e / cols, c = e - r * cols;
    const float4 v = *reinterpret_cast<const float4 *>(x + r * ldx + c);
    const float xs[4] = {v.x, v.y, v.z, v.w};
    uint32_t h[2], m[2], l[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float p[2][3];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float a = xs[2 * i + j];
        const float a1 = bf16r(a), r1 = a - a1;  // exact
        const float a2 = bf16r(r1), r2 = r1 - a2;  // exact
        p[j][0] = a1, p[j][1] = a2, p[j][2] = r2;
      }
      h[i] = pack_bf16x2(p[0][0], p[1][0]);
      m[i] = pack_bf16x2(p[0][1], p[1][1]);
      l[i] = pack_bf16x2(p[0][2], p[1][2]);
    }
    *reinterpret_cast<uint2 *>(out + e) = make_uint2(h[0], h[1]);
    *reinterpret_cast<uint2 *>(out + plane + e) = make_uint2(m[0], m[1]);
    *reinterpret_cast<uint2 *>(out + 2 * plane + e) = make_uint2(l[0], l[1]);
  }
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_split3_bf16(const float *x, int64_t rows, int64_t cols, int64_t ldx, void *out, void *stream) {
  BL_REQUIRE(rows >= 0 && cols >= 0, "bl_split3_bf16: bad shape");
  if (rows == 0 || cols == 0) return BL_OK;
  BL_REQUIRE(x && out, "bl_split3_bf16: null pointer");
  BL_REQUIRE(cols % 4 == 0 && ldx % 4 == 0 && ldx >= cols && aligned_to(x, 16) && aligned_to(out, 8),
             "bl_split3_bf16: cols and ldx must be multiples of 4, x 16-byte aligned");
  const int64_t quads = rows * cols / 4;
  const int64_t blocks = (quads + 255) / 256;
  const int64_t cap = int64_t(num_sms()) * 8;
  split3_kernel<<<int(blocks < cap ? blocks : cap), 256, 0, as_stream(stream)>>>(
      x, rows, cols, ldx, static_cast<__nv_bfloat16 *>(out));
  BL_LAUNCH_CHECK();
  return BL_OK;
}

extern "C" int bl_linear_split3(const void *x3, int64_t m, int64_t k, const void *w3, int64_t n, const float *bias,
                                const float *residual, int64_t ldr, float *y, int64_t ldy, void *stream) {
  BL_REQUIRE(m >= 0 && n >= 0 && k >= 0, "bl_linear_split3: bad shape");
  if (m == 0 || n == 0) return BL_OK;
  BL_REQUIRE(k > 0 && x3 && w3 && y, "bl_linear_split3: null pointer or k = 0");
  BL_REQUIRE(k % 8 == 0 && n % 4 == 0 && ldy % 4 == 0 && ldy >= n, "bl_linear_split3: k % 8, n % 4, ldy % 4 must be 0");
  BL_REQUIRE(aligned_to(x3, 16) && aligned_to(w3, 16) && aligned_to(y, 16),
             "bl_linear_split3: pointers must be 16-byte aligned");
  BL_REQUIRE(!residual || (aligned_to(residual, 16) && ldr % 4 == 0 && ldr >= n),
             "bl_linear_split3: residual must be 16-byte aligned with ldr % 4 == 0 and ldr >= n");
  BL_REQUIRE(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "bl_linear_split3: shape too large");
  // Every CTA streams its tile's A and B rows through the whole K range, so
  // the critical path is (waves of work units) x (bytes one unit loads).
  // Pick the N tile and, for problems with few tiles, a cluster split over K
  // (one wave, BN <= 64) that minimise it.
  int bn = 128, splits = 1;
  {
    const int64_t k_blocks = (k + kBK - 1) / kBK, tiles_m = (m + kBM - 1) / kBM, sms = num_sms();
    int64_t best = -1;
    for (int b : {32, 64, 128}) {
      const int64_t tiles = tiles_m * ((n + b - 1) / b);
      for (int sp = 1; sp <= 8; sp *= 2) {
        if (sp > 1 && (b > 64 || tiles * sp > sms || sp > k_blocks)) break;
        const int64_t waves = (tiles * sp + sms - 1) / sms;
        const int64_t cost = waves * ((k_blocks + sp - 1) / sp) * (3 * (kBM + b) * kBK * 2);
        if (best < 0 || cost < best) best = cost, bn = b, splits = sp;
      }
    }
  }
  CUtensorMap tx, tw, ty;
  {
    uint64_t dims[3] = {uint64_t(k), uint64_t(m), 3};
    uint64_t strides[2] = {uint64_t(k) * 2, uint64_t(m) * uint64_t(k) * 2};
    uint32_t box[3] = {kBK, kBM, 1};
    BL_REQUIRE(encode_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, x3, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_linear_split3: cannot encode the X map");
  }
  {
    uint64_t dims[3] = {uint64_t(k), uint64_t(n), 3};
    uint64_t strides[2] = {uint64_t(k) * 2, uint64_t(n) * uint64_t(k) * 2};
    uint32_t box[3] = {kBK, uint32_t(bn), 1};
    BL_REQUIRE(encode_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, w3, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_linear_split3: cannot encode the W map");
  }
  {
    uint64_t dims[2] = {uint64_t(n), uint64_t(m)};
    uint64_t strides[1] = {uint64_t(ldy) * 4};
    uint32_t box[2] = {32, 32};
    BL_REQUIRE(encode_tmap(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, y, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_linear_split3: cannot encode the Y map");
  }
  LinArgs args{};
  args.m = int(m), args.n = int(n), args.k = int(k);
  args.tiles_m = int((m + kBM - 1) / kBM);
  args.bias = bias;
  args.res = residual, args.ldr = ldr;
  args.y = y, args.ldy = ldy;
  args.splits = 1, args.kb_per_split = 0;
  args.status = device_status_ptr();
  BL_REQUIRE(args.status, "bl_linear_split3: device status word unavailable");
  cudaStream_t s = as_stream(stream);
  if (splits > 1) {
    if (bn == 64) return launch_linear_cluster<64>(tx, tw, args, splits, s);
    return launch_linear_cluster<32>(tx, tw, args, splits, s);
  }
  if (bn == 128) return launch_linear<128>(tx, tw, ty, args, s);
  if (bn == 64) return launch_linear<64>(tx, tw, ty, args, s);
  return launch_linear<32>(tx, tw, ty, args, s);
}
