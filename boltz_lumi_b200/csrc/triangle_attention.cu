// Flash triangle attention on tcgen05 tensor cores (starting and ending node).
//
// For every outer row a of the pair tensor, head h and query b:
//   s(b, c) = bf16(q_s(a, b) . k(a, c))                    q_s = bf16(q / sqrt(d))
//   t(b, c) = bf16(bf16(s + inf * (mask(a, c) - 1)) + bias(h, b, c))
//   o(a, b) = bf16(sum_c softmax_c(t) v(a, c))
//   out(a, b) = bf16(o * s_g(a, b))                         s_g = bf16(sigmoid(g))
// q_s and s_g arrive prepared (the projection kernel writes them), so the
// kernel reads Q straight into the first MMA and the gate straight into the
// epilogue.
// This is the reference's ordered_triangle_forward (triangle.py:32-104 and
// kernels/triangle_softmax.py:90-113) plus upstream _wrap_up's gate, without
// materialising the [I, H, N, N] scores.  The ending node is the same
// computation on z transposed, expressed through row strides and a
// transposed bias plane.  Blackwell structure:
//   * S = Q K^T for a 64-key tile is one pair of tcgen05.mma (M = 128 queries,
//     N = 64 keys, K = 32) into TMEM, double-buffered so the MMA of tile j+1
//     runs while the softmax of tile j is in progress;
//   * each query row is handled by two softmax threads (keys 0..31 and 32..63
//     of every tile, TMEM lane = row).  A thread reads its 32 scores with one
//     tcgen05.ld, applies the ordered rounding (bf16 score -> + mask -> + bias)
//     on packed bf16x2 and computes P = exp2(t log2 e - m log2 e) (fp32 MUFU,
//     rounded to bf16).  The two halves keep separate running maxima and
//     separate O / row-sum accumulators, so they never synchronise per tile;
//     the epilogue merges them (flash-decoding style split of the key axis);
//   * P goes back into TMEM over the columns its S half occupied, and
//     O_h += P_h V_h is a tcgen05.mma with A = P from TMEM and B = V in its
//     natural [key][d] layout read MN-major; the row sums accumulate in
//     registers from the fp32 exponentials (the reference's softmax divides by
//     the fp32 sum too);
//   * O_h is rescaled (tcgen05.ld/st) only when its maximum grows by more than
//     2^8, so P stays <= 256 and rescales are rare;
//   * Q, K, V and the bias tiles arrive by TMA through a 4-deep ring (3-D
//     maps carry the starting/ending-node strides); no multicast.
//   * when the grid still fills the GPU several times over (N >= ~300 at
//     one outer row per CTA row), one CTA runs two or four heads of its
//     (outer row, query tile) back to back: the setup (barriers, TMEM), the
//     mask pass and the key ring are shared, the next head's Q and first key
//     tiles load while the previous head finishes, and only its epilogue sits
//     between two heads (the first P.V of a head waits until the previous
//     head's O has been read).  Measured at N = 512: 288 -> 268 us per launch
//     (starting node), bitwise-identical output.
//   * given W_o (bl_triangle_attention_residual) and four heads per CTA, the
//     epilogue also runs the output projection and the residual add: each head's
//     gated bf16 output goes into TMEM (lane = query row, 64 columns for the
//     128 channels), W_o lands in the drained key ring by TMA, one more
//     tcgen05.mma chain (M = 128, N = 128, K = 128, A from TMEM) accumulates
//     gated . W_o^T into the S columns, and the softmax warps add
//     bf16(D + b_o) into the fp32 z row with vector reductions.  The gated
//     tensor never reaches HBM; measured at N = 512 (starting node, flash +
//     linear_o): 327 -> 308 us, z bitwise equal to the unfused pair of launches.
// Warp roles: warp 0 TMA producer, warp 1 TMEM allocation + MMA issue, warps
// 2..9 softmax and epilogue (TMEM lane quarter = warp % 4; warps 2..5 take key
// half 0, warps 6..9 key half 1).
#include "tc.cuh"

namespace bl {
namespace {

constexpr int kD = 32;
constexpr int kBQ = 128;
constexpr int kBK = 64;
constexpr int kHeads = 4;
constexpr int kMaxTiles = 64;  // n <= 4096
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = (2 + kSoftmaxWarps) * 32;
constexpr int kStages = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // keep P = exp2(x - ref) <= 2^8 before rescaling O

// Shared memory layout (offsets from a 1024-byte aligned base).
constexpr int kQOff = 0;                        // Q [128][32] bf16, 64B-swizzled              8 KB
constexpr int kStageOff = 8192;                 // ring of {K, V, bias}
constexpr int kKBytes = kBK * kD * 2;           // K [64][32] bf16, 64B-swizzled               4 KB
constexpr int kVBytes = kBK * kD * 2;           // V [64][32] bf16, 64B-swizzled               4 KB
constexpr int kBiasBytes = kBQ * kBK * 2;       // bias [128][64] bf16, 128B-swizzled         16 KB
constexpr int kStageBytes = kKBytes + kVBytes + kBiasBytes;
constexpr int kBarOff = kStageOff + kStages * kStageBytes;
constexpr int kMaxOff = kBarOff + 256;          // per-half row maxima exchanged in the epilogue
constexpr int kSumOff = kMaxOff + 2 * kBQ * 4;  // per-half row sums exchanged in the epilogue
constexpr int kFlagOff = kSumOff + 2 * kBQ * 4; // per-key-tile "has masked keys" flags
constexpr int kMaskOff = kFlagOff + kMaxTiles * 4;

// TMEM columns: S/P[b] at 64 b (b = 0, 1; key half h at +32 h), O_h at
// 128 + 32 h; with the fused output, the gated bf16 outputs of the four heads
// (packed two per column) at 192 and linear_o's accumulator over columns 0..127.
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kOCol = 128;
constexpr uint32_t kOStride = kD;
constexpr uint32_t kACol = 192;  // fused output: the gated bf16 outputs of the four heads (A of linear_o)

constexpr uint32_t kNegPad = 0xF14AF14Au;  // bf16x2 (-1e30, -1e30)
// Lower bound of a half-row's reference maximum.  When every key of a thread's
// first tile is padding (n <= 32, key half 1) the maximum would be the pad
// value itself, and t log2 e - m log2 e would leave the fma's rounding residual
// (up to 2^76 at that magnitude) inside exp2, overflowing the register row sum.
// With the floor the padded exponentials underflow to exactly 0; scores of real
// keys stay far above it (masked keys sit at -inf, and the host requires inf <= 1e20).
constexpr float kMaxFloor = -1e29f;

struct TcArgs {
  const __nv_bfloat16 *g;
  int64_t ld, so, si;
  const float *mask;
  int64_t ms_o, ms_k;
  float inf;
  __nv_bfloat16 *out;
  int64_t out_ld;
  int n;
  int heads_per_cta;  // 2 or 4 heads run back to back by one CTA (the kMulti kernel)
  // Fused output (kFuse, four heads per CTA): z[pair][c] += bf16(gated . W_o^T + b_o)
  const float *b_o;
  float *z;
  int64_t z_ld;
  unsigned int *status;
};

__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// Shared-memory reads through 32-bit shared addresses (the generic pointer
// arithmetic on the aligned dynamic window would otherwise hide the state space).
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ int lds32(uint32_t addr) {
  int v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
// (x.lo, x.hi) * (s, s) + (c, c) on the packed fp32x2 pipe (sm_100).
__device__ __forceinline__ void fma_f32x2(float &lo, float &hi, float s, float c) {
  uint64_t x = (uint64_t(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
  const uint64_t sv = (uint64_t(__float_as_uint(s)) << 32) | __float_as_uint(s);
  const uint64_t cv = (uint64_t(__float_as_uint(c)) << 32) | __float_as_uint(c);
  asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(x) : "l"(sv), "l"(cv));
  lo = __uint_as_float(uint32_t(x));
  hi = __uint_as_float(uint32_t(x >> 32));
}
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 64-byte swizzle descriptor (K-major: LBO unused = 16 B; MN-major: LBO = block stride), SBO = 512 B.
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr, uint32_t lbo_bytes) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (uint64_t(512 >> 4) << 32) | (uint64_t(1) << 46) | (uint64_t(4) << 61);
}

__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void red_add_v4(float *addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
// 128-byte swizzle descriptor, K-major (LBO unused), SBO = 1024 B.
__device__ __forceinline__ uint64_t desc_sw128_k(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

// Warp-uniform bounded wait: the whole warp continues only if every lane saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, unsigned int *status, unsigned code) {
  return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, status, code));
}

template <bool kMulti, bool kFuse>
__global__ void __launch_bounds__(kThreads, 2)
    tri_flash_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_bias,
                        const __grid_constant__ CUtensorMap map_wo, const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t smem_base = tc::smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *q_full = bars + 0;               // Q of the current head landed (one phase per head)
  uint64_t *q_empty = bars + 1;              // every S MMA of a head completed: Q may be replaced
  uint64_t *st_full = bars + 2;              // [kStages] K, V, bias of a key tile landed
  uint64_t *st_empty = bars + 2 + kStages;   // [kStages] P.V of that tile completed
  uint64_t *s_full = bars + 2 + 2 * kStages; // [2] S tile in TMEM
  uint64_t *p_full = s_full + 2;             // [2] P tile in TMEM (and O rescaled if needed)
  uint64_t *pv_done = p_full + 2;            // [2] P.V reading TMEM buffer b completed
  uint64_t *o_full = pv_done + 2;            // every P.V of a head done (one phase per head)
  uint64_t *o_free = o_full + 1;             // the softmax warps have read O (one phase per head)
  uint64_t *a_full = o_free + 1;             // fused output: the gated outputs of all heads are in TMEM
  uint64_t *w_full = a_full + 1;             // fused output: W_o landed (in the drained key ring)
  uint64_t *d_full = w_full + 1;             // fused output: linear_o accumulated in TMEM
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(d_full + 1);
  float *row_max = reinterpret_cast<float *>(smem + kMaxOff);
  float *row_sum = reinterpret_cast<float *>(smem + kSumOff);  // [2 heads parity][2 halves][128]
  int *tile_masked = reinterpret_cast<int *>(smem + kFlagOff);
  __nv_bfloat16 *mask_bias = reinterpret_cast<__nv_bfloat16 *>(smem + kMaskOff);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = args.n;
  const int hpc = kMulti ? args.heads_per_cta : 1, groups = kHeads / hpc;
  const int h_begin = (blockIdx.x % groups) * hpc;
  const int q0 = (blockIdx.x / groups) * kBQ;
  const int outer = blockIdx.y;
  const int n_tiles = (n + kBK - 1) / kBK;

  if (tid < kMaxTiles) tile_masked[tid] = 0;
  if (tid == 0) {
    tc::mbar_init(q_full, 1);
    tc::mbar_init(q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&st_full[s], 1);
      tc::mbar_init(&st_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&s_full[b], 1);
      tc::mbar_init(&p_full[b], kSoftmaxWarps);
      tc::mbar_init(&pv_done[b], 1);
    }
    tc::mbar_init(o_full, 1);
    tc::mbar_init(o_free, kSoftmaxWarps);
    tc::mbar_init(a_full, kSoftmaxWarps);
    tc::mbar_init(w_full, 1);
    tc::mbar_init(d_full, 1);
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: the four heads back to back ----------------
    if (lane == 0) {
      tc::prefetch_tmap(&map_q);
      tc::prefetch_tmap(&map_k);
      tc::prefetch_tmap(&map_v);
      tc::prefetch_tmap(&map_bias);
      bool ok = true;
      int g = 0;  // key tiles issued so far over all heads (ring position)
#pragma unroll 1
      for (int hl = 0; hl < hpc && ok; ++hl) {
        const int h = h_begin + hl;
        // Q of head h replaces Q of the previous head once its last S MMA has completed.
        if (hl > 0 && !(ok = tc::mbar_wait(q_empty, (hl - 1) & 1, args.status, 0x20B))) break;
        tc::mbar_arrive_expect_tx(q_full, kBQ * kD * 2);
        tc::tma_load_3d(smem + kQOff, &map_q, q_full, h * kD, q0, outer);
        for (int j = 0; j < n_tiles; ++j, ++g) {
          const int s = g % kStages;
          if (g >= kStages && !(ok = tc::mbar_wait(&st_empty[s], ((g / kStages) & 1) ^ 1u, args.status, 0x201))) break;
          uint8_t *stage = smem + kStageOff + s * kStageBytes;
          tc::mbar_arrive_expect_tx(&st_full[s], kStageBytes);
          tc::tma_load_3d(stage, &map_k, &st_full[s], h * kD, j * kBK, outer);
          tc::tma_load_3d(stage + kKBytes, &map_v, &st_full[s], h * kD, j * kBK, outer);
          tc::tma_load_3d(stage + kKBytes + kVBytes, &map_bias, &st_full[s], j * kBK, q0, h);
        }
      }
      // Fused output: once every P.V of the last head has completed the key ring
      // is drained; W_o (two 128-byte-swizzled K blocks of [128][64]) lands there.
      if (kFuse && ok && tc::mbar_wait(o_full, (hpc - 1) & 1, args.status, 0x20E)) {
        tc::prefetch_tmap(&map_wo);
        tc::mbar_arrive_expect_tx(w_full, 128 * 128 * 2);
        tc::tma_load_2d(smem + kStageOff, &map_wo, w_full, 0, 0);
        tc::tma_load_2d(smem + kStageOff + 128 * 64 * 2, &map_wo, w_full, 64, 0);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16(128, kBK, false, false);
      constexpr uint32_t idesc_pv = tc::idesc_bf16(128, kD, false, true);
      const uint32_t q_addr = tc::smem_u32(smem + kQOff);
      // S of global tile g (head g / n_tiles) into TMEM buffer g & 1.
      auto issue_s = [&](int g) {
        const int s = g % kStages, b = g & 1;
        if (!tc::mbar_wait(&st_full[s], (g / kStages) & 1, args.status, 0x203)) return false;
        // TMEM buffer b still holds P of tile g - 2: its P.V must have finished reading it.
        if (g >= 2 && !tc::mbar_wait(&pv_done[b], ((g - 2) >> 1) & 1, args.status, 0x204)) return false;
        tc::tc_fence_after();
        const uint32_t k_addr = tc::smem_u32(smem + kStageOff + s * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          tc::umma_f16_ss(tmem + uint32_t(b * kBK), desc_sw64(q_addr + kk * 32, 16), desc_sw64(k_addr + kk * 32, 16),
                          idesc_s, kk);
        tc::umma_commit(&s_full[b]);
        return true;
      };
      bool ok = true;
      int g = 0;
#pragma unroll 1
      for (int hl = 0; hl < hpc && ok; ++hl) {
        if (!(ok = tc::mbar_wait(q_full, hl & 1, args.status, 0x202))) break;
        tc::tc_fence_after();
        if (!(ok = issue_s(g))) break;
        if (kMulti && n_tiles == 1) tc::umma_commit(q_empty);
        for (int j = 0; j < n_tiles; ++j, ++g) {
          if (j + 1 < n_tiles) {
            if (!(ok = issue_s(g + 1))) break;
            if (kMulti && j + 2 == n_tiles) tc::umma_commit(q_empty);  // the head's last S MMA: Q may be replaced
          }
          const int s = g % kStages, b = g & 1;
          if (!(ok = tc::mbar_wait(&p_full[b], (g >> 1) & 1, args.status, 0x205))) break;
          // The first P.V of a head overwrites O: the previous head's O must have been read.
          if (j == 0 && hl > 0 && !(ok = tc::mbar_wait(o_free, (hl - 1) & 1, args.status, 0x20C))) break;
          tc::tc_fence_after();
          const uint32_t v_addr = tc::smem_u32(smem + kStageOff + s * kStageBytes + kKBytes);
          const uint32_t lbo = 4096;  // N = 32: one 64-byte N block, LBO unused
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
              tc::umma_f16_ts(tmem + kOCol + half * kOStride, tmem + uint32_t(b * kBK + half * 32 + kk * 8),
                              desc_sw64(v_addr + (half * 2 + kk) * 1024, lbo), idesc_pv, (j | kk) != 0);
          tc::umma_commit(&st_empty[s]);
          tc::umma_commit(&pv_done[b]);
          if (j + 1 == n_tiles) tc::umma_commit(o_full);
        }
      }
      // Fused output: D[128 rows][128] = gated (A, four heads in TMEM) . W_o^T into the
      // S columns (free after the last P.V: MMAs of this thread run in order).
      if (kFuse && ok && tc::mbar_wait(a_full, 0, args.status, 0x20F) &&
          tc::mbar_wait(w_full, 0, args.status, 0x210)) {
        tc::tc_fence_after();
        constexpr uint32_t idesc_o = tc::idesc_bf16(128, 128, false, false);
        const uint32_t w_addr = tc::smem_u32(smem + kStageOff);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc::umma_f16_ts(tmem, tmem + kACol + uint32_t(kk * 8),
                          desc_sw128_k(w_addr + (kk >> 2) * (128 * 64 * 2) + (kk & 3) * 32), idesc_o, kk != 0);
        tc::umma_commit(d_full);
      }
    }
  } else {
    // ---------------- softmax + epilogue: half a query row per thread, four heads ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const uint32_t o_base = lane_base + kOCol + half * kOStride;
    const int qi = q0 + row;
    const int64_t pair = int64_t(outer) * args.so + int64_t(qi) * args.si;
    // The gate rows of all four heads (256 contiguous bytes of the pair row) go to L2 now.
    if (qi < n) asm volatile("prefetch.global.L2 [%0];" ::"l"(args.g + pair * args.ld + half * 64));
    // Mask bias of this outer row (shared by the four heads), 4 keys per
    // thread (bf16; for mask in {0, 1} adding it rounds exactly like the fp32
    // value), and per-tile "any key masked" flags.
    const float *mrow = args.mask + int64_t(outer) * args.ms_o;
    for (int k4 = (tid - 64) * 4; k4 < n_tiles * kBK; k4 += kSoftmaxWarps * 32 * 4) {
      float mb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k4 + e;
        mb[e] = key < n ? args.inf * (__ldg(mrow + int64_t(key) * args.ms_k) - 1.f) : 0.f;
      }
      *reinterpret_cast<uint2 *>(mask_bias + k4) = make_uint2(pack_bf16x2(mb[0], mb[1]), pack_bf16x2(mb[2], mb[3]));
      if (mb[0] != 0.f || mb[1] != 0.f || mb[2] != 0.f || mb[3] != 0.f) atomicOr(&tile_masked[k4 / kBK], 1);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
    bool ok = true;
    int g = 0;
    // Every softmax warp runs the epilogue (and its named barrier) of every head,
    // even after a bounded wait gave up (ok = false: the work is skipped), so the
    // barrier counts always match.
#pragma unroll 1
    for (int hl = 0; hl < hpc; ++hl) {
      const int h = h_begin + hl;
      float m_ref = -INFINITY;  // reference maximum of this half-row's exponentials
      float l_even = 0.f, l_odd = 0.f;  // row sum of the fp32 exponentials (even / odd keys)
      for (int j = 0; j < n_tiles && ok; ++j, ++g) {
        const int s = g % kStages, b = g & 1;
        if (!(ok = warp_wait(&s_full[b], (g >> 1) & 1, args.status, 0x206))) break;
        tc::tc_fence_after();
        uint32_t sv[32];
        tc::tmem_ld_32x32b_x32(lane_base + b * kBK + half * 32, sv);
        if (!(ok = warp_wait(&st_full[s], (g / kStages) & 1, args.status, 0x207))) {
          tc::tmem_ld_wait();
          break;
        }
        const int k0 = j * kBK + half * 32;
        const uint32_t bias_row = smem_base + kStageOff + s * kStageBytes + kKBytes + kVBytes + row * 128;
        uint32_t bw[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 bv = lds128(bias_row + (((half * 4 + c) ^ (row & 7)) << 4));
          bw[4 * c] = bv.x, bw[4 * c + 1] = bv.y, bw[4 * c + 2] = bv.z, bw[4 * c + 3] = bv.w;
        }
        const bool tile_unmasked = lds32(smem_base + kFlagOff + 4 * j) == 0;
        tc::tmem_ld_wait_regs(sv);
        uint32_t t[16];
        if (tile_unmasked) {
#pragma unroll
          for (int pr = 0; pr < 16; ++pr)
            t[pr] = add_bf16x2(cvt_bf16x2(__uint_as_float(sv[2 * pr]), __uint_as_float(sv[2 * pr + 1])), bw[pr]);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 m4 = lds128(smem_base + kMaskOff + 2 * k0 + 16 * c);
            const uint32_t mw[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int pr = 4 * c + e;
              const uint32_t x = cvt_bf16x2(__uint_as_float(sv[2 * pr]), __uint_as_float(sv[2 * pr + 1]));
              t[pr] = add_bf16x2(add_bf16x2(x, mw[e]), bw[pr]);
            }
          }
        }
        const bool tail = k0 + 32 > n;
        if (tail) {
#pragma unroll
          for (int pr = 0; pr < 16; ++pr) {
            const int key = k0 + 2 * pr;
            const uint32_t keep = (key < n ? 0x0000ffffu : 0u) | (key + 1 < n ? 0xffff0000u : 0u);
            t[pr] = (t[pr] & keep) | (kNegPad & ~keep);
          }
        }
        uint32_t mx[4] = {t[0], t[1], t[2], t[3]};
#pragma unroll
        for (int pr = 4; pr < 16; ++pr) mx[pr & 3] = max_bf16x2(mx[pr & 3], t[pr]);
        const uint32_t tmax = max_bf16x2(max_bf16x2(mx[0], mx[1]), max_bf16x2(mx[2], mx[3]));
        const float m_tile = fmaxf(bf16_lo(tmax), bf16_hi(tmax));
        const bool first = j == 0;
        const bool grow = !first && (m_tile - m_ref) * kLog2e > kRescaleLog2;
        if (__any_sync(0xffffffffu, grow)) {
          if (!(ok = warp_wait(&pv_done[(g - 1) & 1], ((g - 1) >> 1) & 1, args.status, 0x208))) break;
          tc::tc_fence_after();
          const float alpha = grow ? fast_exp2((m_ref - m_tile) * kLog2e) : 1.f;
          uint32_t o[32];
          tc::tmem_ld_32x32b_x32(o_base, o);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tc::tmem_st_32x32b_x16(o_base, *reinterpret_cast<const uint32_t(*)[16]>(&o[0]));
          tc::tmem_st_32x32b_x16(o_base + 16, *reinterpret_cast<const uint32_t(*)[16]>(&o[16]));
          l_even *= alpha;
          l_odd *= alpha;
        }
        if (first || grow) m_ref = fmaxf(m_tile, kMaxFloor);
        const float ml = m_ref * kLog2e;
        uint32_t p[16];
#pragma unroll
        for (int pr = 0; pr < 16; ++pr) {
          float x0 = bf16_lo(t[pr]), x1 = bf16_hi(t[pr]);
          fma_f32x2(x0, x1, kLog2e, -ml);
          const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
          l_even += e0;
          l_odd += e1;
          p[pr] = cvt_bf16x2(e0, e1);
        }
        if (tail) {
#pragma unroll
          for (int pr = 0; pr < 16; ++pr) {
            const int key = k0 + 2 * pr;
            p[pr] &= (key < n ? 0x0000ffffu : 0u) | (key + 1 < n ? 0xffff0000u : 0u);
          }
        }
        tc::tmem_st_32x32b_x16(lane_base + b * kBK + half * 32, p);
        tc::tmem_st_wait();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&p_full[b]);
      }
      // Epilogue of head h: merge the two key halves, O / l, bf16, gate, store.
      float *rmax = row_max;  // a warp rewrites it only after every warp started the next head
      rmax[half * kBQ + row] = m_ref;
      row_sum[half * kBQ + row] = l_even + l_odd;
      uint4 gate[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
      if (qi < n) {
        const uint4 *g4 = reinterpret_cast<const uint4 *>(args.g + pair * args.ld + h * kD + half * 16);
        gate[0] = g4[0];
        gate[1] = g4[1];
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
      const float m_other = rmax[(half ^ 1) * kBQ + row];
      const float l_other = row_sum[(half ^ 1) * kBQ + row], l_mine = l_even + l_odd;
      // After the exchange the next head's epilogue may rewrite rmax: every warp
      // has read its partner's value before any warp leaves this barrier pair.
      if (kMulti) asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
      if (!ok || !(ok = warp_wait(o_full, hl & 1, args.status, 0x20A))) continue;
      tc::tc_fence_after();
      uint32_t o0[16], o1[16];
      tc::tmem_ld_32x32b_x16(lane_base + kOCol + half * 16, o0);
      tc::tmem_ld_32x32b_x16(lane_base + kOCol + kOStride + half * 16, o1);
      tc::tmem_ld_wait();
      const float l0 = half == 0 ? l_mine : l_other, l1 = half == 0 ? l_other : l_mine;
      // O has been read: the next head's first P.V may overwrite it.
      if (kMulti && hl + 1 < hpc) {
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(o_free);
      }
      const float m0 = half == 0 ? m_ref : m_other, m1 = half == 0 ? m_other : m_ref;
      const float m = fmaxf(m0, m1);
      const float a0 = fast_exp2((m0 - m) * kLog2e), a1 = fast_exp2((m1 - m) * kLog2e);
      {
        const float inv = fast_rcp(l0 * a0 + l1 * a1);
        uint32_t w8[8];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 gv = gate[c];  // zero for rows past n
          const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = c * 8 + e * 2;
            const float v0 = (__uint_as_float(o0[d]) * a0 + __uint_as_float(o1[d]) * a1) * inv;
            const float v1 = (__uint_as_float(o0[d + 1]) * a0 + __uint_as_float(o1[d + 1]) * a1) * inv;
            const float g0 = bf16_lo(gw[e]), g1 = bf16_hi(gw[e]);  // bf16(sigmoid(g)) from the projection
            w8[4 * c + e] = pack_bf16x2(bf16r(v0) * g0, bf16r(v1) * g1);
          }
        }
        if (kFuse) {
          // Channels h*32 + 16 half .. + 15 of the linear_o operand (TMEM, lane = row).
          tmem_st_x8(lane_base + kACol + uint32_t(h * 16 + half * 8), w8);
          if (hl + 1 == hpc) {
            tc::tmem_st_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(a_full);
          }
        } else if (qi < n) {
          uint4 *o4 = reinterpret_cast<uint4 *>(args.out + pair * args.out_ld + h * kD + half * 16);
          o4[0] = make_uint4(w8[0], w8[1], w8[2], w8[3]);
          o4[1] = make_uint4(w8[4], w8[5], w8[6], w8[7]);
        }
      }
    }
    // Fused output: z[pair][64 half .. 64 half + 63] += bf16(D + b_o) (the block's residual
    // update by linear_o, as upstream's bf16 linear under autocast then the fp32 add).
    if (kFuse && ok && warp_wait(d_full, 0, args.status, 0x211)) {
      tc::tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t dv[32];
        tc::tmem_ld_32x32b_x32(lane_base + uint32_t(half * 64 + cc * 32), dv);
        tc::tmem_ld_wait();
        if (qi < n) {
          const int c0 = half * 64 + cc * 32;
          float *zr = args.z + pair * args.z_ld + c0;
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            red_add_v4(zr + e, bf16r(__uint_as_float(dv[e]) + __ldg(args.b_o + c0 + e)),
                       bf16r(__uint_as_float(dv[e + 1]) + __ldg(args.b_o + c0 + e + 1)),
                       bf16r(__uint_as_float(dv[e + 2]) + __ldg(args.b_o + c0 + e + 2)),
                       bf16r(__uint_as_float(dv[e + 3]) + __ldg(args.b_o + c0 + e + 3)));
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int linear_fused(const void *a, int64_t a_ld, const void *a2, int64_t a2_ld, int64_t k1, const void *w,
                 int64_t w_ld, int64_t m, int64_t n, int64_t k, const float *bias, int gate, float *z, int64_t z_ld,
                 void *out, int64_t out_ld, cudaStream_t stream);

namespace {

bool pair_rows_map(CUtensorMap *map, const void *base, int64_t ld, int64_t so, int64_t si, int n, int n_outer,
                   int box_rows) {
  // Element (column c, inner b, outer a) at base + (a*so + b*si)*ld + c.
  uint64_t dims[3] = {uint64_t(kHeads * kD), uint64_t(n), uint64_t(n_outer)};
  uint64_t strides[2] = {uint64_t(si * ld * 2), uint64_t(so * ld * 2)};
  uint32_t box[3] = {uint32_t(kD), uint32_t(box_rows), 1};
  return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}

}  // namespace
}  // namespace bl

using namespace bl;

namespace bl {
namespace {

// Both C entries: w_o == nullptr writes the gated output to `out`; otherwise
// z (fp32 rows, pair order) += bf16(gated . W_o^T + b_o), with `out` as scratch
// for the gated tensor when the projection cannot run in the epilogue.
int triangle_attention(const void *q, const void *k, const void *v, const void *g, int64_t ld, int64_t so,
                       int64_t si, const void *bias, int64_t bias_ld, int64_t bias_hs, const float *mask,
                       int64_t ms_o, int64_t ms_k, float inf, int64_t heads, int64_t head_dim, int64_t n,
                       int64_t n_outer, void *out, int64_t out_ld, const void *w_o, const float *b_o, float *z,
                       int64_t z_ld, void *stream) {
  BL_REQUIRE(head_dim == kD && heads == kHeads, "bl_triangle_attention: 4 heads x 32 supported");
  BL_REQUIRE(n >= 0 && n_outer >= 0 && n_outer <= n, "bl_triangle_attention: bad shape");
  if (n == 0 || n_outer == 0) return BL_OK;
  BL_REQUIRE(n <= kMaxTiles * kBK, "bl_triangle_attention: at most 4096 tokens");
  BL_REQUIRE(q && k && v && g && bias && mask && out, "bl_triangle_attention: null pointer");
  BL_REQUIRE(inf >= 0.f && inf <= 1e20f, "bl_triangle_attention: inf must lie in [0, 1e20]");
  BL_REQUIRE(ld % 8 == 0 && out_ld % 8 == 0 && bias_ld % 8 == 0 && bias_ld >= n && bias_hs % 8 == 0,
             "bl_triangle_attention: leading dimensions must keep 16-byte rows");
  BL_REQUIRE(aligned_to(q, 16) && aligned_to(k, 16) && aligned_to(v, 16) && aligned_to(g, 16) &&
                 aligned_to(bias, 16) && aligned_to(out, 16),
             "bl_triangle_attention: pointers must be 16-byte aligned");
  CUtensorMap map_q, map_k, map_v, map_bias;
  BL_REQUIRE(pair_rows_map(&map_q, q, ld, so, si, int(n), int(n_outer), kBQ) &&
                 pair_rows_map(&map_k, k, ld, so, si, int(n), int(n_outer), kBK) &&
                 pair_rows_map(&map_v, v, ld, so, si, int(n), int(n_outer), kBK),
             "bl_triangle_attention: cannot encode the q/k/v tensor maps");
  {
    uint64_t dims[3] = {uint64_t(bias_ld), uint64_t(n), uint64_t(kHeads)};
    uint64_t strides[2] = {uint64_t(bias_ld * 2), uint64_t(bias_hs * 2)};
    uint32_t box[3] = {kBK, kBQ, 1};
    BL_REQUIRE(encode_tmap(&map_bias, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, bias, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_triangle_attention: cannot encode the bias tensor map");
  }
  CUtensorMap map_wo = map_bias;  // placeholder unless the output is fused
  if (w_o) {
    BL_REQUIRE(b_o && z && aligned_to(w_o, 16) && aligned_to(z, 16) && z_ld % 4 == 0 && z_ld >= 128,
               "bl_triangle_attention: w_o needs b_o and a 16-byte aligned fp32 z with z_ld % 4 == 0");
    uint64_t dims[2] = {128, 128};
    uint64_t strides[1] = {128 * 2};
    uint32_t box[2] = {64, 128};
    BL_REQUIRE(encode_tmap(&map_wo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_o, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "bl_triangle_attention: cannot encode the W_o tensor map");
  }
  TcArgs args;
  args.b_o = b_o, args.z = z, args.z_ld = z_ld;
  args.g = static_cast<const __nv_bfloat16 *>(g);
  args.ld = ld, args.so = so, args.si = si;
  args.mask = mask, args.ms_o = ms_o, args.ms_k = ms_k;
  args.inf = inf;
  args.out = static_cast<__nv_bfloat16 *>(out);
  args.out_ld = out_ld;
  args.n = int(n);

  args.status = device_status_ptr();
  BL_REQUIRE(args.status, "bl_triangle_attention: device status word unavailable");
  const int n_tiles = int((n + kBK - 1) / kBK);
  const int smem = kMaskOff + n_tiles * kBK * 2 + 1024;
  // Heads run back to back by one CTA (sharing its setup, mask pass and key
  // ring) when the grid still fills the GPU several times over.
  const int64_t q_tiles = (n + kBQ - 1) / kBQ, slots = 2 * int64_t(num_sms());
  const int hpc = q_tiles * n_outer >= 4 * slots ? 4 : 2 * q_tiles * n_outer >= 4 * slots ? 2 : 1;
  args.heads_per_cta = hpc;
  // With w_o and all four heads in one CTA, linear_o and the residual add into z
  // run in the kernel's epilogue; otherwise the gated output goes to `out` and,
  // given w_o, the separate linear (bl_linear_fused's kernel) adds it into z.
  // (Four heads per CTA needs q_tiles * n_outer >= 8 * num_sms, so n > 384 and n_tiles >
  // kStages: when the producer finishes the last head's loads, the o_full phases of the
  // earlier heads have completed and its parity wait names the last head's phase.)
  const bool fuse = w_o && hpc == kHeads && n_tiles > kStages;
  // The separate linear_o runs over rows 0 .. n_outer * n - 1 of out and z: a whole
  // tensor or a starting-node row slab (checked before anything is launched).
  BL_REQUIRE(!w_o || fuse || (so == n && si == 1) || (so == 1 && si == n && n_outer == n),
             "bl_triangle_attention: the unfused w_o path needs contiguous output rows");
  auto kernel = fuse ? tri_flash_tc_kernel<true, true>
                     : hpc > 1 ? tri_flash_tc_kernel<true, false> : tri_flash_tc_kernel<false, false>;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), 232448));
  dim3 grid(unsigned(q_tiles * (kHeads / hpc)), unsigned(n_outer));
  kernel<<<grid, kThreads, smem, as_stream(stream)>>>(map_q, map_k, map_v, map_bias, map_wo, args);
  BL_LAUNCH_CHECK();
  if (w_o && !fuse) {
    return linear_fused(out, out_ld, nullptr, 0, 128, w_o, 128, n_outer * n, 128, 128, b_o, 0, z, z_ld, nullptr, 0,
                        as_stream(stream));
  }
  return BL_OK;
}

}  // namespace
}  // namespace bl

extern "C" int bl_triangle_attention(const void *q, const void *k, const void *v, const void *g, int64_t ld,
                                        int64_t so, int64_t si, const void *bias, int64_t bias_ld, int64_t bias_hs,
                                        const float *mask, int64_t ms_o, int64_t ms_k, float inf, int64_t heads,
                                        int64_t head_dim, int64_t n, int64_t n_outer, void *out, int64_t out_ld,
                                        void *stream) {
  return bl::triangle_attention(q, k, v, g, ld, so, si, bias, bias_ld, bias_hs, mask, ms_o, ms_k, inf, heads,
                                head_dim, n, n_outer, out, out_ld, nullptr, nullptr, nullptr, 0, stream);
}

extern "C" int bl_triangle_attention_residual(const void *q, const void *k, const void *v, const void *g,
                                                 int64_t ld, int64_t so, int64_t si, const void *bias,
                                                 int64_t bias_ld, int64_t bias_hs, const float *mask, int64_t ms_o,
                                                 int64_t ms_k, float inf, int64_t heads, int64_t head_dim, int64_t n,
                                                 int64_t n_outer, void *scratch, int64_t scratch_ld,
                                                 const void *w_o, const float *b_o, float *z, int64_t z_ld,
                                                 void *stream) {
  BL_REQUIRE(w_o, "bl_triangle_attention_residual: w_o is required");
  return bl::triangle_attention(q, k, v, g, ld, so, si, bias, bias_ld, bias_hs, mask, ms_o, ms_k, inf, heads,
                                head_dim, n, n_outer, scratch, scratch_ld, w_o, b_o, z, z_ld, stream);
}
