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
//     natural [key][d] layout read MN-major; a constant block of ones appended
//     to V makes the same MMA produce the row sums of the bf16 P (column 32);
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
constexpr int kOnesOff = kStageOff + kStages * kStageBytes;  // [64][32] ones (V's extra N block)
constexpr int kBarOff = kOnesOff + kVBytes;
constexpr int kMaxOff = kBarOff + 256;          // per-half row maxima exchanged in the epilogue
constexpr int kFlagOff = kMaxOff + 2 * kBQ * 4; // per-key-tile "has masked keys" flags
constexpr int kMaskOff = kFlagOff + kMaxTiles * 4;

// TMEM columns: S/P[b] at 64 b (b = 0, 1; key half h at +32 h),
// O_h | l_h at 128 + 48 h (32 output columns + 16 row-sum columns).
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kOCol = 128;
constexpr uint32_t kOStride = 48;

constexpr uint32_t kNegPad = 0xF14AF14Au;  // bf16x2 (-1e30, -1e30)

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

// Warp-uniform bounded wait: the whole warp continues only if every lane saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, unsigned int *status, unsigned code) {
  return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, status, code));
}

template <bool kMulti>
__global__ void __launch_bounds__(kThreads, 2)
    tri_flash_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_bias,
                        const TcArgs args) {
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
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(o_free + 1);
  float *row_max = reinterpret_cast<float *>(smem + kMaxOff);  // [2 heads parity][2 halves][128]
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
    tc::fence_mbar_init();
  }
  // Ones block read as V's second N block (its swizzle is irrelevant: every element is 1).
  for (int i = tid; i < kVBytes / 16; i += kThreads)
    *reinterpret_cast<uint4 *>(smem + kOnesOff + i * 16) = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  // The ones block is read by the MMA (async proxy).
  tc::fence_proxy_async_smem();
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
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16(128, kBK, false, false);
      constexpr uint32_t idesc_pv = tc::idesc_bf16(128, 48, false, true);
      const uint32_t q_addr = tc::smem_u32(smem + kQOff);
      const uint32_t ones_addr = tc::smem_u32(smem + kOnesOff);
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
          const uint32_t lbo = ones_addr - v_addr;
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
          uint32_t o[32], l16[16];
          tc::tmem_ld_32x32b_x32(o_base, o);
          tc::tmem_ld_32x32b_x16(o_base + 32, l16);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
#pragma unroll
          for (int i = 0; i < 16; ++i) l16[i] = __float_as_uint(__uint_as_float(l16[i]) * alpha);
          tc::tmem_st_32x32b_x16(o_base, *reinterpret_cast<const uint32_t(*)[16]>(&o[0]));
          tc::tmem_st_32x32b_x16(o_base + 16, *reinterpret_cast<const uint32_t(*)[16]>(&o[16]));
          tc::tmem_st_32x32b_x16(o_base + 32, l16);
        }
        if (first || grow) m_ref = m_tile;
        const float ml = m_ref * kLog2e;
        uint32_t p[16];
#pragma unroll
        for (int pr = 0; pr < 16; ++pr) {
          float x0 = bf16_lo(t[pr]), x1 = bf16_hi(t[pr]);
          fma_f32x2(x0, x1, kLog2e, -ml);
          p[pr] = cvt_bf16x2(fast_exp2(x0), fast_exp2(x1));
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
      uint4 gate[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
      if (qi < n) {
        const uint4 *g4 = reinterpret_cast<const uint4 *>(args.g + pair * args.ld + h * kD + half * 16);
        gate[0] = g4[0];
        gate[1] = g4[1];
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
      const float m_other = rmax[(half ^ 1) * kBQ + row];
      // After the exchange the next head's epilogue may rewrite rmax: every warp
      // has read its partner's value before any warp leaves this barrier pair.
      if (kMulti) asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
      if (!ok || !(ok = warp_wait(o_full, hl & 1, args.status, 0x20A))) continue;
      tc::tc_fence_after();
      uint32_t o0[16], o1[16], l0, l1;  // row sums: column 32 of each half's accumulator
      tc::tmem_ld_32x32b_x16(lane_base + kOCol + half * 16, o0);
      tc::tmem_ld_32x32b_x16(lane_base + kOCol + kOStride + half * 16, o1);
      tc::tmem_ld_32x32b_x1(lane_base + kOCol + 32, l0);
      tc::tmem_ld_32x32b_x1(lane_base + kOCol + kOStride + 32, l1);
      tc::tmem_ld_wait();
      // O has been read: the next head's first P.V may overwrite it.
      if (kMulti && hl + 1 < hpc) {
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(o_free);
      }
      const float m0 = half == 0 ? m_ref : m_other, m1 = half == 0 ? m_other : m_ref;
      const float m = fmaxf(m0, m1);
      const float a0 = fast_exp2((m0 - m) * kLog2e), a1 = fast_exp2((m1 - m) * kLog2e);
      if (qi < n) {
        const float inv = fast_rcp(__uint_as_float(l0) * a0 + __uint_as_float(l1) * a1);
        uint4 *o4 = reinterpret_cast<uint4 *>(args.out + pair * args.out_ld + h * kD + half * 16);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 gv = gate[c];
          const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = c * 8 + e * 2;
            const float v0 = (__uint_as_float(o0[d]) * a0 + __uint_as_float(o1[d]) * a1) * inv;
            const float v1 = (__uint_as_float(o0[d + 1]) * a0 + __uint_as_float(o1[d + 1]) * a1) * inv;
            const float g0 = bf16_lo(gw[e]), g1 = bf16_hi(gw[e]);  // bf16(sigmoid(g)) from the projection
            w[e] = pack_bf16x2(bf16r(v0) * g0, bf16r(v1) * g1);
          }
          o4[c] = make_uint4(w[0], w[1], w[2], w[3]);
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

extern "C" int bl_triangle_attention(const void *q, const void *k, const void *v, const void *g, int64_t ld,
                                        int64_t so, int64_t si, const void *bias, int64_t bias_ld, int64_t bias_hs,
                                        const float *mask, int64_t ms_o, int64_t ms_k, float inf, int64_t heads,
                                        int64_t head_dim, int64_t n, int64_t n_outer, void *out, int64_t out_ld,
                                        void *stream) {
  BL_REQUIRE(head_dim == kD && heads == kHeads, "bl_triangle_attention: 4 heads x 32 supported");
  BL_REQUIRE(n >= 0 && n_outer >= 0 && n_outer <= n, "bl_triangle_attention: bad shape");
  if (n == 0 || n_outer == 0) return BL_OK;
  BL_REQUIRE(n <= kMaxTiles * kBK, "bl_triangle_attention: at most 4096 tokens");
  BL_REQUIRE(q && k && v && g && bias && mask && out, "bl_triangle_attention: null pointer");
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
  TcArgs args;
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
  auto kernel = hpc > 1 ? tri_flash_tc_kernel<true> : tri_flash_tc_kernel<false>;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), 232448));
  dim3 grid(unsigned(q_tiles * (kHeads / hpc)), unsigned(n_outer));
  kernel<<<grid, kThreads, smem, as_stream(stream)>>>(map_q, map_k, map_v, map_bias, args);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
