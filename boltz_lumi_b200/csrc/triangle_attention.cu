// Flash triangle attention (starting and ending node) with the upstream bf16
// rounding points and the fused sigmoid output gate.
//
// For every outer row a of the pair tensor, head h and query b:
//   s(b, c) = bf16(q_s(a, b) . k(a, c))                    q_s = bf16(q / sqrt(d))
//   t(b, c) = bf16(bf16(s + inf * (mask(a, c) - 1)) + bias(h, b, c))
//   o(a, b) = bf16(sum_c softmax_c(t) v(a, c))
//   out(a, b) = bf16(o * bf16(sigmoid(g(a, b))))
// This is the reference's ordered_triangle_forward (triangle.py:32-104 and
// kernels/triangle_softmax.py:90-113) plus upstream _wrap_up's gate, without
// materialising the [I, H, N, N] scores.  The ending node is the same
// computation on z transposed; the caller expresses it through row strides
// (pair row of (outer, inner) = outer * so + inner * si) and a transposed bias
// plane, so no transposed copy of z or of q/k/v is made.
//
// Cost model: head dim 32 makes the core exp/issue-bound (N^3 H exponentials
// at 16 MUFU ops/clk/SM vs 4 N^3 H d flops), so the two small contractions
// stay on mma.sync m16n8k16 and the per-score work is kept minimal:
//   cvt.rn.bf16x2 (s) -> add.bf16x2 (mask; skipped on key tiles without
//   masked keys) -> add.bf16x2 (bias, loaded with ldmatrix in fragment
//   layout) -> max.bf16x2 -> one fp32 FFMA + MUFU.EX2 per score -> cvt = P
// (measured on B200: packed ex2.bf16x2 costs two MUFU ops, so the exponent
// runs in fp32, which also keeps t*log2(e) exact).  P feeds the P.V mma
// directly and the row sums come from one extra mma against a ones fragment.
#include "common.cuh"

namespace bl {
namespace {

constexpr int kD = 32;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kBQ = kWarps * 16;  // 128 queries per CTA
constexpr int kBK = 64;           // keys per tile
constexpr int kBiasLd = kBK + 8;  // padded smem row (144 B): conflict-free fragment reads
constexpr int kHeadsPerRow = 4;   // heads (grid.x = heads * query tiles)
constexpr int kMaxTiles = 64;     // key tiles per row: n <= 4096

struct FlashArgs {
  const __nv_bfloat16 *q, *k, *v, *g;
  int64_t ld;      // elements per pair row of q/k/v/g; head h at columns [h*32, h*32+32)
  int64_t so, si;  // pair row of (outer, inner)
  const __nv_bfloat16 *bias;  // bias(h, q, k) at bias + h*bias_hs + q*bias_ld + k
  int64_t bias_ld, bias_hs;
  const float *mask;  // mask(outer, key) at mask + outer*ms_o + key*ms_k
  int64_t ms_o, ms_k;
  float inf;
  float q_divisor;
  __nv_bfloat16 *out;
  int64_t out_ld;
  int n;
};

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Packed bf16x2 arithmetic (each result rounded once to nearest-even).
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
__device__ __forceinline__ uint32_t sub_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t fma_bf16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t ex2_bf16x2(uint32_t a) {
  uint32_t r;
  asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(r) : "r"(a));
  return r;
}
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t splat_lo(uint32_t v) { return (v & 0xffffu) | (v << 16); }
__device__ __forceinline__ uint32_t splat_hi(uint32_t v) { return (v >> 16) | (v & 0xffff0000u); }

constexpr uint32_t kOnes = 0x3F803F80u;      // bf16x2 (1, 1)
constexpr uint32_t kNegInf = 0xFF80FF80u;    // bf16x2 (-inf, -inf): max identity
// Padding keys get -1e30 rather than -inf so (t - m) log2(e) stays finite in
// the two-term fma (inf - inf would give NaN); ex2 of it is exactly 0.
constexpr uint32_t kNegPad = 0xF14AF14Au;    // bf16x2 (-1.0003e30, -1.0003e30)
// log2(e) as an unbiased two-term bf16 constant: c1 = bf16(log2 e), c2 = bf16(log2 e - c1).
constexpr uint32_t kLog2eHi = 0x3FB93FB9u;   // 1.4453125
constexpr uint32_t kLog2eLo = 0xBB2CBB2Cu;   // -0.00262451171875

// [rows][32] bf16 tile, 4 chunks of 16 B per row, chunk c of row r stored at
// c ^ ((r >> 1) & 3): conflict-free for ldmatrix row groups of 8.
__device__ __forceinline__ int qkv_chunk_offset(int row, int chunk) {
  return row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4);
}

struct Smem {
  alignas(128) __nv_bfloat16 q[kBQ * kD];
  alignas(128) __nv_bfloat16 k[2][kBK * kD];
  alignas(128) __nv_bfloat16 v[2][kBK * kD];
  alignas(128) __nv_bfloat16 bias[2][kBQ * kBiasLd];
  int tile_masked[kMaxTiles];
  // followed by the per-key mask bias of this outer row (bf16, dynamic)
};

__global__ void __launch_bounds__(kThreads, 2) tri_flash_kernel(const FlashArgs args) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  __nv_bfloat16 *mask_bias = reinterpret_cast<__nv_bfloat16 *>(smem_raw + sizeof(Smem));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = args.n;
  // Heads of one query tile are adjacent in the grid: they read the same pair rows.
  const int h = blockIdx.x % kHeadsPerRow;
  const int q0 = (blockIdx.x / kHeadsPerRow) * kBQ;
  const int64_t outer = blockIdx.y;
  const int col0 = h * kD;
  const int n_tiles = (n + kBK - 1) / kBK;

  // Per-key additive mask of this outer row (bf16; for mask in {0, 1} adding it
  // rounds exactly like adding the fp32 value) and a flag per key tile that
  // says whether any key of the tile is masked at all.
  if (tid < kMaxTiles) sm.tile_masked[tid] = 0;
  __syncthreads();
  for (int key = tid; key < n_tiles * kBK; key += kThreads) {
    float mb = key < n ? args.inf * (args.mask[outer * args.ms_o + int64_t(key) * args.ms_k] - 1.f) : 0.f;
    mask_bias[key] = __float2bfloat16_rn(mb);
    if (mb != 0.f) atomicOr(&sm.tile_masked[key / kBK], 1);
  }

  // Per-thread load addresses: K/V row (tid / 4, 16-byte chunk tid % 4) and
  // four bias chunks (rows tid / 8 + 32 i, chunk tid % 8), advanced per tile.
  const int kv_row = tid >> 2, kv_chunk = tid & 3;
  const int64_t kv_base = (outer * args.so + int64_t(kv_row) * args.si) * args.ld + col0 + kv_chunk * 8;
  const int64_t kv_step = int64_t(kBK) * args.si * args.ld;
  const int b_row = tid >> 3, b_chunk = tid & 7;
  const __nv_bfloat16 *bias_base = args.bias + int64_t(h) * args.bias_hs + int64_t(q0 + b_row) * args.bias_ld + b_chunk * 8;
  const int64_t bias_rows32 = 32 * args.bias_ld;

  for (int c = tid; c < kBQ * 4; c += kThreads) {
    int row = c >> 2, chunk = c & 3;
    int qi = q0 + row;
    bool valid = qi < n;
    const __nv_bfloat16 *src =
        valid ? args.q + (outer * args.so + int64_t(qi) * args.si) * args.ld + col0 + chunk * 8 : args.q;
    cp_async16(reinterpret_cast<uint8_t *>(sm.q) + qkv_chunk_offset(row, chunk), src, valid);
  }
  auto load_tile = [&](int tile, int buf) {
    const int k0 = tile * kBK;
    const bool kv_valid = k0 + kv_row < n;
    const int64_t off = kv_base + tile * kv_step;
    cp_async16(reinterpret_cast<uint8_t *>(sm.k[buf]) + qkv_chunk_offset(kv_row, kv_chunk),
               kv_valid ? args.k + off : args.k, kv_valid);
    cp_async16(reinterpret_cast<uint8_t *>(sm.v[buf]) + qkv_chunk_offset(kv_row, kv_chunk),
               kv_valid ? args.v + off : args.v, kv_valid);
    const bool col_valid = k0 + b_chunk * 8 < args.bias_ld;
#pragma unroll
    for (int i = 0; i < kBQ / 32; ++i) {
      const bool valid = col_valid && q0 + b_row + 32 * i < n;
      cp_async16(sm.bias[buf] + (b_row + 32 * i) * kBiasLd + b_chunk * 8,
                 valid ? bias_base + i * bias_rows32 + k0 : args.bias, valid);
    }
  };

  load_tile(0, 0);
  cp_async_commit();

  const int g = lane >> 2, t = lane & 3;
  float o_acc[4][4];
  float l_acc[4];  // row sums from the ones-fragment mma: [0] row g, [2] row g + 8
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    l_acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) o_acc[i][j] = 0.f;
  }
  float m_run0 = -INFINITY, m_run1 = -INFINITY;  // running maxima of rows g, g + 8
  uint32_t qf[2][4];
  constexpr float kLog2e = 1.4426950408889634f;

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < n_tiles) load_tile(tile + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    if (tile == 0) {
      // Q fragments, scaled and re-rounded as upstream's in-place q /= sqrt(d).
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int chunk = ks * 2 + (lane >> 4);
        ldmatrix_x4(qf[ks], reinterpret_cast<uint8_t *>(sm.q) + qkv_chunk_offset(row, chunk));
#pragma unroll
        for (int r = 0; r < 4; ++r)
          qf[ks][r] = pack_bf16x2(__fdiv_rn(bf16_lo(qf[ks][r]), args.q_divisor),
                                  __fdiv_rn(bf16_hi(qf[ks][r]), args.q_divisor));
      }
    }

    // S = Q K^T for 64 keys (8 n-tiles of 8 keys) and the ordered rounding in
    // bf16x2: sp[j][0] = row g keys (2t, 2t+1), sp[j][1] = row g + 8.
    const int k0 = tile * kBK;
    const bool masked = sm.tile_masked[tile] != 0;
    uint32_t sp[8][2];
    uint32_t tmax0 = kNegInf, tmax1 = kNegInf;
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
      // Bias fragments of n-tiles 2jp, 2jp+1: [0] row g, [1] row g+8, [2]/[3] next n-tile.
      uint32_t bf[4];
      ldmatrix_x4(bf, sm.bias[buf] + (warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kBiasLd +
                          (jp * 2 + (lane >> 4)) * 8);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int j = jp * 2 + half;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t kf[4];
        ldmatrix_x4(kf, reinterpret_cast<uint8_t *>(sm.k[buf]) + qkv_chunk_offset(j * 8 + (lane & 7), lane >> 3));
        mma_bf16(s, qf[0], kf[0], kf[1]);
        mma_bf16(s, qf[1], kf[2], kf[3]);
        uint32_t p0 = cvt_bf16x2(s[0], s[1]), p1 = cvt_bf16x2(s[2], s[3]);
        if (masked) {
          const uint32_t mb = *reinterpret_cast<const uint32_t *>(mask_bias + k0 + j * 8 + 2 * t);
          p0 = add_bf16x2(p0, mb);
          p1 = add_bf16x2(p1, mb);
        }
        sp[j][0] = add_bf16x2(p0, bf[half * 2 + 0]);
        sp[j][1] = add_bf16x2(p1, bf[half * 2 + 1]);
      }
    }
    if (k0 + kBK > n) {  // last tile: keys past n contribute nothing
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int key = k0 + j * 8 + 2 * t;
        const uint32_t keep = (key < n ? 0x0000ffffu : 0u) | (key + 1 < n ? 0xffff0000u : 0u);
        sp[j][0] = (sp[j][0] & keep) | (kNegPad & ~keep);
        sp[j][1] = (sp[j][1] & keep) | (kNegPad & ~keep);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      tmax0 = max_bf16x2(tmax0, sp[j][0]);
      tmax1 = max_bf16x2(tmax1, sp[j][1]);
    }
    // Row maxima packed as (row g, row g + 8), reduced over the 4-thread quad.
    uint32_t rmax = max_bf16x2((tmax0 & 0xffffu) | (tmax1 << 16), (tmax0 >> 16) | (tmax1 & 0xffff0000u));
    rmax = max_bf16x2(rmax, __shfl_xor_sync(0xffffffffu, rmax, 1));
    rmax = max_bf16x2(rmax, __shfl_xor_sync(0xffffffffu, rmax, 2));
    const float m_new0 = fmaxf(m_run0, bf16_lo(rmax)), m_new1 = fmaxf(m_run1, bf16_hi(rmax));
    if (m_new0 != m_run0 || m_new1 != m_run1) {
      const float alpha0 = fast_exp2((m_run0 - m_new0) * kLog2e);
      const float alpha1 = fast_exp2((m_run1 - m_new1) * kLog2e);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o_acc[i][0] *= alpha0, o_acc[i][1] *= alpha0;
        o_acc[i][2] *= alpha1, o_acc[i][3] *= alpha1;
      }
      l_acc[0] *= alpha0, l_acc[1] *= alpha0, l_acc[2] *= alpha1, l_acc[3] *= alpha1;
      m_run0 = m_new0, m_run1 = m_new1;
    }
    // P = exp2(t log2 e - m log2 e) in fp32 (the bf16 scores convert exactly),
    // rounded to bf16x2 as the A fragments of P.V.
    const float ml0 = m_run0 * kLog2e, ml1 = m_run1 * kLog2e;
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e0 = fast_exp2(fmaf(bf16_lo(sp[j][0]), kLog2e, -ml0));
      const float e1 = fast_exp2(fmaf(bf16_hi(sp[j][0]), kLog2e, -ml0));
      const float e2 = fast_exp2(fmaf(bf16_lo(sp[j][1]), kLog2e, -ml1));
      const float e3 = fast_exp2(fmaf(bf16_hi(sp[j][1]), kLog2e, -ml1));
      const int kk = j >> 1, hi = j & 1;
      pf[kk][hi * 2 + 0] = cvt_bf16x2(e0, e1);
      pf[kk][hi * 2 + 1] = cvt_bf16x2(e2, e3);
    }
    // O += P V (4 k-steps of 16 keys x 4 n-tiles of 8 channels); l += P 1.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t vf[4];
        int row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int chunk = np * 2 + (lane >> 4);
        ldmatrix_x4_trans(vf, reinterpret_cast<uint8_t *>(sm.v[buf]) + qkv_chunk_offset(row, chunk));
        mma_bf16(o_acc[np * 2 + 0], a, vf[0], vf[1]);
        mma_bf16(o_acc[np * 2 + 1], a, vf[2], vf[3]);
      }
      mma_bf16(l_acc, a, kOnes, kOnes);
    }
    __syncthreads();
  }

  // Normalise, round, gate, store.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = q0 + warp * 16 + g + r * 8;
    if (qi >= n) continue;
    const float inv = 1.f / l_acc[r * 2];
    const int64_t pair = outer * args.so + int64_t(qi) * args.si;
    const __nv_bfloat16 *grow = args.g + pair * args.ld + col0;
    __nv_bfloat16 *orow = args.out + pair * args.out_ld + col0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = i * 8 + 2 * t;
      const uint32_t gv = *reinterpret_cast<const uint32_t *>(grow + d);
      float o0 = bf16r(o_acc[i][r * 2 + 0] * inv), o1 = bf16r(o_acc[i][r * 2 + 1] * inv);
      float g0 = bf16r(sigmoidf_fast(bf16_lo(gv))), g1 = bf16r(sigmoidf_fast(bf16_hi(gv)));
      *reinterpret_cast<uint32_t *>(orow + d) = pack_bf16x2(o0 * g0, o1 * g1);
    }
  }
}

// Bias planes from the pair-major projection: natural[h][r][s] = tb[r*n + s][h]
// (starting node) or transposed[h][s][r] (ending node), rows padded to `ld`
// with zeros.
__global__ void bias_planes_kernel(const __nv_bfloat16 *tb, int64_t tb_ld, int heads, int n, int transpose,
                                   __nv_bfloat16 *out, int64_t ld) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int r0 = blockIdx.y * 32, s0 = blockIdx.x * 32, h = blockIdx.z;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int y = ty; y < 32; y += 8) {
    int r = r0 + y, s = s0 + tx;
    tile[y][tx] = (r < n && s < n) ? tb[(int64_t(r) * n + s) * tb_ld + h] : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  __nv_bfloat16 *plane = out + int64_t(h) * n * ld;
  for (int y = ty; y < 32; y += 8) {
    if (!transpose) {
      int r = r0 + y, s = s0 + tx;
      if (r < n && s < ld) plane[int64_t(r) * ld + s] = tile[y][tx];
    } else {
      int row = s0 + y, col = r0 + tx;  // out[s][r]
      if (row < n && col < ld) plane[int64_t(row) * ld + col] = tile[tx][y];
    }
  }
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_triangle_bias_planes(const void *tb, int64_t tb_ld, int64_t heads, int64_t n, int transpose,
                                       void *out, int64_t ld, void *stream) {
  BL_REQUIRE(n >= 0 && heads > 0 && heads <= 64, "bl_triangle_bias_planes: bad shape");
  if (n == 0) return BL_OK;
  BL_REQUIRE(tb && out, "bl_triangle_bias_planes: null pointer");
  BL_REQUIRE(ld >= n && ld <= (n + 31) / 32 * 32 && tb_ld >= heads, "bl_triangle_bias_planes: bad leading dimension");
  dim3 grid((n + 31) / 32, (n + 31) / 32, heads);
  bias_planes_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const __nv_bfloat16 *>(tb), tb_ld, int(heads),
                                                         int(n), transpose, static_cast<__nv_bfloat16 *>(out), ld);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

extern "C" int bl_triangle_attention(const void *q, const void *k, const void *v, const void *g, int64_t ld,
                                     int64_t so, int64_t si, const void *bias, int64_t bias_ld, int64_t bias_hs,
                                     const float *mask, int64_t ms_o, int64_t ms_k, float inf, int64_t heads,
                                     int64_t head_dim, int64_t n, void *out, int64_t out_ld, void *stream) {
  BL_REQUIRE(head_dim == kD, "bl_triangle_attention: head_dim must be 32");
  BL_REQUIRE(heads == kHeadsPerRow, "bl_triangle_attention: 4 heads supported");
  BL_REQUIRE(n >= 0, "bl_triangle_attention: bad shape");
  if (n == 0) return BL_OK;
  BL_REQUIRE(n <= kMaxTiles * kBK, "bl_triangle_attention: at most 4096 tokens");
  BL_REQUIRE(q && k && v && g && bias && mask && out, "bl_triangle_attention: null pointer");
  BL_REQUIRE(ld % 8 == 0 && out_ld % 2 == 0 && bias_ld % 8 == 0 && bias_ld >= n,
             "bl_triangle_attention: leading dimensions must keep 16-byte rows");
  BL_REQUIRE(aligned_to(q, 16) && aligned_to(k, 16) && aligned_to(v, 16) && aligned_to(bias, 16) &&
                 aligned_to(g, 4) && aligned_to(out, 4),
             "bl_triangle_attention: misaligned pointer");
  BL_REQUIRE(bias_hs % 8 == 0, "bl_triangle_attention: bias head stride must be a multiple of 8");
  FlashArgs args;
  args.q = static_cast<const __nv_bfloat16 *>(q);
  args.k = static_cast<const __nv_bfloat16 *>(k);
  args.v = static_cast<const __nv_bfloat16 *>(v);
  args.g = static_cast<const __nv_bfloat16 *>(g);
  args.ld = ld, args.so = so, args.si = si;
  args.bias = static_cast<const __nv_bfloat16 *>(bias);
  args.bias_ld = bias_ld, args.bias_hs = bias_hs;
  args.mask = mask, args.ms_o = ms_o, args.ms_k = ms_k;
  args.inf = inf;
  args.q_divisor = sqrtf(float(head_dim));
  args.out = static_cast<__nv_bfloat16 *>(out);
  args.out_ld = out_ld;
  args.n = int(n);
  const int n_tiles = int((n + kBK - 1) / kBK);
  const size_t smem = sizeof(Smem) + size_t(n_tiles) * kBK * sizeof(__nv_bfloat16);
  BL_REQUIRE(smem <= 227 * 1024, "bl_triangle_attention: too many tokens for the mask buffer");
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(tri_flash_kernel), int(227 * 1024)));
  dim3 grid(unsigned((n + kBQ - 1) / kBQ * kHeadsPerRow), unsigned(n));
  tri_flash_kernel<<<grid, kThreads, smem, as_stream(stream)>>>(args);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
