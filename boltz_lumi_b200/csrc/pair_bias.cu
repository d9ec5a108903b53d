// Pair bias of the single-track attention in one pass over z (fp32):
//
//   bias[h][r] = sum_c LayerNorm(z[r])[c] * w[h][c]        h < heads <= 16, r < rows
//
// i.e. proj_z = LayerNorm(c_z) -> Linear(c_z, heads, bias=False) ->
// permute to [heads, N, N] of upstream AttentionPairBias (the Pairformer
// block's single track, fp32 without autocast).  Unfused: an LN pass writing
// the normalised fp32 pair tensor (128 MiB at N = 512), a GEMM reading it
// back, and a strided permute consumed by a non-vectorised add.
//
// Two threads per pair row.  A CTA stages 128 rows (64 KB of fp32) in shared
// memory with coalesced 16-byte asynchronous copies; thread pair (2 r, 2 r + 1)
// takes row r, each thread the alternate 16-byte chunks of its 128 channels
// (chunks 2 i and 2 i + 1).  Each computes partial row statistics and partial
// heads dot products from shared memory (packed fp32x2 FMA against weights
// read as same-address broadcasts); one shuffle joins the halves.  Rows and
// the transposed weights are XOR-swizzled by 16-byte chunk so that the eight
// lanes of a shared-memory phase (four rows x two halves) hit eight distinct
// bank groups.
#include "common.cuh"

namespace bl {
namespace {

constexpr int kHeads = 16;
constexpr int kC = 128;
constexpr int kRowsPerCta = 128;
constexpr int kThreads = 2 * kRowsPerCta;

// Row r's 16-byte chunk k (channels 4 k .. 4 k + 3) sits at chunk k ^ (2 (r & 3)).
__device__ __forceinline__ int row_chunk(int r, int k) { return k ^ ((r & 3) << 1); }
// Weight row c (16 heads = four 16-byte chunks): chunk q sits at q ^ ((c >> 2) & 1).
__device__ __forceinline__ int w_chunk(int c, int q) { return q ^ ((c >> 2) & 1); }

__global__ void __launch_bounds__(kThreads) pair_bias_kernel(const float *z, int64_t rows, const float *ln_w,
                                                             const float *ln_b, float eps, const float *w,
                                                             int heads, float *out) {
  extern __shared__ float4 smem4[];
  float *tile = reinterpret_cast<float *>(smem4);  // [128][128], chunk-swizzled rows
  float *ws = tile + kRowsPerCta * kC;             // [kC][kHeads]: w transposed, zero past `heads`, swizzled
  float *lnw = ws + kC * kHeads, *lnb = lnw + kC;
  const uint32_t ws_addr = static_cast<uint32_t>(__cvta_generic_to_shared(ws));
  const int t = threadIdx.x;
  for (int i = t; i < kC * kHeads; i += kThreads) {
    const int c = i / kHeads, h = i % kHeads;
    ws[c * kHeads + 4 * w_chunk(c, h >> 2) + (h & 3)] = h < heads ? w[h * kC + c] : 0.f;
  }
  for (int c = t; c < kC; c += kThreads) {
    lnw[c] = ln_w ? ln_w[c] : 1.f;
    lnb[c] = ln_b ? ln_b[c] : 0.f;
  }
  const int row = t >> 1, half = t & 1;
  for (int64_t r0 = int64_t(blockIdx.x) * kRowsPerCta; r0 < rows; r0 += int64_t(gridDim.x) * kRowsPerCta) {
    const int valid = rows - r0 < kRowsPerCta ? int(rows - r0) : kRowsPerCta;
    __syncthreads();  // previous tile's readers are done (and the constants are in place)
    // Coalesced staging with asynchronous copies: 32 consecutive threads copy
    // one 512-byte row; rows past the end are zero-filled.
    const float *src = z + r0 * kC;
#pragma unroll 8
    for (int i = t; i < kRowsPerCta * (kC / 4); i += kThreads) {
      const int r = i / (kC / 4), k = i % (kC / 4);
      const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(tile + r * kC + 4 * row_chunk(r, k)));
      const float *g = src + (r < valid ? i * 4 : 0);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(g), "r"(r < valid ? 16 : 0)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const float *rowp = tile + row * kC;
    // Statistics: mean, then the mean of squared deviations (fp32, four
    // partial sums per thread, joined with the partner thread's).
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int i = 0; i < kC / 8; ++i) {
      const float4 v = *reinterpret_cast<const float4 *>(rowp + 4 * row_chunk(row, 2 * i + half));
      s4[0] += v.x, s4[1] += v.y, s4[2] += v.z, s4[3] += v.w;
    }
    float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    const float mean = sum * (1.f / kC);
    float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int i = 0; i < kC / 8; ++i) {
      const float4 v = *reinterpret_cast<const float4 *>(rowp + 4 * row_chunk(row, 2 * i + half));
      const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
      q4[0] += d0 * d0, q4[1] += d1 * d1, q4[2] += d2 * d2, q4[3] += d3 * d3;
    }
    float sq = (q4[0] + q4[1]) + (q4[2] + q4[3]);
    sq += __shfl_xor_sync(0xffffffffu, sq, 1);
    const float rstd = rsqrtf(sq * (1.f / kC) + eps);
    // Heads in packed pairs (fma.rn.f32x2) over this thread's 64 channels.
    uint64_t acc2[kHeads / 2];
#pragma unroll
    for (int h = 0; h < kHeads / 2; ++h) acc2[h] = 0;
#pragma unroll 2
    for (int i = 0; i < kC / 8; ++i) {
      const int c = 4 * (2 * i + half);
      const float4 v = *reinterpret_cast<const float4 *>(rowp + 4 * row_chunk(row, 2 * i + half));
      const float4 gw = *reinterpret_cast<const float4 *>(lnw + c), gb = *reinterpret_cast<const float4 *>(lnb + c);
      const float y[4] = {(v.x - mean) * rstd * gw.x + gb.x, (v.y - mean) * rstd * gw.y + gb.y,
                          (v.z - mean) * rstd * gw.z + gb.z, (v.w - mean) * rstd * gw.w + gb.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint64_t yy = dup2(y[e]);
        const uint32_t wc = ws_addr + uint32_t((c + e) * kHeads * 4);  // two addresses per warp (the halves)
#pragma unroll
        for (int q = 0; q < kHeads / 4; ++q) {
          uint64_t w01, w23;
          lds_v2b64(wc + 16 * w_chunk(c + e, q), w01, w23);
          ffma2(acc2[2 * q], yy, w01);
          ffma2(acc2[2 * q + 1], yy, w23);
        }
      }
    }
    // Join the halves; thread `half` writes heads 8 half .. 8 half + 7.
    float hv[kHeads];
#pragma unroll
    for (int h = 0; h < kHeads / 2; ++h) {
      hv[2 * h] = lo_f(acc2[h]) + __shfl_xor_sync(0xffffffffu, lo_f(acc2[h]), 1);
      hv[2 * h + 1] = hi_f(acc2[h]) + __shfl_xor_sync(0xffffffffu, hi_f(acc2[h]), 1);
    }
    if (row < valid) {
#pragma unroll
      for (int e = 0; e < kHeads / 2; ++e) {
        const int h = 8 * half + e;
        if (h < heads) out[int64_t(h) * rows + r0 + row] = half ? hv[8 + e] : hv[e];
      }
    }
  }
}

constexpr int kSmemBytes = (kRowsPerCta * kC + kC * kHeads + 2 * kC) * 4;

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_pair_bias(const float *z, int64_t rows, const float *ln_weight, const float *ln_bias, float eps,
                            const float *w, int64_t heads, float *out, void *stream) {
  BL_REQUIRE(rows >= 0 && heads >= 1 && heads <= kHeads, "bl_pair_bias: rows >= 0 and 1 <= heads <= 16");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(z && w && out && eps > 0.f, "bl_pair_bias: null pointer or eps <= 0");
  BL_REQUIRE(aligned_to(z, 16), "bl_pair_bias: z must be 16-byte aligned");
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(pair_bias_kernel), kSmemBytes));
  const int64_t tiles = (rows + kRowsPerCta - 1) / kRowsPerCta;
  const int64_t cap = int64_t(num_sms()) * 3;  // three 75 KB CTAs per SM
  pair_bias_kernel<<<int(tiles < cap ? tiles : cap), kThreads, kSmemBytes, as_stream(stream)>>>(
      z, rows, ln_weight, ln_bias, eps, w, int(heads), out);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
