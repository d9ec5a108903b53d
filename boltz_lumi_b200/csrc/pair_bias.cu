// Pair bias of the single-track attention in one pass over z (fp32):
//
//   bias[h][r] = sum_c LayerNorm(z[r])[c] * w[h][c]        h < 16, r < rows
//
// i.e. proj_z = LayerNorm(c_z) -> Linear(c_z, heads, bias=False) ->
// permute to [heads, N, N] of upstream AttentionPairBias (the Pairformer
// block's single track, fp32 without autocast).  Unfused: an LN pass writing
// the normalised fp32 pair tensor (128 MiB at N = 512), a GEMM reading it
// back, and a strided permute consumed by a non-vectorised add.
//
// One warp per two rows: each lane holds 4 channels of both rows and the
// matching 4 weights of every head; the 32 partial head sums are reduced
// with a butterfly reduce-scatter so lane L ends with (row L / 16, head L % 16).
#include "common.cuh"

namespace bl {
namespace {

constexpr int kHeads = 16;

template <int HALF> __device__ __forceinline__ void reduce_scatter_step(float (&v)[32], int lane) {
  const bool upper = (lane & HALF) != 0;
#pragma unroll
  for (int i = 0; i < HALF; ++i) {
    const float send = upper ? v[i] : v[i + HALF];
    const float keep = upper ? v[i + HALF] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, HALF);
  }
}

__global__ void __launch_bounds__(256) pair_bias_kernel(const float *z, int64_t rows, const float *ln_w,
                                                        const float *ln_b, float eps, const float *w, int heads,
                                                        float *out) {
  const int lane = threadIdx.x & 31;
  float lw[4], lb[4], wh[kHeads][4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    lw[e] = ln_w ? ln_w[lane * 4 + e] : 1.f;
    lb[e] = ln_b ? ln_b[lane * 4 + e] : 0.f;
  }
#pragma unroll
  for (int h = 0; h < kHeads; ++h) {
    const float4 x = h < heads ? *reinterpret_cast<const float4 *>(w + h * 128 + lane * 4) : make_float4(0, 0, 0, 0);
    wh[h][0] = x.x, wh[h][1] = x.y, wh[h][2] = x.z, wh[h][3] = x.w;
  }
  const int64_t pairs = (rows + 1) / 2;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t p = blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5); p < pairs; p += warps) {
    const int64_t r0 = 2 * p;
    float v[2][4];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float4 x = r0 + q < rows ? *reinterpret_cast<const float4 *>(z + (r0 + q) * 128 + lane * 4)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
      v[q][0] = x.x, v[q][1] = x.y, v[q][2] = x.z, v[q][3] = x.w;
    }
    float mean[2], var[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) mean[q] = (v[q][0] + v[q][1]) + (v[q][2] + v[q][3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int q = 0; q < 2; ++q) mean[q] += __shfl_xor_sync(0xffffffffu, mean[q], o);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      mean[q] *= 1.f / 128.f;
      float sq = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float d = v[q][e] - mean[q];
        sq += d * d;
      }
      var[q] = sq;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int q = 0; q < 2; ++q) var[q] += __shfl_xor_sync(0xffffffffu, var[q], o);
    float part[32];  // index q * 16 + h
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float rstd = rsqrtf(var[q] * (1.f / 128.f) + eps);
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = (v[q][e] - mean[q]) * rstd * lw[e] + lb[e];
#pragma unroll
      for (int h = 0; h < kHeads; ++h)
        part[q * 16 + h] = (y[0] * wh[h][0] + y[1] * wh[h][1]) + (y[2] * wh[h][2] + y[3] * wh[h][3]);
    }
    reduce_scatter_step<16>(part, lane);
    reduce_scatter_step<8>(part, lane);
    reduce_scatter_step<4>(part, lane);
    reduce_scatter_step<2>(part, lane);
    reduce_scatter_step<1>(part, lane);
    const int64_t row = r0 + (lane >> 4);
    const int h = lane & 15;
    if (row < rows && h < heads) out[int64_t(h) * rows + row] = part[0];
  }
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_pair_bias(const float *z, int64_t rows, const float *ln_weight, const float *ln_bias, float eps,
                            const float *w, int64_t heads, float *out, void *stream) {
  BL_REQUIRE(rows >= 0 && heads >= 1 && heads <= kHeads, "bl_pair_bias: rows >= 0 and 1 <= heads <= 16");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(z && w && out && eps > 0.f, "bl_pair_bias: null pointer or eps <= 0");
  BL_REQUIRE(aligned_to(z, 16) && aligned_to(w, 16), "bl_pair_bias: z and w must be 16-byte aligned");
  const int64_t pairs = (rows + 1) / 2;
  int64_t blocks = (pairs + 7) / 8, cap = int64_t(num_sms()) * 8;
  pair_bias_kernel<<<int(blocks < cap ? blocks : cap), 256, 0, as_stream(stream)>>>(z, rows, ln_weight, ln_bias, eps,
                                                                                   w, int(heads), out);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
