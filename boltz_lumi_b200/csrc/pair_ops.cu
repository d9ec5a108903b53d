// Pair-track layout kernels that sit between the tensor-core GEMMs of the
// triangle multiplication and the pair transition.
#include "common.cuh"

namespace bl {
namespace {

__device__ __forceinline__ float gate_value(float p, float g) { return bf16r(p * bf16r(sigmoidf_fast(g))); }

// Gate + mask the joint projection of a triangle multiplication and write the
// two operands as natural channel-first planes:
//   a[c][r][s] = bf16(bf16(p[r,s,c] * bf16(sigmoid(g[r,s,c]))) * mask[r,s])      c < 128
//   b[c][r][s] = same with channel 128 + c
// (multiplication_gate_hip.cu:16-20,41-42; einsum operands of multiplication.py).
// One CTA: one row r, 64 consecutive s, all 256 channels.
constexpr int kPlaneTile = 64;

__global__ void __launch_bounds__(256) pack_planes_kernel(const __nv_bfloat16 *pg, int64_t pg_ld, const float *mask,
                                                          int n, int64_t plane_ld, __nv_bfloat16 *a,
                                                          __nv_bfloat16 *b) {
  __shared__ __nv_bfloat16 tile[256][kPlaneTile + 2];
  const int r = blockIdx.y, s0 = blockIdx.x * kPlaneTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Each warp gates 8 pairs; lane covers channels 8*lane .. 8*lane+7 of p and g.
  for (int ps = warp; ps < kPlaneTile; ps += 8) {
    const int s = s0 + ps;
    float v[8];
    if (s < n) {
      const int64_t pair = int64_t(r) * n + s;
      const float m = mask[pair];
      const __nv_bfloat16 *row = pg + pair * pg_ld;
      uint4 pv = *reinterpret_cast<const uint4 *>(row + lane * 8);
      uint4 gv = *reinterpret_cast<const uint4 *>(row + 256 + lane * 8);
      const uint32_t *p32 = &pv.x, *g32 = &gv.x;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        v[2 * w] = bf16r(gate_value(bf16_lo(p32[w]), bf16_lo(g32[w])) * m);
        v[2 * w + 1] = bf16r(gate_value(bf16_hi(p32[w]), bf16_hi(g32[w])) * m);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) tile[lane * 8 + e][ps] = __float2bfloat16_rn(v[e]);
  }
  __syncthreads();
  // Each warp writes channel rows: 64 s values = 128 B per channel.
  const int64_t plane = int64_t(n) * plane_ld;
  for (int c = warp; c < 256; c += 8) {
    __nv_bfloat16 *dst = (c < 128 ? a + int64_t(c) * plane : b + int64_t(c - 128) * plane) + int64_t(r) * plane_ld;
    for (int ps = lane; ps < kPlaneTile; ps += 32) {
      const int s = s0 + ps;
      if (s < n) dst[s] = tile[c][ps];
      else if (s < plane_ld) dst[s] = __float2bfloat16_rn(0.f);
    }
  }
}

// out[r][c] = bf16(bf16(silu(x[r][c])) * x[r][w + c]) for the joint fc1|fc2
// projection of the pair transition (pair_transition.py:20-28, pair_hip.cu:12-17).
__global__ void swiglu_rows_vec_kernel(const __nv_bfloat16 *x, int64_t x_ld, int64_t rows, int width,
                                       __nv_bfloat16 *out, int64_t out_ld) {
  const int vecs = width / 8;
  const int64_t total = rows * vecs;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = t / vecs;
    const int c = int(t % vecs) * 8;
    uint4 av = *reinterpret_cast<const uint4 *>(x + row * x_ld + c);
    uint4 bv = *reinterpret_cast<const uint4 *>(x + row * x_ld + width + c);
    const uint32_t *a32 = &av.x, *b32 = &bv.x;
    uint4 r;
    uint32_t *r32 = &r.x;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      float a0 = bf16_lo(a32[w]), a1 = bf16_hi(a32[w]);
      float s0 = bf16r(a0 / (1.f + __expf(-a0))), s1 = bf16r(a1 / (1.f + __expf(-a1)));
      r32[w] = pack_bf16x2(s0 * bf16_lo(b32[w]), s1 * bf16_hi(b32[w]));
    }
    *reinterpret_cast<uint4 *>(out + row * out_ld + c) = r;
  }
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_trimul_pack_planes(const void *pg, int64_t pg_ld, const float *mask, int64_t n, int64_t plane_ld,
                                     void *a_planes, void *b_planes, void *stream) {
  BL_REQUIRE(n >= 0 && n <= 65535, "bl_trimul_pack_planes: bad token count");
  if (n == 0) return BL_OK;
  BL_REQUIRE(pg && mask && a_planes && b_planes, "bl_trimul_pack_planes: null pointer");
  BL_REQUIRE(pg_ld >= 512 && pg_ld % 8 == 0 && aligned_to(pg, 16), "bl_trimul_pack_planes: projection rows must be 16-byte aligned and hold p|g");
  BL_REQUIRE(plane_ld >= n, "bl_trimul_pack_planes: plane row stride too small");
  dim3 grid(unsigned((n + kPlaneTile - 1) / kPlaneTile), unsigned(n));
  pack_planes_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const __nv_bfloat16 *>(pg), pg_ld, mask, int(n),
                                                          plane_ld, static_cast<__nv_bfloat16 *>(a_planes),
                                                          static_cast<__nv_bfloat16 *>(b_planes));
  BL_LAUNCH_CHECK();
  return BL_OK;
}

extern "C" int bl_swiglu_rows(const void *x, int64_t x_ld, int64_t rows, int64_t width, void *out, int64_t out_ld,
                              void *stream) {
  BL_REQUIRE(rows >= 0 && width > 0, "bl_swiglu_rows: bad shape");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(x && out, "bl_swiglu_rows: null pointer");
  BL_REQUIRE(width % 8 == 0 && x_ld % 8 == 0 && out_ld % 8 == 0 && x_ld >= 2 * width && out_ld >= width &&
                 aligned_to(x, 16) && aligned_to(out, 16),
             "bl_swiglu_rows: rows must be 16-byte aligned multiples of 8 elements");
  int64_t total = rows * (width / 8);
  int64_t blocks = (total + 255) / 256, cap = int64_t(num_sms()) * 16;
  swiglu_rows_vec_kernel<<<int(blocks < cap ? blocks : cap), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16 *>(x), x_ld, rows, int(width), static_cast<__nv_bfloat16 *>(out), out_ld);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
