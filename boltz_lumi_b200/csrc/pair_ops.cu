// SwiGLU over the joint fc1|fc2 rows of the unfused pair transition (the
// shapes the fused transition kernel does not cover, and the allocation-free
// entry point).
#include "common.cuh"

namespace bl {
namespace {

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
