// LayerNorm kernels (K-LN of the reference, kernels/multiplication_hip.cu).
//
// Row-major: one warp per row, the row held in registers (128-bit loads for
// fp32, 64-bit for bf16), two-pass mean/variance with warp shuffles.
// Channel-first [128, M] -> [M, 128]: a 32-row tile is transposed through
// shared memory so both the plane reads and the row writes stay coalesced.
#include "common.cuh"

namespace bl {

template <typename T> struct Vec4;
template <> struct Vec4<float> {
  static __device__ __forceinline__ void load(const float *p, float v[4]) {
    float4 x = *reinterpret_cast<const float4 *>(p);
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
  }
  static __device__ __forceinline__ void store(float *p, const float v[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <> struct Vec4<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float v[4]) {
    uint2 x = *reinterpret_cast<const uint2 *>(p);
    v[0] = bf16_lo(x.x), v[1] = bf16_hi(x.x), v[2] = bf16_lo(x.y), v[3] = bf16_hi(x.y);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float v[4]) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  }
};

// cols == 128 * V exactly; vector-aligned rows.
template <typename Tin, typename Tout, int V>
__global__ void layernorm_rows_vec_kernel(const Tin *x, const float *w, const float *b, Tout *out, int64_t rows,
                                          float eps) {
  constexpr int C = 128 * V;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int64_t row = blockIdx.x * int64_t(warps) + (threadIdx.x >> 5); row < rows;
       row += int64_t(gridDim.x) * warps) {
    float v[V][4];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      Vec4<Tin>::load(x + row * C + j * 128 + lane * 4, v[j]);
      sum += (v[j][0] + v[j][1]) + (v[j][2] + v[j][3]);
    }
    const float mean = warp_sum(sum) * (1.f / C);
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float d = v[j][e] - mean;
        sq += d * d;
      }
    const float rstd = rsqrtf(warp_sum(sq) * (1.f / C) + eps);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float r[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int c = j * 128 + lane * 4 + e;
        float y = (v[j][e] - mean) * rstd;
        if (w) y = y * w[c];
        if (b) y = y + b[c];
        r[e] = y;
      }
      Vec4<Tout>::store(out + row * C + j * 128 + lane * 4, r);
    }
  }
}

// fp32 rows -> LayerNorm -> three bf16 planes (the fp32 linears' operand form).
template <int V>
__global__ void layernorm_split3_kernel(const float *x, const float *w, const float *b, __nv_bfloat16 *out,
                                        int64_t rows, float eps) {
  constexpr int C = 128 * V;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int64_t plane = rows * C;
  for (int64_t row = blockIdx.x * int64_t(warps) + (threadIdx.x >> 5); row < rows;
       row += int64_t(gridDim.x) * warps) {
    float v[V][4];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      Vec4<float>::load(x + row * C + j * 128 + lane * 4, v[j]);
      sum += (v[j][0] + v[j][1]) + (v[j][2] + v[j][3]);
    }
    const float mean = warp_sum(sum) * (1.f / C);
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float d = v[j][e] - mean;
        sq += d * d;
      }
    const float rstd = rsqrtf(warp_sum(sq) * (1.f / C) + eps);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float r[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int c = j * 128 + lane * 4 + e;
        float y = (v[j][e] - mean) * rstd;
        if (w) y = y * w[c];
        if (b) y = y + b[c];
        r[e] = y;
      }
      store_split3_4(out, plane, row * C + j * 128 + lane * 4, r[0], r[1], r[2], r[3]);
    }
  }
}

// Any width, any alignment: two passes over global memory.
template <typename Tin, typename Tout>
__global__ void layernorm_rows_generic_kernel(const Tin *x, const float *w, const float *b, Tout *out,
                                              int64_t rows, int64_t cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int64_t row = blockIdx.x * int64_t(warps) + (threadIdx.x >> 5); row < rows;
       row += int64_t(gridDim.x) * warps) {
    const Tin *xr = x + row * cols;
    float sum = 0.f;
    for (int64_t c = lane; c < cols; c += 32) sum += load_as_float(xr + c);
    const float mean = warp_sum(sum) / float(cols);
    float sq = 0.f;
    for (int64_t c = lane; c < cols; c += 32) {
      float d = load_as_float(xr + c) - mean;
      sq += d * d;
    }
    const float rstd = rsqrtf(warp_sum(sq) / float(cols) + eps);
    for (int64_t c = lane; c < cols; c += 32) {
      float y = (load_as_float(xr + c) - mean) * rstd;
      if (w) y = y * w[c];
      if (b) y = y + b[c];
      store_from_float(out + row * cols + c, y);
    }
  }
}

// Channel-first input: channel c of row m at x[c * plane + (m / inner) * ld + m % inner]
// (a dense [128, M] tensor is inner = ld = plane = M).  Block = 8 warps, 32 rows per tile.
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256) layernorm_channel_first_kernel(const Tin *x, const float *w,
                                                                      const float *b, Tout *out, int64_t m,
                                                                      int64_t inner, int64_t ld, int64_t plane,
                                                                      float eps) {
  __shared__ float tile[128][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t start = blockIdx.x * 32ll; start < m; start += int64_t(gridDim.x) * 32) {
    // Coalesced plane reads: warp w reads channels w, w+8, ...; lane = row.
    const int64_t row_l = start + lane;
    const int64_t offset = (row_l / inner) * ld + row_l % inner;
    for (int c = warp; c < 128; c += 8) {
      tile[c][lane] = row_l < m ? load_as_float(x + int64_t(c) * plane + offset) : 0.f;
    }
    __syncthreads();
    // Each warp normalises 4 rows; lane holds channels lane*4 .. lane*4+3.
    for (int r = warp; r < 32; r += 8) {
      int64_t row = start + r;
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = tile[lane * 4 + e][r];
      float mean = warp_sum((v[0] + v[1]) + (v[2] + v[3])) * (1.f / 128.f);
      float sq = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float d = v[e] - mean;
        sq += d * d;
      }
      float rstd = rsqrtf(warp_sum(sq) * (1.f / 128.f) + eps);
      if (row < m) {
        float y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int c = lane * 4 + e;
          y[e] = (v[e] - mean) * rstd;
          if (w) y[e] = y[e] * w[c];
          if (b) y[e] = y[e] + b[c];
        }
        Vec4<Tout>::store(out + row * 128 + lane * 4, y);
      }
    }
    __syncthreads();
  }
}

template <typename Tin, typename Tout>
static int launch_channel_first(const Tin *x, int64_t rows, int64_t inner, int64_t ld, int64_t plane,
                                const float *w, const float *b, float eps, Tout *out, cudaStream_t s) {
  BL_REQUIRE(aligned_to(out, 8 * sizeof(Tout) / 2), "bl_layernorm: output misaligned");
  int64_t blocks = (rows + 31) / 32, cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  layernorm_channel_first_kernel<Tin, Tout><<<int(blocks), 256, 0, s>>>(x, w, b, out, rows, inner, ld, plane, eps);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

template <typename Tin, typename Tout>
static int launch_layernorm(const Tin *x, int64_t rows, int64_t cols, int channel_first, const float *w,
                            const float *b, float eps, Tout *out, cudaStream_t s) {
  const int threads = 256;
  int64_t cap = int64_t(num_sms()) * 16;
  if (channel_first) {
    BL_REQUIRE(cols == 128, "bl_layernorm: channel-first input needs 128 channels");
    return launch_channel_first(x, rows, rows, rows, rows, w, b, eps, out, s);
  }
  int64_t blocks = (rows + 7) / 8;
  if (blocks > cap) blocks = cap;
  bool vec = cols % 128 == 0 && cols <= 1024 && aligned_to(x, 4 * sizeof(Tin)) && aligned_to(out, 4 * sizeof(Tout));
  if (vec) {
    switch (cols / 128) {
#define BL_LN_CASE(V)                                                                               \
  case V:                                                                                          \
    layernorm_rows_vec_kernel<Tin, Tout, V><<<int(blocks), threads, 0, s>>>(x, w, b, out, rows, eps); \
    break;
      BL_LN_CASE(1)
      BL_LN_CASE(2)
      BL_LN_CASE(3)
      BL_LN_CASE(4)
      BL_LN_CASE(5)
      BL_LN_CASE(6)
      BL_LN_CASE(7)
      BL_LN_CASE(8)
#undef BL_LN_CASE
    }
  } else {
    layernorm_rows_generic_kernel<Tin, Tout><<<int(blocks), threads, 0, s>>>(x, w, b, out, rows, cols, eps);
  }
  BL_LAUNCH_CHECK();
  return BL_OK;
}

}  // namespace bl

using namespace bl;

extern "C" int bl_layernorm(const void *x, int x_dtype, int64_t rows, int64_t cols, int channel_first,
                            const float *weight, const float *bias, float eps, void *out, int out_dtype,
                            void *stream) {
  BL_REQUIRE(x_dtype == BL_F32 || x_dtype == BL_BF16, "bl_layernorm: bad input dtype");
  BL_REQUIRE(out_dtype == BL_F32 || out_dtype == BL_BF16, "bl_layernorm: bad output dtype");
  BL_REQUIRE(rows >= 0 && cols > 0, "bl_layernorm: bad shape");
  BL_REQUIRE(eps > 0.f, "bl_layernorm: eps must be positive");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(x && out, "bl_layernorm: null pointer");
  auto s = as_stream(stream);
  if (x_dtype == BL_F32) {
    if (out_dtype == BL_F32)
      return launch_layernorm(static_cast<const float *>(x), rows, cols, channel_first, weight, bias, eps,
                              static_cast<float *>(out), s);
    return launch_layernorm(static_cast<const float *>(x), rows, cols, channel_first, weight, bias, eps,
                            static_cast<__nv_bfloat16 *>(out), s);
  }
  if (out_dtype == BL_F32)
    return launch_layernorm(static_cast<const __nv_bfloat16 *>(x), rows, cols, channel_first, weight, bias, eps,
                            static_cast<float *>(out), s);
  return launch_layernorm(static_cast<const __nv_bfloat16 *>(x), rows, cols, channel_first, weight, bias, eps,
                          static_cast<__nv_bfloat16 *>(out), s);
}

extern "C" int bl_layernorm_split3(const float *x, int64_t rows, int64_t cols, const float *weight,
                                   const float *bias, float eps, void *out3, void *stream) {
  BL_REQUIRE(rows >= 0 && cols > 0, "bl_layernorm_split3: bad shape");
  BL_REQUIRE(eps > 0.f, "bl_layernorm_split3: eps must be positive");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(x && out3, "bl_layernorm_split3: null pointer");
  BL_REQUIRE(cols % 128 == 0 && cols <= 1024 && aligned_to(x, 16) && aligned_to(out3, 8),
             "bl_layernorm_split3: cols must be a multiple of 128 (<= 1024), x 16-byte aligned");
  auto s = as_stream(stream);
  int64_t blocks = (rows + 7) / 8, cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  auto *o = static_cast<__nv_bfloat16 *>(out3);
  switch (cols / 128) {
#define BL_LN3_CASE(V) \
  case V:              \
    layernorm_split3_kernel<V><<<int(blocks), 256, 0, s>>>(x, weight, bias, o, rows, eps); \
    break;
    BL_LN3_CASE(1)
    BL_LN3_CASE(2)
    BL_LN3_CASE(3)
    BL_LN3_CASE(4)
    BL_LN3_CASE(5)
    BL_LN3_CASE(6)
    BL_LN3_CASE(7)
    BL_LN3_CASE(8)
#undef BL_LN3_CASE
  }
  BL_LAUNCH_CHECK();
  return BL_OK;
}
