// Memory-bound kernels of the pair path: sigmoid gating, gate+mask packing,
// SiLU-mul, fp32 diffusion epilogues and the ordered bias softmax.
//
// All of them stream HBM once: 128-bit loads/stores where the pointers allow,
// grid-stride loops sized to the SM count, fp32 math with the bf16 rounding
// points of upstream's eager path.
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"

namespace bl {

__device__ unsigned int g_device_status = 0;

unsigned int *device_status_ptr() {
  // One address per device: the symbol is resolved on the current device.
  static thread_local int cached_device = -1;
  static thread_local unsigned int *cached = nullptr;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_device) {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_status) != cudaSuccess) return nullptr;
    cached = static_cast<unsigned int *>(ptr);
    cached_device = dev;
  }
  return cached;
}

cudaError_t ensure_smem_limit(const void *kernel, int bytes) {
  static std::mutex lock;
  static std::vector<std::pair<const void *, int>> done;  // (kernel, device)
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> guard(lock);
  for (auto &entry : done)
    if (entry.first == kernel && entry.second == dev) return cudaSuccess;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) done.emplace_back(kernel, dev);
  return err;
}

namespace {
thread_local std::string t_last_error;
}

void set_error(const char *fmt, ...) {
  char buffer[1024];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buffer, sizeof(buffer), fmt, args);
  va_end(args);
  t_last_error = buffer;
}

static int grid_for(int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  int64_t cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return int(blocks);
}

// ---------------------------------------------------------------------------
// gate: out = bf16(p * bf16(sigmoid(g)))  (multiplication_gate_hip.cu:16-25)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gated(float p, float g) { return bf16r(p * bf16r(sigmoidf_fast(g))); }

__global__ void gate_vec_kernel(const uint4 *p, const uint4 *g, uint4 *out, int64_t vecs) {
  for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < vecs;
       v += int64_t(gridDim.x) * blockDim.x) {
    uint4 pv = p[v], gv = g[v], r;
    const uint32_t *pa = &pv.x, *ga = &gv.x;
    uint32_t *ra = &r.x;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      ra[w] = pack_bf16x2(gated(bf16_lo(pa[w]), bf16_lo(ga[w])), gated(bf16_hi(pa[w]), bf16_hi(ga[w])));
    out[v] = r;
  }
}

__global__ void gate_scalar_kernel(const __nv_bfloat16 *p, const __nv_bfloat16 *g, __nv_bfloat16 *out,
                                   int64_t begin, int64_t n) {
  for (int64_t i = begin + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(gated(__bfloat162float(p[i]), __bfloat162float(g[i])));
}

// ---------------------------------------------------------------------------
// silu_mul: out = bf16(bf16(silu(a)) * b)  (pair_hip.cu:12-17)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_mul(float a, float b) {
  return bf16r(bf16r(a / (1.f + __expf(-a))) * b);
}

__global__ void silu_vec_kernel(const uint4 *a, const uint4 *b, uint4 *out, int64_t vecs) {
  for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < vecs;
       v += int64_t(gridDim.x) * blockDim.x) {
    uint4 av = a[v], bv = b[v], r;
    const uint32_t *aa = &av.x, *ba = &bv.x;
    uint32_t *ra = &r.x;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      ra[w] = pack_bf16x2(silu_mul(bf16_lo(aa[w]), bf16_lo(ba[w])), silu_mul(bf16_hi(aa[w]), bf16_hi(ba[w])));
    out[v] = r;
  }
}

__global__ void silu_scalar_kernel(const __nv_bfloat16 *a, const __nv_bfloat16 *b, __nv_bfloat16 *out,
                                   int64_t begin, int64_t n) {
  for (int64_t i = begin + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(silu_mul(__bfloat162float(a[i]), __bfloat162float(b[i])));
}

// ---------------------------------------------------------------------------
// Gate + mask + channel-first pack (multiplication_gate_hip.cu:27-60).
// Tile: 32 x 32 pairs x 8 channels; one 16-byte load per pair and operand.
// ---------------------------------------------------------------------------
constexpr int kPackTile = 32;
constexpr int kPackChannels = 8;

__global__ void __launch_bounds__(256) gate_pack_kernel(const __nv_bfloat16 *p, const __nv_bfloat16 *g,
                                                        int64_t stride, const float *mask, int n,
                                                        int outgoing, __nv_bfloat16 *left,
                                                        __nv_bfloat16 *right) {
  __shared__ __nv_bfloat16 tile[2][kPackChannels][kPackTile][kPackTile + 2];
  const int r0 = blockIdx.y * kPackTile, s0 = blockIdx.x * kPackTile;
  const int c0 = blockIdx.z * kPackChannels;
  // Load: thread -> (pair r, s); each pair contributes 8 channels of a and of b.
  for (int idx = threadIdx.x; idx < kPackTile * kPackTile; idx += blockDim.x) {
    int r = idx / kPackTile, s = idx % kPackTile;
    int gr = r0 + r, gs = s0 + s;
    float av[kPackChannels], bv[kPackChannels];
    if (gr < n && gs < n) {
      int64_t pair = int64_t(gr) * n + gs;
      float m = mask[pair];
      const __nv_bfloat16 *pp = p + pair * stride + c0, *gp = g + pair * stride + c0;
      uint4 pa = *reinterpret_cast<const uint4 *>(pp), ga = *reinterpret_cast<const uint4 *>(gp);
      uint4 pb = *reinterpret_cast<const uint4 *>(pp + 128), gb = *reinterpret_cast<const uint4 *>(gp + 128);
      const uint32_t *pa32 = &pa.x, *ga32 = &ga.x, *pb32 = &pb.x, *gb32 = &gb.x;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        av[2 * w] = bf16r(gated(bf16_lo(pa32[w]), bf16_lo(ga32[w])) * m);
        av[2 * w + 1] = bf16r(gated(bf16_hi(pa32[w]), bf16_hi(ga32[w])) * m);
        bv[2 * w] = bf16r(gated(bf16_lo(pb32[w]), bf16_lo(gb32[w])) * m);
        bv[2 * w + 1] = bf16r(gated(bf16_hi(pb32[w]), bf16_hi(gb32[w])) * m);
      }
    } else {
#pragma unroll
      for (int c = 0; c < kPackChannels; ++c) av[c] = bv[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < kPackChannels; ++c) {
      tile[0][c][r][s] = __float2bfloat16_rn(av[c]);
      tile[1][c][r][s] = __float2bfloat16_rn(bv[c]);
    }
  }
  __syncthreads();
  // Store rows of 32 contiguous elements.  Natural: plane[c][r][s] = v[r][s];
  // transposed: plane[c][s][r] = v[r][s].
  for (int idx = threadIdx.x; idx < kPackChannels * kPackTile * kPackTile; idx += blockDim.x) {
    int c = idx / (kPackTile * kPackTile), rem = idx % (kPackTile * kPackTile);
    int row = rem / kPackTile, col = rem % kPackTile;
    int64_t plane = int64_t(c0 + c) * n * n;
    // Natural orientation for left/outgoing and right/incoming.
    int nr = r0 + row, ns = s0 + col;
    // Transposed orientation: output row = s0 + row, output column = r0 + col.
    int tr = s0 + row, ts = r0 + col;
    if (outgoing) {
      if (nr < n && ns < n) left[plane + int64_t(nr) * n + ns] = tile[0][c][row][col];
      if (tr < n && ts < n) right[plane + int64_t(tr) * n + ts] = tile[1][c][col][row];
    } else {
      if (tr < n && ts < n) left[plane + int64_t(tr) * n + ts] = tile[0][c][col][row];
      if (nr < n && ns < n) right[plane + int64_t(nr) * n + ns] = tile[1][c][row][col];
    }
  }
}

__global__ void gate_split_kernel(const __nv_bfloat16 *p, const __nv_bfloat16 *g, int64_t stride,
                                  const float *mask, int64_t pairs, __nv_bfloat16 *a, __nv_bfloat16 *b) {
  // One thread per (pair, 8-channel group): 16 groups per pair.
  int64_t groups = pairs * 16;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < groups;
       t += int64_t(gridDim.x) * blockDim.x) {
    int64_t pair = t >> 4;
    int c = int(t & 15) * 8;
    float m = mask[pair];
    const __nv_bfloat16 *pp = p + pair * stride + c, *gp = g + pair * stride + c;
    uint4 pa = *reinterpret_cast<const uint4 *>(pp), ga = *reinterpret_cast<const uint4 *>(gp);
    uint4 pb = *reinterpret_cast<const uint4 *>(pp + 128), gb = *reinterpret_cast<const uint4 *>(gp + 128);
    uint4 ra, rb;
    const uint32_t *pa32 = &pa.x, *ga32 = &ga.x, *pb32 = &pb.x, *gb32 = &gb.x;
    uint32_t *ra32 = &ra.x, *rb32 = &rb.x;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      ra32[w] = pack_bf16x2(gated(bf16_lo(pa32[w]), bf16_lo(ga32[w])) * m,
                            gated(bf16_hi(pa32[w]), bf16_hi(ga32[w])) * m);
      rb32[w] = pack_bf16x2(gated(bf16_lo(pb32[w]), bf16_lo(gb32[w])) * m,
                            gated(bf16_hi(pb32[w]), bf16_hi(gb32[w])) * m);
    }
    *reinterpret_cast<uint4 *>(a + pair * 128 + c) = ra;
    *reinterpret_cast<uint4 *>(b + pair * 128 + c) = rb;
  }
}

// ---------------------------------------------------------------------------
// fp32 diffusion epilogues (diffusion_hip.cu:13-27).  Multiply and add round
// separately, as in the eager path: no FMA contraction.
// ---------------------------------------------------------------------------
template <int KIND> __device__ __forceinline__ float epilogue_value(float a, float b, float c) {
  if constexpr (KIND == BL_EPI_MODULATION) {
    float product = __fmul_rn(sigmoidf_acc(b), a);
    return __fadd_rn(product, c);
  } else if constexpr (KIND == BL_EPI_GATE) {
    return __fmul_rn(sigmoidf_acc(a), b);
  } else if constexpr (KIND == BL_EPI_SWIGLU) {
    // a: first half (silu input), b: second half.
    return __fmul_rn(a / (1.f + expf(-a)), b);
  } else {
    // a: first half (value), b: second half (gate input), c: a_to_b.
    float activation = b / (1.f + expf(-b));
    return __fmul_rn(__fmul_rn(activation, a), c);
  }
}

// The epilogue result as three bf16 planes (the fp32 linears' operand form);
// cols % 4 == 0, 16-byte aligned operands.
template <int KIND>
__global__ void diffusion_epilogue_split3_kernel(const float *a, const float *b, const float *c,
                                                 __nv_bfloat16 *out, int64_t rows, int64_t cols) {
  const int64_t width = cols / 4, total = rows * width, plane = rows * cols;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = t / width, col = t % width;
    float4 av, bv, cv = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (KIND == BL_EPI_GATED_SWIGLU || KIND == BL_EPI_SWIGLU) {
      const float4 *a4 = reinterpret_cast<const float4 *>(a) + row * 2 * width;
      av = a4[col];
      bv = a4[width + col];
      if constexpr (KIND == BL_EPI_GATED_SWIGLU) cv = reinterpret_cast<const float4 *>(b)[t];
    } else {
      av = reinterpret_cast<const float4 *>(a)[t];
      bv = reinterpret_cast<const float4 *>(b)[t];
      if constexpr (KIND == BL_EPI_MODULATION) cv = reinterpret_cast<const float4 *>(c)[t];
    }
    store_split3_4(out, plane, 4 * t, epilogue_value<KIND>(av.x, bv.x, cv.x), epilogue_value<KIND>(av.y, bv.y, cv.y),
                   epilogue_value<KIND>(av.z, bv.z, cv.z), epilogue_value<KIND>(av.w, bv.w, cv.w));
  }
}

template <int KIND, bool VEC>
__global__ void diffusion_epilogue_kernel(const float *a, const float *b, const float *c, float *out,
                                          int64_t rows, int64_t cols) {
  const int64_t width = VEC ? cols / 4 : cols;
  const int64_t total = rows * width;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    int64_t row = t / width, col = t % width;
    if constexpr (VEC) {
      float4 av, bv, cv = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (KIND == BL_EPI_GATED_SWIGLU || KIND == BL_EPI_SWIGLU) {
        const float4 *a4 = reinterpret_cast<const float4 *>(a) + row * 2 * width;
        av = a4[col];
        bv = a4[width + col];
        if constexpr (KIND == BL_EPI_GATED_SWIGLU) cv = reinterpret_cast<const float4 *>(b)[t];
      } else {
        av = reinterpret_cast<const float4 *>(a)[t];
        bv = reinterpret_cast<const float4 *>(b)[t];
        if constexpr (KIND == BL_EPI_MODULATION) cv = reinterpret_cast<const float4 *>(c)[t];
      }
      float4 r = make_float4(epilogue_value<KIND>(av.x, bv.x, cv.x), epilogue_value<KIND>(av.y, bv.y, cv.y),
                             epilogue_value<KIND>(av.z, bv.z, cv.z), epilogue_value<KIND>(av.w, bv.w, cv.w));
      reinterpret_cast<float4 *>(out)[t] = r;
    } else {
      float av, bv, cv = 0.f;
      if constexpr (KIND == BL_EPI_GATED_SWIGLU || KIND == BL_EPI_SWIGLU) {
        av = a[row * 2 * cols + col];
        bv = a[row * 2 * cols + cols + col];
        if constexpr (KIND == BL_EPI_GATED_SWIGLU) cv = b[t];
      } else {
        av = a[t];
        bv = b[t];
        if constexpr (KIND == BL_EPI_MODULATION) cv = c[t];
      }
      out[t] = epilogue_value<KIND>(av, bv, cv);
    }
  }
}

// ---------------------------------------------------------------------------
// Fused AdaLN modulation: out = sigmoid(scale) * LN(a) + shift (no affine LN).
// One warp per row; the row stays in registers when cols <= 32 * 4 * MAXV.
// ---------------------------------------------------------------------------
template <int MAXV, bool SPLIT>
__global__ void adaln_modulate_kernel(const float *a, const float *scale, const float *shift, void *out_,
                                      int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int vecs = cols >> 2;  // float4 per row
  for (int64_t row = blockIdx.x * int64_t(warps) + (threadIdx.x >> 5); row < rows;
       row += int64_t(gridDim.x) * warps) {
    const float4 *a4 = reinterpret_cast<const float4 *>(a + row * cols);
    float4 v[MAXV];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      int idx = lane + 32 * j;
      v[j] = idx < vecs ? a4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
      sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
    const float mean = warp_sum(sum) / float(cols);
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      int idx = lane + 32 * j;
      if (idx < vecs) {
        float dx = v[j].x - mean, dy = v[j].y - mean, dz = v[j].z - mean, dw = v[j].w - mean;
        sq += (dx * dx + dy * dy) + (dz * dz + dw * dw);
      }
    }
    const float rstd = rsqrtf(warp_sum(sq) / float(cols) + eps);
    const float4 *s4 = reinterpret_cast<const float4 *>(scale + row * cols);
    const float4 *b4 = reinterpret_cast<const float4 *>(shift + row * cols);
    float4 *o4 = reinterpret_cast<float4 *>(static_cast<float *>(out_) + row * cols);
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      int idx = lane + 32 * j;
      if (idx < vecs) {
        float4 sc = s4[idx], sh = b4[idx], r;
        r.x = epilogue_value<BL_EPI_MODULATION>((v[j].x - mean) * rstd, sc.x, sh.x);
        r.y = epilogue_value<BL_EPI_MODULATION>((v[j].y - mean) * rstd, sc.y, sh.y);
        r.z = epilogue_value<BL_EPI_MODULATION>((v[j].z - mean) * rstd, sc.z, sh.z);
        r.w = epilogue_value<BL_EPI_MODULATION>((v[j].w - mean) * rstd, sc.w, sh.w);
        if constexpr (SPLIT)
          store_split3_4(static_cast<__nv_bfloat16 *>(out_), rows * cols, row * cols + 4 * idx, r.x, r.y, r.z, r.w);
        else
          o4[idx] = r;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Ordered bias softmax over materialised scores (triangle_softmax.py:90-113):
// one warp per score row, online max/sum, then a second pass that writes.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void triangle_softmax_kernel(const T *scores, const T *bias, const float *mask, T *out,
                                        int64_t batch, int64_t outer, int64_t heads, int64_t n,
                                        int64_t s0, int64_t s1, int64_t s2, int64_t s3, int64_t s4,
                                        int64_t b0, int64_t b1, int64_t b2, int64_t b3, int64_t m0,
                                        int64_t m1, int64_t m2) {
  constexpr bool kBf16 = sizeof(T) == 2;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int64_t rows = batch * outer * heads * n;
  for (int64_t row = blockIdx.x * int64_t(warps) + (threadIdx.x >> 5); row < rows;
       row += int64_t(gridDim.x) * warps) {
    int64_t q = row % n, h = (row / n) % heads, i = (row / (n * heads)) % outer, b = row / (n * heads * outer);
    const T *srow = scores + b * s0 + i * s1 + h * s2 + q * s3;
    const T *brow = bias + b * b0 + h * b1 + q * b2;
    const float *mrow = mask + b * m0 + i * m1;
    auto value = [&](int64_t k) {
      float v = load_as_float(srow + k * s4) + mrow[k * m2];
      if (kBf16) v = bf16r(v);
      v = v + load_as_float(brow + k * b3);
      if (kBf16) v = bf16r(v);
      return v;
    };
    float m = -INFINITY, sum = 0.f;
    for (int64_t k = lane; k < n; k += 32) {
      float v = value(k);
      float nm = fmaxf(m, v);
      sum = sum * expf(m - nm) + expf(v - nm);
      m = nm;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, sum, o);
      float nm = fmaxf(m, om);
      float a = (m == -INFINITY) ? 0.f : sum * expf(m - nm);
      float c = (om == -INFINITY) ? 0.f : os * expf(om - nm);
      sum = a + c;
      m = nm;
    }
    T *orow = out + row * n;
    for (int64_t k = lane; k < n; k += 32) store_from_float(orow + k, __fdiv_rn(expf(value(k) - m), sum));
  }
}

}  // namespace bl

using namespace bl;

extern "C" {

const char *bl_last_error(void) { return bl::t_last_error.c_str(); }

int bl_version(void) { return 1; }

int bl_device_status(int reset) {
  BL_CUDA(cudaDeviceSynchronize());
  unsigned int value = 0;
  BL_CUDA(cudaMemcpyFromSymbol(&value, bl::g_device_status, sizeof(value)));
  if (reset) {
    unsigned int zero = 0;
    BL_CUDA(cudaMemcpyToSymbol(bl::g_device_status, &zero, sizeof(zero)));
  }
  return int(value);
}

int bl_gate(const void *p, const void *g, void *out, int64_t n, void *stream) {
  BL_REQUIRE(n >= 0, "bl_gate: negative size");
  if (n == 0) return BL_OK;
  BL_REQUIRE(p && g && out, "bl_gate: null pointer");
  auto s = as_stream(stream);
  const auto *pb = static_cast<const __nv_bfloat16 *>(p);
  const auto *gb = static_cast<const __nv_bfloat16 *>(g);
  auto *ob = static_cast<__nv_bfloat16 *>(out);
  int64_t body = 0;
  if (aligned_to(p, 16) && aligned_to(g, 16) && aligned_to(out, 16)) {
    int64_t vecs = n / 8;
    if (vecs) {
      gate_vec_kernel<<<grid_for(vecs, 256), 256, 0, s>>>(reinterpret_cast<const uint4 *>(pb),
                                                          reinterpret_cast<const uint4 *>(gb),
                                                          reinterpret_cast<uint4 *>(ob), vecs);
      BL_LAUNCH_CHECK();
    }
    body = vecs * 8;
  }
  if (body < n) {
    gate_scalar_kernel<<<grid_for(n - body, 256), 256, 0, s>>>(pb, gb, ob, body, n);
    BL_LAUNCH_CHECK();
  }
  return BL_OK;
}

int bl_silu_mul(const void *a, const void *b, void *out, int64_t n, void *stream) {
  BL_REQUIRE(n >= 0, "bl_silu_mul: negative size");
  if (n == 0) return BL_OK;
  BL_REQUIRE(a && b && out, "bl_silu_mul: null pointer");
  auto s = as_stream(stream);
  const auto *ab = static_cast<const __nv_bfloat16 *>(a);
  const auto *bb = static_cast<const __nv_bfloat16 *>(b);
  auto *ob = static_cast<__nv_bfloat16 *>(out);
  int64_t body = 0;
  if (aligned_to(a, 16) && aligned_to(b, 16) && aligned_to(out, 16)) {
    int64_t vecs = n / 8;
    if (vecs) {
      silu_vec_kernel<<<grid_for(vecs, 256), 256, 0, s>>>(reinterpret_cast<const uint4 *>(ab),
                                                          reinterpret_cast<const uint4 *>(bb),
                                                          reinterpret_cast<uint4 *>(ob), vecs);
      BL_LAUNCH_CHECK();
    }
    body = vecs * 8;
  }
  if (body < n) {
    silu_scalar_kernel<<<grid_for(n - body, 256), 256, 0, s>>>(ab, bb, ob, body, n);
    BL_LAUNCH_CHECK();
  }
  return BL_OK;
}

static int check_gate_operands(const char *name, const void *p, const void *g, int64_t stride,
                               const float *mask, int64_t n) {
  BL_REQUIRE(n >= 0 && n <= (1 << 20), "%s: bad token count %lld", name, (long long)n);
  BL_REQUIRE(stride == 256 || stride == 512, "%s: pair stride must be 256 or 512", name);
  BL_REQUIRE(p && g && mask, "%s: null pointer", name);
  BL_REQUIRE(aligned_to(p, 16) && aligned_to(g, 16), "%s: p/g must be 16-byte aligned", name);
  return BL_OK;
}

int bl_gate_pack(const void *p, const void *g, int64_t pair_stride, const float *mask, int64_t n,
                 int outgoing, void *left, void *right, void *stream) {
  int rc = check_gate_operands("bl_gate_pack", p, g, pair_stride, mask, n);
  if (rc) return rc;
  if (n == 0) return BL_OK;
  BL_REQUIRE(left && right, "bl_gate_pack: null output");
  dim3 grid((n + kPackTile - 1) / kPackTile, (n + kPackTile - 1) / kPackTile, 128 / kPackChannels);
  gate_pack_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16 *>(p), static_cast<const __nv_bfloat16 *>(g), pair_stride, mask,
      int(n), outgoing, static_cast<__nv_bfloat16 *>(left), static_cast<__nv_bfloat16 *>(right));
  BL_LAUNCH_CHECK();
  return BL_OK;
}

int bl_gate_split(const void *p, const void *g, int64_t pair_stride, const float *mask, int64_t n,
                  void *a, void *b, void *stream) {
  int rc = check_gate_operands("bl_gate_split", p, g, pair_stride, mask, n);
  if (rc) return rc;
  if (n == 0) return BL_OK;
  BL_REQUIRE(a && b && aligned_to(a, 16) && aligned_to(b, 16), "bl_gate_split: outputs must be 16-byte aligned");
  int64_t pairs = n * n;
  gate_split_kernel<<<grid_for(pairs * 16, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16 *>(p), static_cast<const __nv_bfloat16 *>(g), pair_stride, mask, pairs,
      static_cast<__nv_bfloat16 *>(a), static_cast<__nv_bfloat16 *>(b));
  BL_LAUNCH_CHECK();
  return BL_OK;
}

int bl_diffusion_epilogue(const float *a, const float *b, const float *c, float *out, int64_t rows,
                          int64_t cols, int kind, void *stream) {
  BL_REQUIRE(kind == BL_EPI_MODULATION || kind == BL_EPI_GATE || kind == BL_EPI_GATED_SWIGLU ||
                 kind == BL_EPI_SWIGLU,
             "bl_diffusion_epilogue: unknown kind %d", kind);
  BL_REQUIRE(rows >= 0 && cols >= 0, "bl_diffusion_epilogue: negative shape");
  if (rows == 0 || cols == 0) return BL_OK;
  BL_REQUIRE(a && (b || kind == BL_EPI_SWIGLU) && out, "bl_diffusion_epilogue: null pointer");
  BL_REQUIRE(kind != BL_EPI_MODULATION || c, "bl_diffusion_epilogue: MODULATION needs c");
  bool vec = cols % 4 == 0 && aligned_to(a, 16) && aligned_to(b, 16) && aligned_to(out, 16) &&
             (kind != BL_EPI_MODULATION || aligned_to(c, 16));
  int64_t items = rows * (vec ? cols / 4 : cols);
  auto s = as_stream(stream);
  int blocks = grid_for(items, 256);
#define BL_EPI_CASE(K)                                                                              \
  case K:                                                                                          \
    if (vec)                                                                                       \
      diffusion_epilogue_kernel<K, true><<<blocks, 256, 0, s>>>(a, b, c, out, rows, cols);         \
    else                                                                                           \
      diffusion_epilogue_kernel<K, false><<<blocks, 256, 0, s>>>(a, b, c, out, rows, cols);        \
    break;
  switch (kind) {
    BL_EPI_CASE(BL_EPI_MODULATION)
    BL_EPI_CASE(BL_EPI_GATE)
    BL_EPI_CASE(BL_EPI_GATED_SWIGLU)
    BL_EPI_CASE(BL_EPI_SWIGLU)
  }
#undef BL_EPI_CASE
  BL_LAUNCH_CHECK();
  return BL_OK;
}

int bl_adaln_modulate(const float *a, const float *scale, const float *shift, float *out, int64_t rows,
                      int64_t cols, float eps, void *stream) {
  BL_REQUIRE(rows >= 0 && cols > 0, "bl_adaln_modulate: bad shape");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(a && scale && shift && out, "bl_adaln_modulate: null pointer");
  BL_REQUIRE(cols % 4 == 0 && cols <= 32 * 4 * 16, "bl_adaln_modulate: cols must be a multiple of 4 and <= 2048");
  BL_REQUIRE(aligned_to(a, 16) && aligned_to(scale, 16) && aligned_to(shift, 16) && aligned_to(out, 16),
             "bl_adaln_modulate: pointers must be 16-byte aligned");
  BL_REQUIRE(eps > 0.f, "bl_adaln_modulate: eps must be positive");
  auto s = as_stream(stream);
  int blocks = grid_for(rows, 8);
  if (cols <= 512)
    adaln_modulate_kernel<4, false><<<blocks, 256, 0, s>>>(a, scale, shift, out, rows, int(cols), eps);
  else if (cols <= 1024)
    adaln_modulate_kernel<8, false><<<blocks, 256, 0, s>>>(a, scale, shift, out, rows, int(cols), eps);
  else
    adaln_modulate_kernel<16, false><<<blocks, 256, 0, s>>>(a, scale, shift, out, rows, int(cols), eps);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

int bl_adaln_modulate_split3(const float *a, const float *scale, const float *shift, void *out3, int64_t rows,
                             int64_t cols, float eps, void *stream) {
  BL_REQUIRE(rows >= 0 && cols > 0, "bl_adaln_modulate_split3: bad shape");
  if (rows == 0) return BL_OK;
  BL_REQUIRE(a && scale && shift && out3, "bl_adaln_modulate_split3: null pointer");
  BL_REQUIRE(cols % 4 == 0 && cols <= 32 * 4 * 16, "bl_adaln_modulate_split3: cols must be a multiple of 4, <= 2048");
  BL_REQUIRE(aligned_to(a, 16) && aligned_to(scale, 16) && aligned_to(shift, 16) && aligned_to(out3, 8),
             "bl_adaln_modulate_split3: misaligned pointer");
  BL_REQUIRE(eps > 0.f, "bl_adaln_modulate_split3: eps must be positive");
  auto s = as_stream(stream);
  int blocks = grid_for(rows, 8);
  if (cols <= 512)
    adaln_modulate_kernel<4, true><<<blocks, 256, 0, s>>>(a, scale, shift, out3, rows, int(cols), eps);
  else if (cols <= 1024)
    adaln_modulate_kernel<8, true><<<blocks, 256, 0, s>>>(a, scale, shift, out3, rows, int(cols), eps);
  else
    adaln_modulate_kernel<16, true><<<blocks, 256, 0, s>>>(a, scale, shift, out3, rows, int(cols), eps);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

int bl_diffusion_epilogue_split3(const float *a, const float *b, const float *c, void *out3, int64_t rows,
                                 int64_t cols, int kind, void *stream) {
  BL_REQUIRE(kind == BL_EPI_MODULATION || kind == BL_EPI_GATE || kind == BL_EPI_GATED_SWIGLU ||
                 kind == BL_EPI_SWIGLU,
             "bl_diffusion_epilogue_split3: unknown kind %d", kind);
  BL_REQUIRE(rows >= 0 && cols >= 0, "bl_diffusion_epilogue_split3: negative shape");
  if (rows == 0 || cols == 0) return BL_OK;
  BL_REQUIRE(a && (b || kind == BL_EPI_SWIGLU) && out3 && (kind != BL_EPI_MODULATION || c),
             "bl_diffusion_epilogue_split3: null pointer");
  BL_REQUIRE(cols % 4 == 0 && aligned_to(a, 16) && aligned_to(b, 16) && aligned_to(out3, 8) &&
                 (kind != BL_EPI_MODULATION || aligned_to(c, 16)),
             "bl_diffusion_epilogue_split3: cols % 4 == 0 and 16-byte aligned operands");
  auto s = as_stream(stream);
  int blocks = grid_for(rows * (cols / 4), 256);
  auto *o = static_cast<__nv_bfloat16 *>(out3);
  if (kind == BL_EPI_MODULATION)
    diffusion_epilogue_split3_kernel<BL_EPI_MODULATION><<<blocks, 256, 0, s>>>(a, b, c, o, rows, cols);
  else if (kind == BL_EPI_GATE)
    diffusion_epilogue_split3_kernel<BL_EPI_GATE><<<blocks, 256, 0, s>>>(a, b, c, o, rows, cols);
  else if (kind == BL_EPI_SWIGLU)
    diffusion_epilogue_split3_kernel<BL_EPI_SWIGLU><<<blocks, 256, 0, s>>>(a, b, c, o, rows, cols);
  else
    diffusion_epilogue_split3_kernel<BL_EPI_GATED_SWIGLU><<<blocks, 256, 0, s>>>(a, b, c, o, rows, cols);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

int bl_triangle_softmax(const void *scores, int dtype, int64_t batch, int64_t outer, int64_t heads, int64_t n,
                        const int64_t *ss, const void *bias, const int64_t *bs, const float *mask,
                        const int64_t *ms, void *out, void *stream) {
  BL_REQUIRE(dtype == BL_F32 || dtype == BL_BF16, "bl_triangle_softmax: dtype must be f32 or bf16");
  BL_REQUIRE(batch >= 0 && outer >= 0 && heads >= 0 && n >= 0, "bl_triangle_softmax: negative shape");
  int64_t rows = batch * outer * heads * n;
  if (rows == 0) return BL_OK;
  BL_REQUIRE(scores && bias && mask && out && ss && bs && ms, "bl_triangle_softmax: null pointer");
  auto s = as_stream(stream);
  int blocks = grid_for(rows, 8);
  if (dtype == BL_F32)
    triangle_softmax_kernel<float><<<blocks, 256, 0, s>>>(
        static_cast<const float *>(scores), static_cast<const float *>(bias), mask, static_cast<float *>(out),
        batch, outer, heads, n, ss[0], ss[1], ss[2], ss[3], ss[4], bs[0], bs[1], bs[2], bs[3], ms[0], ms[1],
        ms[2]);
  else
    triangle_softmax_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(scores), static_cast<const __nv_bfloat16 *>(bias), mask,
        static_cast<__nv_bfloat16 *>(out), batch, outer, heads, n, ss[0], ss[1], ss[2], ss[3], ss[4], bs[0],
        bs[1], bs[2], bs[3], ms[0], ms[1], ms[2]);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

}  // extern "C"
