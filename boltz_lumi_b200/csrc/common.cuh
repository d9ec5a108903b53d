// Shared host/device helpers for the sm_100a kernels of the Boltz-2 pair path.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "boltz_b200.h"

namespace bl {

// ---------------------------------------------------------------------------
// Host-side error reporting: every C-ABI entry point returns a BL_* status and
// leaves a message for bl_last_error() on failure.
// ---------------------------------------------------------------------------
void set_error(const char *fmt, ...);

#define BL_REQUIRE(cond, ...)                                                                      \
  do {                                                                                             \
    if (!(cond)) {                                                                                 \
      ::bl::set_error(__VA_ARGS__);                                                                \
      return BL_ERR_INVALID;                                                                       \
    }                                                                                              \
  } while (0)

#define BL_CUDA(call)                                                                              \
  do {                                                                                             \
    cudaError_t err_ = (call);                                                                     \
    if (err_ != cudaSuccess) {                                                                     \
      ::bl::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(err_), __FILE__,         \
                      __LINE__);                                                                   \
      return BL_ERR_CUDA;                                                                          \
    }                                                                                              \
  } while (0)

// Check the launch that was just issued (configuration errors only; execution
// errors surface at the caller's next synchronisation).
#define BL_LAUNCH_CHECK() BL_CUDA(cudaGetLastError())

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned_to(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int num_sms() {
  static int count = 0;
  if (!count) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (count <= 0) count = 148;
  }
  return count;
}

// ---------------------------------------------------------------------------
// Device-side failure flag: bounded waits record where they gave up instead of
// hanging; the host reads it back with bl_device_status().  Kernels receive
// its device address as a parameter (the library is built without -rdc).
// ---------------------------------------------------------------------------
unsigned int *device_status_ptr();

// Raise a kernel's dynamic shared-memory limit once per (kernel, device).
cudaError_t ensure_smem_limit(const void *kernel, int bytes);

// ---------------------------------------------------------------------------
// bf16 helpers.  Round-to-nearest-even conversions match torch's .to(bfloat16).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ float bf16_to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ float load_as_float(const T *p);
template <> __device__ __forceinline__ float load_as_float<float>(const float *p) { return *p; }
template <> __device__ __forceinline__ float load_as_float<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(*p);
}

template <typename T> __device__ __forceinline__ void store_from_float(T *p, float v);
template <> __device__ __forceinline__ void store_from_float<float>(float *p, float v) { *p = v; }
template <> __device__ __forceinline__ void store_from_float<__nv_bfloat16>(__nv_bfloat16 *p, float v) {
  *p = __float2bfloat16_rn(v);
}

// Sigmoid as torch computes it for a bf16/fp32 tensor: 1 / (1 + exp(-x)) in fp32.
__device__ __forceinline__ float sigmoidf_fast(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoidf_acc(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Packed fp32 pairs (sm_100 fma.rn.f32x2): the pair lives in one 64-bit register.
__device__ __forceinline__ void lds_v2b64(uint32_t addr, uint64_t &a, uint64_t &b) {
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}
__device__ __forceinline__ uint64_t lds_b64(uint32_t addr) {
  uint64_t v;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(addr));
  return v;
}
// acc.{lo,hi} += a.{lo,hi} * b.{lo,hi}
__device__ __forceinline__ void ffma2(uint64_t &acc, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ uint64_t dup2(float x) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %1};" : "=l"(v) : "f"(x));
  return v;
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }

// Four fp32 values as three bf16 planes (x = x1 + x2 + x3, x1 = bf16(x),
// x2 = bf16(x - x1), x3 = bf16(x - x1 - x2); both subtractions exact): the
// operand form of bl_linear_split3.  Element e (a multiple of 4) of each
// plane; planes are `plane` elements apart.
__device__ __forceinline__ void store_split3_4(__nv_bfloat16 *planes, int64_t plane, int64_t e, float v0, float v1,
                                               float v2, float v3) {
  const float v[4] = {v0, v1, v2, v3};
  float p1[4], p2[4], p3[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    p1[i] = bf16r(v[i]);
    const float r1 = v[i] - p1[i];
    p2[i] = bf16r(r1);
    p3[i] = r1 - p2[i];
  }
  *reinterpret_cast<uint2 *>(planes + e) = make_uint2(pack_bf16x2(p1[0], p1[1]), pack_bf16x2(p1[2], p1[3]));
  *reinterpret_cast<uint2 *>(planes + plane + e) = make_uint2(pack_bf16x2(p2[0], p2[1]), pack_bf16x2(p2[2], p2[3]));
  *reinterpret_cast<uint2 *>(planes + 2 * plane + e) =
      make_uint2(pack_bf16x2(p3[0], p3[1]), pack_bf16x2(p3[2], p3[3]));
}

__device__ __forceinline__ void store_split3_1(__nv_bfloat16 *planes, int64_t plane, int64_t e, float v) {
  const float p1 = bf16r(v), r1 = v - p1, p2 = bf16r(r1);
  planes[e] = __float2bfloat16_rn(p1);
  planes[plane + e] = __float2bfloat16_rn(p2);
  planes[2 * plane + e] = __float2bfloat16_rn(r1 - p2);
}

}  // namespace bl
