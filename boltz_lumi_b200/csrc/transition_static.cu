// Pair transition with no device allocation anywhere in the call.
//
// Who needs this: hosts that do not let a plugin allocate device memory while
// they run inference.  Examples are serving runtimes that reserve all of HBM
// up front in their own pool (cudaMalloc then fails, because nothing is left
// outside the pool) and plugin interfaces that hand a kernel only its input
// and output buffers.  cudaMalloc and cudaFree can also stall or synchronise
// the device, which such hosts avoid on their hot path.
//
// The other pair-transition path of this library (bl_layernorm ->
// bl_batched_gemm -> bl_swiglu_rows -> bl_linear_fused, driven from Python)
// keeps its intermediates in buffers the caller allocates.  This entry point
// computes the same thing with its intermediates in one fixed array compiled
// into the library instead.
#include <mutex>

#include "common.cuh"

namespace {

// Shape of the Boltz-2 pair transition this entry point covers.
constexpr int64_t kDim = 128;      // pair channels
constexpr int64_t kHidden = 512;   // SwiGLU width (4x expansion)
// Largest number of pair rows one call may process.
constexpr int64_t kMaxRows = 1024;

// Intermediates per row: normalised input (bf16), joint fc1|fc2 projection
// (bf16), SwiGLU activation (bf16).
constexpr size_t kNormBytes = size_t(kMaxRows) * kDim * 2;
constexpr size_t kJointBytes = size_t(kMaxRows) * 2 * kHidden * 2;
constexpr size_t kActBytes = size_t(kMaxRows) * kHidden * 2;
constexpr size_t kScratchBytes = kNormBytes + kJointBytes + kActBytes;  // 3.25 MiB

// Every GPU that loads the library holds this array until the process exits.
// All calls on a device share it, so calls that overlap on the GPU (for
// example on two streams at once) race on it.
static __device__ __align__(256) unsigned char g_transition_scratch[kScratchBytes];

// Device address of the array, looked up once per device.  In host code the
// array's name is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress with that device current.  The cached address belongs
// to the device's primary context: after cudaDeviceReset (or anything else
// that destroys that context) it no longer points at the array, so this entry
// point must not be used across a device reset within one process.
constexpr int kMaxDevices = 64;
std::mutex g_setup_lock;
unsigned char *g_scratch_ptr[kMaxDevices] = {};

int scratch_for_current_device(unsigned char **out) {
  int dev = 0;
  BL_CUDA(cudaGetDevice(&dev));
  BL_REQUIRE(dev >= 0 && dev < kMaxDevices, "bl_pair_transition_static: device index %d out of range", dev);
  std::lock_guard<std::mutex> guard(g_setup_lock);
  if (!g_scratch_ptr[dev]) {
    void *ptr = nullptr;
    BL_CUDA(cudaGetSymbolAddress(&ptr, g_transition_scratch));
    g_scratch_ptr[dev] = static_cast<unsigned char *>(ptr);
  }
  *out = g_scratch_ptr[dev];
  return BL_OK;
}

}  // namespace

extern "C" int bl_pair_transition_static(const float *x, int64_t rows, const float *ln_weight, const float *ln_bias,
                                         float eps, const void *w12, const void *w3, void *out, void *stream) {
  BL_REQUIRE(rows >= 0, "bl_pair_transition_static: negative row count");
  BL_REQUIRE(rows <= kMaxRows,
             "bl_pair_transition_static: %lld rows exceed the built-in scratch limit of %lld rows; "
             "split the call or use the caller-allocated path",
             (long long)rows, (long long)kMaxRows);
  if (rows == 0) return BL_OK;
  BL_REQUIRE(x && w12 && w3 && out, "bl_pair_transition_static: null pointer");
  BL_REQUIRE(bl::aligned_to(x, 16) && bl::aligned_to(w12, 16) && bl::aligned_to(w3, 16) && bl::aligned_to(out, 16),
             "bl_pair_transition_static: x, w12, w3 and out must be 16-byte aligned");
  unsigned char *scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  void *norm = scratch;
  void *joint = scratch + kNormBytes;
  void *act = scratch + kNormBytes + kJointBytes;
  // Every intermediate is written in full before it is read, so nothing left
  // over from an earlier call needs clearing.
  rc = bl_layernorm(x, BL_F32, rows, kDim, 0, ln_weight, ln_bias, eps, norm, BL_BF16, stream);
  if (rc) return rc;
  rc = bl_batched_gemm(norm, 0, kDim, 0, w12, 0, kDim, 0, joint, 2 * kHidden, 0, 1, rows, 2 * kHidden, kDim, nullptr,
                       stream);
  if (rc) return rc;
  rc = bl_swiglu_rows(joint, 2 * kHidden, rows, kHidden, act, kHidden, stream);
  if (rc) return rc;
  return bl_linear_fused(act, kHidden, nullptr, 0, kHidden, w3, kHidden, rows, kDim, kHidden, nullptr, 0, nullptr, 0,
                         out, kDim, stream);
}
