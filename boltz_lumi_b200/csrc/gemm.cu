// Batched bf16 GEMM on tcgen05 tensor cores with TMA-fed operands.
//
//   acc[b](m, n) = sum_k A[b](m, k) * B[b](n, k)  (+ bias[n]),  fp32 accumulate
//
// A and B may each be K-major or MN-major in global memory; the MN-major form
// lets the incoming triangle multiplication (O[i,j,c] = sum_k a[k,i,c] b[k,j,c])
// read its channel planes without a transpose pass.  This kernel replaces the
// reference's torch.bmm / torch.matmul / F.linear calls (multiplication.py:122,
// triangle.py:194,208, pair_transition.py:158-165) and fuses what follows them:
//
//   EPI_STORE          C = bf16(acc + bias)
//   EPI_RESIDUAL       Z += bf16(acc + bias)                 (fp32 Z, the pair tensor; TMA reduce-add)
//   EPI_GATE_STORE     C[:, c] = bf16(bf16(acc[c]) * bf16(sigmoid(bf16(acc[w + c]))))
//   EPI_GATE_RESIDUAL  Z[:, c] += that value                  (w = BN / 2)
// The gate forms are the output gate of the triangle multiplication
// (multiplication.py:135-137): p_out and g_out computed as one GEMM.
//
// Persistent, warp-specialised CTA (192 threads, one per SM):
//   warp 0      TMA producer over a STAGES-deep shared-memory ring
//   warp 1      TMEM allocation + single-thread tcgen05.mma issue
//   warps 2..5  epilogue: tcgen05.ld -> math -> swizzled staging -> TMA store
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile t overlaps the main loop of tile t+1.  Residual epilogues add into
// the fp32 Z with TMA reduce-add (no Z load on the SM).
#include "tc.cuh"

namespace bl {

bool encode_tmap(CUtensorMap *map, CUtensorMapDataType type, int rank, const void *base, const uint64_t *dims,
                 const uint64_t *strides_bytes, const uint32_t *box, CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult query;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &query) != cudaSuccess ||
        query != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = encode(map, type, cuuint32_t(rank), const_cast<void *>(base), d, s, b, e,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_GATE_STORE = 2, EPI_GATE_RESIDUAL = 3 };

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kStagingBytes = 4096;  // bf16 store: 32 rows x 64 bf16; residual: 32 rows x 32 fp32

struct GemmArgs {
  int m, n, k, batch;
  int tiles_m, tiles_n;
  int k_split;  // K blocks < k_split come from tma_a, the rest from tma_a2 (K-concatenated operands)
  const float *bias;
  unsigned int *status;
};

template <int BN, int EPI> struct GemmShape {
  static constexpr bool kResidual = EPI == EPI_RESIDUAL || EPI == EPI_GATE_RESIDUAL;
  static constexpr bool kGate = EPI == EPI_GATE_STORE || EPI == EPI_GATE_RESIDUAL;
  static constexpr int kOutWidth = kGate ? BN / 2 : BN;  // output columns per tile
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN == 256 ? 4 : 5;  // 4 x 48 KB + 32 KB staging fits in 227 KB
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kStagingPerWarp = 2 * kStagingBytes;  // double-buffered 4 KB boxes
  static constexpr int kStagingTotal = 4 * kStagingPerWarp;
  static constexpr int kBarrierOffset = kRingBytes + kStagingTotal;
  static constexpr int kSmemBytes = kBarrierOffset + 256 + 1024;  // barriers + alignment slack
  static constexpr uint32_t kTmemCols = 2 * BN;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ float gate_pair(float p, float g) {
  return bf16r(bf16r(p) * bf16r(sigmoidf_fast(bf16r(g))));
}

template <bool A_MN, bool B_MN, int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_a2,
                     const __grid_constant__ CUtensorMap tma_b, const __grid_constant__ CUtensorMap tma_c,
                     const GemmArgs args) {
  using S = GemmShape<BN, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::kBarrierOffset);
  uint64_t *empty = full + S::kStages;
  uint64_t *acc_full = empty + S::kStages;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_per_batch = args.tiles_m * args.tiles_n;
  const int total_tiles = tiles_per_batch * args.batch;
  const int k_blocks = (args.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 4);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tma_a);
    tc::prefetch_tmap(&tma_a2);
    tc::prefetch_tmap(&tma_b);
    tc::prefetch_tmap(&tma_c);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, S::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const int b = tile / tiles_per_batch, rem = tile % tiles_per_batch;
        const int m0 = (rem / args.tiles_n) * kBM, n0 = (rem % args.tiles_n) * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1u, args.status, 0x101)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * S::kStageBytes;
          uint8_t *sb = sa + S::kABytes;
          tc::mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          const int k0 = kb * kBK;
          const CUtensorMap *map_a = kb < args.k_split ? &tma_a : &tma_a2;
          const int ka = kb < args.k_split ? k0 : k0 - args.k_split * kBK;
          if constexpr (A_MN) {
            tc::tma_load_3d(sa, map_a, &full[stage], m0, ka, b);
            tc::tma_load_3d(sa + 8192, map_a, &full[stage], m0 + 64, ka, b);
          } else {
            tc::tma_load_3d(sa, map_a, &full[stage], ka, m0, b);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int t = 0; t < BN / 64; ++t) tc::tma_load_3d(sb + t * 8192, &tma_b, &full[stage], n0 + t * 64, k0, b);
          } else {
            tc::tma_load_3d(sb, &tma_b, &full[stage], k0, n0, b);
          }
          if (++stage == S::kStages) stage = 0, phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        if (!tc::mbar_wait(&acc_empty[acc], acc_phase ^ 1u, args.status, 0x102)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, args.status, 0x103)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t a_desc = A_MN ? tc::desc_sw128(sa + kk * 2048, 8192) : tc::desc_sw128(sa + kk * 32, 16);
            const uint64_t b_desc = B_MN ? tc::desc_sw128(sb + kk * 2048, 8192) : tc::desc_sw128(sb + kk * 32, 16);
            tc::umma_f16_ss(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0);
          }
          tc::umma_commit(&empty[stage]);
          if (++stage == S::kStages) stage = 0, phase ^= 1u;
        }
        tc::umma_commit(&acc_full[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1u;
      }
    }
  } else {
    // Epilogue warps 2..5 own TMEM lane quarters (warp % 4).
    const int quarter = warp & 3;
    uint8_t *staging = smem + S::kRingBytes + quarter * S::kStagingPerWarp;
    int acc = 0;
    uint32_t acc_phase = 0;
    int chunk_count = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      const int b = tile / tiles_per_batch, rem = tile % tiles_per_batch;
      const int m0 = (rem / args.tiles_n) * kBM, n0 = (rem % args.tiles_n) * BN;
      const int row0 = m0 + quarter * 32;
      if (!tc::mbar_wait(&acc_full[acc], acc_phase, args.status, 0x104)) break;
      tc::tc_fence_after();
      const uint32_t tbase = tc::tmem_addr(tmem_base, quarter * 32, acc * BN);
      if constexpr (S::kResidual) {
        // Z += y as a TMA reduce-add of each [32 rows][32 fp32] box: the SM
        // never loads Z (the add happens at L2, fp32 round-to-nearest).
#pragma unroll 1
        for (int cc = 0; cc < S::kOutWidth / 32; ++cc) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(tbase + cc * 32, r);
          float out[32];
          if constexpr (S::kGate) {
            uint32_t gr[32];
            tc::tmem_ld_32x32b_x32(tbase + S::kOutWidth + cc * 32, gr);
            tc::tmem_ld_wait_regs(r, gr);
#pragma unroll
            for (int j = 0; j < 32; ++j) out[j] = gate_pair(__uint_as_float(r[j]), __uint_as_float(gr[j]));
          } else {
            tc::tmem_ld_wait();
            const int c0 = n0 + cc * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int c = c0 + j;
              out[j] = bf16r(__uint_as_float(r[j]) + (args.bias && c < args.n ? __ldg(args.bias + c) : 0.f));
            }
          }
          uint8_t *buf = staging + (chunk_count & 1) * kStagingBytes;
          if (lane == 0) tc::bulk_wait_read<1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4 *>(buf + lane * 128 + ((j ^ (lane & 7)) * 16)) =
                make_float4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tc::tma_reduce_add_2d(&tma_c, buf, cc * 32, row0);
            tc::bulk_commit();
          }
          ++chunk_count;
        }
      } else {
#pragma unroll 1
        for (int cc = 0; cc < S::kOutWidth / 64; ++cc) {
          uint32_t r0[32], r1[32];
          tc::tmem_ld_32x32b_x32(tbase + cc * 64, r0);
          tc::tmem_ld_32x32b_x32(tbase + cc * 64 + 32, r1);
          uint32_t packed[32];
          if constexpr (S::kGate) {
            uint32_t g0[32], g1[32];
            tc::tmem_ld_32x32b_x32(tbase + S::kOutWidth + cc * 64, g0);
            tc::tmem_ld_32x32b_x32(tbase + S::kOutWidth + cc * 64 + 32, g1);
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              packed[j] = pack_bf16x2(gate_pair(__uint_as_float(r0[2 * j]), __uint_as_float(g0[2 * j])),
                                      gate_pair(__uint_as_float(r0[2 * j + 1]), __uint_as_float(g0[2 * j + 1])));
              packed[16 + j] = pack_bf16x2(gate_pair(__uint_as_float(r1[2 * j]), __uint_as_float(g1[2 * j])),
                                           gate_pair(__uint_as_float(r1[2 * j + 1]), __uint_as_float(g1[2 * j + 1])));
            }
          } else {
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v0 = __uint_as_float(r0[2 * j]), v1 = __uint_as_float(r0[2 * j + 1]);
              float w0 = __uint_as_float(r1[2 * j]), w1 = __uint_as_float(r1[2 * j + 1]);
              if (args.bias) {
                const int c = n0 + cc * 64 + 2 * j;
                v0 += c < args.n ? args.bias[c] : 0.f;
                v1 += c + 1 < args.n ? args.bias[c + 1] : 0.f;
                w0 += c + 32 < args.n ? args.bias[c + 32] : 0.f;
                w1 += c + 33 < args.n ? args.bias[c + 33] : 0.f;
              }
              packed[j] = pack_bf16x2(v0, v1);
              packed[16 + j] = pack_bf16x2(w0, w1);
            }
          }
          uint8_t *buf = staging + (chunk_count & 1) * kStagingBytes;
          if (lane == 0) tc::bulk_wait_read<1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 v = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
            *reinterpret_cast<uint4 *>(buf + lane * 128 + ((j ^ (lane & 7)) * 16)) = v;
          }
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tc::tma_store_3d(&tma_c, buf, (S::kGate ? 0 : n0) + cc * 64, row0, b);
            tc::bulk_commit();
          }
          ++chunk_count;
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) acc = 0, acc_phase ^= 1u;
    }
    if (lane == 0) tc::bulk_wait<0>();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

template <bool A_MN, bool B_MN, int BN, int EPI>
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &ta2, const CUtensorMap &tb, const CUtensorMap &tcm,
                const GemmArgs &args, cudaStream_t stream) {
  using S = GemmShape<BN, EPI>;
  auto kernel = gemm_bf16_kernel<A_MN, B_MN, BN, EPI>;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(kernel), S::kSmemBytes));
  int total = args.tiles_m * args.tiles_n * args.batch;
  int grid = total < num_sms() ? total : num_sms();
  kernel<<<grid, kThreads, S::kSmemBytes, stream>>>(ta, ta2, tb, tcm, args);
  BL_LAUNCH_CHECK();
  return BL_OK;
}

}  // namespace

// Encode the 3-D map of an operand tile.  `mn_major`: rows of the stored
// matrix run along K (elements contiguous along M/N).
static bool operand_map(CUtensorMap *map, const void *ptr, bool mn_major, int64_t rows_mn, int64_t k, int64_t ld,
                        int64_t batch_stride, int64_t batch, int box_mn) {
  uint64_t dims[3], strides[2];
  uint32_t box[3];
  if (mn_major) {
    dims[0] = uint64_t(rows_mn), dims[1] = uint64_t(k);
    box[0] = 64, box[1] = 64;
  } else {
    dims[0] = uint64_t(k), dims[1] = uint64_t(rows_mn);
    box[0] = 64, box[1] = uint32_t(box_mn);
  }
  dims[2] = uint64_t(batch);
  box[2] = 1;
  strides[0] = uint64_t(ld) * 2;
  strides[1] = uint64_t(batch_stride) * 2;
  return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ptr, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int BN, int EPI>
static int dispatch_majors(bool a_mn, bool b_mn, const CUtensorMap &ta, const CUtensorMap &tb,
                           const CUtensorMap &tcm, const GemmArgs &args, cudaStream_t stream) {
  if (a_mn && b_mn) return launch_gemm<true, true, BN, EPI>(ta, ta, tb, tcm, args, stream);
  if (a_mn) return launch_gemm<true, false, BN, EPI>(ta, ta, tb, tcm, args, stream);
  if (b_mn) return launch_gemm<false, true, BN, EPI>(ta, ta, tb, tcm, args, stream);
  return launch_gemm<false, false, BN, EPI>(ta, ta, tb, tcm, args, stream);
}

int batched_gemm_bf16(const void *a, bool a_mn, int64_t a_ld, int64_t a_bs, const void *b, bool b_mn, int64_t b_ld,
                      int64_t b_bs, void *c, int64_t c_ld, int64_t c_bs, int64_t batch, int64_t m, int64_t n,
                      int64_t k, const float *bias, cudaStream_t stream) {
  BL_REQUIRE(batch >= 0 && m >= 0 && n >= 0 && k >= 0, "gemm: negative shape");
  if (batch == 0 || m == 0 || n == 0) return BL_OK;
  BL_REQUIRE(k > 0, "gemm: k must be positive");
  BL_REQUIRE(a && b && c, "gemm: null pointer");
  BL_REQUIRE(aligned_to(a, 16) && aligned_to(b, 16) && aligned_to(c, 16), "gemm: pointers must be 16-byte aligned");
  BL_REQUIRE(a_ld % 8 == 0 && b_ld % 8 == 0 && c_ld % 8 == 0, "gemm: leading dimensions must be multiples of 8");
  BL_REQUIRE((batch == 1) || (a_bs % 8 == 0 && b_bs % 8 == 0 && c_bs % 8 == 0),
             "gemm: batch strides must be multiples of 8");
  BL_REQUIRE(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31) && batch < (1ll << 31), "gemm: shape too large");
  BL_REQUIRE(a_ld >= (a_mn ? m : k) && b_ld >= (b_mn ? n : k) && c_ld >= n, "gemm: leading dimension too small");
  const int bn = n > 128 ? 256 : 128;
  // A 1-batch map still needs a valid batch stride.
  if (batch == 1) {
    a_bs = a_bs ? a_bs : a_ld * (a_mn ? k : m);
    b_bs = b_bs ? b_bs : b_ld * (b_mn ? k : n);
    c_bs = c_bs ? c_bs : c_ld * m;
    a_bs = (a_bs + 7) / 8 * 8, b_bs = (b_bs + 7) / 8 * 8, c_bs = (c_bs + 7) / 8 * 8;
  }
  CUtensorMap ta, tb, tcm;
  BL_REQUIRE(operand_map(&ta, a, a_mn, m, k, a_ld, a_bs, batch, kBM), "gemm: cannot encode the A tensor map");
  BL_REQUIRE(operand_map(&tb, b, b_mn, n, k, b_ld, b_bs, batch, bn), "gemm: cannot encode the B tensor map");
  {
    uint64_t dims[3] = {uint64_t(n), uint64_t(m), uint64_t(batch)};
    uint64_t strides[2] = {uint64_t(c_ld) * 2, uint64_t(c_bs) * 2};
    uint32_t box[3] = {64, 32, 1};
    BL_REQUIRE(encode_tmap(&tcm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, c, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "gemm: cannot encode the C tensor map");
  }
  GemmArgs args;
  args.m = int(m), args.n = int(n), args.k = int(k), args.batch = int(batch);
  args.tiles_m = int((m + kBM - 1) / kBM);
  args.tiles_n = int((n + bn - 1) / bn);
  args.k_split = int((k + kBK - 1) / kBK);
  args.bias = bias;
  args.status = device_status_ptr();
  BL_REQUIRE(args.status, "gemm: device status word unavailable");
  if (bn == 256) return dispatch_majors<256, EPI_STORE>(a_mn, b_mn, ta, tb, tcm, args, stream);
  return dispatch_majors<128, EPI_STORE>(a_mn, b_mn, ta, tb, tcm, args, stream);
}

// Linear layer over pair rows with a fused epilogue (single N tile per row block).
int linear_fused(const void *a, int64_t a_ld, const void *a2, int64_t a2_ld, int64_t k1, const void *w,
                 int64_t w_ld, int64_t m, int64_t n, int64_t k, const float *bias, int gate, float *z, int64_t z_ld,
                 void *out, int64_t out_ld, cudaStream_t stream) {
  BL_REQUIRE(m >= 0 && k > 0, "linear: bad shape");
  if (m == 0) return BL_OK;
  BL_REQUIRE(a && w && (z || out) && !(z && out), "linear: exactly one of z (residual) and out must be given");
  if (!a2) k1 = k;
  BL_REQUIRE(k1 > 0 && k1 <= k && k1 % kBK == 0 || k1 == k, "linear: the A split must fall on a 64-column boundary");
  BL_REQUIRE(gate ? n == 256 : n == 128, "linear: n must be 128 (or 256 = p|g with gate)");
  BL_REQUIRE(!(gate && bias), "linear: the gate form takes no bias");
  BL_REQUIRE(aligned_to(a, 16) && aligned_to(w, 16) && a_ld % 8 == 0 && w_ld % 8 == 0 && w_ld >= k,
             "linear: operands must have 16-byte aligned rows");
  BL_REQUIRE(m < (1ll << 31) && k < (1ll << 31), "linear: shape too large");
  const int width = gate ? int(n / 2) : int(n);
  CUtensorMap ta, ta2, tb, tcm;
  BL_REQUIRE(a_ld >= k1, "linear: A leading dimension too small");
  BL_REQUIRE(operand_map(&ta, a, false, m, k1, a_ld, a_ld * m, 1, kBM), "linear: cannot encode the A tensor map");
  if (a2) {
    BL_REQUIRE(aligned_to(a2, 16) && a2_ld % 8 == 0 && a2_ld >= k - k1, "linear: second A operand misaligned");
    BL_REQUIRE(operand_map(&ta2, a2, false, m, k - k1, a2_ld, a2_ld * m, 1, kBM),
               "linear: cannot encode the second A tensor map");
  } else {
    ta2 = ta;
  }
  BL_REQUIRE(operand_map(&tb, w, false, n, k, w_ld, w_ld * n, 1, int(n)), "linear: cannot encode the W tensor map");
  if (z) {
    BL_REQUIRE(aligned_to(z, 16) && z_ld % 4 == 0 && z_ld >= width, "linear: z rows must be 16-byte aligned");
    uint64_t dims[2] = {uint64_t(width), uint64_t(m)};
    uint64_t strides[1] = {uint64_t(z_ld) * 4};
    uint32_t box[2] = {32, 32};
    BL_REQUIRE(encode_tmap(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, z, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "linear: cannot encode the Z tensor map");
  } else {
    BL_REQUIRE(aligned_to(out, 16) && out_ld % 8 == 0 && out_ld >= width, "linear: out rows must be 16-byte aligned");
    uint64_t dims[3] = {uint64_t(width), uint64_t(m), 1};
    uint64_t strides[2] = {uint64_t(out_ld) * 2, uint64_t(out_ld) * 2 * uint64_t(m)};
    uint32_t box[3] = {64, 32, 1};
    BL_REQUIRE(encode_tmap(&tcm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B),
               "linear: cannot encode the output tensor map");
  }
  GemmArgs args;
  args.m = int(m), args.n = int(n), args.k = int(k), args.batch = 1;
  args.tiles_m = int((m + kBM - 1) / kBM);
  args.tiles_n = 1;
  args.k_split = int(a2 ? k1 / kBK : (k + kBK - 1) / kBK);
  args.bias = bias;
  args.status = device_status_ptr();
  BL_REQUIRE(args.status, "linear: device status word unavailable");
  if (gate) {
    if (z) return launch_gemm<false, false, 256, EPI_GATE_RESIDUAL>(ta, ta2, tb, tcm, args, stream);
    return launch_gemm<false, false, 256, EPI_GATE_STORE>(ta, ta2, tb, tcm, args, stream);
  }
  if (z) return launch_gemm<false, false, 128, EPI_RESIDUAL>(ta, ta2, tb, tcm, args, stream);
  return launch_gemm<false, false, 128, EPI_STORE>(ta, ta2, tb, tcm, args, stream);
}

}  // namespace bl

extern "C" int bl_batched_gemm(const void *a, int a_mn_major, int64_t a_ld, int64_t a_batch_stride, const void *b,
                               int b_mn_major, int64_t b_ld, int64_t b_batch_stride, void *c, int64_t c_ld,
                               int64_t c_batch_stride, int64_t batch, int64_t m, int64_t n, int64_t k,
                               const float *bias, void *stream) {
  return bl::batched_gemm_bf16(a, a_mn_major != 0, a_ld, a_batch_stride, b, b_mn_major != 0, b_ld, b_batch_stride, c,
                               c_ld, c_batch_stride, batch, m, n, k, bias, bl::as_stream(stream));
}

extern "C" int bl_linear_fused(const void *a, int64_t a_ld, const void *a2, int64_t a2_ld, int64_t k1, const void *w,
                               int64_t w_ld, int64_t m, int64_t n, int64_t k, const float *bias, int gate, float *z,
                               int64_t z_ld, void *out, int64_t out_ld, void *stream) {
  return bl::linear_fused(a, a_ld, a2, a2_ld, k1, w, w_ld, m, n, k, bias, gate, z, z_ld, out, out_ld,
                          bl::as_stream(stream));
}
