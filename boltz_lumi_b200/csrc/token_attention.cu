// Attention core of the diffusion token transformer's AttentionPairBias, fp32:
//
//   o[b, q, h] = sigmoid(g[b, q, h]) * sum_k softmax_k(s) v[b, k, h],
//   s(q, k) = (q[b, q, h] . k[b, k, h]) * scale + bias[b', h, q, k] + inf * (mask[b, k] - 1)
//
// upstream attentionv2 with a prepared (dense) pair bias, which the reference
// runs unfused in fp32 with autocast off (pair_bias.py:28-36: einsum,
// + bias, + mask term, softmax, einsum, then the sigmoid gate).  The [B, H, N, N] scores never reach
// HBM here.  b' = b / bias_batch_div lets one bias serve the `multiplicity`
// diffusion samples of an input without repeating it.
//
// fp32 rules out the bf16 tensor cores, so this is a CUDA-core flash kernel:
// one CTA = 64 queries of one (batch, head), 128 threads, two CTAs per SM.
// Thread (tq, tk) = (t / 8, t % 8) owns queries 4 tq .. 4 tq + 3 and keys
// tk + 8 j (j < 8) of every 64-key tile for S, and output dims
// tk * D / 8 .. of its 4 queries for O.  Per key tile:
//   * K, V, the 64 x 64 bias block and the 64 mask values of the NEXT tile
//     are in flight (cp.async, double-buffered) while this one is computed;
//   * S accumulates on the packed fp32x2 pipe (even / odd head dims in the two
//     halves, summed once per tile): 64 fma.rn.f32x2 per 12 16-byte loads;
//   * the online softmax needs one max-reduction over the row's 8 lanes;
//     row sums stay per lane until the end;
//   * P overwrites the bias block it was computed from (each element by the
//     thread that read it), and O += P V on the fp32x2 pipe.
// When the grid would leave most SMs idle (few tokens, heads and samples:
// the diffusion steps at a few hundred tokens), the key range is
// split over a thread-block cluster of 2 or 4 CTAs on the same 64 queries.
// Each CTA runs the same loop over its share of the key tiles and parks its
// per-row (max, sum, O) in its own shared memory; after a cluster barrier
// CTA r merges rows [64 r / split, 64 (r + 1) / split) across the cluster
// through distributed shared memory (flash-decoding merge, no global
// scratch), applies the gate and stores.
#include "common.cuh"

namespace bl {
namespace {

constexpr int kBQ = 64, kBK = 64, kThreads = 128;
constexpr int kPld = kBK + 4;  // bias / P row (floats); 16-byte aligned rows

struct TokArgs {
  const float *q, *k, *v, *g;  // g (gate logits) may be null
  int64_t sb, si, sh;  // element strides of q/k/v/g: batch, token, head (dims contiguous)
  const float *bias;
  int64_t bias_sb, bias_sh, bias_sq, bias_sk;
  int bias_div;
  int bias_vec;       // bias rows dense and 16-byte aligned: staged in 16-byte chunks
  const float *mask;  // [B][N] at mask + b * mask_sb + k, or null
  int64_t mask_sb;
  float scale, inf;
  int heads, n;
  int nq;      // queries per batch entry (rows of q / g / bias / out); n for self-attention
  float *out;  // [B][nq][H][d] contiguous, or null when out3 is set
  __nv_bfloat16 *out3;  // [3][B * N][H * d] bf16 planes of the output, or null
  int batch;
  int split;  // CTAs per cluster sharing one query tile's key range (kSplit kernels)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// fp32 at the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ float ld_peer_f32(const float *local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}
template <int D, bool kSplit>
__global__ void __launch_bounds__(kThreads, 2) token_attention_kernel(const TokArgs a) {
  constexpr int kLd = D + 4;   // padded row (floats): conflict-free 16-byte row reads
  constexpr int kDpt = D / 8;  // output dims per thread
  constexpr bool kPairs = kDpt % 2 == 0;
  extern __shared__ float4 smem4[];
  float *qs = reinterpret_cast<float *>(smem4);  // [64][kLd]
  float *ks = qs + kBQ * kLd;                    // [2][64][kLd]
  float *vs = ks + 2 * kBK * kLd;                // [2][64][kLd]
  float *bs = vs + 2 * kBK * kLd;                // [2][64][kPld]: bias block, then P
  float *ms = bs + 2 * kBQ * kPld;               // [2][64]: mask values

  const int t = threadIdx.x, tq = t >> 3, tk = t & 7;
  // With kSplit the cluster (split, 1, 1) shares one query tile: rank = x % split.
  const int split = kSplit ? a.split : 1;
  const int rank = kSplit ? int(blockIdx.x) % split : 0;
  const int q0 = (kSplit ? int(blockIdx.x) / split : int(blockIdx.x)) * kBQ, h = blockIdx.y, b = blockIdx.z;
  const int n = a.n, nq = a.nq;
  const float *qb = a.q + b * a.sb + h * a.sh, *kb = a.k + b * a.sb + h * a.sh, *vb = a.v + b * a.sb + h * a.sh;
  const float *bias = a.bias + int64_t(b / a.bias_div) * a.bias_sb + h * a.bias_sh;
  const float *mask = a.mask ? a.mask + b * a.mask_sb : nullptr;

  // Q tile (rows past n are zero).
  constexpr int kChunks = D / 4;  // 16-byte chunks per row
  for (int i = t; i < kBQ * kChunks; i += kThreads) {
    const int r = i / kChunks, c = i % kChunks;
    const bool ok = q0 + r < nq;
    cp_async16(smem_u32(qs + r * kLd + 4 * c), qb + (ok ? int64_t(q0 + r) * a.si + 4 * c : 0), ok ? 16 : 0);
  }
  auto load_tile = [&](int tile, int buf) {
    const int k0 = tile * kBK;
    for (int i = t; i < kBK * kChunks; i += kThreads) {
      const int r = i / kChunks, c = i % kChunks;
      const bool ok = k0 + r < n;
      const int64_t off = ok ? int64_t(k0 + r) * a.si + 4 * c : 0;
      cp_async16(smem_u32(ks + (buf * kBK + r) * kLd + 4 * c), kb + off, ok ? 16 : 0);
      cp_async16(smem_u32(vs + (buf * kBK + r) * kLd + 4 * c), vb + off, ok ? 16 : 0);
    }
    float *bt = bs + buf * kBQ * kPld;
    if (a.bias_vec) {
#pragma unroll 4
      for (int i = t; i < kBQ * (kBK / 4); i += kThreads) {
        const int r = i >> 4, c = 4 * (i & 15);
        const int qi = q0 + r, kj = k0 + c;
        const int left = n - kj;
        const int bytes = qi < nq ? (left >= 4 ? 16 : left > 0 ? 4 * left : 0) : 0;
        cp_async16(smem_u32(bt + r * kPld + c), bias + (bytes ? int64_t(qi) * a.bias_sq + kj : 0), bytes);
      }
    } else {
#pragma unroll 4
      for (int i = t; i < kBQ * kBK; i += kThreads) {
        const int r = i >> 6, c = i & 63;
        const bool ok = q0 + r < nq && k0 + c < n;
        cp_async4(smem_u32(bt + r * kPld + c),
                  bias + (ok ? int64_t(q0 + r) * a.bias_sq + int64_t(k0 + c) * a.bias_sk : 0), ok);
      }
    }
    if (mask && t < kBK) cp_async4(smem_u32(ms + buf * kBK + t), mask + (k0 + t < n ? k0 + t : 0), k0 + t < n);
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int n_tiles = (n + kBK - 1) / kBK;
  const int t_begin = rank * n_tiles / split, t_end = (rank + 1) * n_tiles / split;  // >= 1 tile each
  load_tile(t_begin, 0);

  float m[4], l[4], o[4][kDpt];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY, l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < kDpt; ++e) o[i][e] = 0.f;
  }
  constexpr float kLog2e = 1.4426950408889634f;
  const uint32_t q_base = smem_u32(qs + 4 * tq * kLd);

  for (int tile = t_begin; tile < t_end; ++tile) {
    const int buf = (tile - t_begin) & 1, k0 = tile * kBK;
    if (tile + 1 < t_end) {
      load_tile(tile + 1, buf ^ 1);  // the buffers were released by the barrier that ended tile - 1
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();

    // S = Q K^T for queries 4 tq + i and keys tk + 8 j; even / odd dims in the two halves.
    uint64_t acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0;
    const uint32_t k_base = smem_u32(ks + (buf * kBK + tk) * kLd);
#pragma unroll 3
    for (int e = 0; e < D; e += 4) {
      uint64_t qa[4], qz[4], ka[8], kz[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) lds_v2b64(q_base + (i * kLd + e) * 4, qa[i], qz[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) lds_v2b64(k_base + (8 * j * kLd + e) * 4, ka[j], kz[j]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ffma2(acc[i][j], qa[i], ka[j]);
          ffma2(acc[i][j], qz[i], kz[j]);
        }
    }
    // Logits (log2 domain), the row max over the 8 lanes, P into the bias block.
    float mk[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int key = tk + 8 * j;
      mk[j] = k0 + key < n ? (mask ? a.inf * (ms[buf * kBK + key] - 1.f) : 0.f) : -INFINITY;
    }
    float *bt = bs + buf * kBQ * kPld + 4 * tq * kPld + tk;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float sc[8], mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sc[j] = ((lo_f(acc[i][j]) + hi_f(acc[i][j])) * a.scale + bt[i * kPld + 8 * j]) + mk[j];
        mx = fmaxf(mx, sc[j]);
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m[i], mx);
      const float alpha = exp2f((m[i] - m_new) * kLog2e);  // 0 on the first tile (m = -inf)
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // s - max first (exact for logits on the same binade grid, e.g. two
        // masked keys near -inf), then the base change; padding keys: exp2(-inf) = 0.
        const float p = exp2f((sc[j] - m_new) * kLog2e);
        sum += p;
        bt[i * kPld + 8 * j] = p;
      }
      l[i] = fmaf(l[i], alpha, sum);  // this lane's share of the row sum
      m[i] = m_new;
#pragma unroll
      for (int e = 0; e < kDpt; ++e) o[i][e] *= alpha;
    }
    __syncwarp();  // a query row's P is written and read by the same 8 lanes
    // O += P V: 4 queries x kDpt contiguous dims (tk * kDpt ...).
    const float *pt = bs + buf * kBQ * kPld + 4 * tq * kPld;
    const uint32_t v_base = smem_u32(vs + buf * kBK * kLd + tk * kDpt);
#pragma unroll 2
    for (int kk = 0; kk < kBK; kk += 4) {
      float4 pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4 *>(pt + i * kPld + kk);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if constexpr (kPairs) {
          uint64_t vv[kDpt / 2];
#pragma unroll
          for (int e = 0; e < kDpt / 2; ++e) vv[e] = lds_b64(v_base + ((kk + u) * kLd + 2 * e) * 4);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p = u == 0 ? pv[i].x : u == 1 ? pv[i].y : u == 2 ? pv[i].z : pv[i].w;
            const uint64_t pp = dup2(p);
#pragma unroll
            for (int e = 0; e < kDpt / 2; ++e) {
              uint64_t acc2 = (uint64_t(__float_as_uint(o[i][2 * e + 1])) << 32) | __float_as_uint(o[i][2 * e]);
              ffma2(acc2, pp, vv[e]);
              o[i][2 * e] = lo_f(acc2), o[i][2 * e + 1] = hi_f(acc2);
            }
          }
        } else {
          const float *vr = vs + buf * kBK * kLd + (kk + u) * kLd + tk * kDpt;
          float vv[kDpt];
#pragma unroll
          for (int e = 0; e < kDpt; ++e) vv[e] = vr[e];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p = u == 0 ? pv[i].x : u == 1 ? pv[i].y : u == 2 ? pv[i].z : pv[i].w;
#pragma unroll
            for (int e = 0; e < kDpt; ++e) o[i][e] = fmaf(p, vv[e], o[i][e]);
          }
        }
      }
    }
    __syncthreads();  // K / V / bias buffer `buf` is free for the tile after next
  }
  if constexpr (kSplit) {
    // Partials into the Q tile (no longer read): row r holds O at [0, D),
    // the row maximum at D and the row sum at D + 1.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], off);
      float *row = qs + (4 * tq + i) * kLd;
#pragma unroll
      for (int e = 0; e < kDpt; ++e) row[tk * kDpt + e] = o[i][e];
      if (tk == 0) row[D] = m[i], row[D + 1] = l[i];
    }
    cluster_sync_all();  // every CTA's partials are visible cluster-wide
    // kThreads / rows threads per merged row; all peer loads of a row are
    // independent (issued together), then the weighted sums.
    const int rows = kBQ / split, tpr = kThreads / rows;
    const int r = rank * rows + t / tpr, part = t % tpr;
    const int qi = q0 + r;
    const float *row = qs + r * kLd;
    float mp[4], lp[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      mp[p] = p < split ? ld_peer_f32(row + D, uint32_t(p)) : -INFINITY;
      lp[p] = p < split ? ld_peer_f32(row + D + 1, uint32_t(p)) : 0.f;
    }
    const float mx = fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3]));
    float w[4], sum = 0.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      w[p] = p < split ? exp2f((mp[p] - mx) * kLog2e) : 0.f;
      sum = fmaf(lp[p], w[p], sum);
    }
    const float inv = 1.f / sum;
    const int64_t at0 = ((int64_t(b) * nq + qi) * a.heads + h) * D;
    const float *gr = a.g ? a.g + b * a.sb + h * a.sh + int64_t(qi) * a.si : nullptr;
    for (int d0 = part; d0 < D; d0 += 4 * tpr) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f}, ov[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int d = d0 + u * tpr;
          ov[u][p] = p < split && d < D ? ld_peer_f32(row + d, uint32_t(p)) : 0.f;
        }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[u] = fmaf(ov[u][p], w[p], acc[u]);
        const int d = d0 + u * tpr;
        if (qi < nq && d < D) {
          const float y = acc[u] * inv;
          const float out_v = gr ? y * (1.f / (1.f + expf(-gr[d]))) : y;
          if (a.out3)
            store_split3_1(a.out3, int64_t(a.batch) * nq * a.heads * D, at0 + d, out_v);
          else
            a.out[at0 + d] = out_v;
        }
      }
    }
    cluster_sync_all();  // peers may still be reading this CTA's partials
  } else {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], off);
    const int qi = q0 + 4 * tq + i;
    if (qi >= nq) continue;
    const float inv = 1.f / l[i];
    const int64_t at = ((int64_t(b) * nq + qi) * a.heads + h) * D + tk * kDpt;
    float *dst = a.out + at;
    const float *gr = a.g ? a.g + b * a.sb + h * a.sh + int64_t(qi) * a.si + tk * kDpt : nullptr;
#pragma unroll
    for (int e = 0; e < kDpt; ++e) {
      const float y = o[i][e] * inv;
      const float out_v = gr ? y * (1.f / (1.f + expf(-gr[e]))) : y;
      if (a.out3)
        store_split3_1(a.out3, int64_t(a.batch) * nq * a.heads * D, at + e, out_v);
      else
        dst[e] = out_v;
    }
  }
  }
}

template <int D> int launch_token(TokArgs a, int batch, cudaStream_t stream) {
  constexpr int kLd = D + 4;
  const int smem = (kBQ * kLd + 4 * kBK * kLd + 2 * kBQ * kPld + 2 * kBK) * 4;
  const int q_tiles = (a.nq + kBQ - 1) / kBQ;
  // Split the key range over a cluster when the grid would occupy at most
  // half of the SMs (measured on B200: 18 -> 15 us at 117 tokens, 25 -> 17 us
  // at 200-256 tokens, 16 heads; neutral at 96-128 CTAs, 4 % slower at 256).
  const int64_t ctas = int64_t(q_tiles) * a.heads * batch, sms = num_sms();
  int split = 1;
  if (2 * ctas <= sms && q_tiles >= 2) split = (q_tiles >= 4 && 4 * ctas <= 2 * sms) ? 4 : 2;
  if (split == 1) {
    BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(token_attention_kernel<D, false>), smem));
    dim3 grid(q_tiles, a.heads, batch);
    token_attention_kernel<D, false><<<grid, kThreads, smem, stream>>>(a);
    BL_LAUNCH_CHECK();
    return BL_OK;
  }
  a.split = split;
  BL_CUDA(ensure_smem_limit(reinterpret_cast<const void *>(token_attention_kernel<D, true>), smem));
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(unsigned(q_tiles * split), unsigned(a.heads), unsigned(batch));
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  BL_CUDA(cudaLaunchKernelEx(&config, token_attention_kernel<D, true>, a));
  BL_LAUNCH_CHECK();
  return BL_OK;
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_token_attention(const float *q, const float *k, const float *v, const float *g, int64_t sb,
                                  int64_t si, int64_t sh,
                                  const float *bias, int64_t bias_sb, int64_t bias_sh, int64_t bias_sq,
                                  int64_t bias_sk, int64_t bias_batch_div, const float *mask, int64_t mask_sb,
                                  float scale, float inf, int64_t batch, int64_t heads, int64_t n, int64_t n_q,
                                  int64_t head_dim, float *out, void *out3, void *stream) {
  if (n_q == 0) n_q = n;
  BL_REQUIRE(batch >= 0 && heads > 0 && n >= 0 && n_q >= 0, "bl_token_attention: bad shape");
  if (batch == 0 || n == 0 || n_q == 0) return BL_OK;
  BL_REQUIRE(head_dim == 24 || head_dim == 32 || head_dim == 48 || head_dim == 64,
             "bl_token_attention: head_dim 24, 32, 48 or 64");
  BL_REQUIRE(q && k && v && bias && (out || out3) && bias_batch_div >= 1, "bl_token_attention: null pointer");
  BL_REQUIRE(aligned_to(q, 16) && aligned_to(k, 16) && aligned_to(v, 16) && aligned_to(g, 4) && si % 4 == 0 &&
                 sh % 4 == 0 &&
                 sb % 4 == 0,
             "bl_token_attention: q/k/v rows must be 16-byte aligned");
  BL_REQUIRE(n < (1 << 20) && n_q < (1 << 20) && heads < 65536 && batch < 65536, "bl_token_attention: shape too large");
  TokArgs a{};
  a.q = q, a.k = k, a.v = v, a.g = g, a.sb = sb, a.si = si, a.sh = sh;
  a.bias = bias, a.bias_sb = bias_sb, a.bias_sh = bias_sh, a.bias_sq = bias_sq, a.bias_sk = bias_sk;
  a.bias_div = int(bias_batch_div);
  a.bias_vec = bias_sk == 1 && bias_sq % 4 == 0 && bias_sh % 4 == 0 && (bias_batch_div >= batch || bias_sb % 4 == 0) &&
               aligned_to(bias, 16);
  a.mask = mask, a.mask_sb = mask_sb;
  a.scale = scale, a.inf = inf;
  a.heads = int(heads), a.n = int(n), a.nq = int(n_q);
  a.out = out, a.out3 = static_cast<__nv_bfloat16 *>(out3), a.batch = int(batch);
  cudaStream_t s = as_stream(stream);
  if (head_dim == 24) return launch_token<24>(a, int(batch), s);
  if (head_dim == 32) return launch_token<32>(a, int(batch), s);
  if (head_dim == 48) return launch_token<48>(a, int(batch), s);
  return launch_token<64>(a, int(batch), s);
}
