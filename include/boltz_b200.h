/*
 * boltz_b200.h -- C ABI of the B200 (sm_100a) kernels for Boltz-2's pair path.
 *
 * Every entry point takes plain device pointers, element counts and a
 * cudaStream_t passed as void*, launches asynchronously on that stream and
 * returns a BL_* status.  On failure bl_last_error() holds a message (per
 * calling thread).  No entry point allocates device memory: intermediate
 * buffers are passed in by the caller, except for bl_pair_transition_static,
 * whose intermediates live in a fixed array compiled into the library (see
 * its declaration).  Inference only: nothing here records autograd state.
 *
 * Each declaration names the reference interface it replaces
 * (lauritsf/boltz-lumi, path relative to src/boltz_lumi/).
 */
#ifndef BOLTZ_B200_H
#define BOLTZ_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define BL_API __attribute__((visibility("default")))
#else
#define BL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum {
  BL_OK = 0,
  BL_ERR_INVALID = 1,     /* bad shape, dtype, alignment or pointer          */
  BL_ERR_CUDA = 2,        /* a CUDA runtime call failed                       */
  BL_ERR_UNSUPPORTED = 3, /* valid request outside what the kernels cover     */
  BL_ERR_TIMEOUT = 4      /* a bounded device-side wait gave up               */
};

/* Element types. */
enum { BL_F32 = 0, BL_BF16 = 1 };

/* Diffusion epilogue kinds; values match the reference's operation codes
 * (diffusion.py:27 MODULATION, GATE, GATED_SWIGLU = 0, 1, 3). */
enum { BL_EPI_MODULATION = 0, BL_EPI_GATE = 1, BL_EPI_GATED_SWIGLU = 3 };
/* silu(a[:, :cols]) * a[:, cols:] (an fp32 Transition's fc1 | fc2 product,
 * the Pairformer's transition_s); no counterpart code in the reference, which
 * leaves 2 unused. */
enum { BL_EPI_SWIGLU = 2 };

/* Message for the last failed call on this thread ("" if none). */
BL_API const char *bl_last_error(void);

/* ABI version of this library. */
BL_API int bl_version(void);

/* Device-side status word of the current device: 0 when every bounded wait
 * completed, otherwise a code naming the wait that gave up.  reset != 0
 * clears it.  Synchronises the device. */
BL_API int bl_device_status(int reset);

/* Self-test of the bounded device-side wait used by every tensor-core kernel:
 * one thread waits on an mbarrier phase with a limit of limit_ns (at most
 * 2 s).  arrive != 0 completes the phase first (the wait succeeds, the status
 * word stays 0); arrive == 0 leaves it incomplete, so the wait gives up after
 * limit_ns, records 0x7F01 in the status word (read it with
 * bl_device_status) and the kernel returns normally.  Diagnostic only; no
 * counterpart in the reference. */
BL_API int bl_wait_selftest(int arrive, int64_t limit_ns, void *stream);

/*
 * LayerNorm over `cols` channels, fp32 statistics.
 * Replaces kernels/multiplication_hip.cu:149 `multiplication_norm`
 * (bound as extension("multiplication").norm, used at triangle.py:240 and
 * multiplication.py:88,124).
 *   channel_first = 0: x is [rows, cols] row-major.
 *   channel_first = 1: x is [cols, rows] (one plane per channel); cols must be 128.
 * out is [rows, cols] row-major.  weight / bias may be NULL (no affine).
 */
BL_API int bl_layernorm(const void *x, int x_dtype, int64_t rows, int64_t cols, int channel_first,
                 const float *weight, const float *bias, float eps, void *out, int out_dtype,
                 void *stream);

/*
 * Sigmoid gate: out = bf16(p * bf16(sigmoid(g))), all bf16, n elements.
 * Replaces kernels/multiplication_gate_hip.cu:81 `multiplication_gate`
 * (extension("multiplication_gate").gate, multiplication.py:137).
 */
BL_API int bl_gate(const void *p, const void *g, void *out, int64_t n, void *stream);

/*
 * Gate, mask and pack the triangle-multiplication operands into
 * channel-first planes for a per-channel batched matmul.
 * Replaces kernels/multiplication_gate_hip.cu:140 `multiplication_gate_pack`
 * (multiplication.py:106).  p, g: bf16 [n, n, 256] with row stride
 * `pair_stride` elements (256 dense, 512 for a joint projection); mask: fp32
 * [n, n].  Outputs left, right: bf16 [128, n, n]:
 *   outgoing: left[c][i][k] = a[i][k][c], right[c][k][j] = b[j][k][c]
 *   incoming: left[c][i][k] = a[k][i][c], right[c][k][j] = b[k][j][c]
 * where a / b are channels 0..127 / 128..255 of bf16(p * bf16(sigmoid(g))) * mask.
 */
BL_API int bl_gate_pack(const void *p, const void *g, int64_t pair_stride, const float *mask, int64_t n,
                 int outgoing, void *left, void *right, void *stream);

/*
 * Gate and mask into channel-last halves: a, b bf16 [n*n, 128].
 * Replaces kernels/multiplication_gate_hip.cu:96 `multiplication_gate_split`
 * (multiplication.py:110).
 */
BL_API int bl_gate_split(const void *p, const void *g, int64_t pair_stride, const float *mask, int64_t n,
                  void *a, void *b, void *stream);

/*
 * out = bf16(bf16(silu(a)) * b), all bf16, n elements, any alignment.
 * Replaces kernels/pair_hip.cu:42 `pair_silu_mul` (pair_transition.py:161).
 */
BL_API int bl_silu_mul(const void *a, const void *b, void *out, int64_t n, void *stream);

/*
 * fp32 diffusion epilogues over rows x cols outputs (contiguous):
 *   MODULATION:   out = sigmoid(b) * a + c
 *   GATE:         out = sigmoid(a) * b
 *   GATED_SWIGLU: a is [rows, 2*cols]; out = silu(a[:, cols:]) * a[:, :cols] * b
 *   SWIGLU:       a is [rows, 2*cols]; out = silu(a[:, :cols]) * a[:, cols:]   (b unused, may be NULL)
 * Replaces kernels/diffusion_hip.cu:80 `diffusion_epilogue` (diffusion.py:52-68).
 */
BL_API int bl_diffusion_epilogue(const float *a, const float *b, const float *c, float *out,
                          int64_t rows, int64_t cols, int kind, void *stream);

/*
 * Fused AdaLN modulation: out = sigmoid(scale) * LayerNorm(a) + shift, where
 * the LayerNorm has no affine (upstream AdaLN.a_norm).  fp32, [rows, cols].
 * Fuses the a_norm call and the MODULATION epilogue of diffusion.py:52-57.
 */
BL_API int bl_adaln_modulate(const float *a, const float *scale, const float *shift, float *out,
                      int64_t rows, int64_t cols, float eps, void *stream);

/*
 * Ordered bias softmax of materialised triangle scores:
 *   p = softmax(round(round(s + mask) + bias)) rounded to the score dtype.
 * Replaces kernels/triangle_softmax.py:120 `ordered_softmax` and
 * kernels/triangle_block_softmax_hip.cu:120 `triangle_block_softmax`
 * (triangle.py:88-100).  scores: [B, I, H, N, N] of `dtype` with element
 * strides ss[5]; bias: `dtype`, indexed by (b, h, q, k) with strides bs[4];
 * mask: fp32 indexed by (b, i, k) with strides ms[3]; out: contiguous
 * [B, I, H, N, N] of `dtype`.
 */
BL_API int bl_triangle_softmax(const void *scores, int dtype, int64_t batch, int64_t outer, int64_t heads,
                        int64_t n, const int64_t *ss, const void *bias, const int64_t *bs,
                        const float *mask, const int64_t *ms, void *out, void *stream);

/*
 * Batched bf16 GEMM on tcgen05 tensor cores, fp32 accumulation, bf16 output:
 *   C[b](m, n) = sum_k A[b](m, k) * B[b](n, k) + bias[n]   (bias may be NULL)
 * Replaces the torch.bmm / torch.matmul calls of the reference path
 * (multiplication.py:122 `torch.bmm(left, right)`, triangle.py:194,208).
 * A is K-major (A[b][m][k] at a + b*a_batch_stride + m*a_ld + k) or, with
 * a_mn_major, MN-major (A[b][k][m] at a + b*a_batch_stride + k*a_ld + m);
 * likewise B.  C[b][m][n] at c + b*c_batch_stride + m*c_ld + n.
 * Pointers 16-byte aligned; leading dimensions and batch strides multiples
 * of 8 elements.  Rows/columns past m, n, k are handled by the TMA bounds.
 */
BL_API int bl_batched_gemm(const void *a, int a_mn_major, int64_t a_ld, int64_t a_batch_stride,
                           const void *b, int b_mn_major, int64_t b_ld, int64_t b_batch_stride, void *c,
                           int64_t c_ld, int64_t c_batch_stride, int64_t batch, int64_t m, int64_t n,
                           int64_t k, const float *bias, void *stream);

/*
 * Linear layer over pair rows on tcgen05 with a fused epilogue; one N tile
 * per row block.  acc = [A | A2] . W^T, where A [m, k1] (row stride a_ld) and
 * the optional A2 [m, k - k1] (row stride a2_ld) are concatenated along K
 * (k1 a multiple of 64), W bf16 [n, k] (row stride w_ld).
 *   gate = 0, n = 128: y = bf16(acc + bias)                          (bias may be NULL)
 *   gate = 1, n = 256: y[:, c] = bf16(bf16(acc[c]) * bf16(sigmoid(bf16(acc[128 + c]))))
 * Exactly one of z / out: z (fp32 rows of z_ld) receives z += y, the residual
 * update of the Pairformer block; out (bf16 rows of out_ld) receives y.
 * Replaces the output linears of the reference path and the gate that follows
 * them: linear_o of upstream _wrap_up (triangle.py:104), p_out / g_out and the
 * K-gate `gate` (multiplication.py:135-137), fc3 (pair_transition.py:165).
 */
BL_API int bl_linear_fused(const void *a, int64_t a_ld, const void *a2, int64_t a2_ld, int64_t k1,
                           const void *w, int64_t w_ld, int64_t m, int64_t n, int64_t k,
                           const float *bias, int gate, float *z, int64_t z_ld, void *out,
                           int64_t out_ld, void *stream);

/*
 * Triangle-attention input stage in one pass over the fp32 pair rows
 * x [n_outer*n][128] (16-byte aligned; n_outer = n for a whole pair tensor,
 * fewer for a row slab of a sharded one):
 *   x_hat = bf16(LayerNorm(x))                                  (fp32 statistics)
 *   y[r][0:512] = bf16(x_hat[r] . w^T + bias)                   w bf16 [512][128] = q | k | v | g rows
 *   proj[r] = bf16(y_q * q_scale) | y_k | y_v | bf16(sigmoid(y_g))  (the flash kernel's operands)
 *   bias_planes[h][q][k] = bf16(x_hat[q*n + k] . w_heads[h])    (transpose = 0, starting node)
 *   bias_planes[h][k][q] = same                                 (transpose = 1, ending node)
 * bias (fp32 [512]) may be NULL; w_heads is bf16 [4][128]; proj rows are
 * proj_ld >= 512 elements (multiple of 8); bias plane h at bias_planes + h*bias_hs,
 * rows of bias_ld elements.
 * Replaces the layer_norm fast path (triangle.py:107-146), the q/k/v/g
 * linears of _prep_qkv (triangle.py:80, upstream Attention) and upstream's
 * triangle-bias `linear` that feed ordered_triangle_forward (triangle.py:32).
 */
BL_API int bl_attention_projection(const float *x, int64_t n, int64_t n_outer, const float *ln_weight,
                                   const float *ln_bias, float eps, const void *w, const float *bias,
                                   float q_scale, const void *w_heads, int transpose, void *proj,
                                   int64_t proj_ld, void *bias_planes, int64_t bias_ld, int64_t bias_hs,
                                   void *stream);

/*
 * Triangle-multiplication input stage in one pass over the fp32 pair rows
 * x [n_outer*n][128] (outer index i < n_outer, inner k < n):
 *   x_hat = bf16(LayerNorm(x)) -> xn [n*n][128]
 *   p = x_hat . w[0:256]^T, g = x_hat . w[256:512]^T        (bf16 results; w = [p_in; g_in])
 *   planes[c][i][k] = bf16(bf16(p_c * bf16(sigmoid(g_c))) * mask[i*n + k])   c < 256
 * planes is bf16 [256][n_outer][plane_ld] (channels 0..127 = a, 128..255 = b),
 * plane_ld >= n and a multiple of 8.  Replaces norm_in + p_in/g_in + the
 * gate/pack/split kernels and layout copies of multiplication.py:48-120
 * (multiplication_gate_hip.cu:16-58).
 */
BL_API int bl_trimul_projection(const float *x, int64_t n, int64_t n_outer, const float *ln_weight,
                                const float *ln_bias, float eps, const void *w, const float *mask, void *planes,
                                int64_t plane_ld, void *xn, void *stream);

/*
 * Pair transition in one pass over fp32 rows x [rows][128]:
 *   x_hat = bf16(LayerNorm(x)), u = bf16(bf16(silu(bf16(x_hat fc1^T))) * bf16(x_hat fc2^T)),
 *   y = bf16(u fc3^T)
 * then z += y (z fp32 [rows][128], may alias x) or out = y (bf16 [rows][128]);
 * exactly one of z and out is non-NULL.  w12 is bf16 [1024][128] (fc1 rows
 * then fc2 rows), w3 is bf16 [128][512].  Replaces upstream
 * Transition.forward (pair_transition.py:8-28) including the pair_silu_mul
 * kernel (kernels/pair_hip.cu:42-64); the hidden activations stay on chip.
 */
BL_API int bl_pair_transition(const float *x, int64_t rows, const float *ln_weight, const float *ln_bias,
                              float eps, const void *w12, const void *w3, float *z, void *out, void *stream);

/*
 * Output stage of the triangle multiplication:
 *   o_hat = bf16(LayerNorm(O)) over the 128 channels of the product planes
 *           prod bf16 [128][n_outer][ld] (O_c[i][j] at c*n_outer*ld + i*ld + j, i < n_outer),
 *   y = bf16(bf16(o_hat p_out^T) * bf16(sigmoid(bf16(x_hat g_out^T))))
 * with x_hat = xn bf16 [n_outer*n][128] and w_out = bf16 [256][128] (p_out rows
 * then g_out rows); then z += y (fp32 [n_outer*n][128]) or out = y (bf16), exactly one
 * non-NULL.  ld is a multiple of 8, pointers 16-byte aligned.  Replaces
 * norm_out + p_out + g_out + the gate of multiplication.py:124-137 and the
 * Pairformer's residual add.
 */
BL_API int bl_trimul_output(const void *prod, int64_t n, int64_t n_outer, int64_t ld, const float *ln_weight,
                            const float *ln_bias, float eps, const void *xn, const void *w_out, float *z,
                            void *out, void *stream);

/*
 * Pair bias of the single-track attention, fp32, in one pass over z:
 *   out[h][r] = sum_c LayerNorm(z[r])[c] * w[h][c]     z [rows][128], w [heads][128], heads <= 16
 * (the LayerNorm has fp32 statistics and optional affine ln_weight/ln_bias).
 * Replaces upstream AttentionPairBias.proj_z (LayerNorm -> Linear(c_z, heads,
 * bias=False) -> permute to [heads, N, N]) of the Pairformer block.
 */
BL_API int bl_pair_bias(const float *z, int64_t rows, const float *ln_weight, const float *ln_bias, float eps,
                        const float *w, int64_t heads, float *out, void *stream);

/*
 * Pair-transition activation on the joint fc1|fc2 projection:
 *   out[r][c] = bf16(bf16(silu(x[r][c])) * x[r][width + c]).
 * Replaces kernels/pair_hip.cu:42 `pair_silu_mul` on separate fc1/fc2
 * outputs (pair_transition.py:157-165).
 */
BL_API int bl_swiglu_rows(const void *x, int64_t x_ld, int64_t rows, int64_t width, void *out,
                          int64_t out_ld, void *stream);

/*
 * Flash triangle attention with fused output gate (bf16):
 *   out(a, b) = bf16(bf16(softmax_c(bf16(bf16(bf16(q_s . k) + inf*(mask-1)) + bias)) v) * s_g)
 * where q_s = bf16(q / sqrt(32)) and s_g = bf16(sigmoid(g)) are passed in
 * already prepared (bl_attention_projection writes them).  Replaces
 * triangle.py:139 `ordered_triangle_forward` (q k^T, ordered bias softmax,
 * p v) and the gate of upstream Attention._wrap_up.  q_s, k, v, s_g:
 * bf16 pair rows of ld elements, head h at columns h*32..h*32+31, pair row of
 * (outer a, inner b) = a*so + b*si (starting node: so = n, si = 1; ending
 * node: so = 1, si = n).  bias(h, b, c) at bias + h*bias_hs + b*bias_ld + c.
 * mask(a, c) at mask + a*ms_o + c*ms_k (fp32).  out rows of out_ld elements
 * at the same pair rows.  n is the key / query extent, n_outer the number of
 * outer rows a processed (n for a whole pair tensor, fewer for a row slab).
 * heads must be 4 and head_dim 32, n <= 4096, 0 <= inf <= 1e20; all pointers
 * 16-byte aligned, ld / out_ld / bias_ld / bias_hs multiples of 8.  Runs on
 * tcgen05 tensor cores (scores and P in TMEM, TMA-fed key tiles).
 */
BL_API int bl_triangle_attention(const void *q, const void *k, const void *v, const void *g, int64_t ld,
                                 int64_t so, int64_t si, const void *bias, int64_t bias_ld,
                                 int64_t bias_hs, const float *mask, int64_t ms_o, int64_t ms_k,
                                 float inf, int64_t heads, int64_t head_dim, int64_t n, int64_t n_outer,
                                 void *out, int64_t out_ld, void *stream);

/*
 * Triangle attention followed by its output projection and the block's
 * residual add (fp32 z):
 *   z[pair] += bf16(out(a, b) . W_o^T + b_o)
 * with out(a, b) as in bl_triangle_attention and pair = a*so + b*si.
 * Replaces, on top of bl_triangle_attention's span, linear_o of upstream
 * _wrap_up (triangle.py:104) and the Pairformer's residual add of the
 * triangle-attention update.
 * w_o: bf16 [128][128] row-major (linear_o.weight), b_o: fp32 [128];
 * z: fp32 rows of z_ld elements (z_ld a multiple of 4, 16-byte aligned).
 * scratch: bf16 rows of scratch_ld elements at the same pair rows, written
 * only when the projection runs as a separate GEMM (fewer than four heads per
 * CTA at this size; the output rows must then be contiguous: starting node,
 * or ending node over the whole tensor).  When the grid fills the GPU eight
 * times over (4 * ceil(n / 128) * n_outer >= 32 * SMs) the projection runs in
 * the attention kernel's epilogue and the gated tensor never reaches memory.
 * Either way z equals bl_triangle_attention + bl_linear_fused bit for bit.
 */
BL_API int bl_triangle_attention_residual(const void *q, const void *k, const void *v, const void *g,
                                          int64_t ld, int64_t so, int64_t si, const void *bias,
                                          int64_t bias_ld, int64_t bias_hs, const float *mask, int64_t ms_o,
                                          int64_t ms_k, float inf, int64_t heads, int64_t head_dim, int64_t n,
                                          int64_t n_outer, void *scratch, int64_t scratch_ld, const void *w_o,
                                          const float *b_o, float *z, int64_t z_ld, void *stream);

/*
 * Attention core of the diffusion token transformer, fp32 end to end:
 *   out[b][i][h][:] = sigmoid(g[b][i][h][:]) * sum_j softmax_j(s) v[b][j][h][:],
 *   s = (q[b][i][h] . k[b][j][h]) * scale + bias[b / bias_batch_div][h][i][j]
 *       + inf * (mask[b][j] - 1)
 * q, k, v and the gate logits g (NULL: no gate): fp32, element (b, i, h, e)
 * at b*sb + i*si + h*sh + e (strides multiples of 4, q/k/v 16-byte aligned); bias: element (b', h, i, j) at
 * b'*bias_sb + h*bias_sh + i*bias_sq + j*bias_sk, so a layer's slice of the
 * prepared [B, L*H, N, N] token bias is passed without a copy and one bias
 * row serves the bias_batch_div diffusion samples of its input; mask: fp32
 * at b*mask_sb + j, or NULL for none; head_dim 24, 32, 48 or 64; out: fp32
 * [batch][n_q][heads][head_dim] contiguous.  n_q queries (rows of q, g, bias and
 * out; 0 means n) attend over the n keys: a rank of the row-sharded block passes
 * its own query rows (pointers offset to them) against all keys.  Replaces the
 * einsum / bias / mask / softmax / einsum and the gate product of
 * pair_bias.py:28-36 (prepared_forward).
 * With out3 != NULL the result is written instead as three bf16 planes
 * [3][batch * n_q][heads * head_dim] (the operand form of bl_linear_split3,
 * for proj_o) and out may be NULL.
 */
BL_API int bl_token_attention(const float *q, const float *k, const float *v, const float *g, int64_t sb,
                              int64_t si, int64_t sh,
                              const float *bias, int64_t bias_sb, int64_t bias_sh, int64_t bias_sq,
                              int64_t bias_sk, int64_t bias_batch_div, const float *mask, int64_t mask_sb,
                              float scale, float inf, int64_t batch, int64_t heads, int64_t n, int64_t n_q,
                              int64_t head_dim, float *out, void *out3, void *stream);

/*
 * fp32-accurate linear layers on the bf16 tensor cores (three-way split).
 * bl_split3_bf16: out = bf16 planes [3][rows][cols] with x = x1 + x2 + x3
 *   (x1 = bf16(x), x2 = bf16(x - x1), x3 = bf16(x - x1 - x2); |x - sum| <=
 *   2^-27 |x|); x fp32 rows of ldx elements; cols and ldx multiples of 4.
 * bl_linear_split3: y[i][j] = sum_k x[i][k] w[j][k] + bias[j] from the split
 *   planes x3 [3][m][k] and w3 [3][n][k] (bl_split3_bf16 of x and of the fp32
 *   weight), keeping every cross product down to 2^-24 relative (error
 *   within 2^-17 of the largest output); y fp32 rows of ldy; k % 8 == 0,
 *   n % 4 == 0, ldy % 4 == 0, pointers 16-byte aligned; bias may be NULL;
 *   residual (fp32 rows of ldr, NULL for none) is added to y: the block's
 *   s = s + proj_o(o) and s = s + fc3(h) without a separate add pass.
 * Replaces the fp32 linears the reference leaves to the BLAS: the diffusion
 * AdaLN / ConditionedTransitionBlock projections (diffusion.py:55-68) and the
 * AttentionPairBias projections (pair_bias.py:22-28, 36).
 */
BL_API int bl_split3_bf16(const float *x, int64_t rows, int64_t cols, int64_t ldx, void *out, void *stream);
BL_API int bl_linear_split3(const void *x3, int64_t m, int64_t k, const void *w3, int64_t n, const float *bias,
                            const float *residual, int64_t ldr, float *y, int64_t ldy, void *stream);

/*
 * Producers of fp32-linear operands that write the three bf16 planes
 * [3][rows][cols] (as bl_split3_bf16 would) instead of fp32, saving the
 * separate split pass:
 *   bl_layernorm_split3:          LayerNorm of fp32 rows (cols % 128 == 0, <= 1024),
 *                                 the s_norm of AdaLN (diffusion.py:55-57);
 *   bl_adaln_modulate_split3:     bl_adaln_modulate's result (the conditioned
 *                                 transition's a', diffusion.py:63-65);
 *   bl_diffusion_epilogue_split3: bl_diffusion_epilogue's result (cols % 4 == 0;
 *                                 GATED_SWIGLU's b feeds b_to_a, diffusion.py:66-68).
 */
BL_API int bl_layernorm_split3(const float *x, int64_t rows, int64_t cols, const float *weight, const float *bias,
                               float eps, void *out3, void *stream);
BL_API int bl_adaln_modulate_split3(const float *a, const float *scale, const float *shift, void *out3, int64_t rows,
                                    int64_t cols, float eps, void *stream);
BL_API int bl_diffusion_epilogue_split3(const float *a, const float *b, const float *c, void *out3, int64_t rows,
                                        int64_t cols, int kind, void *stream);

/*
 * Pair transition (LayerNorm -> fc1|fc2 -> SwiGLU -> fc3, the bf16-autocast
 * contract) that allocates no device memory.  This entry point has no
 * counterpart in the reference; it exists for callers that may not allocate
 * device memory while they run inference -- hosts that keep all of HBM in
 * their own pool, or plugin interfaces that pass a kernel only its inputs
 * and outputs.  The intermediates live in a fixed array compiled into the
 * library (3.25 MiB, held on every GPU that loads the library until exit).
 *   x: fp32 [rows, 128]; ln_weight, ln_bias: fp32 [128] (may be NULL);
 *   w12: bf16 [1024, 128] (fc1 rows then fc2 rows); w3: bf16 [128, 512];
 *   out: bf16 [rows, 128].  rows <= 1024, otherwise BL_ERR_INVALID.
 *   x, w12, w3 and out must be 16-byte aligned.
 * Runs on the current device.  Its first call on a device looks up the
 * array's device address, so make that first call before any stream
 * capture.  The address is kept for the life of the process: do not use
 * this entry point across a cudaDeviceReset.  All calls on a device share
 * the array: calls that overlap on the GPU (e.g. on two streams) race; calls
 * ordered on one stream do not.
 */
BL_API int bl_pair_transition_static(const float *x, int64_t rows, const float *ln_weight,
                                     const float *ln_bias, float eps, const void *w12, const void *w3,
                                     void *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BOLTZ_B200_H */
