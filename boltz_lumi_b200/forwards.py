"""Replacement forwards of the upstream Boltz-2 modules on the pair hot path.

Each function takes the module as ``self`` (it is bound with
``types.MethodType`` exactly like the reference's adapter, adapters.py:24-47)
and reads only upstream attribute names, so it works both on upstream Boltz
2.2.1 modules and on the standalone classes of :mod:`boltz_lumi_b200.layers`.

Numerics follow upstream's eager path under bf16 autocast for the trunk
(TriangleAttention, TriangleMultiplication, Transition) and plain fp32 for the
diffusion AdaLN / ConditionedTransitionBlock.  All compute runs in the sm_100a
kernels of ``libboltz_b200.so``; there is no CPU path.

The trunk forwards return the bf16 update like upstream.  Given
``residual=z`` (an fp32 pair tensor of the same shape) they instead add the
update into ``z`` inside the last GEMM's epilogue and return ``z``: this is
how the Pairformer block applies ``z = z + op(z)`` without a separate pass.
"""

import torch
import torch.nn.functional as F

from . import _lib, atom_conditioning, kernels
from ._lib import call, stream_of

_BF16 = torch.bfloat16
# fp32(1 / fp32(sqrt(32))): the factor torch's CUDA kernel applies for q / sqrt(32).
_Q_SCALE = float(torch.tensor(1.0, dtype=torch.float32) / torch.tensor(32.0, dtype=torch.float32).sqrt())

def _pad8(n):
    return (n + 7) // 8 * 8


def _cached(module, name, params, build):
    """Derived weights, rebuilt when any source parameter changes identity,
    in-place version or storage (a move to another device or dtype makes new
    storage): the invalidation events of the reference's cache key
    (multiplication.py:29-40), checked with cheap attribute reads."""
    key = tuple((id(p), p._version, p.data_ptr()) for p in params if p is not None)
    cached = getattr(module, name, None)
    if cached is None or cached[0] != key:
        with torch.no_grad():
            cached = (key, build())
        setattr(module, name, cached)
    return cached[1]


def _check_pair_input(x, mask, c=128):
    if not x.is_cuda:
        raise RuntimeError("pair ops need CUDA tensors")
    if x.dim() != 4 or x.shape[1] != x.shape[2] or x.shape[-1] != c:
        raise RuntimeError(f"expected a pair tensor [B, N, N, {c}], got {tuple(x.shape)}")
    if mask is not None and tuple(mask.shape) != tuple(x.shape[:-1]):
        raise RuntimeError("pair mask must be [B, N, N]")


def _check_residual(residual, x):
    if residual is None:
        return
    if residual.dtype != torch.float32 or not residual.is_contiguous() or residual.shape != x.shape:
        raise RuntimeError("residual must be a contiguous fp32 tensor shaped like the input")


def _f32(t):
    return None if t is None else t.float().contiguous()


def _layer_norm_bf16(x2d, norm):
    return kernels.layer_norm(x2d, _f32(norm.weight), _f32(getattr(norm, "bias", None)), norm.eps, out_dtype=_BF16)


def _linear_bf16(x2d, weight_bf16, bias=None):
    """Autocast linear on tcgen05: bf16 operands, fp32 accumulation, bf16 result."""
    return kernels.bmm(x2d.unsqueeze(0), weight_bf16.unsqueeze(0), bias=bias).squeeze(0)


def _linear_out(a, w, rows, k, stream, bias=None, a2=None, k1=None, gate=False, residual=None, out=None):
    """bl_linear_fused: residual (fp32 rows += y) or out (bf16 rows = y)."""
    n = w.shape[0]
    call("bl_linear_fused", a.data_ptr(), a.stride(0), None if a2 is None else a2.data_ptr(),
         0 if a2 is None else a2.stride(0), k if k1 is None else k1, w.data_ptr(), w.stride(0), rows, n, k,
         None if bias is None else bias.data_ptr(), int(gate),
         None if residual is None else residual.data_ptr(), 0 if residual is None else residual.shape[-1],
         None if out is None else out.data_ptr(), 0 if out is None else out.shape[-1], stream)


def _split_weight(module, name, weights, biases=None):
    """bf16 split planes [3, N, K] of the row-concatenated fp32 ``weights``
    (and their joint fp32 bias, zeros where a part has none), cached on the
    module until a source parameter changes."""
    biases = list(biases) if biases is not None else [None] * len(weights)
    params = tuple(weights) + tuple(b for b in biases if b is not None)

    def build():
        w = torch.cat([x.float() for x in weights], 0).contiguous()
        bias = None
        if any(b is not None for b in biases):
            bias = torch.cat([b.float() if b is not None else torch.zeros(x.shape[0], device=w.device)
                              for x, b in zip(weights, biases)]).contiguous()
        return kernels.split3(w), bias

    return _cached(module, name, params, build)


def _linear32(module, name, x, weights, biases=None, x3=None):
    """fp32 ``x @ [W_1; W_2; ...]^T + bias`` (upstream's fp32 nn.Linear calls,
    autocast off) on the tensor cores via the three-way bf16 split
    (bl_linear_split3); shapes it does not cover stay on cuBLAS fp32."""
    k = x.shape[-1]
    if x.dtype == torch.float32 and x.is_cuda and k % 8 == 0:
        w3, bias = _split_weight(module, name, weights, biases)
        n = w3.shape[1]
        if n % 4 == 0:
            if x3 is None:
                x3 = kernels.split3_fast(x)
            y = torch.empty(*x.shape[:-1], n, device=x.device, dtype=torch.float32)
            kernels.linear_split3_fast(x3, w3, bias, y)
            return y
    w = torch.cat(list(weights), 0) if len(weights) > 1 else weights[0]
    bias = None
    if biases is not None and any(b is not None for b in biases):
        bias = torch.cat([b if b is not None else w.new_zeros(p.shape[0]) for p, b in zip(weights, biases)])
    return F.linear(x, w, bias)


def _linear32_planes(module, name, x3, lead, weights, biases=None, residual=None):
    """:func:`_linear32` on an input already in split form (x3 = bf16 [3, rows, K],
    written by a fused producer); the output is fp32 [*lead, N], plus ``residual``
    (contiguous fp32 [*lead, N]) when given, added inside the kernel's epilogue."""
    w3, bias = _split_weight(module, name, weights, biases)
    n = w3.shape[1]
    if n % 4 == 0:
        y = torch.empty(*lead, n, device=x3.device, dtype=torch.float32)
        if residual is not None and (not residual.is_contiguous() or residual.dtype != torch.float32):
            residual = residual.float().contiguous()
        kernels.linear_split3_fast(x3, w3, bias, y, residual=residual)
        return y
    x = x3.float().sum(0).view(*lead, x3.shape[-1])  # exact to 2^-27 relative
    w = torch.cat(list(weights), 0) if len(weights) > 1 else weights[0]
    y = F.linear(x, w, bias)
    return y if residual is None else y + residual


def _split_input(x):
    """split3(x) when x can feed bl_linear_split3, else None."""
    return kernels.split3_fast(x) if x.dtype == torch.float32 and x.is_cuda and x.shape[-1] % 8 == 0 else None


# ---------------------------------------------------------------------------
# Triangle attention (starting / ending node)
# ---------------------------------------------------------------------------
def _attention_weights(module):
    mha = module.mha
    params = (mha.linear_q.weight, mha.linear_k.weight, mha.linear_v.weight, mha.linear_g.weight,
              mha.linear_g.bias, module.linear.weight, mha.linear_o.weight, mha.linear_o.bias)

    def build():
        w = torch.cat([mha.linear_q.weight, mha.linear_k.weight, mha.linear_v.weight, mha.linear_g.weight], 0)
        bias = torch.zeros(w.shape[0], device=w.device, dtype=torch.float32)
        bias[384:512] = mha.linear_g.bias
        return dict(w_in=w.to(_BF16).contiguous(), b_in=bias, w_heads=module.linear.weight.to(_BF16).contiguous(),
                    w_out=mha.linear_o.weight.to(_BF16).contiguous(), b_out=mha.linear_o.bias.float().contiguous())

    return _cached(module, "_bl_attention_weights", params, build)


def _attention_supported(module):
    mha = module.mha
    return (getattr(mha, "c_hidden", None) == 32 and getattr(mha, "no_heads", None) == 4
            and mha.linear_q.weight.shape == (128, 128) and mha.linear_q.bias is None)


def triangle_attention_forward(self, x, mask=None, chunk_size=None, use_kernels=False, residual=None):
    """Upstream ``TriangleAttention.forward(x, mask, chunk_size, use_kernels)``.

    Returns the bf16 update (or, with ``residual``, adds it into that fp32 z).
    Row chunking is irrelevant here: the flash kernel never materialises the scores.
    """
    _check_pair_input(x, mask)
    _check_residual(residual, x)
    if not _attention_supported(self):
        raise RuntimeError("triangle attention kernels cover c_z = 128, 4 heads x 32 only")
    starting = getattr(self, "starting", True)
    batch, n = x.shape[0], x.shape[1]
    if mask is None:
        mask = x.new_ones(x.shape[:-1], dtype=torch.float32)
    mask = mask.float().contiguous()
    w = _attention_weights(self)
    width = w["w_in"].shape[0]
    n_pad = _pad8(n)
    out = None if residual is not None else torch.empty(batch, n, n, 128, device=x.device, dtype=_BF16)
    stream = stream_of(x)
    ln = self.layer_norm
    rows = n * n
    for b in range(batch):
        xb = x[b].reshape(rows, 128).float().contiguous()
        bias = torch.empty(4, n, n_pad, device=x.device, dtype=_BF16)
        proj = torch.empty(rows, 512, device=x.device, dtype=_BF16)  # q_s | k | v | sigmoid(g)
        # LayerNorm, the q/k/v/g projection and the 128 -> 4 triangle-bias
        # projection in one pass; bias planes are [h][query][key] (transposed
        # for the ending node).
        # q leaves as bf16(q * fp32(1 / sqrt(32))) (torch's CUDA division by a
        # host scalar) and g as bf16(sigmoid(g)).
        call("bl_attention_projection", xb.data_ptr(), n, n, _f32(ln.weight).data_ptr(), _f32(ln.bias).data_ptr(),
             float(ln.eps), w["w_in"].data_ptr(), w["b_in"].data_ptr(), _Q_SCALE, w["w_heads"].data_ptr(),
             int(not starting), proj.data_ptr(), 512, bias.data_ptr(), n_pad, n * n_pad, stream)
        gated = torch.empty(rows, 128, device=x.device, dtype=_BF16)
        so, si = (n, 1) if starting else (1, n)
        ms_o, ms_k = (n, 1) if starting else (1, n)
        base = proj.data_ptr()
        args = (base, base + 128 * 2, base + 256 * 2, base + 384 * 2, width, so, si, bias.data_ptr(), n_pad,
                n * n_pad, mask[b].data_ptr(), ms_o, ms_k, float(getattr(self, "inf", 1e9)), 4, 32, n, n,
                gated.data_ptr(), 128)
        if residual is not None:
            # linear_o and the residual add run in the attention kernel's epilogue
            # when four heads share a CTA (else as one more GEMM launch, same bits).
            call("bl_triangle_attention_residual", *args, w["w_out"].data_ptr(), w["b_out"].data_ptr(),
                 residual[b].data_ptr(), 128, stream)
        else:
            call("bl_triangle_attention", *args, stream)
            _linear_out(gated, w["w_out"], rows, 128, stream, bias=w["b_out"], out=out[b].view(rows, 128))
        del proj, bias
    return residual if residual is not None else out


def triangle_attention_forward_fp32(self, x, mask=None, chunk_size=None, use_kernels=False):
    """Upstream ``TriangleAttention.forward`` in fp32 mode: fp32 input, autocast off.

    The reference's fast path accepts this case too (triangle.py:47-51: ``q_x.dtype`` fp32 and
    autocast disabled); upstream then computes every linear, the scores and the softmax in
    fp32 and returns fp32.  Here:

    1. ``bl_layernorm_split3``: LayerNorm of each pair row, written as the three bf16 split
       planes of the next linear's operand;
    2. ``bl_linear_split3``: q | k | v | g (linear_g's bias) and the 128 -> 4 triangle-bias
       projection as one fp32-accurate tensor-core GEMM, [N*N, 516];
    3. ``bl_token_attention``: fp32 flash attention per outer row, reading q / k / v / g, the
       bias planes and the mask through strides (the ending node is the same call on z
       transposed: swapped row strides, a transposed bias view and a transposed mask), with
       sigmoid(g) applied in its epilogue and its output written as split planes;
    4. ``bl_linear_split3``: linear_o with its bias.

    Returns fp32 [B, N, N, 128].  Error: within 1e-4 of upstream's fp32 eager path on O(1)
    outputs (the split linears keep every product to 2^-24 relative).
    """
    _check_pair_input(x, mask)
    if not _attention_supported(self):
        raise RuntimeError("triangle attention kernels cover c_z = 128, 4 heads x 32 only")
    if x.dtype != torch.float32:
        raise RuntimeError("fp32-mode triangle attention takes fp32 input")
    starting = getattr(self, "starting", True)
    batch, n = x.shape[0], x.shape[1]
    if mask is None:
        mask = x.new_ones(x.shape[:-1], dtype=torch.float32)
    mask = mask.float()
    mha, ln = self.mha, self.layer_norm
    out = torch.empty(batch, n, n, 128, device=x.device, dtype=torch.float32)
    if n == 0 or batch == 0:
        return out
    stream = stream_of(x)
    width = 516  # q | k | v | g | 4 bias heads
    with torch.autocast("cuda", enabled=False):
        for b in range(batch):
            x3 = kernels.layer_norm_split3(x[b].reshape(n * n, 128), ln.weight, ln.bias, ln.eps)
            proj = _linear32_planes(self, "_bl_w3_tri_fp32", x3, (n, n),
                                    [mha.linear_q.weight, mha.linear_k.weight, mha.linear_v.weight,
                                     mha.linear_g.weight, self.linear.weight],
                                    [None, None, None, mha.linear_g.bias, None])
            heads = proj[..., 512:516]  # [i, j, h]
            if starting:  # outer row i, inner j: element (a, b) at a*N*W + b*W
                strides = (n * width, width, 32)
                bias = heads.permute(2, 0, 1).unsqueeze(0)  # bias[h][q][k] = lin(LN(z))[q, k, h]
                mask_rows = mask[b].contiguous()
            else:  # z transposed: outer row a = column of z, inner b = row of z
                strides = (width, n * width, 32)
                bias = heads.permute(2, 1, 0).unsqueeze(0)  # lin(LN(z^T))[q, k, h] = lin(LN(z))[k, q, h]
                mask_rows = mask[b].t().contiguous()
            out3 = torch.empty(3, n * n, 128, device=x.device, dtype=torch.bfloat16)
            base = proj.data_ptr()
            kernels.launch_token_attention(base, base + 128 * 4, base + 256 * 4, base + 384 * 4, strides, bias,
                                           mask_rows, float(getattr(self, "inf", 1e9)), n, 4, n, 32, None, stream,
                                           out3=out3)
            del proj
            y = _linear32_planes(self, "_bl_w3_tri_fp32_o", out3, (n, n), [mha.linear_o.weight],
                                 [mha.linear_o.bias])
            out[b].copy_(y if starting else y.transpose(0, 1))
    return out


# ---------------------------------------------------------------------------
# Triangle multiplication (outgoing / incoming)
# ---------------------------------------------------------------------------
def _multiplication_weights(module):
    params = (module.p_in.weight, module.g_in.weight, module.p_out.weight, module.g_out.weight)

    def build():
        w_in = torch.cat([module.p_in.weight, module.g_in.weight], 0)
        # Block-diagonal [p_out 0; 0 g_out] over the K-concatenation [LN_out(o) | LN_in(x)].
        w_out = torch.zeros(256, 256, device=w_in.device, dtype=torch.float32)
        w_out[:128, :128] = module.p_out.weight
        w_out[128:, 128:] = module.g_out.weight
        w_pg = torch.cat([module.p_out.weight, module.g_out.weight], 0)  # [256][128]
        return dict(w_in=w_in.to(_BF16).contiguous(), w_out=w_out.to(_BF16).contiguous(),
                    w_pg=w_pg.to(_BF16).contiguous())

    return _cached(module, "_bl_multiplication_weights", params, build)


def _is_outgoing(module):
    if hasattr(module, "outgoing"):
        return bool(module.outgoing)
    return type(module).__name__ == "TriangleMultiplicationOutgoing"


def triangle_multiplication_forward(self, x, mask, use_kernels=False, residual=None):
    """Upstream ``TriangleMultiplication{Outgoing,Incoming}.forward(x, mask, use_kernels)``
    (the reference's ``normalized_forward``, multiplication.py:48-137).  Returns bf16
    (or, with ``residual``, adds into that fp32 z)."""
    _check_pair_input(x, mask)
    _check_residual(residual, x)
    if self.p_in.weight.shape != (256, 128) or self.p_in.bias is not None:
        raise RuntimeError("triangle multiplication kernels cover dim = 128 without projection biases")
    outgoing = _is_outgoing(self)
    batch, n = x.shape[0], x.shape[1]
    mask = mask.float().contiguous()
    w = _multiplication_weights(self)
    n_pad = _pad8(n)
    rows = n * n
    out = None if residual is not None else torch.empty(batch, n, n, 128, device=x.device, dtype=_BF16)
    stream = stream_of(x)
    for b in range(batch):
        xb = x[b].reshape(rows, 128).float().contiguous()
        xn = torch.empty(rows, 128, device=x.device, dtype=_BF16)
        planes = torch.empty(256, n, n_pad, device=x.device, dtype=_BF16)
        # LayerNorm, p_in | g_in, the sigmoid gate and the mask in one pass,
        # written as channel planes a = planes[:128], b = planes[128:].
        call("bl_trimul_projection", xb.data_ptr(), n, n, _f32(self.norm_in.weight).data_ptr(),
             _f32(self.norm_in.bias).data_ptr(), float(self.norm_in.eps), w["w_in"].data_ptr(), mask[b].data_ptr(),
             planes.data_ptr(), n_pad, xn.data_ptr(), stream)
        a, bp = planes[:128], planes[128:]
        prod = torch.empty_like(a)
        plane = n * n_pad
        # outgoing: O_c = A_c B_c^T over planes [i][k] (K-major);
        # incoming: O_c = A_c^T B_c over planes [k][i] (MN-major).
        mn = int(not outgoing)
        call("bl_batched_gemm", a.data_ptr(), mn, n_pad, plane, bp.data_ptr(), mn, n_pad, plane, prod.data_ptr(),
             n_pad, plane, 128, n, n, n, None, stream)
        del a, bp, planes
        # LayerNorm over the product's channel planes, p_out, g_out(x_hat), the
        # gate and the residual add in one kernel.
        norm = self.norm_out
        args = (prod.data_ptr(), n, n, n_pad, _f32(norm.weight).data_ptr(), _f32(norm.bias).data_ptr(),
                float(norm.eps), xn.data_ptr(), w["w_pg"].data_ptr())
        if residual is not None:
            call("bl_trimul_output", *args, residual[b].data_ptr(), None, stream)
        else:
            call("bl_trimul_output", *args, None, out[b].data_ptr(), stream)
        del prod
    return residual if residual is not None else out


# ---------------------------------------------------------------------------
# Pair transition
# ---------------------------------------------------------------------------
def _transition_weights(module):
    params = (module.fc1.weight, module.fc2.weight, module.fc3.weight)

    def build():
        return dict(w12=torch.cat([module.fc1.weight, module.fc2.weight], 0).to(_BF16).contiguous(),
                    w3=module.fc3.weight.to(_BF16).contiguous())

    return _cached(module, "_bl_transition_weights", params, build)


def transition_forward(self, x, chunk_size=None, residual=None):
    """Upstream ``Transition.forward(x, chunk_size)`` under bf16 autocast
    (the reference's pair_transition.py:8-28).  Returns bf16 (or adds into ``residual``)."""
    if not x.is_cuda:
        raise RuntimeError("transition kernels need CUDA tensors")
    _check_residual(residual, x)
    dim, hidden = x.shape[-1], self.fc1.weight.shape[0]
    out_dim = self.fc3.weight.shape[0]
    if dim % 8 or hidden % 64 or any(f.bias is not None for f in (self.fc1, self.fc2, self.fc3)):
        raise RuntimeError("transition kernels need bias-free layers, dim % 8 == 0 and hidden % 64 == 0")
    w = _transition_weights(self)
    rows = x.numel() // dim
    stream = stream_of(x)
    if dim == 128 and hidden == 512 and out_dim == 128:
        # One fused kernel: LN, fc1|fc2, SwiGLU and fc3 with the hidden
        # activations on chip; the residual lands as a reduce-add into z.
        xf = x.reshape(rows, dim).float().contiguous()
        norm = self.norm
        args = (xf.data_ptr(), rows, _f32(norm.weight).data_ptr(), _f32(norm.bias).data_ptr(), float(norm.eps),
                w["w12"].data_ptr(), w["w3"].data_ptr())
        if residual is not None:
            call("bl_pair_transition", *args, residual.data_ptr(), None, stream)
            return residual
        out = torch.empty(rows, out_dim, device=x.device, dtype=_BF16)
        call("bl_pair_transition", *args, None, out.data_ptr(), stream)
        return out.view(*x.shape[:-1], out_dim)
    xn = _layer_norm_bf16(x.reshape(rows, dim).contiguous(), self.norm)
    h12 = _linear_bf16(xn, w["w12"])
    del xn
    h = torch.empty(rows, hidden, device=x.device, dtype=_BF16)
    call("bl_swiglu_rows", h12.data_ptr(), 2 * hidden, rows, hidden, h.data_ptr(), hidden, stream)
    del h12
    if out_dim == 128:
        if residual is not None:
            _linear_out(h, w["w3"], rows, hidden, stream, residual=residual.view(rows, out_dim))
            return residual
        out = torch.empty(rows, out_dim, device=x.device, dtype=_BF16)
        _linear_out(h, w["w3"], rows, hidden, stream, out=out)
        return out.view(*x.shape[:-1], out_dim)
    y = _linear_bf16(h, w["w3"]).view(*x.shape[:-1], out_dim)
    if residual is not None:
        return residual.add_(y)
    return y


# ---------------------------------------------------------------------------
# Diffusion AdaLN / ConditionedTransitionBlock (fp32, no autocast)
# ---------------------------------------------------------------------------
def adaln_forward(self, a, s):
    """Upstream ``AdaLN.forward(a, s)`` (the reference's diffusion.py:52-57), fp32."""
    if a.dtype != torch.float32 or s.dtype != torch.float32:
        raise RuntimeError("AdaLN kernels are fp32")

    with torch.autocast("cuda", enabled=False):
        scale, shift = _adaln_conditioning(self, s)
        return kernels.adaln_modulate(a, scale, shift, self.a_norm.eps)


def _adaln_conditioning(self, s):
    """AdaLN's (s_scale(s_norm(s)), s_bias(s_norm(s))); depends on s only, so
    reused across steps inside atom_conditioning_cache."""

    def conditioning():
        cols = s.shape[-1]
        if cols % 128 == 0 and cols <= 1024:
            # LayerNorm straight into the linears' split operand form.
            sn3 = kernels.layer_norm_split3(s, self.s_norm.weight, getattr(self.s_norm, "bias", None),
                                            self.s_norm.eps)
            lead = s.shape[:-1]
            return (_linear32_planes(self, "_bl_w3_scale", sn3, lead, [self.s_scale.weight], [self.s_scale.bias]),
                    _linear32_planes(self, "_bl_w3_shift", sn3, lead, [self.s_bias.weight], [self.s_bias.bias]))
        sn = kernels.layer_norm(s, self.s_norm.weight, getattr(self.s_norm, "bias", None), self.s_norm.eps,
                                out_dtype=torch.float32)
        sn3 = _split_input(sn)
        return (_linear32(self, "_bl_w3_scale", sn, [self.s_scale.weight], [self.s_scale.bias], x3=sn3),
                _linear32(self, "_bl_w3_shift", sn, [self.s_bias.weight], [self.s_bias.bias], x3=sn3))

    return atom_conditioning.lookup(self, "adaln", s, conditioning)


def conditioned_transition_forward(self, a, s):
    """Upstream ``ConditionedTransitionBlock.forward(a, s)`` (diffusion.py:60-68), fp32."""
    with torch.autocast("cuda", enabled=False):
        dim, lead = a.shape[-1], a.shape[:-1]
        inner = self.a_to_b.weight.shape[0]
        op = self.output_projection[0]
        gate = atom_conditioning.lookup(self, "gate", s, lambda: _linear32(self, "_bl_w3_gate", s, [op.weight], [op.bias]))
        if dim % 8 == 0 and dim <= 2048 and inner % 8 == 0 and a.dtype == torch.float32:
            # a' = AdaLN(a, s) and b = SwiGLU(...) leave their kernels as the
            # split operands of the linears that consume them.
            scale, shift = _adaln_conditioning(self.adaln, s)
            a3 = kernels.adaln_modulate_split3(a, scale, shift, self.adaln.a_norm.eps)
            projected = _linear32_planes(self, "_bl_w3_swish", a3, lead, [self.swish_gate[0].weight],
                                         [self.swish_gate[0].bias])
            third = _linear32_planes(self, "_bl_w3_atob", a3, lead, [self.a_to_b.weight], [self.a_to_b.bias])
            b3 = kernels.epilogue_split3(projected, third, None, kernels.GATED_SWIGLU)
            out = _linear32_planes(self, "_bl_w3_btoa", b3, lead, [self.b_to_a.weight], [self.b_to_a.bias])
        else:
            a = adaln_forward(self.adaln, a, s)
            a3 = _split_input(a)
            projected = _linear32(self, "_bl_w3_swish", a, [self.swish_gate[0].weight], [self.swish_gate[0].bias],
                                  x3=a3)
            third = _linear32(self, "_bl_w3_atob", a, [self.a_to_b.weight], [self.a_to_b.bias], x3=a3)
            b = kernels.epilogue(projected.contiguous(), third.contiguous(), None, kernels.GATED_SWIGLU)
            out = _linear32(self, "_bl_w3_btoa", b, [self.b_to_a.weight], [self.b_to_a.bias])
        return kernels.epilogue(gate.contiguous(), out.contiguous(), None, kernels.GATE)


# ---------------------------------------------------------------------------
# AttentionPairBias with a given (prepared) bias: diffusion token transformer
# ---------------------------------------------------------------------------
_TOKEN_HEAD_DIMS = (24, 32, 48, 64)


def prepare_token_bias(value):
    """The diffusion token bias [B, N, N, L*H] with dense head-major storage.

    Same logical shape and values (fp32); only the memory order changes to
    [B, L*H, N, N], so each layer's [B, H, N, N] slice is read row by row by
    the attention kernel (the reference's prepare_token_bias, pair_bias.py:6-12).
    """
    return value.permute(0, 3, 1, 2).contiguous().float().permute(0, 2, 3, 1)


def token_attention_supported(module, s, k_in, bias, mask=None):
    """Shapes and dtypes the fused fp32 token attention covers."""
    heads, d = module.num_heads, module.head_dim
    return (d in _TOKEN_HEAD_DIMS and heads * d == module.c_s and s.dim() == 3 and s.dtype == torch.float32
            and s.is_cuda and k_in.dtype == torch.float32 and k_in.shape == s.shape and s.shape[-1] == module.c_s
            and bias.dim() == 4 and tuple(bias.shape[1:]) == (heads, s.shape[1], s.shape[1])
            and bias.shape[0] >= 1 and s.shape[0] % bias.shape[0] == 0 and bias.device == s.device
            and (mask is None or tuple(mask.shape) == tuple(s.shape[:2]))
            and all(p.bias is None for p in (module.proj_k, module.proj_v, module.proj_g)))


def attend_with_bias(self, s, bias, mask, k_in, s3=None, residual=None):
    """Upstream attentionv2 ``AttentionPairBias`` after ``proj_z``: projections,
    fused fp32 attention with bias, key mask and sigmoid gate, then ``proj_o``.

    ``bias`` is fp32 [B', H, N, N] (any strides, B' dividing the batch: sample
    ``b`` reads bias ``b // (B / B')``).  When ``k_in is s`` the four input
    projections run as one GEMM over stacked weights; ``s3`` may pass s
    already in split form (a fused producer wrote it), with ``s`` then only
    giving the shape.  With ``residual`` the result is ``residual + attention``
    (the add runs in proj_o's epilogue).
    """
    if not token_attention_supported(self, s, k_in, bias, mask):
        raise RuntimeError(f"token attention covers fp32 CUDA s [B, N, H*d] with d in {_TOKEN_HEAD_DIMS}, "
                           f"bias [B', H, N, N] and mask [B, N]; got s {tuple(s.shape)}, bias {tuple(bias.shape)}")
    b, n = s.shape[0], s.shape[1]
    heads, d, c = self.num_heads, self.head_dim, self.c_s
    if torch.is_autocast_enabled("cuda"):  # the reference's math is fp32 throughout
        with torch.autocast("cuda", enabled=False):
            return attend_with_bias(self, s, bias, mask, k_in, s3=s3, residual=residual)
    if bias.dtype != torch.float32:
        bias = bias.float()
    if mask is not None and (mask.dtype != torch.float32 or mask.stride(-1) != 1):
        mask = mask.float().contiguous()
    if b == 0 or n == 0:
        out = self.proj_o(s.new_zeros(b, n, c))
        return out if residual is None else out + residual
    out3 = torch.empty(3, b * n, c, device=s.device, dtype=torch.bfloat16)  # the output, as proj_o's operand
    stream = stream_of(s)
    if k_in is s:
        # One GEMM for q | k | v | g; the kernel reads the four column blocks in place.
        weights = [self.proj_q.weight, self.proj_k.weight, self.proj_v.weight, self.proj_g.weight]
        biases = [self.proj_q.bias, None, None, None]
        if s3 is not None:
            proj = _linear32_planes(self, "_bl_w3_qkvg", s3, (b, n), weights, biases)
        else:
            proj = _linear32(self, "_bl_w3_qkvg", s, weights, biases)
        base = proj.data_ptr()
        kernels.launch_token_attention(base, base + 4 * c, base + 8 * c, base + 12 * c, (n * 4 * c, 4 * c, d), bias,
                                       mask, self.inf, b, heads, n, d, None, stream, out3=out3)
    else:  # four contiguous [B, N, c_s] projections share one stride layout
        s3, k3 = _split_input(s), _split_input(k_in)
        q = _linear32(self, "_bl_w3_q", s, [self.proj_q.weight], [self.proj_q.bias], x3=s3)
        k = _linear32(self, "_bl_w3_k", k_in, [self.proj_k.weight], x3=k3)
        v = _linear32(self, "_bl_w3_v", k_in, [self.proj_v.weight], x3=k3)
        g = _linear32(self, "_bl_w3_g", s, [self.proj_g.weight], x3=s3)
        kernels.launch_token_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), (n * c, c, d), bias,
                                       mask, self.inf, b, heads, n, d, None, stream, out3=out3)
    return _linear32_planes(self, "_bl_w3_o", out3, (b, n), [self.proj_o.weight], [self.proj_o.bias],
                            residual=residual)


def token_attention_forward(self, s, z, mask, k_in, multiplicity=1):
    """Upstream ``AttentionPairBias.forward(s, z, mask, k_in, multiplicity)``
    with a prepared bias (the reference's prepared_forward, pair_bias.py:15-36).

    ``z`` is the layer's slice of the dense token bias, [B, N, N, H]; upstream's
    ``proj_z`` (a heads-first rearrange when ``compute_pair_bias`` is off)
    turns it into the [B, H, N, N] view the kernel reads in place, and the
    ``multiplicity`` diffusion samples of one input share one bias row
    without the reference's ``repeat_interleave`` copy.
    """
    bias = self.proj_z(z)
    if bias.shape[0] * multiplicity not in (s.shape[0], 1):
        raise RuntimeError(f"bias batch {bias.shape[0]} x multiplicity {multiplicity} != batch {s.shape[0]}")
    return attend_with_bias(self, s, bias, mask, k_in)


# ---------------------------------------------------------------------------
# Reference-compatible entry points (the reference rebinds pieces of modules)
# ---------------------------------------------------------------------------
def normalization_forward(self, x):
    """Upstream triangle ``LayerNorm.forward(x)`` (triangle.py:107-146): fp32
    statistics, bf16 output for the autocast linears that consume it."""
    c = x.shape[-1]
    return kernels.layer_norm(x.reshape(-1, c), _f32(self.weight), _f32(self.bias), self.eps,
                              out_dtype=_BF16).view(x.shape)


__all__ = [
    "adaln_forward",
    "attend_with_bias",
    "prepare_token_bias",
    "token_attention_forward",
    "conditioned_transition_forward",
    "normalization_forward",
    "transition_forward",
    "triangle_attention_forward",
    "triangle_attention_forward_fp32",
    "triangle_multiplication_forward",
]
