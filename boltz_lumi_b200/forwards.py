"""Replacement forwards of the upstream Boltz-2 modules on the pair hot path.

Each function takes the module as ``self`` (it is bound with
``types.MethodType`` exactly like the reference's adapter, adapters.py:24-47)
and reads only upstream attribute names, so it works both on upstream Boltz
2.2.1 modules and on the standalone classes of :mod:`boltz_lumi_b200.layers`.

Numerics follow upstream's eager path under bf16 autocast for the trunk
(TriangleAttention, TriangleMultiplication, Transition) and plain fp32 for the
diffusion AdaLN / ConditionedTransitionBlock.  All compute runs in the sm_100a
kernels of ``libboltz_b200.so``; there is no CPU path.
"""

import torch
import torch.nn.functional as F

from . import _lib, kernels
from ._lib import call, stream_of

_BF16 = torch.bfloat16


def _pad8(n):
    return (n + 7) // 8 * 8


def _cached(module, name, params, build):
    """Derived weights, rebuilt when any source parameter changes identity,
    version, device or dtype (the reference's cache key, multiplication.py:29-40)."""
    key = tuple((id(p), p._version, p.device, p.dtype) for p in params if p is not None)
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


def _layer_norm_bf16(x2d, norm):
    return kernels.layer_norm(x2d, norm.weight.float().contiguous() if norm.weight is not None else None,
                              norm.bias.float().contiguous() if getattr(norm, "bias", None) is not None else None,
                              norm.eps, out_dtype=_BF16)


def _linear_bf16(x2d, weight_bf16, bias=None):
    """Autocast linear on tcgen05: bf16 operands, fp32 accumulation, bf16 result."""
    return kernels.bmm(x2d.unsqueeze(0), weight_bf16.unsqueeze(0), bias=bias).squeeze(0)


# ---------------------------------------------------------------------------
# Triangle attention (starting / ending node)
# ---------------------------------------------------------------------------
def _attention_weights(module):
    mha = module.mha
    params = (mha.linear_q.weight, mha.linear_k.weight, mha.linear_v.weight, mha.linear_g.weight,
              mha.linear_g.bias, module.linear.weight, mha.linear_o.weight, mha.linear_o.bias)

    def build():
        h = module.linear.weight.shape[0]
        w = torch.zeros(512 + _pad8(h), mha.linear_q.weight.shape[1], device=mha.linear_q.weight.device,
                        dtype=torch.float32)
        w[0:128] = mha.linear_q.weight
        w[128:256] = mha.linear_k.weight
        w[256:384] = mha.linear_v.weight
        w[384:512] = mha.linear_g.weight
        w[512:512 + h] = module.linear.weight
        bias = torch.zeros(w.shape[0], device=w.device, dtype=torch.float32)
        bias[384:512] = mha.linear_g.bias
        return dict(w_in=w.to(_BF16).contiguous(), b_in=bias, w_out=mha.linear_o.weight.to(_BF16).contiguous(),
                    b_out=mha.linear_o.bias.float().contiguous())

    return _cached(module, "_bl_attention_weights", params, build)


def _attention_supported(module):
    mha = module.mha
    return (getattr(mha, "c_hidden", None) == 32 and getattr(mha, "no_heads", None) == 4
            and mha.linear_q.weight.shape == (128, 128) and mha.linear_q.bias is None)


def triangle_attention_forward(self, x, mask=None, chunk_size=None, use_kernels=False):
    """Upstream ``TriangleAttention.forward(x, mask, chunk_size, use_kernels)``.

    Returns the bf16 update (the caller adds it to z).  Row chunking is
    irrelevant here: the flash kernel never materialises the scores.
    """
    _check_pair_input(x, mask)
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
    out = torch.empty(batch, n, n, 128, device=x.device, dtype=_BF16)
    stream = stream_of(x)
    for b in range(batch):
        xn = _layer_norm_bf16(x[b].reshape(n * n, 128), self.layer_norm)
        proj = _linear_bf16(xn, w["w_in"], w["b_in"])  # [n*n, 520]: q | k | v | g | tri-bias
        bias = torch.empty(4, n, n_pad, device=x.device, dtype=_BF16)
        call("bl_triangle_bias_planes", proj.data_ptr() + 512 * 2, width, 4, n, int(not starting),
             bias.data_ptr(), n_pad, stream)
        gated = torch.empty(n * n, 128, device=x.device, dtype=_BF16)
        so, si = (n, 1) if starting else (1, n)
        ms_o, ms_k = (n, 1) if starting else (1, n)
        base = proj.data_ptr()
        call("bl_triangle_attention", base, base + 128 * 2, base + 256 * 2, base + 384 * 2, width, so, si,
             bias.data_ptr(), n_pad, n * n_pad, mask[b].data_ptr(), ms_o, ms_k, float(getattr(self, "inf", 1e9)),
             4, 32, n, gated.data_ptr(), 128, stream)
        out[b] = _linear_bf16(gated, w["w_out"], w["b_out"]).view(n, n, 128)
    return out


# ---------------------------------------------------------------------------
# Triangle multiplication (outgoing / incoming)
# ---------------------------------------------------------------------------
def _multiplication_weights(module):
    params = (module.p_in.weight, module.g_in.weight, module.p_out.weight, module.g_out.weight)

    def build():
        return dict(w_in=torch.cat([module.p_in.weight, module.g_in.weight], 0).to(_BF16).contiguous(),
                    w_pout=module.p_out.weight.to(_BF16).contiguous(),
                    w_gout=module.g_out.weight.to(_BF16).contiguous())

    return _cached(module, "_bl_multiplication_weights", params, build)


def _is_outgoing(module):
    if hasattr(module, "outgoing"):
        return bool(module.outgoing)
    return type(module).__name__ == "TriangleMultiplicationOutgoing"


def triangle_multiplication_forward(self, x, mask, use_kernels=False):
    """Upstream ``TriangleMultiplication{Outgoing,Incoming}.forward(x, mask, use_kernels)``
    (the reference's ``normalized_forward``, multiplication.py:48-137).  Returns bf16."""
    _check_pair_input(x, mask)
    if self.p_in.weight.shape != (256, 128) or self.p_in.bias is not None:
        raise RuntimeError("triangle multiplication kernels cover dim = 128 without projection biases")
    outgoing = _is_outgoing(self)
    batch, n = x.shape[0], x.shape[1]
    mask = mask.float().contiguous()
    w = _multiplication_weights(self)
    n_pad = _pad8(n)
    out = torch.empty(batch, n, n, 128, device=x.device, dtype=_BF16)
    stream = stream_of(x)
    for b in range(batch):
        xn = _layer_norm_bf16(x[b].reshape(n * n, 128), self.norm_in)
        pg = _linear_bf16(xn, w["w_in"])  # [n*n, 512]: p | g
        a = torch.empty(128, n, n_pad, device=x.device, dtype=_BF16)
        bp = torch.empty_like(a)
        call("bl_trimul_pack_planes", pg.data_ptr(), 512, mask[b].data_ptr(), n, n_pad, a.data_ptr(), bp.data_ptr(),
             stream)
        del pg
        prod = torch.empty_like(a)
        plane = n * n_pad
        # outgoing: O_c = A_c B_c^T over planes [i][k] (K-major);
        # incoming: O_c = A_c^T B_c over planes [k][i] (MN-major).
        mn = int(not outgoing)
        call("bl_batched_gemm", a.data_ptr(), mn, n_pad, plane, bp.data_ptr(), mn, n_pad, plane, prod.data_ptr(),
             n_pad, plane, 128, n, n, n, None, stream)
        del a, bp
        normed = torch.empty(n * n, 128, device=x.device, dtype=_BF16)
        call("bl_layernorm_planes", prod.data_ptr(), n, n_pad, self.norm_out.weight.float().contiguous().data_ptr(),
             self.norm_out.bias.float().contiguous().data_ptr(), float(self.norm_out.eps), normed.data_ptr(),
             _lib.BL_BF16, stream)
        del prod
        p = _linear_bf16(normed, w["w_pout"])
        g = _linear_bf16(xn, w["w_gout"])
        out[b] = kernels.gate(p, g).view(n, n, 128)
    return out


# ---------------------------------------------------------------------------
# Pair transition
# ---------------------------------------------------------------------------
def _transition_weights(module):
    params = (module.fc1.weight, module.fc2.weight, module.fc3.weight)

    def build():
        return dict(w12=torch.cat([module.fc1.weight, module.fc2.weight], 0).to(_BF16).contiguous(),
                    w3=module.fc3.weight.to(_BF16).contiguous())

    return _cached(module, "_bl_transition_weights", params, build)


def transition_forward(self, x, chunk_size=None):
    """Upstream ``Transition.forward(x, chunk_size)`` under bf16 autocast
    (the reference's pair_transition.py:8-28).  Returns bf16."""
    if not x.is_cuda:
        raise RuntimeError("transition kernels need CUDA tensors")
    dim, hidden = x.shape[-1], self.fc1.weight.shape[0]
    if dim % 8 or hidden % 8 or any(f.bias is not None for f in (self.fc1, self.fc2, self.fc3)):
        raise RuntimeError("transition kernels need bias-free layers with widths that are multiples of 8")
    w = _transition_weights(self)
    rows = x.numel() // dim
    xn = _layer_norm_bf16(x.reshape(rows, dim).contiguous(), self.norm)
    h12 = _linear_bf16(xn, w["w12"])
    h = torch.empty(rows, hidden, device=x.device, dtype=_BF16)
    call("bl_swiglu_rows", h12.data_ptr(), 2 * hidden, rows, hidden, h.data_ptr(), hidden, stream_of(x))
    del h12
    return _linear_bf16(h, w["w3"]).view(*x.shape[:-1], w["w3"].shape[0])


# ---------------------------------------------------------------------------
# Diffusion AdaLN / ConditionedTransitionBlock (fp32, no autocast)
# ---------------------------------------------------------------------------
def adaln_forward(self, a, s):
    """Upstream ``AdaLN.forward(a, s)`` (the reference's diffusion.py:52-57), fp32."""
    if a.dtype != torch.float32 or s.dtype != torch.float32:
        raise RuntimeError("AdaLN kernels are fp32")
    with torch.autocast("cuda", enabled=False):
        sn = kernels.layer_norm(s, self.s_norm.weight, getattr(self.s_norm, "bias", None), self.s_norm.eps,
                                out_dtype=torch.float32)
        scale = F.linear(sn, self.s_scale.weight, self.s_scale.bias)
        shift = F.linear(sn, self.s_bias.weight, self.s_bias.bias)
        return kernels.adaln_modulate(a, scale, shift, self.a_norm.eps)


def conditioned_transition_forward(self, a, s):
    """Upstream ``ConditionedTransitionBlock.forward(a, s)`` (diffusion.py:60-68), fp32."""
    with torch.autocast("cuda", enabled=False):
        a = adaln_forward(self.adaln, a, s)
        projected = F.linear(a, self.swish_gate[0].weight, self.swish_gate[0].bias)
        third = F.linear(a, self.a_to_b.weight, self.a_to_b.bias)
        b = kernels.epilogue(projected.contiguous(), third.contiguous(), None, kernels.GATED_SWIGLU)
        gate = F.linear(s, self.output_projection[0].weight, self.output_projection[0].bias)
        return kernels.epilogue(gate.contiguous(), F.linear(b, self.b_to_a.weight, self.b_to_a.bias).contiguous(),
                                None, kernels.GATE)


# ---------------------------------------------------------------------------
# Reference-compatible entry points (the reference rebinds pieces of modules)
# ---------------------------------------------------------------------------
def normalization_forward(self, x):
    """Upstream triangle ``LayerNorm.forward(x)`` (triangle.py:107-146): fp32
    statistics, bf16 output for the autocast linears that consume it."""
    c = x.shape[-1]
    return kernels.layer_norm(x.reshape(-1, c), self.weight.float().contiguous(), self.bias.float().contiguous(),
                              self.eps, out_dtype=_BF16).view(x.shape)


__all__ = [
    "adaln_forward",
    "conditioned_transition_forward",
    "normalization_forward",
    "transition_forward",
    "triangle_attention_forward",
    "triangle_multiplication_forward",
]
