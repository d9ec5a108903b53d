"""CPU restatement of the upstream Boltz 2.2.1 modules on the hot path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Parameter names and
constructor signatures follow the upstream modules the reference rebinds, so a
``state_dict`` moves between the product layers and these classes unchanged.

Each forward takes ``bf16=True`` to emulate upstream under bf16 autocast (the
trunk contract) or ``bf16=False`` for plain fp32 eager semantics (the
diffusion contract, and the fp32 mode of the trunk).

Assumptions that the reference does not pin and upstream cannot confirm here
(they follow the public OpenFold/AF3/Boltz-2 definitions):

* ``Attention``: ``linear_q/k/v`` have no bias, ``linear_g`` and ``linear_o``
  have biases; the triangle-bias ``linear`` has no bias; ``inf = 1e9``.
* every ``Linear`` of TriangleMultiplication and Transition is bias-free;
* LayerNorm eps is 1e-5 everywhere;
* AdaLN: ``a_norm`` has no affine, ``s_norm`` has a weight and no bias,
  ``s_scale`` has a bias, ``s_bias`` has none;
* ConditionedTransitionBlock: ``swish_gate[0]``, ``a_to_b``, ``b_to_a`` are
  bias-free, ``output_projection[0]`` has a bias; SwiGLU is
  ``silu(x[..., h:]) * x[..., :h]``;
* the Pairformer block order is TriMulOut, TriMulIn, TriAttStart, TriAttEnd,
  Transition(z), then the fp32 single track AttentionPairBias + Transition(s)
  (AF3 supplementary Algorithm 17).
"""

import math

import torch
from torch import nn

from .numerics import GATE, GATED_SWIGLU, MODULATION, bf16_round, diffusion_epilogue, linear_bf16, sigmoid_bf16, silu_bf16


def _linear(x, layer, bf16):
    if bf16:
        return linear_bf16(x, layer.weight, layer.bias)
    return nn.functional.linear(x, layer.weight, layer.bias)


def _layer_norm(x, norm):
    """fp32 LayerNorm (autocast runs layer_norm in fp32 on an fp32 input)."""
    return nn.functional.layer_norm(
        x.float(), norm.normalized_shape, norm.weight, norm.bias, norm.eps
    )


class LayerNorm(nn.LayerNorm):
    """LayerNorm exposing ``c_in`` as the OpenFold variant does (``triangle.py:226``)."""

    def __init__(self, c_in, eps=1e-5, elementwise_affine=True, bias=True):
        super().__init__(c_in, eps=eps, elementwise_affine=elementwise_affine, bias=bias)
        self.c_in = (c_in,)


def ordered_bias_softmax(scores, mask_bias, tri_bias, bf16=True):
    """``(s + mask) -> round -> (+ bias) -> round -> softmax -> round``.

    Follows the reference's ordered softmax (``kernels/triangle_softmax.py:90-113``)
    and the reference test's own expression (``tests/test_triangle_softmax.py:44-47``):
    in-place adds on the score tensor round to the score dtype after each add.
    """
    s = scores.float()
    if bf16:
        s = bf16_round(s + mask_bias.float())
        s = bf16_round(s + tri_bias.float())
        return bf16_round(torch.softmax(s, dim=-1))
    return torch.softmax(s + mask_bias.float() + tri_bias.float(), dim=-1)


class Attention(nn.Module):
    """Gated multi-head attention of the triangle layers (``triangle.py:32-104``)."""

    def __init__(self, c_q, c_k, c_v, c_hidden, no_heads, gating=True):
        super().__init__()
        self.c_q, self.c_hidden, self.no_heads = c_q, c_hidden, no_heads
        self.linear_q = nn.Linear(c_q, c_hidden * no_heads, bias=False)
        self.linear_k = nn.Linear(c_k, c_hidden * no_heads, bias=False)
        self.linear_v = nn.Linear(c_v, c_hidden * no_heads, bias=False)
        self.linear_o = nn.Linear(c_hidden * no_heads, c_q)
        self.linear_g = nn.Linear(c_q, c_hidden * no_heads)

    def forward(self, q_x, kv_x, tri_bias, mask_bias, bf16=True):
        """q_x, kv_x: [*, I, J, C]; tri_bias: [*, 1, H, J, J]; mask_bias: [*, I, 1, 1, J]."""
        h, d = self.no_heads, self.c_hidden
        q = _linear(q_x, self.linear_q, bf16)
        k = _linear(kv_x, self.linear_k, bf16)
        v = _linear(kv_x, self.linear_v, bf16)
        q = q.view(q.shape[:-1] + (h, d)).transpose(-2, -3)
        k = k.view(k.shape[:-1] + (h, d)).transpose(-2, -3)
        v = v.view(v.shape[:-1] + (h, d)).transpose(-2, -3)
        # _prep_qkv(apply_scale=True) divides q after the projection (triangle.py:80).
        q = q / math.sqrt(d)
        if bf16:
            q = bf16_round(q)
        s = q @ k.transpose(-1, -2)
        if bf16:
            s = bf16_round(s)
        p = ordered_bias_softmax(s, mask_bias, tri_bias, bf16)
        o = p @ v
        if bf16:
            o = bf16_round(o)
        o = o.transpose(-2, -3)  # [*, I, J, H, d]
        g = _linear(q_x, self.linear_g, bf16)
        g = sigmoid_bf16(g) if bf16 else torch.sigmoid(g)
        o = o * g.view(g.shape[:-1] + (h, d))
        if bf16:
            o = bf16_round(o)
        o = o.reshape(o.shape[:-2] + (h * d,))
        return _linear(o, self.linear_o, bf16)


class TriangleAttention(nn.Module):
    """Triangle self-attention around the starting node (upstream TriangleAttention)."""

    starting = True

    def __init__(self, c_in, c_hidden, no_heads, starting=None, inf=1e9):
        super().__init__()
        if starting is not None:
            self.starting = starting
        self.c_in, self.c_hidden, self.no_heads, self.inf = c_in, c_hidden, no_heads, inf
        self.layer_norm = LayerNorm(c_in)
        self.linear = nn.Linear(c_in, no_heads, bias=False)
        self.mha = Attention(c_in, c_in, c_in, c_hidden, no_heads)

    def forward(self, x, mask=None, chunk_size=None, bf16=True, row_chunk=64, rows=None):
        """x: [B, N, N, C] fp32; mask: [B, N, N].  Returns the bf16-valued update.

        ``rows`` limits the computation to the first outer rows (of z, or of z
        transposed for the ending node); the largest parity case (N = 2511)
        checks that many rows only.
        """
        if mask is None:
            mask = x.new_ones(x.shape[:-1])
        if not self.starting:
            x = x.transpose(-2, -3)
            mask = mask.transpose(-1, -2)
        x = _layer_norm(x, self.layer_norm)
        mask_bias = (self.inf * (mask.float() - 1))[..., :, None, None, :]
        tri_bias = _linear(x, self.linear, bf16).permute(0, 3, 1, 2).unsqueeze(-4)
        # Row chunking is exact: rows of the pair tensor attend independently
        # (upstream chunk_layer, triangle.py:81-86); it only bounds CPU memory.
        outs = []
        limit = x.shape[-3] if rows is None else min(rows, x.shape[-3])
        for i0 in range(0, limit, row_chunk):
            i1 = min(i0 + row_chunk, limit)
            xs = x[..., i0:i1, :, :]
            outs.append(self.mha(xs, xs, tri_bias, mask_bias[..., i0:i1, :, :, :], bf16))
        out = torch.cat(outs, dim=-3)
        if not self.starting:
            out = out.transpose(-2, -3)
        return out


class TriangleAttentionEndingNode(TriangleAttention):
    """Triangle attention around the ending node: runs on z transposed."""

    starting = False


class _TriangleMultiplication(nn.Module):
    outgoing = True

    def __init__(self, dim=128):
        super().__init__()
        self.norm_in = nn.LayerNorm(dim, eps=1e-5)
        self.p_in = nn.Linear(dim, 2 * dim, bias=False)
        self.g_in = nn.Linear(dim, 2 * dim, bias=False)
        self.norm_out = nn.LayerNorm(dim)
        self.p_out = nn.Linear(dim, dim, bias=False)
        self.g_out = nn.Linear(dim, dim, bias=False)

    def forward(self, x, mask, bf16=True):
        """Follows ``multiplication.py:48-137`` and ``multiplication_gate_hip.cu:16-58``."""
        x = _layer_norm(x, self.norm_in)
        x_in = x
        p = _linear(x, self.p_in, bf16)
        g = _linear(x, self.g_in, bf16)
        if bf16:
            x = bf16_round(p * sigmoid_bf16(g))
        else:
            x = p * torch.sigmoid(g)
        # bf16 * fp32 mask promotes to fp32; the einsum under autocast rounds again.
        x = x * mask.float().unsqueeze(-1)
        a, b = torch.chunk(x, 2, dim=-1)
        if bf16:
            a, b = bf16_round(a), bf16_round(b)
        if self.outgoing:
            o = torch.einsum("bikd,bjkd->bijd", a, b)
        else:
            o = torch.einsum("bkid,bkjd->bijd", a, b)
        if bf16:
            o = bf16_round(o)
        o = _layer_norm(o, self.norm_out)
        p = _linear(o, self.p_out, bf16)
        g = _linear(x_in, self.g_out, bf16)
        if bf16:
            return bf16_round(p * sigmoid_bf16(g))
        return p * torch.sigmoid(g)


class TriangleMultiplicationOutgoing(_TriangleMultiplication):
    outgoing = True


class TriangleMultiplicationIncoming(_TriangleMultiplication):
    outgoing = False


class Transition(nn.Module):
    """SwiGLU transition (``pair_transition.py:8-28``)."""

    def __init__(self, dim=128, hidden=512, out_dim=None):
        super().__init__()
        out_dim = out_dim or dim
        self.norm = nn.LayerNorm(dim, eps=1e-5)
        self.fc1 = nn.Linear(dim, hidden, bias=False)
        self.fc2 = nn.Linear(dim, hidden, bias=False)
        self.fc3 = nn.Linear(hidden, out_dim, bias=False)
        self.silu = nn.SiLU()
        self.hidden = hidden

    def forward(self, x, bf16=True):
        x = _layer_norm(x, self.norm)
        a = _linear(x, self.fc1, bf16)
        b = _linear(x, self.fc2, bf16)
        if bf16:
            h = bf16_round(silu_bf16(a) * b)
        else:
            h = nn.functional.silu(a) * b
        return _linear(h, self.fc3, bf16)


class AdaLN(nn.Module):
    """Adaptive LayerNorm of the diffusion transformer (``diffusion.py:52-57``)."""

    def __init__(self, dim, dim_single_cond):
        super().__init__()
        self.a_norm = nn.LayerNorm(dim, elementwise_affine=False, bias=False)
        self.s_norm = nn.LayerNorm(dim_single_cond, bias=False)
        self.s_scale = nn.Linear(dim_single_cond, dim)
        self.s_bias = nn.Linear(dim_single_cond, dim, bias=False)

    def forward(self, a, s):
        a = _layer_norm(a, self.a_norm)
        s = _layer_norm(s, self.s_norm)
        # diffusion_hip.cu:15-18: the multiply and the add round separately.
        return diffusion_epilogue(MODULATION, a, self.s_scale(s), self.s_bias(s))


class ConditionedTransitionBlock(nn.Module):
    """Conditioned SwiGLU transition (``diffusion.py:60-68``)."""

    def __init__(self, dim_single, dim_single_cond, expansion_factor=2):
        super().__init__()
        self.adaln = AdaLN(dim_single, dim_single_cond)
        inner = int(dim_single * expansion_factor)
        self.swish_gate = nn.Sequential(nn.Linear(dim_single, inner * 2, bias=False))
        self.a_to_b = nn.Linear(dim_single, inner, bias=False)
        self.b_to_a = nn.Linear(inner, dim_single, bias=False)
        self.output_projection = nn.Sequential(nn.Linear(dim_single_cond, dim_single), nn.Sigmoid())

    def forward(self, a, s):
        a = self.adaln(a, s)
        b = diffusion_epilogue(GATED_SWIGLU, self.swish_gate[0](a), self.a_to_b(a))
        return diffusion_epilogue(GATE, self.output_projection[0](s), self.b_to_a(b))


class AttentionPairBias(nn.Module):
    """fp32 single-track attention with pair bias (``pair_bias.py:15-36``)."""

    def __init__(self, c_s, c_z=None, num_heads=None, inf=1e6, compute_pair_bias=True):
        super().__init__()
        self.c_s, self.num_heads, self.head_dim, self.inf = c_s, num_heads, c_s // num_heads, inf
        self.compute_pair_bias = compute_pair_bias
        self.proj_q = nn.Linear(c_s, c_s)
        self.proj_k = nn.Linear(c_s, c_s, bias=False)
        self.proj_v = nn.Linear(c_s, c_s, bias=False)
        self.proj_g = nn.Linear(c_s, c_s, bias=False)
        if compute_pair_bias:
            self.proj_z = nn.Sequential(nn.LayerNorm(c_z), nn.Linear(c_z, num_heads, bias=False))
        self.proj_o = nn.Linear(c_s, c_s, bias=False)

    def forward(self, s, z, mask, k_in):
        b = s.shape[0]
        q = self.proj_q(s).view(b, -1, self.num_heads, self.head_dim)
        k = self.proj_k(k_in).view(b, -1, self.num_heads, self.head_dim)
        v = self.proj_v(k_in).view(b, -1, self.num_heads, self.head_dim)
        if self.compute_pair_bias:
            bias = self.proj_z[1](_layer_norm(z, self.proj_z[0])).permute(0, 3, 1, 2)
        else:
            bias = z
        g = torch.sigmoid(self.proj_g(s))
        attn = torch.einsum("bihd,bjhd->bhij", q, k)
        attn = attn / (self.head_dim ** 0.5) + bias
        attn = attn + (1 - mask[:, None, None].float()) * -self.inf
        attn = attn.softmax(dim=-1)
        o = torch.einsum("bhij,bjhd->bihd", attn, v).reshape(b, -1, self.c_s)
        return self.proj_o(g * o)


class PairformerLayer(nn.Module):
    """One Boltz-2 Pairformer block (AF3 supplementary Algorithm 17)."""

    def __init__(self, token_s=384, token_z=128, num_heads=16, pairwise_head_width=32,
                 pairwise_num_heads=4):
        super().__init__()
        self.pre_norm_s = nn.LayerNorm(token_s)
        self.attention = AttentionPairBias(token_s, token_z, num_heads)
        self.tri_mul_out = TriangleMultiplicationOutgoing(token_z)
        self.tri_mul_in = TriangleMultiplicationIncoming(token_z)
        self.tri_att_start = TriangleAttention(token_z, pairwise_head_width, pairwise_num_heads)
        self.tri_att_end = TriangleAttentionEndingNode(token_z, pairwise_head_width, pairwise_num_heads)
        self.transition_s = Transition(token_s, token_s * 4)
        self.transition_z = Transition(token_z, token_z * 4)

    def forward(self, s, z, mask, pair_mask, bf16=True):
        z = z + self.tri_mul_out(z, pair_mask, bf16=bf16)
        z = z + self.tri_mul_in(z, pair_mask, bf16=bf16)
        z = z + self.tri_att_start(z, pair_mask, bf16=bf16)
        z = z + self.tri_att_end(z, pair_mask, bf16=bf16)
        z = z + self.transition_z(z, bf16=bf16)
        s_normed = _layer_norm(s, self.pre_norm_s)
        s = s + self.attention(s_normed, z, mask, s_normed)
        s = s + self.transition_s(s, bf16=False)
        return s, z


def randomize(module, std=0.08, generator=None):
    """Seeded weights as in the reference test (``tests/test_operator_additions.py:43-47``):
    N(0, std), with mean 1 for normalisation weights."""
    with torch.no_grad():
        for name, parameter in module.named_parameters():
            mean = 1.0 if "norm" in name and name.endswith("weight") else 0.0
            parameter.copy_(torch.randn(parameter.shape, generator=generator) * std + mean)
    return module
