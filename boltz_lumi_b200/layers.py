"""Standalone modules with upstream Boltz-2 constructors and parameter names.

They let the B200 path run without the upstream package installed (tests,
benchmarks, other hosts) and load upstream ``state_dict``s unchanged.  Their
forwards are the kernel-backed functions of :mod:`boltz_lumi_b200.forwards`;
they are inference-only and raise rather than fall back to eager code.
"""


import torch
import torch.nn.functional as F
from torch import nn

from . import _lib, forwards, kernels


def _inference_only(module):
    if module.training or torch.is_grad_enabled():
        raise RuntimeError(f"{type(module).__name__}: the B200 kernels are inference-only; "
                           "use torch.inference_mode() and module.eval()")


class LayerNorm(nn.LayerNorm):
    """LayerNorm exposing ``c_in`` like the triangle-attention variant upstream."""

    def __init__(self, c_in, eps=1e-5, elementwise_affine=True, bias=True):
        super().__init__(c_in, eps=eps, elementwise_affine=elementwise_affine, bias=bias)
        self.c_in = (c_in,)


class Attention(nn.Module):
    """Parameter container of the gated triangle attention (``mha``)."""

    def __init__(self, c_q, c_k, c_v, c_hidden, no_heads):
        super().__init__()
        self.c_q, self.c_hidden, self.no_heads = c_q, c_hidden, no_heads
        self.linear_q = nn.Linear(c_q, c_hidden * no_heads, bias=False)
        self.linear_k = nn.Linear(c_k, c_hidden * no_heads, bias=False)
        self.linear_v = nn.Linear(c_v, c_hidden * no_heads, bias=False)
        self.linear_o = nn.Linear(c_hidden * no_heads, c_q)
        self.linear_g = nn.Linear(c_q, c_hidden * no_heads)


class TriangleAttention(nn.Module):
    starting = True

    def __init__(self, c_in, c_hidden, no_heads, starting=None, inf=1e9):
        super().__init__()
        if starting is not None:
            self.starting = starting
        self.c_in, self.c_hidden, self.no_heads, self.inf = c_in, c_hidden, no_heads, inf
        self.layer_norm = LayerNorm(c_in)
        self.linear = nn.Linear(c_in, no_heads, bias=False)
        self.mha = Attention(c_in, c_in, c_in, c_hidden, no_heads)

    def forward(self, x, mask=None, chunk_size=None, use_kernels=False):
        _inference_only(self)
        return forwards.triangle_attention_forward(self, x, mask, chunk_size, use_kernels)


class TriangleAttentionEndingNode(TriangleAttention):
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

    def forward(self, x, mask, use_kernels=False):
        _inference_only(self)
        return forwards.triangle_multiplication_forward(self, x, mask, use_kernels)


class TriangleMultiplicationOutgoing(_TriangleMultiplication):
    outgoing = True


class TriangleMultiplicationIncoming(_TriangleMultiplication):
    outgoing = False


class Transition(nn.Module):
    def __init__(self, dim=128, hidden=512, out_dim=None):
        super().__init__()
        out_dim = out_dim or dim
        self.norm = nn.LayerNorm(dim, eps=1e-5)
        self.fc1 = nn.Linear(dim, hidden, bias=False)
        self.fc2 = nn.Linear(dim, hidden, bias=False)
        self.fc3 = nn.Linear(hidden, out_dim, bias=False)
        self.silu = nn.SiLU()
        self.hidden = hidden

    def forward(self, x, chunk_size=None):
        _inference_only(self)
        return forwards.transition_forward(self, x, chunk_size)


class AdaLN(nn.Module):
    def __init__(self, dim, dim_single_cond):
        super().__init__()
        self.a_norm = nn.LayerNorm(dim, elementwise_affine=False, bias=False)
        self.s_norm = nn.LayerNorm(dim_single_cond, bias=False)
        self.s_scale = nn.Linear(dim_single_cond, dim)
        self.s_bias = nn.Linear(dim_single_cond, dim, bias=False)

    def forward(self, a, s):
        _inference_only(self)
        return forwards.adaln_forward(self, a, s)


class ConditionedTransitionBlock(nn.Module):
    def __init__(self, dim_single, dim_single_cond, expansion_factor=2):
        super().__init__()
        self.adaln = AdaLN(dim_single, dim_single_cond)
        inner = int(dim_single * expansion_factor)
        self.swish_gate = nn.Sequential(nn.Linear(dim_single, inner * 2, bias=False))
        self.a_to_b = nn.Linear(dim_single, inner, bias=False)
        self.b_to_a = nn.Linear(inner, dim_single, bias=False)
        self.output_projection = nn.Sequential(nn.Linear(dim_single_cond, dim_single), nn.Sigmoid())

    def forward(self, a, s):
        _inference_only(self)
        return forwards.conditioned_transition_forward(self, a, s)


class _HeadsFirst(nn.Module):
    """``proj_z`` of a bias-consuming AttentionPairBias: [B, N, N, H] -> [B, H, N, N]
    as a view (upstream's ``Rearrange("b ... h -> b h ...")``)."""

    def forward(self, z):
        return z.permute(0, 3, 1, 2)


class AttentionPairBias(nn.Module):
    """fp32 single-track attention with pair bias (upstream attentionv2).

    With ``compute_pair_bias`` the bias is LayerNorm(z) . W_z (the Pairformer
    block); without it ``z`` is the bias itself, [B, N, N, H] (the diffusion
    token transformer's layer slice of the prepared token bias).
    """

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
        else:
            self.proj_z = _HeadsFirst()
        self.proj_o = nn.Linear(c_s, c_s, bias=False)

    def pair_bias(self, z):
        """LayerNorm(z) . W_z in one pass, head-major [b, heads, N, N] (fp32)."""
        ln, lin = self.proj_z[0], self.proj_z[1]
        b, n = z.shape[0], z.shape[1]
        zf = z.float().contiguous()
        bias = torch.empty(b, self.num_heads, n, n, device=z.device, dtype=torch.float32)
        w_z = lin.weight.float().contiguous()
        stream = _lib.stream_of(z)
        for i in range(b):
            _lib.call("bl_pair_bias", zf[i].data_ptr(), n * n, _lib.ptr(ln.weight), _lib.ptr(ln.bias),
                      float(ln.eps), w_z.data_ptr(), self.num_heads, bias[i].data_ptr(), stream)
        return bias

    def forward(self, s, z, mask, k_in, multiplicity=1):
        _inference_only(self)
        if not self.compute_pair_bias:
            return forwards.token_attention_forward(self, s, z, mask, k_in, multiplicity)
        return self.attend(s, self.pair_bias(z), mask, k_in)

    def attend(self, s, bias, mask, k_in, residual=None):
        """The attention given the pair bias [b', heads, N, N] (fp32, b' dividing b), plus
        ``residual`` when given (added in proj_o's epilogue)."""
        return forwards.attend_with_bias(self, s, bias, mask, k_in, residual=residual)


class _FP32Transition(Transition):
    """Single-track transition: upstream runs it in fp32 without autocast."""

    def forward(self, x, chunk_size=None, residual=None):
        """fc3(silu(fc1(LN(x))) * fc2(LN(x))), plus ``residual`` when given (added in
        fc3's epilogue: the block's s = s + transition_s(s) in one pass)."""
        _inference_only(self)
        cols, hidden = x.shape[-1], self.fc1.weight.shape[0]
        if cols % 128 == 0 and cols <= 1024 and hidden % 8 == 0:
            # LayerNorm and silu(fc1) * fc2 leave their kernels as the split
            # operands of fc1 | fc2 and fc3.
            lead = x.shape[:-1]
            xn3 = kernels.layer_norm_split3(x, self.norm.weight, self.norm.bias, self.norm.eps)
            h = forwards._linear32_planes(self, "_bl_w3_fc12", xn3, lead, [self.fc1.weight, self.fc2.weight])
            h3 = kernels.epilogue_split3(h, None, None, kernels.SWIGLU)
            return forwards._linear32_planes(self, "_bl_w3_fc3", h3, lead, [self.fc3.weight], residual=residual)
        xn = kernels.layer_norm(x.contiguous(), self.norm.weight, self.norm.bias, self.norm.eps,
                                out_dtype=torch.float32)
        h = forwards._linear32(self, "_bl_w3_fc12", xn, [self.fc1.weight, self.fc2.weight])
        a, b = h.split(hidden, dim=-1)
        y = forwards._linear32(self, "_bl_w3_fc3", F.silu(a) * b, [self.fc3.weight])
        return y if residual is None else y + residual


class PairformerLayer(nn.Module):
    """One Boltz-2 Pairformer block; pair updates are added to z in fp32."""

    def __init__(self, token_s=384, token_z=128, num_heads=16, pairwise_head_width=32, pairwise_num_heads=4):
        super().__init__()
        self.pre_norm_s = nn.LayerNorm(token_s)
        self.attention = AttentionPairBias(token_s, token_z, num_heads)
        self.tri_mul_out = TriangleMultiplicationOutgoing(token_z)
        self.tri_mul_in = TriangleMultiplicationIncoming(token_z)
        self.tri_att_start = TriangleAttention(token_z, pairwise_head_width, pairwise_num_heads)
        self.tri_att_end = TriangleAttentionEndingNode(token_z, pairwise_head_width, pairwise_num_heads)
        self.transition_s = _FP32Transition(token_s, token_s * 4)
        self.transition_z = Transition(token_z, token_z * 4)

    def forward(self, s, z, mask, pair_mask):
        """Returns (s, z); z (contiguous fp32) is updated in place: each pair op adds
        its bf16 update inside its last GEMM's epilogue (z = z + op(z) upstream)."""
        _inference_only(self)
        if z.dtype != torch.float32 or not z.is_contiguous():
            z = z.float().contiguous()
        forwards.triangle_multiplication_forward(self.tri_mul_out, z, pair_mask, residual=z)
        forwards.triangle_multiplication_forward(self.tri_mul_in, z, pair_mask, residual=z)
        forwards.triangle_attention_forward(self.tri_att_start, z, pair_mask, residual=z)
        forwards.triangle_attention_forward(self.tri_att_end, z, pair_mask, residual=z)
        forwards.transition_forward(self.transition_z, z, residual=z)
        s = s.contiguous()
        att = self.attention
        if s.shape[-1] % 128 == 0 and s.shape[-1] <= 1024:
            # LN(s) goes straight into the q | k | v | g projection's split operand.
            s3 = kernels.layer_norm_split3(s, self.pre_norm_s.weight, self.pre_norm_s.bias, self.pre_norm_s.eps)
            # s + attention(...) and s + transition_s(s): the residual adds run in
            # the epilogues of proj_o and fc3 (new tensors; the caller's s is unchanged).
            s = forwards.attend_with_bias(att, s, att.pair_bias(z), mask, s, s3=s3, residual=s)
        else:
            s_normed = kernels.layer_norm(s, self.pre_norm_s.weight, self.pre_norm_s.bias, self.pre_norm_s.eps,
                                          out_dtype=torch.float32)
            s = s + att(s_normed, z, mask, s_normed)
        s = self.transition_s(s, residual=s)
        return s, z
