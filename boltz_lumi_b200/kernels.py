"""Torch-facing wrappers of the C-ABI kernels (one per reference native op).

Each function mirrors a native function of the reference (the pybind11
bindings of ``kernels/*_hip.cpp`` and the Triton ``ordered_softmax``): same
argument meaning, a freshly allocated output, inference only, and the current
CUDA stream of the input's device.  Errors raise ``RuntimeError``; there is
no fallback path.
"""

import functools

import torch

from . import _lib
from ._lib import call, ptr, stream_of


def _require_inference(*tensors):
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise RuntimeError("boltz_lumi_b200 kernels are inference-only (grad mode with requires_grad inputs)")


def _require_cuda(*tensors):
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("boltz_lumi_b200 kernels need CUDA tensors")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError("all tensors must be on the same device")
    return device


def norm(x, weight, bias, eps, channel_first=False, bf16_output=True):
    """LayerNorm over 128 channels (reference ``extension("multiplication").norm``,
    ``kernels/multiplication_hip.cu:149``).

    Row-major ``x`` is [M, C]; channel-first ``x`` is [128, M].  Returns [M, C]
    in bf16 (``bf16_output``) or fp32.
    """
    _require_inference(x)
    _require_cuda(x, weight, bias)
    if x.dim() != 2 or not x.is_contiguous():
        raise RuntimeError("norm expects a contiguous 2-D tensor")
    rows, cols = (x.shape[1], x.shape[0]) if channel_first else (x.shape[0], x.shape[1])
    for v in (weight, bias):
        if v is not None and (v.dtype != torch.float32 or v.numel() != cols or not v.is_contiguous()):
            raise RuntimeError("norm weight/bias must be contiguous fp32 with one value per channel")
    out = torch.empty(rows, cols, device=x.device, dtype=torch.bfloat16 if bf16_output else torch.float32)
    call("bl_layernorm", x.data_ptr(), _lib.dtype_code(x.dtype), rows, cols, int(channel_first), ptr(weight),
         ptr(bias), float(eps), out.data_ptr(), _lib.dtype_code(out.dtype), stream_of(x))
    return out


def layer_norm(x, weight, bias, eps, out_dtype=None):
    """LayerNorm over the last dimension of any-rank ``x`` (fp32 statistics)."""
    _require_inference(x)
    _require_cuda(x, weight, bias)
    x = x.contiguous()
    cols = x.shape[-1]
    out = torch.empty(x.shape, device=x.device, dtype=out_dtype or x.dtype)
    call("bl_layernorm", x.data_ptr(), _lib.dtype_code(x.dtype), x.numel() // max(cols, 1), cols, 0,
         ptr(weight), ptr(bias), float(eps), out.data_ptr(), _lib.dtype_code(out.dtype), stream_of(x))
    return out


def gate(p, g):
    """``bf16(p * bf16(sigmoid(g)))`` (reference ``multiplication_gate_hip.cu:81``)."""
    _require_inference(p, g)
    _require_cuda(p, g)
    if p.shape != g.shape or p.dtype != torch.bfloat16 or g.dtype != torch.bfloat16:
        raise RuntimeError("gate expects two bf16 tensors of the same shape")
    p, g = p.contiguous(), g.contiguous()
    out = torch.empty_like(p)
    call("bl_gate", p.data_ptr(), g.data_ptr(), out.data_ptr(), p.numel(), stream_of(p))
    return out


def _gate_operands(p, g, mask):
    _require_inference(p, g)
    _require_cuda(p, g, mask)
    if p.dtype != torch.bfloat16 or g.dtype != torch.bfloat16:
        raise RuntimeError("gate operands must be bf16")
    if p.dim() != 4 or p.shape[0] != 1 or p.shape[1] != p.shape[2] or p.shape[3] != 256:
        raise RuntimeError("expected projections of shape [1, N, N, 256]")
    stride = p.stride(2)
    if stride not in (256, 512) or p.stride(3) != 1 or p.stride(1) != p.shape[2] * stride or g.stride() != p.stride():
        raise RuntimeError("expected dense or joint-projection rows")
    if mask.dtype != torch.float32 or not mask.is_contiguous() or mask.numel() * 256 != p.shape[1] * p.shape[2] * 256:
        raise RuntimeError("mask must be contiguous fp32 [1, N, N]")
    return p.shape[1], stride


def pack(p, g, mask, outgoing):
    """Gate, mask and channel-first pack (reference ``multiplication_gate_hip.cu:140``)."""
    n, stride = _gate_operands(p, g, mask)
    left = torch.empty(128, n, n, device=p.device, dtype=torch.bfloat16)
    right = torch.empty_like(left)
    call("bl_gate_pack", p.data_ptr(), g.data_ptr(), stride, mask.data_ptr(), n, int(bool(outgoing)),
         left.data_ptr(), right.data_ptr(), stream_of(p))
    return left, right


def split(p, g, mask):
    """Gate and mask into channel-last halves (reference ``multiplication_gate_hip.cu:96``)."""
    n, stride = _gate_operands(p, g, mask)
    a = torch.empty(1, n, n, 128, device=p.device, dtype=torch.bfloat16)
    b = torch.empty_like(a)
    call("bl_gate_split", p.data_ptr(), g.data_ptr(), stride, mask.data_ptr(), n, a.data_ptr(), b.data_ptr(),
         stream_of(p))
    return a, b


def silu_mul(a, b):
    """``bf16(bf16(silu(a)) * b)`` (reference ``kernels/pair_hip.cu:42``)."""
    _require_inference(a, b)
    _require_cuda(a, b)
    if a.shape != b.shape or a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise RuntimeError("silu_mul expects two bf16 tensors of the same shape")
    if not (a.is_contiguous() and b.is_contiguous()):
        raise RuntimeError("silu_mul expects contiguous inputs")
    out = torch.empty_like(a)
    call("bl_silu_mul", a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), stream_of(a))
    return out


MODULATION, GATE, GATED_SWIGLU = _lib.BL_EPI_MODULATION, _lib.BL_EPI_GATE, _lib.BL_EPI_GATED_SWIGLU
SWIGLU = _lib.BL_EPI_SWIGLU  # silu(a[:, :C]) * a[:, C:] (an fp32 Transition's fc1 | fc2 product)


def epilogue(a, b, c, kind):
    """fp32 diffusion epilogues (reference ``kernels/diffusion_hip.cu:80``)."""
    _require_inference(a, b, c)
    _require_cuda(a, b, c)
    if kind not in (MODULATION, GATE, GATED_SWIGLU, SWIGLU):
        raise RuntimeError(f"unknown epilogue kind {kind}")
    for t in (a, b, c):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise RuntimeError("epilogue expects contiguous fp32 tensors")
    shape = list(a.shape)
    cols = shape[-1]
    if kind in (GATED_SWIGLU, SWIGLU):
        if cols % 2:
            raise RuntimeError("SwiGLU epilogues need an even last dimension")
        cols //= 2
        shape[-1] = cols
    out = torch.empty(shape, device=a.device, dtype=torch.float32)
    if (kind != SWIGLU and tuple(b.shape) != tuple(shape)) or \
            (kind == MODULATION and (c is None or tuple(c.shape) != tuple(shape))):
        raise RuntimeError("epilogue operand shapes disagree")
    rows = out.numel() // max(cols, 1)
    call("bl_diffusion_epilogue", a.data_ptr(), ptr(b), ptr(c), out.data_ptr(), rows, cols, kind, stream_of(a))
    return out


def adaln_modulate(a, scale, shift, eps):
    """``sigmoid(scale) * LayerNorm(a) + shift`` with a non-affine LayerNorm (fp32)."""
    _require_inference(a, scale, shift)
    _require_cuda(a, scale, shift)
    a, scale, shift = a.contiguous(), scale.contiguous(), shift.contiguous()
    if not (a.dtype == scale.dtype == shift.dtype == torch.float32) or not (a.shape == scale.shape == shift.shape):
        raise RuntimeError("adaln_modulate expects fp32 tensors of one shape")
    out = torch.empty_like(a)
    cols = a.shape[-1]
    call("bl_adaln_modulate", a.data_ptr(), scale.data_ptr(), shift.data_ptr(), out.data_ptr(),
         a.numel() // max(cols, 1), cols, float(eps), stream_of(a))
    return out


def ordered_softmax(scores, bias, mask):
    """``softmax(round(round(s + mask) + bias))`` over materialised triangle scores.

    Reference ``kernels/triangle_softmax.py:120`` / ``triangle_block_softmax_hip.cu:120``.
    ``scores`` [B, I, H, N, N]; ``bias`` broadcastable as [B, 1, H, N, N];
    ``mask`` fp32 broadcastable as [B, I, 1, 1, N].
    """
    _require_inference(scores, bias)
    _require_cuda(scores, bias, mask)
    if scores.dim() != 5 or scores.shape[-1] != scores.shape[-2]:
        raise RuntimeError("expected square score matrices [B, I, H, N, N]")
    if bias.dtype != scores.dtype or mask.dtype != torch.float32:
        raise RuntimeError("bias must share the score dtype; mask must be fp32")
    b, i, h, n, _ = scores.shape
    bias = bias.expand(b, 1, h, n, n)
    mask = mask.expand(b, i, 1, 1, n)
    out = torch.empty(scores.shape, device=scores.device, dtype=scores.dtype)
    ss = _lib.int64_array(scores.stride())
    bs = _lib.int64_array((bias.stride(0), bias.stride(2), bias.stride(3), bias.stride(4)))
    ms = _lib.int64_array((mask.stride(0), mask.stride(1), mask.stride(4)))
    call("bl_triangle_softmax", scores.data_ptr(), _lib.dtype_code(scores.dtype), b, i, h, n, ss, bias.data_ptr(), bs,
         mask.data_ptr(), ms, out.data_ptr(), stream_of(scores))
    return out


def _operand_layout(t, name):
    """Return (mn_major, ld, batch_stride) for a [batch, rows, k]-shaped view."""
    if t.stride(-1) == 1:
        return False, t.stride(-2), t.stride(0)
    if t.stride(-2) == 1:
        return True, t.stride(-1), t.stride(0)
    raise RuntimeError(f"{name} needs one unit stride among its last two dimensions")


def bmm(a, b_t, bias=None, out=None):
    """``out[b] = a[b] @ b_t[b]^T (+ bias)`` in bf16 on tcgen05 tensor cores.

    ``a`` [B, M, K] and ``b_t`` [B, N, K] may each be K-contiguous or
    M/N-contiguous (e.g. ``x.transpose(1, 2)`` of a dense tensor); nothing is copied.
    """
    _require_inference(a, b_t)
    _require_cuda(a, b_t, bias)
    if a.dtype != torch.bfloat16 or b_t.dtype != torch.bfloat16:
        raise RuntimeError("bmm operands must be bf16")
    if a.dim() != 3 or b_t.dim() != 3 or a.shape[0] != b_t.shape[0] or a.shape[2] != b_t.shape[2]:
        raise RuntimeError("bmm expects a [B, M, K] and b_t [B, N, K]")
    batch, m, k = a.shape
    n = b_t.shape[1]
    a_mn, a_ld, a_bs = _operand_layout(a, "a")
    b_mn, b_ld, b_bs = _operand_layout(b_t, "b_t")
    if out is None:
        out = torch.empty(batch, m, n, device=a.device, dtype=torch.bfloat16)
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != n):
        raise RuntimeError("bias must be fp32 with N elements")
    call("bl_batched_gemm", a.data_ptr(), int(a_mn), a_ld, a_bs, b_t.data_ptr(), int(b_mn), b_ld, b_bs,
         out.data_ptr(), out.stride(1), out.stride(0), batch, m, n, k, ptr(bias), stream_of(a))
    return out


@functools.lru_cache(maxsize=None)
def attention_scale(head_dim):
    """fp32(1 / fp32(sqrt(head_dim))): the factor torch's CUDA division by the
    Python scalar ``head_dim ** 0.5`` applies (pair_bias.py:31)."""
    return float(torch.tensor(1.0, dtype=torch.float32) / torch.tensor(head_dim ** 0.5, dtype=torch.float32))


def launch_token_attention(q_ptr, k_ptr, v_ptr, g_ptr, strides, bias, mask, inf, batch, heads, n, d, out, stream,
                           out3=None, n_q=0):
    """bl_token_attention on raw operand pointers sharing ``strides`` (batch,
    token, head) -- no validation; callers have checked shapes and dtypes.
    With ``out3`` (bf16 [3, batch * n_q, heads * d]) the result is written as the
    split planes instead of into ``out``.  ``n_q`` (0: n) queries from q_ptr / g_ptr
    and the bias rows attend over n keys."""
    mask_ptr, mask_sb = (None, 0) if mask is None else (mask.data_ptr(), mask.stride(0))
    bs = bias.stride()
    call("bl_token_attention", q_ptr, k_ptr, v_ptr, g_ptr, strides[0], strides[1], strides[2], bias.data_ptr(),
         bs[0], bs[1], bs[2], bs[3], batch // bias.shape[0], mask_ptr, mask_sb, attention_scale(d), float(inf),
         batch, heads, n, n_q, d, ptr(out), ptr(out3), stream)
    return out


def token_attention(q, k, v, bias, mask, inf, gate=None, scale=None):
    """Fused fp32 attention of the diffusion token transformer (and the
    Pairformer's single track): ``sigmoid(gate) * softmax(q k^T * scale + bias
    + inf * (mask - 1)) v`` per head, the core of pair_bias.py:28-36.

    ``q``, ``k``, ``v`` (and ``gate``): fp32 [B, N, H, d] views with a common
    stride layout and contiguous head dims (e.g. slices of one joint
    projection).  ``bias``: fp32 [Bb, H, N, N] with any strides, where ``Bb``
    divides ``B`` -- sample ``b`` reads bias ``b // (B // Bb)``, which is the
    reference's ``repeat_interleave(multiplicity, 0)`` without the copy.
    ``mask``: [B, N] key mask or None.  Returns fp32 [B, N, H, d].
    """
    _require_inference(q, k, v, gate, bias, mask)
    _require_cuda(q, k, v, gate, bias, mask)
    tensors = [q, k, v] + ([gate] if gate is not None else [])
    if any(t.dtype != torch.float32 for t in tensors + [bias]):
        raise RuntimeError("token attention operands must be fp32")
    if any(t.dim() != 4 or t.shape != q.shape or t.stride() != q.stride() for t in tensors):
        raise RuntimeError("q, k, v and gate must be [B, N, H, d] views with the same strides")
    batch, n, heads, d = q.shape
    if q.stride(3) != 1:
        raise RuntimeError("q/k/v head dims must be contiguous")
    if bias.dim() != 4 or tuple(bias.shape[1:]) != (heads, n, n) or bias.shape[0] < 1 or batch % bias.shape[0]:
        raise RuntimeError(f"bias must be [B', {heads}, {n}, {n}] with B' dividing {batch}, got {tuple(bias.shape)}")
    mask_sb = 0
    if mask is not None:
        if tuple(mask.shape) != (batch, n):
            raise RuntimeError("mask must be [B, N]")
        mask = mask.float()
        if mask.stride(1) != 1:
            mask = mask.contiguous()
        mask_sb = mask.stride(0)
    if scale is None:
        scale = attention_scale(d)
    out = torch.empty(batch, n, heads, d, device=q.device, dtype=torch.float32)
    if n == 0 or batch == 0:
        return out
    call("bl_token_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), ptr(gate), q.stride(0), q.stride(1),
         q.stride(2), bias.data_ptr(), bias.stride(0), bias.stride(1), bias.stride(2), bias.stride(3),
         batch // bias.shape[0], ptr(mask), mask_sb, float(scale), float(inf), batch, heads, n, 0, d, out.data_ptr(),
         None, stream_of(q))
    return out


def split3(x):
    """fp32 ``x`` [..., K] -> bf16 planes [3, rows, K] with x = x1 + x2 + x3
    (bl_split3_bf16); the operand form of :func:`linear_f32`."""
    _require_cuda(x)
    if x.dtype != torch.float32:
        raise RuntimeError("split3 expects fp32")
    cols = x.shape[-1]
    x2 = x.reshape(-1, cols)
    if x2.stride(-1) != 1 or x2.data_ptr() % 16 or x2.stride(0) % 4:
        x2 = x2.contiguous()
    out = torch.empty(3, x2.shape[0], cols, device=x.device, dtype=torch.bfloat16)
    call("bl_split3_bf16", x2.data_ptr(), x2.shape[0], cols, x2.stride(0), out.data_ptr(), stream_of(x))
    return out


def split3_fast(x):
    """:func:`split3` for callers that have checked x (fp32, CUDA, K % 8 == 0)."""
    cols = x.shape[-1]
    if not x.is_contiguous():
        x = x.contiguous()
    rows = x.numel() // cols
    out = torch.empty(3, rows, cols, device=x.device, dtype=torch.bfloat16)
    call("bl_split3_bf16", x.data_ptr(), rows, cols, cols, out.data_ptr(), _lib.current_stream_handle())
    return out


def linear_split3_fast(x3, w3, bias, y, residual=None):
    """bl_linear_split3 into the contiguous fp32 ``y`` [..., N] for callers
    that have checked the operands (x3 = split3(x), w3 = split3(W)); with
    ``residual`` (contiguous fp32 [..., N]) the result is y = x W^T + bias + residual."""
    m, k = x3.shape[1], x3.shape[2]
    n = w3.shape[1]
    call("bl_linear_split3", x3.data_ptr(), m, k, w3.data_ptr(), n, ptr(bias), ptr(residual),
         0 if residual is None else n, y.data_ptr(), n, _lib.current_stream_handle())
    return y


def linear_f32(x, w3, bias=None, x3=None):
    """fp32 ``x @ W^T + bias`` on the tensor cores (error within 2^-17 of the largest output)
    (bl_linear_split3).  ``w3`` = ``split3(W)`` (bf16 [3, N, K]); ``x3`` may
    pass ``split3(x)`` when one input feeds several linears."""
    _require_inference(x)
    _require_cuda(x, w3, bias)
    k = x.shape[-1]
    n = w3.shape[1]
    if w3.shape != (3, n, k) or w3.dtype != torch.bfloat16:
        raise RuntimeError(f"w3 must be bf16 [3, N, {k}]")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != n or not bias.is_contiguous()):
        raise RuntimeError("bias must be contiguous fp32 with N elements")
    if x3 is None:
        x3 = split3(x)
    m = x3.shape[1]
    y = torch.empty(*x.shape[:-1], n, device=x.device, dtype=torch.float32)
    return linear_split3_fast(x3, w3, bias, y)


def layer_norm_split3(x, weight, bias, eps):
    """LayerNorm of fp32 rows written as split planes [3, rows, C] (bl_layernorm_split3);
    C % 128 == 0 and <= 1024."""
    cols = x.shape[-1]
    x = x.contiguous()
    rows = x.numel() // cols
    out = torch.empty(3, rows, cols, device=x.device, dtype=torch.bfloat16)
    call("bl_layernorm_split3", x.data_ptr(), rows, cols, ptr(weight), ptr(bias), float(eps), out.data_ptr(),
         _lib.current_stream_handle())
    return out


def adaln_modulate_split3(a, scale, shift, eps):
    """:func:`adaln_modulate` written as split planes [3, rows, C]."""
    a, scale, shift = a.contiguous(), scale.contiguous(), shift.contiguous()
    cols = a.shape[-1]
    rows = a.numel() // cols
    out = torch.empty(3, rows, cols, device=a.device, dtype=torch.bfloat16)
    call("bl_adaln_modulate_split3", a.data_ptr(), scale.data_ptr(), shift.data_ptr(), out.data_ptr(), rows, cols,
         float(eps), _lib.current_stream_handle())
    return out


def epilogue_split3(a, b, c, kind):
    """:func:`epilogue` written as split planes [3, rows, C] (C = output width)."""
    cols = a.shape[-1] // 2 if kind in (GATED_SWIGLU, SWIGLU) else a.shape[-1]
    rows = a.numel() // a.shape[-1]
    out = torch.empty(3, rows, cols, device=a.device, dtype=torch.bfloat16)
    call("bl_diffusion_epilogue_split3", a.data_ptr(), ptr(b), ptr(c), out.data_ptr(), rows, cols, kind,
         _lib.current_stream_handle())
    return out
