"""bf16-autocast rounding emulation used by the CPU oracle (test infrastructure).

Upstream Boltz runs the trunk with fp32 storage under ``torch.autocast(bfloat16)``
(reference ``multiplication.py:59-62``, ``triangle.py:118,125-126``).  Under
autocast a ``Linear`` rounds its inputs and weights to bf16, accumulates in
fp32 and rounds the result to bf16; pointwise ops on bf16 tensors compute in
fp32 and round once.  These helpers make every such rounding explicit so the
oracle can run in fp32 on the CPU and still land on the same values.
"""

import torch


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    """Round an fp32 tensor to the nearest bf16 value (ties to even), kept fp32."""
    return x.to(torch.bfloat16).to(torch.float32)


def linear_bf16(x: torch.Tensor, weight: torch.Tensor, bias=None) -> torch.Tensor:
    """Autocast ``F.linear``: bf16 operands, fp32 accumulation, bf16 result."""
    y = bf16_round(x) @ bf16_round(weight).t()
    if bias is not None:
        y = y + bf16_round(bias)
    return bf16_round(y)


def sigmoid_bf16(x: torch.Tensor) -> torch.Tensor:
    """``torch.sigmoid`` on a bf16 tensor: fp32 math, one rounding to bf16.

    The reference rounds the sigmoid to bf16 before the gating multiply
    (``kernels/multiplication_gate_hip.cu:16-20``).
    """
    return bf16_round(torch.sigmoid(bf16_round(x)))


def silu_bf16(x: torch.Tensor) -> torch.Tensor:
    """``F.silu`` on a bf16 tensor, rounded to bf16 (``kernels/pair_hip.cu:12-17``)."""
    return bf16_round(torch.nn.functional.silu(bf16_round(x)))


# Diffusion epilogue operation codes (the reference's diffusion.py:27).
MODULATION, GATE, GATED_SWIGLU = 0, 1, 3


def diffusion_epilogue(kind: int, a: torch.Tensor, b: torch.Tensor, c=None) -> torch.Tensor:
    """The fp32 diffusion epilogues (``kernels/diffusion_hip.cu:13-27``), no autocast.

    * MODULATION: ``sigmoid(b) * a + c`` (AdaLN, the multiply and add round separately);
    * GATE: ``sigmoid(a) * b`` (the conditioned transition's output gate);
    * GATED_SWIGLU: ``silu(a[..., h:]) * a[..., :h] * b`` with ``a`` of width 2h
      (swish_gate's projection times a_to_b's).
    """
    if kind == MODULATION:
        return torch.sigmoid(b) * a + c
    if kind == GATE:
        return torch.sigmoid(a) * b
    if kind == GATED_SWIGLU:
        half = a.shape[-1] // 2
        return torch.nn.functional.silu(a[..., half:]) * a[..., :half] * b
    raise ValueError(f"unknown diffusion epilogue kind {kind}")
