"""CPU: pin the oracle's explicit-rounding restatement to the golden vectors.

tests/golden/kernel_expressions.pt holds the reference tests' own reference
expressions evaluated with torch's native bf16 arithmetic (see
tests/golden/make_golden.py); the oracle must reproduce them.
"""

from pathlib import Path

import pytest
import torch

from oracle import numerics
from oracle.modules import ordered_bias_softmax

GOLDEN = torch.load(Path(__file__).resolve().parent / "golden" / "kernel_expressions.pt")


@pytest.mark.parametrize("index", range(4))
def test_ordered_softmax_matches_reference_expression(index):
    case = GOLDEN["ordered_softmax"][index]
    bf16 = case["scores"].dtype == torch.bfloat16
    got = ordered_bias_softmax(case["scores"].float(), case["mask"], case["bias"].float(), bf16=bf16)
    expected = case["expected"].float()
    # Both sides round every intermediate to bf16; the softmax itself differs
    # only in fp32 summation order.
    tol = 2 ** -8 if bf16 else 1e-6
    assert (got - expected).abs().max().item() <= tol


@pytest.mark.parametrize("index", range(6))
def test_silu_mul_matches_reference_expression(index):
    case = GOLDEN["silu"][index]
    got = numerics.bf16_round(numerics.silu_bf16(case["a"].float()) * case["b"].float())
    assert torch.equal(got, case["expected"].float())


def test_sigmoid_gate_matches_reference_expression():
    case = GOLDEN["gate"]
    got = numerics.bf16_round(case["p"].float() * numerics.sigmoid_bf16(case["g"].float()))
    assert torch.equal(got, case["expected"].float())
    got = numerics.bf16_round(case["pm"].float() * numerics.sigmoid_bf16(case["gm"].float()))
    got = got * case["mask"][..., None]
    assert case["expected_masked"].dtype == torch.float32  # bf16 * fp32 mask promotes
    assert torch.equal(got, case["expected_masked"])


def test_diffusion_epilogues_match_reference_expressions():
    """The oracle's diffusion epilogues (the ones its AdaLN and ConditionedTransitionBlock
    call) reproduce the reference expressions' golden values bitwise."""
    case = GOLDEN["epilogue"]
    a, b, c, wide = case["a"], case["b"], case["c"], case["wide"]
    assert torch.equal(numerics.diffusion_epilogue(numerics.MODULATION, a, b, c), case["modulation"])
    assert torch.equal(numerics.diffusion_epilogue(numerics.GATE, a, b), case["gate"])
    assert torch.equal(numerics.diffusion_epilogue(numerics.GATED_SWIGLU, wide, b), case["swiglu"])


def test_oracle_diffusion_modules_use_the_pinned_epilogues():
    """AdaLN and ConditionedTransitionBlock of the oracle equal their formulas written out
    with the same expressions the golden epilogue values pin."""
    import oracle

    g = torch.Generator().manual_seed(3)
    block = oracle.randomize(oracle.ConditionedTransitionBlock(64, 64), std=0.1, generator=g)
    a = torch.randn(5, 64, generator=g)
    s = torch.randn(5, 64, generator=g)
    ada = block.adaln
    an = torch.nn.functional.layer_norm(a, (64,), eps=ada.a_norm.eps)
    sn = torch.nn.functional.layer_norm(s, (64,), ada.s_norm.weight, None, ada.s_norm.eps)
    modulated = torch.sigmoid(ada.s_scale(sn)) * an + ada.s_bias(sn)
    assert torch.allclose(ada(a, s), modulated, atol=1e-6)
    x = block.swish_gate[0](modulated)
    bb = torch.nn.functional.silu(x[:, 64 * 2:]) * x[:, :64 * 2] * block.a_to_b(modulated)
    expected = torch.sigmoid(block.output_projection[0](s)) * block.b_to_a(bb)
    assert torch.allclose(block(a, s), expected, atol=1e-5)


def test_oracle_module_shapes_and_masks():
    """Fully masked rows attend uniformly (upstream's -1e9 bias rounds to one bf16 value)."""
    import oracle

    torch.manual_seed(0)
    att = oracle.randomize(oracle.TriangleAttention(128, 32, 4))
    x = torch.randn(1, 9, 9, 128)
    mask = torch.ones(1, 9, 9)
    mask[:, 3, :] = 0
    out = att(x, mask)
    assert out.shape == x.shape and torch.isfinite(out).all()
