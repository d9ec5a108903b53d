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
    case = GOLDEN["epilogue"]
    a, b, c, wide = case["a"], case["b"], case["c"], case["wide"]
    assert torch.allclose(torch.sigmoid(b) * a + c, case["modulation"], atol=0, rtol=0)
    assert torch.allclose(torch.sigmoid(a) * b, case["gate"], atol=0, rtol=0)
    swiglu = torch.nn.functional.silu(wide[:, 768:]) * wide[:, :768] * b
    assert torch.allclose(swiglu, case["swiglu"], atol=0, rtol=0)


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
