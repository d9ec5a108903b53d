"""Parity of the tcgen05 flash triangle-attention kernel against the CPU oracle
(same cases and tolerance as the module tests)."""

import pytest
import torch

import oracle
from conftest import assert_close
from test_modules_gpu import BF16_ATOL, build, pair_mask

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from boltz_lumi_b200 import forwards, layers


@pytest.fixture
def tc_entry(monkeypatch):
    monkeypatch.setattr(forwards, "ATTENTION_ENTRY", "bl_triangle_attention_tc")


@pytest.mark.parametrize("ending", [False, True])
@pytest.mark.parametrize("n,kind", [(17, "ones"), (64, "partial"), (117, "ones"), (117, "partial"),
                                    (130, "partial"), (200, "ones"), (256, "fractional")])
def test_triangle_attention_tc(tc_entry, ending, n, kind):
    cls = (layers.TriangleAttentionEndingNode, oracle.TriangleAttentionEndingNode) if ending else \
        (layers.TriangleAttention, oracle.TriangleAttention)
    mod, ref = build(*cls, 128, 32, 4)
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(n))
    mask = pair_mask(n, kind)
    expected = ref(x, mask, chunk_size=32)
    with torch.inference_mode():
        actual = mod(x.cuda(), mask.cuda(), chunk_size=32)
    assert_close(actual.float(), expected, atol=BF16_ATOL)


def test_triangle_attention_tc_matches_mma_kernel(monkeypatch):
    """Both kernels compute the same thing on a large case (N = 512, masked tail)."""
    n = 512
    mod, _ = build(layers.TriangleAttention, oracle.TriangleAttention, 128, 32, 4, std=1 / 128 ** 0.5)
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(3)).cuda()
    mask = pair_mask(n, "partial", masked_tokens=51).cuda()
    with torch.inference_mode():
        a = mod(x, mask)
        monkeypatch.setattr(forwards, "ATTENTION_ENTRY", "bl_triangle_attention_tc")
        b = mod(x, mask)
    assert_close(b.float(), a.float(), atol=BF16_ATOL)
