"""Parity at the benchmarked configurations, against the oracle run on the GPU as the checker.

The measurement configurations, exactly:

* C2: TriangleAttention starting and ending node at N = 512, z ~ N(0, 1), tokens 461..511
  (the last 10 %) masked in rows and columns, weights N(0, 1/128) with unit-mean norm
  weights, the triangle bias from the module's own linear(LN(z));
* C3: TriangleMultiplication outgoing and incoming and the pair Transition at N = 768,
  z ~ N(0, 1), mask all ones;
* the bench workload: one full Pairformer block at N = 512 with the bench's seeded weights
  and inputs.

The oracle (same torch restatement as on the CPU, fp32 with explicit bf16 rounding points)
runs on the GPU here only because it would take minutes on the CPU at these sizes; it is
the checker, never the thing measured.

Per-op bound: max(2e-2, one bf16 ulp of the expected value) per element plus relative L2
<= 1e-2.  Above |y| = 2.56 one bf16 ulp of the output itself exceeds 2e-2, and a different
fp32 accumulation order can flip that final rounding; a masking or indexing error shows up
as a relative L2 error of 10 % or more.  The measured errors are recorded (see
``conftest.record_parity``).
"""

import pytest
import torch

import oracle
from conftest import assert_close, record_parity

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from boltz_lumi_b200 import layers

BF16_ATOL = 2e-2
BF16_ULP = 2.0 ** -7
REL_L2 = 1e-2
STD = 128 ** -0.5  # weights N(0, 1/128), the bench's initialisation


def seeded(product_cls, oracle_cls, *args, seed):
    ref = oracle.randomize(oracle_cls(*args), std=STD, generator=torch.Generator().manual_seed(seed))
    mod = product_cls(*args)
    mod.load_state_dict(ref.state_dict())
    return mod.cuda().eval(), ref.cuda().eval()


def tail_masked(n, first_masked):
    mask = torch.ones(1, n, n, device="cuda")
    mask[:, first_masked:, :] = 0
    mask[:, :, first_masked:] = 0
    return mask


@pytest.mark.parametrize("ending", [False, True])
def test_c2_triangle_attention_n512_last_tenth_masked(ending):
    n, first_masked = 512, 461
    cls = (layers.TriangleAttentionEndingNode, oracle.TriangleAttentionEndingNode) if ending else \
        (layers.TriangleAttention, oracle.TriangleAttention)
    mod, ref = seeded(*cls, 128, 32, 4, seed=2024 + ending)
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(512)).cuda()
    mask = tail_masked(n, first_masked)
    with torch.inference_mode():
        expected = ref(x, mask, chunk_size=32)
        actual = mod(x, mask, chunk_size=32)
    info = assert_close(actual.float(), expected, atol=BF16_ATOL, rtol=BF16_ULP, rel_l2=REL_L2)
    record_parity(f"C2 TriangleAttention{'EndingNode' if ending else ''} N=512 tokens>=461 masked", info)


@pytest.mark.parametrize("op", ["outgoing", "incoming", "transition"])
def test_c3_n768(op):
    n = 768
    if op == "transition":
        mod, ref = seeded(layers.Transition, oracle.Transition, 128, 512, seed=768)
    elif op == "incoming":
        mod, ref = seeded(layers.TriangleMultiplicationIncoming, oracle.TriangleMultiplicationIncoming, 128,
                          seed=769)
    else:
        mod, ref = seeded(layers.TriangleMultiplicationOutgoing, oracle.TriangleMultiplicationOutgoing, 128,
                          seed=770)
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(7680)).cuda()
    mask = torch.ones(1, n, n, device="cuda")
    with torch.inference_mode():
        if op == "transition":
            expected, actual = ref(x), mod(x)
        else:
            expected, actual = ref(x, mask), mod(x, mask)
    info = assert_close(actual.float(), expected, atol=BF16_ATOL, rtol=BF16_ULP, rel_l2=REL_L2)
    record_parity(f"C3 {op} N=768", info)


def _bench_block():
    """The bench's block: oracle.randomize draws N(0, 1/128) (unit-mean norm weights) in
    named-parameter order from one seeded generator, as bench.py's seeded_block does."""
    ref = oracle.randomize(oracle.PairformerLayer(), std=STD, generator=torch.Generator().manual_seed(1234))
    mod = layers.PairformerLayer()
    mod.load_state_dict(ref.state_dict())
    return mod.cuda().eval(), ref.cuda().eval()


def test_block_n512_per_op_then_chained():
    """One Pairformer block at N = 512 (the metric's workload).

    First every op is checked alone on the same input (the oracle's chained z), each within
    the per-op bound; then the chained block.  The chained z takes five bf16 updates, each
    within its per-op bound, so its bound is the sum of the five (0.1 absolute with one
    bf16 ulp relative) plus relative L2 <= 1e-2; s (the fp32 single track) is checked the
    same way with the attention bias from that z."""
    n = 512
    mod, ref = _bench_block()
    g = torch.Generator().manual_seed(1000)
    s = torch.randn(1, n, 384, generator=g).cuda()
    z = torch.randn(1, n, n, 128, generator=g).cuda()
    mask = torch.ones(1, n, device="cuda")
    pmask = torch.ones(1, n, n, device="cuda")
    with torch.inference_mode():
        zc = z.clone()
        for name in ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end", "transition_z"):
            op_ref, op = getattr(ref, name), getattr(mod, name)
            if name == "transition_z":
                expected, actual = op_ref(zc), op(zc)
            else:
                expected, actual = op_ref(zc, pmask), op(zc, pmask)
            info = assert_close(actual.float(), expected, atol=BF16_ATOL, rtol=BF16_ULP, rel_l2=REL_L2)
            record_parity(f"block N=512 {name} (shared input)", info)
            zc = zc + expected
        s_expected, z_expected = ref(s, z.clone(), mask, pmask)
        s_actual, z_actual = mod(s, z.clone(), mask, pmask)
    info_z = assert_close(z_actual, z_expected, atol=5 * BF16_ATOL, rtol=BF16_ULP, rel_l2=REL_L2)
    record_parity("block N=512 chained z", info_z)
    info_s = assert_close(s_actual, s_expected, atol=5 * BF16_ATOL, rtol=BF16_ULP, rel_l2=REL_L2)
    record_parity("block N=512 chained s", info_s)


def test_block_n512_single_track_shared_input():
    """The fp32 single track alone on the oracle's z and s: AttentionPairBias (pair bias from
    LN(z)) and transition_s, fp32 contract 1e-4 on O(1) outputs, relative L2 <= 1e-4."""
    n = 512
    mod, ref = _bench_block()
    g = torch.Generator().manual_seed(1001)
    s = torch.randn(1, n, 384, generator=g).cuda()
    z = torch.randn(1, n, n, 128, generator=g).cuda()
    mask = torch.ones(1, n, device="cuda")
    with torch.inference_mode():
        sn = torch.nn.functional.layer_norm(s, (384,), ref.pre_norm_s.weight, ref.pre_norm_s.bias, 1e-5)
        expected = ref.attention(sn, z, mask, sn)
        actual = mod.attention(sn, z, mask, sn)
        info = assert_close(actual, expected, atol=1e-3, rel_l2=1e-4)
        record_parity("block N=512 attention_pair_bias (shared input)", info)
        expected = ref.transition_s(s, bf16=False)
        actual = mod.transition_s(s)
        info = assert_close(actual, expected, atol=1e-3, rel_l2=1e-4)
        record_parity("block N=512 transition_s (shared input)", info)
