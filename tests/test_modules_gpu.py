"""Module-level parity of the B200 path against the CPU oracle (upstream semantics).

Case lists follow tests/test_operator_additions.py of the reference (token
counts with tails, masked tokens, zero / ones / partial / fractional masks,
N(0, 0.08) weights with unit-mean norms) at sizes the CPU oracle finishes in
seconds.  Tolerances: per-op max abs error 2e-2 for the bf16 trunk ops,
1e-4 for the fp32 diffusion ops.
"""

import pytest
import torch

import oracle
from conftest import assert_close

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from boltz_lumi_b200 import layers

BF16_ATOL = 2e-2
FP32_ATOL = 1e-4
# Above |y| = 2.56 one bf16 ulp of the output itself exceeds 2e-2, and an
# fp32 accumulation-order difference can flip the output's final rounding:
# large-N cases allow max(2e-2, one bf16 ulp) per element and bound the
# relative L2 error.
BF16_ULP = 2.0 ** -7
BF16_REL_L2 = 1e-2


def build(product_cls, oracle_cls, *args, seed=732991, std=0.08):
    ref = oracle_cls(*args)
    oracle.randomize(ref, std=std, generator=torch.Generator().manual_seed(seed))
    mod = product_cls(*args)
    mod.load_state_dict(ref.state_dict())
    return mod.cuda().eval(), ref.eval()


def pair_mask(n, kind, masked_tokens=3, seed=5):
    mask = torch.ones(1, n, n)
    if kind == "zero":
        mask.zero_()
    elif kind == "partial":
        mask[:, -masked_tokens:, :] = 0
        mask[:, :, -masked_tokens:] = 0
    elif kind == "partial_rows":  # the reference's multiplication case: rows only
        mask[:, -masked_tokens:, :] = 0
    elif kind == "fractional":
        mask = torch.rand(1, n, n, generator=torch.Generator().manual_seed(seed))
    return mask


@pytest.mark.parametrize("ending", [False, True])
@pytest.mark.parametrize("n,kind", [(17, "ones"), (64, "partial"), (117, "ones"), (117, "partial"),
                                    (130, "partial"), (200, "ones")])
def test_triangle_attention(ending, n, kind):
    cls = (layers.TriangleAttentionEndingNode, oracle.TriangleAttentionEndingNode) if ending else \
        (layers.TriangleAttention, oracle.TriangleAttention)
    mod, ref = build(*cls, 128, 32, 4)
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(n))
    mask = pair_mask(n, kind)
    expected = ref(x, mask, chunk_size=32)
    with torch.inference_mode():
        actual = mod(x.cuda(), mask.cuda(), chunk_size=32)
    assert actual.dtype == torch.bfloat16
    assert_close(actual.float(), expected, atol=BF16_ATOL)


@pytest.mark.parametrize("ending", [False, True])
@pytest.mark.parametrize("n,kind,rows", [(312, "ones", None), (312, "partial", None), (576, "ones", None),
                                         (576, "partial", None), (1134, "partial", None), (2511, "partial", 48)])
def test_triangle_attention_reference_sizes(ending, n, kind, rows):
    """The reference's own attention case list (test_operator_additions.py:60-67: N = 312, 576,
    1134, 2511, x * 0.3, the last three tokens masked).  At these sizes the oracle runs on the
    GPU as the checker (same torch restatement, fp32); at N = 2511 it computes the first
    `rows` outer rows (rows attend independently) and the kernel output is compared there.
    Bound: max(2e-2, one bf16 ulp of the expected value) per element, relative L2 <= 1e-2."""
    cls = (layers.TriangleAttentionEndingNode, oracle.TriangleAttentionEndingNode) if ending else \
        (layers.TriangleAttention, oracle.TriangleAttention)
    mod, ref = build(*cls, 128, 32, 4)
    ref = ref.cuda()
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(1, n, n, 128, generator=g) * 0.3).cuda()
    mask = pair_mask(n, kind).cuda()
    with torch.inference_mode():
        expected = ref(x, mask, chunk_size=32, rows=rows)
        actual = mod(x, mask, chunk_size=32)
    if rows is not None:
        actual = actual[:, :, :rows] if ending else actual[:, :rows]
    assert actual.shape == expected.shape
    assert_close(actual.float(), expected, atol=BF16_ATOL, rtol=BF16_ULP, rel_l2=BF16_REL_L2)


@pytest.mark.parametrize("ending", [False, True])
@pytest.mark.parametrize("n,kind", [(200, "partial"), (312, "ones"), (450, "partial"), (576, "ones"),
                                    (1134, "partial")])
def test_triangle_attention_residual(ending, n, kind):
    """z += TriangleAttention(z) through bl_triangle_attention_residual (linear_o and the
    residual add in the attention kernel's epilogue at N >= 385, one more GEMM below):
    bit-identical to z + the module's bf16 output, so the parity of the module output
    carries over.  N = 450 ends in a partial query tile; 200 and 312 take the separate
    GEMM (one and two heads per CTA)."""
    from boltz_lumi_b200 import forwards

    cls = (layers.TriangleAttentionEndingNode, oracle.TriangleAttentionEndingNode) if ending else \
        (layers.TriangleAttention, oracle.TriangleAttention)
    mod, _ = build(*cls, 128, 32, 4)
    g = torch.Generator().manual_seed(n + 1)
    z = (torch.randn(1, n, n, 128, generator=g) * 0.3).cuda()
    mask = pair_mask(n, kind).cuda()
    with torch.inference_mode():
        expected = z + mod(z, mask).float()
        forwards.triangle_attention_forward(mod, z, mask, residual=z)
    assert torch.isfinite(z).all()
    assert torch.equal(z, expected), (z - expected).abs().max().item()


def test_triangle_attention_residual_rejects_strided_slab():
    """Below four heads per CTA the residual entry runs linear_o as a separate GEMM over
    contiguous rows; an ending-node slab (n_outer < n) is refused before any launch and
    z is left untouched."""
    from boltz_lumi_b200 import _lib

    n, n_outer, n8 = 200, 40, 200
    dev = "cuda"
    proj = torch.zeros(n * n, 512, device=dev, dtype=torch.bfloat16)
    bias = torch.zeros(4, n, n8, device=dev, dtype=torch.bfloat16)
    mask = torch.ones(n, n, device=dev)
    w_o = torch.zeros(128, 128, device=dev, dtype=torch.bfloat16)
    b_o = torch.zeros(128, device=dev)
    z = torch.ones(n * n, 128, device=dev)
    scratch = torch.empty(n * n, 128, device=dev, dtype=torch.bfloat16)
    base = proj.data_ptr()
    with pytest.raises(RuntimeError, match="contiguous output rows"):
        _lib.call("bl_triangle_attention_residual", base, base + 256, base + 512, base + 768, 512, 1, n,
                  bias.data_ptr(), n8, n * n8, mask.data_ptr(), 1, n, 1e9, 4, 32, n, n_outer, scratch.data_ptr(), 128,
                  w_o.data_ptr(), b_o.data_ptr(), z.data_ptr(), 128, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(z, torch.ones_like(z))


@pytest.mark.parametrize("ending", [False, True])
@pytest.mark.parametrize("n,kind", [(17, "ones"), (64, "partial"), (130, "partial"), (200, "ones"), (312, "partial")])
def test_triangle_attention_fp32_mode(ending, n, kind):
    """fp32 mode: fp32 input with autocast off (the reference's fast path accepts it,
    triangle.py:47-51).  An upstream-named module (the oracle's class) is rebound by
    adapters.install and called without autocast; the result is fp32 and within the fp32
    contract (1e-4) of upstream's fp32 semantics (the oracle with bf16=False)."""
    import copy

    from torch import nn

    from boltz_lumi_b200 import adapters

    cls = oracle.TriangleAttentionEndingNode if ending else oracle.TriangleAttention
    ref = oracle.randomize(cls(128, 32, 4), std=128 ** -0.5, generator=torch.Generator().manual_seed(n))
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(n + 3))
    mask = pair_mask(n, kind)
    expected = ref(x, mask, chunk_size=32, bf16=False)
    model = nn.Module()
    model.pairformer = nn.Module()
    model.pairformer.tri_att = copy.deepcopy(ref).cuda().eval()
    assert adapters.install(model) == 1
    with torch.inference_mode():
        actual = model.pairformer.tri_att(x.cuda(), mask.cuda(), chunk_size=32)
    assert actual.dtype == torch.float32
    info = assert_close(actual, expected, atol=FP32_ATOL)
    assert info["relative_l2_error"] < 1e-5, info


def test_triangle_attention_fp32_mode_differs_from_bf16_contract():
    """The fp32 path is not the bf16 path in disguise: on the same module and input the
    bf16-autocast result differs from the fp32 one by far more than the fp32 tolerance."""
    from boltz_lumi_b200 import forwards

    mod, ref = build(layers.TriangleAttention, oracle.TriangleAttention, 128, 32, 4, std=128 ** -0.5)
    x = torch.randn(1, 48, 48, 128, generator=torch.Generator().manual_seed(9)).cuda()
    with torch.inference_mode():
        y32 = forwards.triangle_attention_forward_fp32(mod, x)
        y16 = forwards.triangle_attention_forward(mod, x)
    assert (y32 - y16.float()).abs().max().item() > 10 * FP32_ATOL


@pytest.mark.parametrize("incoming", [False, True])
@pytest.mark.parametrize("n", [312, 576])
@pytest.mark.parametrize("kind", ["zero", "ones", "partial", "partial_rows", "fractional"])
def test_triangle_multiplication_reference_sizes(incoming, n, kind):
    """The reference's multiplication cases at N = 312 and 576 (test_operator_additions.py:68,
    112-130: x * 0.3, masks zero / ones / last two rows / uniform; plus rows and columns),
    oracle on the GPU as the checker.  Bound: max(2e-2, one bf16 ulp of the expected value)
    per element, relative L2 <= 1e-2."""
    cls = (layers.TriangleMultiplicationIncoming, oracle.TriangleMultiplicationIncoming) if incoming else \
        (layers.TriangleMultiplicationOutgoing, oracle.TriangleMultiplicationOutgoing)
    mod, ref = build(*cls, 128)
    ref = ref.cuda()
    x = (torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(n + 1)) * 0.3).cuda()
    mask = pair_mask(n, kind, masked_tokens=2).cuda()
    with torch.inference_mode():
        expected = ref(x, mask)
        actual = mod(x, mask)
    assert_close(actual.float(), expected, atol=BF16_ATOL, rtol=BF16_ULP, rel_l2=BF16_REL_L2)


@pytest.mark.parametrize("incoming", [False, True])
@pytest.mark.parametrize("n", [7, 64, 117, 128])
@pytest.mark.parametrize("kind", ["zero", "ones", "partial", "partial_rows", "fractional"])
def test_triangle_multiplication(incoming, n, kind):
    cls = (layers.TriangleMultiplicationIncoming, oracle.TriangleMultiplicationIncoming) if incoming else \
        (layers.TriangleMultiplicationOutgoing, oracle.TriangleMultiplicationOutgoing)
    mod, ref = build(*cls, 128)
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(n + 1))
    mask = pair_mask(n, kind, masked_tokens=2)
    expected = ref(x, mask)
    with torch.inference_mode():
        actual = mod(x.cuda(), mask.cuda())
    assert_close(actual.float(), expected, atol=BF16_ATOL)


@pytest.mark.parametrize("n", [17, 117, 312])
def test_pair_transition(n):
    mod, ref = build(layers.Transition, oracle.Transition, 128, 512, std=0.05)
    x = torch.randn(1, n, n, 128, generator=torch.Generator().manual_seed(n + 2))
    with torch.inference_mode():
        for value in (x, x[:, ::2]):  # dense and strided inputs (test_pair_transition.py:57-61)
            expected = ref(value)
            actual = mod(value.cuda())
            assert expected.abs().max() > 0
            assert_close(actual.float(), expected, atol=BF16_ATOL)


@pytest.mark.parametrize("n", [17, 117, 312, 576])
def test_pair_transition_reference_cases(n):
    """The reference's transition cases (test_pair_transition.py:52-66): x [2, n, 128],
    weights N(0, 0.05), dense and strided (x[:, ::2]) inputs."""
    mod, ref = build(layers.Transition, oracle.Transition, 128, 512, std=0.05, seed=81)
    x = torch.randn(2, n, 128, generator=torch.Generator().manual_seed(81 + n))
    with torch.inference_mode():
        for value in (x, x[:, ::2]):
            expected = ref(value)
            actual = mod(value.cuda())
            assert expected.abs().max() > 0
            assert_close(actual.float(), expected, atol=BF16_ATOL)


@pytest.mark.parametrize("dim,hidden", [(64, 256), (256, 1024), (128, 256)])
def test_pair_transition_other_widths(dim, hidden):
    """Widths other than the trunk's 128 -> 512 -> 128 (the template module's
    pair stack runs c_z = 64 with hidden 256) take the unfused-width path:
    LayerNorm, fc1|fc2 GEMM, SwiGLU, fc3 GEMM on the same kernels."""
    mod, ref = build(layers.Transition, oracle.Transition, dim, hidden, std=0.05)
    x = torch.randn(1, 37, 37, dim, generator=torch.Generator().manual_seed(dim + hidden))
    expected = ref(x)
    with torch.inference_mode():
        actual = mod(x.cuda())
    assert actual.shape == (1, 37, 37, dim)
    assert_close(actual.float(), expected, atol=BF16_ATOL)


@pytest.mark.parametrize("rows", [1, 129, 5000])
def test_pair_transition_residual_in_place(rows):
    """z += Transition(z) with z both the input and the residual (the block's
    in-place update); ragged row counts exercise the last partial tile."""
    from boltz_lumi_b200 import forwards

    mod, ref = build(layers.Transition, oracle.Transition, 128, 512, std=0.05)
    z = torch.randn(rows, 128, generator=torch.Generator().manual_seed(rows))
    expected = z + ref(z)
    with torch.inference_mode():
        zc = z.cuda()
        forwards.transition_forward(mod, zc, residual=zc)
    assert_close(zc.cpu(), expected, atol=BF16_ATOL)


# fp32 diffusion ops: weights ~ N(0, 1/fan_in) keep outputs O(1), where a 1e-4
# absolute bound is meaningful (N(0, 0.08) at width 1536 gives outputs in the tens).
@pytest.mark.parametrize("tokens,dim", [(384, 768), (1000, 128), (5, 768)])
def test_adaln(tokens, dim):
    mod, ref = build(layers.AdaLN, oracle.AdaLN, dim, dim, std=dim ** -0.5)
    a = torch.randn(2, tokens, dim, generator=torch.Generator().manual_seed(1))
    s = torch.randn(2, tokens, dim, generator=torch.Generator().manual_seed(2))
    expected = ref(a, s)
    with torch.inference_mode():
        actual = mod(a.cuda(), s.cuda())
    assert_close(actual, expected, atol=FP32_ATOL)


@pytest.mark.parametrize("tokens,dim", [(384, 768), (300, 128)])
def test_conditioned_transition(tokens, dim):
    mod, ref = build(layers.ConditionedTransitionBlock, oracle.ConditionedTransitionBlock, dim, dim,
                     std=dim ** -0.5)
    a = torch.randn(1, tokens, dim, generator=torch.Generator().manual_seed(3))
    s = torch.randn(1, tokens, dim, generator=torch.Generator().manual_seed(4))
    expected = ref(a, s)
    with torch.inference_mode():
        actual = mod(a.cuda(), s.cuda())
    assert_close(actual, expected, atol=FP32_ATOL)


def test_pairformer_block_c1():
    """Block parity config: one block at N = 64, s ~ N(0,1) [1,64,384], z ~ N(0,1), pair mask ones."""
    n = 64
    mod, ref = build(layers.PairformerLayer, oracle.PairformerLayer, std=1 / 128 ** 0.5)
    g = torch.Generator().manual_seed(11)
    s = torch.randn(1, n, 384, generator=g)
    z = torch.randn(1, n, n, 128, generator=g)
    mask = torch.ones(1, n)
    pmask = torch.ones(1, n, n)
    s_ref, z_ref = ref(s, z.clone(), mask, pmask)
    with torch.inference_mode():
        s_out, z_out = mod(s.cuda(), z.cuda(), mask.cuda(), pmask.cuda())
    # Five bf16 updates accumulate into z; the single track is fp32 on top of z.
    info_z = assert_close(z_out, z_ref, atol=5 * BF16_ATOL)
    info_s = assert_close(s_out, s_ref, atol=5 * BF16_ATOL)
    assert info_z["relative_l2_error"] < 1e-2 and info_s["relative_l2_error"] < 1e-2, (info_z, info_s)


def test_inference_only():
    mod = layers.Transition(128, 512).cuda()
    with pytest.raises(RuntimeError, match="inference-only"):
        mod(torch.randn(1, 4, 4, 128, device="cuda"))
