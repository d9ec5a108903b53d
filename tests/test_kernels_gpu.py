"""Parity of the memory-bound kernels and the tcgen05 GEMM against the CPU oracle.

Case lists follow the reference tests: tails, unaligned offsets, strided masks,
non-default streams (tests/test_pair_transition.py:34-78,
tests/test_triangle_softmax.py:14-47).  Tolerances are written per test.
"""

import pytest
import torch

from conftest import assert_close
from oracle import numerics
from oracle.modules import ordered_bias_softmax

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from boltz_lumi_b200 import kernels

BF16_ULP = 2.0 ** -8  # half-ulp-safe relative bound for one bf16 rounding difference


def gen(seed):
    return torch.Generator().manual_seed(seed)


# ---------------------------------------------------------------------------
# LayerNorm
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("cols", [128, 384, 768, 100])
@pytest.mark.parametrize("in_dtype,out_dtype", [(torch.float32, torch.bfloat16), (torch.float32, torch.float32),
                                                (torch.bfloat16, torch.bfloat16)])
def test_layer_norm_rows(cols, in_dtype, out_dtype):
    g = gen(1)
    x = (torch.randn(1000, cols, generator=g) * 3 + 0.5).to(in_dtype)
    w = torch.randn(cols, generator=g) * 0.1 + 1
    b = torch.randn(cols, generator=g) * 0.1
    expected = torch.nn.functional.layer_norm(x.float(), (cols,), w, b, 1e-5)
    actual = kernels.layer_norm(x.cuda(), w.cuda(), b.cuda(), 1e-5, out_dtype=out_dtype)
    if out_dtype == torch.float32:
        assert_close(actual, expected, atol=1e-5)
    else:
        assert_close(actual.float(), numerics.bf16_round(expected), atol=1e-6, rtol=2 * BF16_ULP)


@pytest.mark.parametrize("rows,heads", [(1, 16), (1001, 16), (4096, 4), (37, 1)])
def test_pair_bias(rows, heads):
    """bl_pair_bias = LayerNorm(z) . W^T in fp32, written head-major [heads][rows]."""
    from boltz_lumi_b200 import _lib

    g = gen(7)
    z = torch.randn(rows, 128, generator=g) * 2 + 0.3
    w_ln, b_ln = torch.randn(128, generator=g) * 0.1 + 1, torch.randn(128, generator=g) * 0.1
    w = torch.randn(heads, 128, generator=g) * 128 ** -0.5
    expected = (torch.nn.functional.layer_norm(z.double(), (128,), w_ln.double(), b_ln.double(), 1e-5)
                @ w.double().T).T.float()
    out = torch.empty(heads, rows, device="cuda")
    zc, wc, w_lnc, b_lnc = z.cuda(), w.cuda(), w_ln.cuda(), b_ln.cuda()  # referenced until the call returns
    _lib.call("bl_pair_bias", zc.data_ptr(), rows, w_lnc.data_ptr(), b_lnc.data_ptr(), 1e-5,
              wc.data_ptr(), heads, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert_close(out.cpu(), expected, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("m", [1, 17, 1000, 4099])
def test_norm_channel_first(m):
    g = gen(2)
    x = torch.randn(128, m, generator=g) * 2
    w = torch.randn(128, generator=g) * 0.08 + 1
    b = torch.randn(128, generator=g) * 0.08
    expected = torch.nn.functional.layer_norm(x.t(), (128,), w, b, 1e-5)
    actual = kernels.norm(x.cuda(), w.cuda(), b.cuda(), 1e-5, channel_first=True, bf16_output=False)
    assert_close(actual, expected, atol=1e-5)
    actual = kernels.norm(x.bfloat16().cuda(), w.cuda(), b.cuda(), 1e-5, channel_first=True, bf16_output=True)
    expected = torch.nn.functional.layer_norm(x.bfloat16().float().t(), (128,), w, b, 1e-5)
    assert_close(actual.float(), numerics.bf16_round(expected), atol=1e-6, rtol=2 * BF16_ULP)


def test_norm_without_affine_and_empty():
    x = torch.randn(5, 768, generator=gen(3))
    actual = kernels.layer_norm(x.cuda(), None, None, 1e-5, out_dtype=torch.float32)
    assert_close(actual, torch.nn.functional.layer_norm(x, (768,), eps=1e-5), atol=1e-5)
    empty = kernels.layer_norm(torch.empty(0, 128, device="cuda"), None, None, 1e-5)
    assert empty.shape == (0, 128)


# ---------------------------------------------------------------------------
# Gates, SiLU-mul
# ---------------------------------------------------------------------------
SIZES = (0, 1, 17, 257, 512, 513, 117 * 512, 312 * 512)


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("offset", (0, 1))
def test_silu_mul(size, offset):
    g = gen(81)
    a = (torch.randn(size + 2, generator=g) * 20).bfloat16()
    b = torch.randn(size + 2, generator=g).bfloat16()
    a_s, b_s = a[offset:offset + size], b[offset:offset + size]
    expected = numerics.bf16_round(numerics.silu_bf16(a_s.float()) * b_s.float())
    actual = kernels.silu_mul(a.cuda()[offset:offset + size], b.cuda()[offset:offset + size])
    assert_close(actual.float(), expected, atol=1e-30, rtol=2 * BF16_ULP)


def test_silu_mul_nondefault_stream():
    g = gen(82)
    a = torch.randn(513, generator=g).bfloat16()
    b = torch.randn(513, generator=g).bfloat16()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        actual = kernels.silu_mul(a.cuda(), b.cuda())
    stream.synchronize()
    expected = numerics.bf16_round(numerics.silu_bf16(a.float()) * b.float())
    assert_close(actual.float(), expected, atol=1e-30, rtol=2 * BF16_ULP)


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("offset", (0, 1))
def test_gate(size, offset):
    g = gen(83)
    p = (torch.randn(size + 2, generator=g) * 3).bfloat16()
    q = (torch.randn(size + 2, generator=g) * 4).bfloat16()
    expected = numerics.bf16_round(p[offset:offset + size].float() * numerics.sigmoid_bf16(q[offset:offset + size].float()))
    actual = kernels.gate(p.cuda()[offset:offset + size], q.cuda()[offset:offset + size])
    assert_close(actual.float(), expected, atol=1e-30, rtol=2 * BF16_ULP)


def _gated_halves(p, g, mask):
    x = numerics.bf16_round(p.float() * numerics.sigmoid_bf16(g.float()))
    x = numerics.bf16_round(x * mask.float().unsqueeze(-1))
    return x[..., :128], x[..., 128:]


@pytest.mark.parametrize("n", [7, 33, 117])
@pytest.mark.parametrize("joint", [False, True])
@pytest.mark.parametrize("mask_kind", ["ones", "partial", "fractional"])
def test_pack_and_split(n, joint, mask_kind):
    g = gen(84)
    width = 512 if joint else 256
    p = torch.randn(1, n, n, width, generator=g).bfloat16()
    q = torch.randn(1, n, n, width, generator=g).bfloat16()
    mask = torch.ones(1, n, n)
    if mask_kind == "partial":
        mask[:, -2:, :] = 0
    if mask_kind == "fractional":
        mask = torch.rand(1, n, n, generator=g)
    pv, qv = p[..., :256], q[..., :256]
    a, b = _gated_halves(pv, qv, mask)
    pc, qc, mc = p.cuda()[..., :256], q.cuda()[..., :256], mask.cuda()
    for outgoing in (True, False):
        left, right = kernels.pack(pc, qc, mc, outgoing)
        a0, b0 = a[0], b[0]  # [n, n, 128]
        if outgoing:
            exp_left = a0.permute(2, 0, 1)  # left[c][i][k] = a[i][k][c]
            exp_right = b0.permute(2, 1, 0)  # right[c][k][j] = b[j][k][c]
        else:
            exp_left = a0.permute(2, 1, 0)  # left[c][i][k] = a[k][i][c]
            exp_right = b0.permute(2, 0, 1)  # right[c][k][j] = b[k][j][c]
        assert_close(left.float(), exp_left, atol=1e-30, rtol=2 * BF16_ULP)
        assert_close(right.float(), exp_right, atol=1e-30, rtol=2 * BF16_ULP)
    sa, sb = kernels.split(pc, qc, mc)
    assert_close(sa.float(), a, atol=1e-30, rtol=2 * BF16_ULP)
    assert_close(sb.float(), b, atol=1e-30, rtol=2 * BF16_ULP)


# ---------------------------------------------------------------------------
# fp32 diffusion epilogues (1e-4 fp32 contract)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rows,cols", [(1, 4), (37, 768), (5, 3), (384, 128)])
def test_diffusion_epilogues(rows, cols):
    g = gen(85)
    a = torch.randn(rows, cols, generator=g) * 3
    b = torch.randn(rows, cols, generator=g) * 3
    c = torch.randn(rows, cols, generator=g)
    wide = torch.randn(rows, 2 * cols, generator=g) * 3
    ac, bc, cc, wc = a.cuda(), b.cuda(), c.cuda(), wide.cuda()
    assert_close(kernels.epilogue(ac, bc, cc, kernels.MODULATION), torch.sigmoid(b) * a + c, atol=1e-5)
    assert_close(kernels.epilogue(ac, bc, None, kernels.GATE), torch.sigmoid(a) * b, atol=1e-5)
    swiglu = torch.nn.functional.silu(wide[:, cols:]) * wide[:, :cols] * b
    assert_close(kernels.epilogue(wc, bc, None, kernels.GATED_SWIGLU), swiglu, atol=1e-4)


@pytest.mark.parametrize("rows,cols", [(3, 128), (384, 768), (50, 1536)])
def test_adaln_modulate(rows, cols):
    g = gen(86)
    a = torch.randn(rows, cols, generator=g) * 2 + 1
    scale = torch.randn(rows, cols, generator=g)
    shift = torch.randn(rows, cols, generator=g)
    expected = torch.sigmoid(scale) * torch.nn.functional.layer_norm(a, (cols,), eps=1e-5) + shift
    actual = kernels.adaln_modulate(a.cuda(), scale.cuda(), shift.cuda(), 1e-5)
    assert_close(actual, expected, atol=1e-4)


# ---------------------------------------------------------------------------
# Ordered bias softmax (tests/test_triangle_softmax.py case list)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [117, 129, 257, 312, 513, 576, 1023, 1024, 1134, 1734, 2511])
def test_ordered_softmax(dtype, n):
    if n > 1024 and dtype != torch.bfloat16:
        pytest.skip("the reference runs fp32 scores up to 1024 only (test_triangle_softmax.py:29-30)")
    g = gen(46)
    scores = (torch.randn(1, 3, 4, n, n, generator=g) * 5).to(dtype)
    bias = (torch.randn(1, 1, 4, n, n, generator=g) * 2).to(dtype)
    mask = torch.zeros(1, n, 1, 1, 3).transpose(1, 4)
    mask[:, :, :, :, -3:] = -1e9
    mask[:, 1] = -1e9
    expected = ordered_bias_softmax(scores.float(), mask, bias.float(), bf16=dtype == torch.bfloat16)
    actual = kernels.ordered_softmax(scores.cuda(), bias.cuda(), mask.cuda())
    atol = 4e-3 if dtype == torch.bfloat16 else 1e-5
    assert_close(actual.float(), expected, atol=atol)


# ---------------------------------------------------------------------------
# tcgen05 batched GEMM
# ---------------------------------------------------------------------------
def _view(t, mn_major):
    """Return a [B, R, K] view that is R-contiguous when mn_major."""
    if not mn_major:
        return t.contiguous()
    return t.transpose(1, 2).contiguous().transpose(1, 2)


@pytest.mark.parametrize("batch,m,n,k", [(1, 128, 128, 64), (2, 256, 512, 192), (3, 200, 136, 72),
                                         (4, 117, 120, 120), (1, 1000, 256, 128), (2, 64, 384, 512)])
@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
def test_batched_gemm(batch, m, n, k, a_mn, b_mn):
    g = gen(87)
    a = torch.randn(batch, m, k, generator=g).bfloat16()
    b = torch.randn(batch, n, k, generator=g).bfloat16()
    bias = torch.randn(n, generator=g) if (m + n) % 2 == 0 else None
    expected = a.float() @ b.float().transpose(1, 2)
    if bias is not None:
        expected = expected + bias
    expected = numerics.bf16_round(expected)
    av, bv = _view(a.cuda(), a_mn), _view(b.cuda(), b_mn)
    if (a_mn and m % 8) or (b_mn and n % 8):
        pytest.skip("MN-major operands need a row stride that is a multiple of 8 elements")
    actual = kernels.bmm(av, bv, bias=None if bias is None else bias.cuda())
    # fp32 accumulation-order differences can flip one bf16 rounding.
    assert_close(actual.float(), expected, atol=1e-3 * k ** 0.5, rtol=2 * BF16_ULP)


# ---------------------------------------------------------------------------
# tcgen05 linear with fused epilogues (residual add into fp32 z, gate pair)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("m", [1, 127, 1000, 4096 + 64])
@pytest.mark.parametrize("gate", [False, True])
@pytest.mark.parametrize("residual", [False, True])
def test_linear_fused(m, gate, residual):
    from boltz_lumi_b200._lib import call

    g = gen(88)
    k1, k = (128, 256) if gate else (512, 512)
    n = 256 if gate else 128
    a = torch.randn(m, k1, generator=g).bfloat16()
    a2 = torch.randn(m, k - k1, generator=g).bfloat16() if gate else None
    w = (torch.randn(n, k, generator=g) / k ** 0.5).bfloat16()
    bias = None if gate else torch.randn(n, generator=g)
    full = a.float() if a2 is None else torch.cat([a.float(), a2.float()], 1)
    acc = full @ w.float().t()
    if gate:
        y = numerics.bf16_round(numerics.bf16_round(acc[:, :128]) * numerics.sigmoid_bf16(acc[:, 128:]))
    else:
        y = numerics.bf16_round(acc + bias)
    z0 = torch.randn(m, 128, generator=g)
    ac, wc = a.cuda(), w.cuda()
    a2c = a2.cuda() if a2 is not None else None
    bc = bias.cuda() if bias is not None else None
    zc = z0.cuda() if residual else None
    out = None if residual else torch.empty(m, 128, device="cuda", dtype=torch.bfloat16)
    call("bl_linear_fused", ac.data_ptr(), k1, None if a2c is None else a2c.data_ptr(), k - k1, k1, wc.data_ptr(), k,
         m, n, k, None if bc is None else bc.data_ptr(), int(gate), None if zc is None else zc.data_ptr(), 128,
         None if out is None else out.data_ptr(), 128, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    # The gate composes three bf16 roundings (p, sigmoid, product): allow two ulps.
    rtol = 4 * BF16_ULP if gate else 2 * BF16_ULP
    if residual:
        assert_close(zc.cpu() - z0, y, atol=1e-5, rtol=rtol)
    else:
        assert_close(out.float(), y, atol=1e-5, rtol=rtol)


# ---------------------------------------------------------------------------
# Kernels against the committed golden vectors (reference test expressions)
# ---------------------------------------------------------------------------
def _golden():
    from pathlib import Path

    return torch.load(Path(__file__).resolve().parent / "golden" / "kernel_expressions.pt")


def test_golden_ordered_softmax():
    for case in _golden()["ordered_softmax"]:
        bf16 = case["scores"].dtype == torch.bfloat16
        got = kernels.ordered_softmax(case["scores"].cuda(), case["bias"].cuda(), case["mask"].cuda())
        assert_close(got.float(), case["expected"].float(), atol=4e-3 if bf16 else 1e-5)


def test_golden_silu_and_gate():
    for case in _golden()["silu"]:
        got = kernels.silu_mul(case["a"].cuda(), case["b"].cuda())
        assert_close(got.float(), case["expected"].float(), atol=1e-30, rtol=2 * BF16_ULP)
    case = _golden()["gate"]
    got = kernels.gate(case["p"].cuda(), case["g"].cuda())
    assert_close(got.float(), case["expected"].float(), atol=1e-30, rtol=2 * BF16_ULP)


def test_golden_diffusion_epilogues():
    case = _golden()["epilogue"]
    a, b, c, wide = (case[k].cuda() for k in ("a", "b", "c", "wide"))
    assert_close(kernels.epilogue(a, b, c, kernels.MODULATION), case["modulation"], atol=1e-5)
    assert_close(kernels.epilogue(a, b, None, kernels.GATE), case["gate"], atol=1e-5)
    assert_close(kernels.epilogue(wide, b, None, kernels.GATED_SWIGLU), case["swiglu"], atol=1e-4)
