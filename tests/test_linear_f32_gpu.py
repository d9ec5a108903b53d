"""fp32-accurate tensor-core linear (bl_split3_bf16 + bl_linear_split3) on B200.

The three-way bf16 split must reconstruct fp32 to 2^-27 relative, and the
six-product GEMM must match a float64 reference to 2^-17 of the largest
output (a few times an fp32 SGEMM's error: the tensor core's fp32
accumulation of the dominant product is slightly coarser), far inside the
1e-4 bound of the fp32 diffusion ops.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from boltz_lumi_b200 import kernels


def test_split3_reconstructs():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(333, 96, generator=g) * torch.logspace(-6, 6, 96)
    x3 = kernels.split3(x.cuda()).double().cpu()
    assert x3.shape == (3, 333, 96)
    rel = ((x3.sum(0) - x.double()).abs() / x.double().abs().clamp_min(1e-30)).max().item()
    assert rel <= 2.0 ** -26
    assert torch.equal(x3[0].float(), x.bfloat16().float())  # the first plane is bf16(x)


@pytest.mark.parametrize("m,n,k,with_bias", [(117, 3072, 768, True), (40, 768, 768, False), (512, 1536, 384, True),
                                             (1, 4, 8, True), (300, 100, 72, False), (2000, 768, 768, True),
                                             (129, 260, 1536, True), (117, 768, 768, True), (100, 100, 1096, True),
                                             (8, 768, 136, False), (300, 768, 768, True), (256, 3072, 768, False)])
def test_linear_matches_fp64(m, n, k, with_bias):
    g = torch.Generator().manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) * k ** -0.5
    bias = torch.randn(n, generator=g) if with_bias else None
    ref = x.double() @ w.double().T + (bias.double() if with_bias else 0)
    with torch.inference_mode():
        y = kernels.linear_f32(x.cuda(), kernels.split3(w.cuda()), None if bias is None else bias.cuda())
        y_cublas = torch.nn.functional.linear(x.cuda(), w.cuda(), None if bias is None else bias.cuda())
    err = (y.double().cpu() - ref).abs().max().item()
    err_cublas = (y_cublas.double().cpu() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert y.shape == (m, n) and y.dtype == torch.float32
    assert err <= 2.0 ** -17 * scale, (err, err_cublas, scale)


def test_linear_batched_input_and_shared_split():
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 50, 384, generator=g).cuda()
    w1, w2 = (torch.randn(n, 384, generator=g).cuda() * 0.05 for n in (768, 384))
    with torch.inference_mode():
        x3 = kernels.split3(x)
        y1 = kernels.linear_f32(x, kernels.split3(w1), x3=x3)
        y2 = kernels.linear_f32(x, kernels.split3(w2), x3=x3)
    assert y1.shape == (2, 50, 768) and y2.shape == (2, 50, 384)
    for y, w in ((y1, w1), (y2, w2)):
        ref = (x.double() @ w.double().T)
        assert (y.double() - ref).abs().max().item() <= 1e-5


@pytest.mark.parametrize("m,n,k", [(117, 768, 768), (100, 100, 1096), (64, 1536, 768), (300, 768, 768)])
def test_skinny_cluster_split_is_deterministic(m, n, k):
    """m <= 128 with few N tiles splits K over a thread-block cluster and
    reduces the partials in rank order through distributed shared memory:
    repeated calls must agree bitwise."""
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g).cuda()
    w3 = kernels.split3((torch.randn(n, k, generator=g) * k ** -0.5).cuda())
    bias = torch.randn(n, generator=g).cuda()
    with torch.inference_mode():
        ys = [kernels.linear_f32(x, w3, bias) for _ in range(3)]
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    ref = x.double() @ w3.double().sum(0).T + bias.double()
    assert (ys[0].double() - ref).abs().max().item() <= 2.0 ** -17 * ref.abs().max().item()


@pytest.mark.parametrize("rows,cols", [(117, 768), (5, 128), (300, 384)])
def test_fused_split_producers_match_split3(rows, cols):
    """The producers that write split planes directly (LayerNorm, AdaLN
    modulation, diffusion epilogue, token attention) must give exactly
    split3 of their fp32 results."""
    g = torch.Generator().manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=g).cuda()
    w, b = (torch.randn(cols, generator=g).cuda() for _ in range(2))
    sc, sh = (torch.randn(rows, cols, generator=g).cuda() for _ in range(2))
    with torch.inference_mode():
        ln = kernels.layer_norm(x, w, b, 1e-5, out_dtype=torch.float32)
        assert torch.equal(kernels.layer_norm_split3(x, w, b, 1e-5), kernels.split3(ln))
        mod = kernels.adaln_modulate(x, sc, sh, 1e-5)
        assert torch.equal(kernels.adaln_modulate_split3(x, sc, sh, 1e-5), kernels.split3(mod))
        a2 = torch.randn(rows, 2 * cols, generator=g).cuda()
        for kind, args in ((kernels.GATED_SWIGLU, (a2, x, None)), (kernels.GATE, (x, sc, None)),
                           (kernels.MODULATION, (x, sc, sh))):
            ref = kernels.epilogue(*args, kind)
            assert torch.equal(kernels.epilogue_split3(*args, kind), kernels.split3(ref)), kind


def test_token_attention_split_output():
    g = torch.Generator().manual_seed(3)
    b, n, h, d = 2, 70, 16, 48
    q, k, v, gate = (torch.randn(b, n, h, d, generator=g).cuda() for _ in range(4))
    bias = torch.randn(b, h, n, n, generator=g).cuda()
    mask = torch.ones(b, n).cuda()
    with torch.inference_mode():
        out = kernels.token_attention(q, k, v, bias, mask, 1e6, gate=gate)
        out3 = torch.empty(3, b * n, h * d, device="cuda", dtype=torch.bfloat16)
        kernels.launch_token_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), gate.data_ptr(),
                                       q.stride()[:3], bias, mask, 1e6, b, h, n, d, None,
                                       torch.cuda.current_stream().cuda_stream, out3=out3)
    torch.cuda.synchronize()
    assert torch.equal(out3, kernels.split3(out.view(b * n, h * d)))


def test_swiglu_epilogue():
    """SWIGLU (the fp32 transition's silu(fc1) * fc2 on the joint fc1 | fc2
    output) against torch, and its split form against split3."""
    g = torch.Generator().manual_seed(12)
    h = torch.randn(300, 2 * 1536, generator=g).cuda() * 4
    with torch.inference_mode():
        ref = torch.nn.functional.silu(h[:, :1536]) * h[:, 1536:]
        out = kernels.epilogue(h, None, None, kernels.SWIGLU)
        assert (out - ref).abs().max().item() <= 1e-6 * ref.abs().max().item()
        assert torch.equal(kernels.epilogue_split3(h, None, None, kernels.SWIGLU), kernels.split3(out))


@pytest.mark.parametrize("m,n,k", [(117, 768, 768), (512, 384, 1536), (2000, 768, 768), (40, 100, 72)])
def test_linear_with_residual(m, n, k):
    """y = x W^T + bias + residual (the single track's s + proj_o(o) and s + fc3(h)) on both
    the one-CTA tiles and the K-split cluster path; the residual is read, not modified."""
    g = torch.Generator().manual_seed(m * 7 + n)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) * k ** -0.5
    bias = torch.randn(n, generator=g)
    res = torch.randn(m, n, generator=g) * 3
    ref = x.double() @ w.double().T + bias.double() + res.double()
    with torch.inference_mode():
        rc = res.cuda()
        keep = rc.clone()
        y = torch.empty(m, n, device="cuda")
        kernels.linear_split3_fast(kernels.split3(x.cuda()), kernels.split3(w.cuda()), bias.cuda(), y, residual=rc)
    assert torch.equal(rc, keep)
    err = (y.double().cpu() - ref).abs().max().item()
    assert err <= 2.0 ** -17 * ref.abs().max().item() + 1e-6, err
