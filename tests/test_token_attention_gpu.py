"""Diffusion token-transformer AttentionPairBias on B200 against torch fp32.

The reference computes this attention unfused in fp32 with autocast off
(pair_bias.py:15-36, prepared_forward): einsum -> / sqrt(d) + bias -> + the key
mask term -> softmax -> einsum -> gate -> proj_o.  ``_reference_core`` and
``_reference_forward`` restate exactly that in torch fp32; the fused kernel
(bl_token_attention) must agree within the fp32 bound of 1e-4 absolute.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from boltz_lumi_b200 import adapters, forwards, kernels, layers

TOL = 1e-4  # fp32 mode: per-op max abs error


def _reference_core(q, k, v, bias, mask, inf, multiplicity=1):
    """pair_bias.py:29-34 on [B, N, H, d] fp32 operands and a [B', H, N, N] bias."""
    d = q.shape[-1]
    if multiplicity != 1 or not bias.is_contiguous():
        bias = bias.repeat_interleave(multiplicity, 0)
    attn = torch.einsum("bihd,bjhd->bhij", q.float(), k.float())
    attn = attn / (d ** 0.5) + bias.float()
    if mask is not None:
        attn = attn + (1 - mask[:, None, None].float()) * -inf
    attn = attn.softmax(dim=-1)
    return torch.einsum("bhij,bjhd->bihd", attn, v.float())


def _reference_forward(module, s, z, mask, k_in, multiplicity=1):
    """pair_bias.py:21-36 (prepared_forward) with upstream's proj_z rearrange."""
    b = s.shape[0]
    q = module.proj_q(s).view(b, -1, module.num_heads, module.head_dim)
    k = module.proj_k(k_in).view(b, -1, module.num_heads, module.head_dim)
    v = module.proj_v(k_in).view(b, -1, module.num_heads, module.head_dim)
    bias = z.permute(0, 3, 1, 2)
    gate = module.proj_g(s).sigmoid()
    out = _reference_core(q, k, v, bias, mask, module.inf, multiplicity).reshape(b, -1, module.c_s)
    return module.proj_o(gate * out)


def _mask(batch, n, gen, p_zero=0.2):
    m = (torch.rand(batch, n, generator=gen) > p_zero).float()
    m[:, 0] = 1.0
    return m.cuda()


# (2, 128, 16, 48) and (1, 65, 2, 64) run the two-CTA key split, (1, 256, 16, 48)
# and (1, 230, 8, 24) the four-CTA split (small grids), the rest one CTA per query tile.
@pytest.mark.parametrize("batch,n,heads,d", [(1, 17, 16, 48), (2, 128, 16, 48), (1, 300, 16, 24),
                                             (3, 64, 4, 32), (1, 65, 2, 64), (1, 1, 16, 48),
                                             (1, 256, 16, 48), (1, 230, 8, 24)])
def test_core_matches_torch(batch, n, heads, d):
    gen = torch.Generator().manual_seed(n * 7 + d)
    q, k, v, g = (torch.randn(batch, n, heads, d, generator=gen).cuda() for _ in range(4))
    bias = torch.randn(batch, heads, n, n, generator=gen).cuda() * 2
    mask = _mask(batch, n, gen)
    with torch.inference_mode():
        out = kernels.token_attention(q, k, v, bias, mask, 1e6, gate=g)
        ref = torch.sigmoid(g) * _reference_core(q, k, v, bias, mask, 1e6)
        plain = kernels.token_attention(q, k, v, bias, None, 1e6)
        ref_plain = _reference_core(q, k, v, bias, None, 1e6)
    torch.cuda.synchronize()
    assert (out - ref).abs().max().item() <= TOL
    assert (plain - ref_plain).abs().max().item() <= TOL


def test_layer_slice_of_prepared_bias_and_multiplicity():
    """A layer's [B, H, N, N] slice of the dense [B, N, N, L*H] token bias, shared
    by `multiplicity` samples, read in place (no repeat_interleave copy)."""
    gen = torch.Generator().manual_seed(5)
    layers_, heads, d, n, mult = 3, 16, 48, 96, 3
    raw = torch.randn(1, n, n, layers_ * heads, generator=gen).cuda()
    prepared = forwards.prepare_token_bias(raw)
    assert torch.equal(prepared, raw)
    q, k, v = (torch.randn(mult, n, heads, d, generator=gen).cuda() for _ in range(3))
    mask = _mask(mult, n, gen)
    for layer in range(layers_):
        bias = prepared.view(1, n, n, layers_, heads)[:, :, :, layer].permute(0, 3, 1, 2)
        assert bias.stride(-1) == 1  # dense rows after preparation
        with torch.inference_mode():
            out = kernels.token_attention(q, k, v, bias, mask, 1e6)
            ref = _reference_core(q, k, v, bias, mask, 1e6, multiplicity=mult)
        assert (out - ref).abs().max().item() <= TOL
    # An unprepared bias (head stride 1, key stride L*H) gives the same values.
    bias_raw = raw.view(1, n, n, layers_, heads)[:, :, :, 1].permute(0, 3, 1, 2)
    bias_dense = prepared.view(1, n, n, layers_, heads)[:, :, :, 1].permute(0, 3, 1, 2)
    with torch.inference_mode():
        a = kernels.token_attention(q, k, v, bias_raw, mask, 1e6)
        b = kernels.token_attention(q, k, v, bias_dense, mask, 1e6)
    assert torch.equal(a, b)


def test_fully_masked_sample_and_large_logits():
    """All keys masked gives upstream's finite -inf term (uniform over the biased
    scores); large biases stay finite through the online softmax."""
    gen = torch.Generator().manual_seed(8)
    batch, n, heads, d = 2, 130, 16, 48
    q, k, v = (torch.randn(batch, n, heads, d, generator=gen).cuda() for _ in range(3))
    bias = (torch.randn(batch, heads, n, n, generator=gen) * 30).cuda()
    mask = torch.ones(batch, n).cuda()
    mask[1] = 0.0
    with torch.inference_mode():
        out = kernels.token_attention(q, k, v, bias, mask, 1e6)
        ref = _reference_core(q, k, v, bias, mask, 1e6)
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() <= TOL


def test_empty_and_invalid():
    q = torch.empty(1, 0, 16, 48, device="cuda")
    bias = torch.empty(1, 16, 0, 0, device="cuda")
    assert kernels.token_attention(q, q, q, bias, None, 1e6).shape == (1, 0, 16, 48)
    q = torch.randn(1, 8, 4, 40, device="cuda")  # head_dim 40 is not covered
    with pytest.raises(RuntimeError, match="head_dim"):
        kernels.token_attention(q, q, q, torch.zeros(1, 4, 8, 8, device="cuda"), None, 1e6)
    q = torch.randn(2, 8, 4, 32, device="cuda")
    with pytest.raises(RuntimeError, match="bias"):
        kernels.token_attention(q, q, q, torch.zeros(3, 4, 8, 8, device="cuda"), None, 1e6)


@pytest.mark.parametrize("n,mult,same_keys", [(40, 1, True), (200, 2, True), (64, 1, False)])
def test_module_forward_matches_reference(n, mult, same_keys):
    torch.manual_seed(n)
    module = layers.AttentionPairBias(768, num_heads=16, compute_pair_bias=False).cuda().eval()
    gen = torch.Generator().manual_seed(n + 1)
    s = torch.randn(mult, n, 768, generator=gen).cuda()
    k_in = s if same_keys else torch.randn(mult, n, 768, generator=gen).cuda()
    z = forwards.prepare_token_bias(torch.randn(1, n, n, 2 * 16, generator=gen).cuda())
    z = z.view(1, n, n, 2, 16)[:, :, :, 1]
    mask = _mask(mult, n, gen)
    with torch.inference_mode():
        out = module(s, z, mask, k_in, multiplicity=mult)
        ref = _reference_forward(module, s, z, mask, k_in, multiplicity=mult)
    assert out.shape == ref.shape == (mult, n, 768)
    assert (out - ref).abs().max().item() <= TOL


class _UpstreamAttentionPairBias(layers.AttentionPairBias):
    """Stand-in whose class forward is upstream's eager math (the fallback)."""

    def forward(self, s, z, mask, k_in, multiplicity=1):
        return _reference_forward(self, s, z, mask, k_in, multiplicity)


AttentionPairBias = type("AttentionPairBias", (_UpstreamAttentionPairBias,), {})


class _AtomDiffusion(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.score_model = torch.nn.Module()
        self.score_model.token_transformer = torch.nn.Module()
        self.score_model.token_transformer.layers = torch.nn.ModuleList(
            [AttentionPairBias(768, num_heads=16, compute_pair_bias=False) for _ in range(2)])

    def sample(self, s, mask, diffusion_conditioning=None, multiplicity=1):
        bias = diffusion_conditioning["token_trans_bias"]
        n = bias.shape[1]
        bias = bias.view(bias.shape[0], n, n, 2, 16)
        for i, layer in enumerate(self.score_model.token_transformer.layers):
            s = s + layer(s, bias[:, :, :, i], mask, s, multiplicity)
        return s


def test_installed_model_matches_upstream():
    """install() rebinds the token transformer and wraps sample(); the result
    equals the upstream forwards on the unprepared bias within fp32 tolerance."""
    torch.manual_seed(3)
    model = torch.nn.Module()
    model.structure_module = _AtomDiffusion()
    model = model.cuda().eval()
    gen = torch.Generator().manual_seed(4)
    n, mult = 70, 2
    s = torch.randn(mult, n, 768, generator=gen).cuda()
    mask = _mask(mult, n, gen)
    cond = {"token_trans_bias": torch.randn(1, n, n, 32, generator=gen).cuda()}
    with torch.inference_mode():
        ref = model.structure_module.sample(s, mask, diffusion_conditioning=cond, multiplicity=mult)
        assert adapters.install(model) == 2
        out = model.structure_module.sample(s, mask, diffusion_conditioning=cond, multiplicity=mult)
    adapters.uninstall(model)
    assert "sample" not in model.structure_module.__dict__
    assert (out - ref).abs().max().item() <= 2 * TOL


@pytest.mark.parametrize("n,r0,nq,heads,d", [(256, 64, 64, 16, 24), (512, 128, 128, 16, 24), (200, 0, 100, 8, 48),
                                             (130, 65, 65, 4, 32)])
def test_query_rows_subset(n, r0, nq, heads, d):
    """n_q < n: the queries r0 .. r0 + n_q (q / g pointers and bias rows offset to them) over
    all n keys, as a rank of the row-sharded block runs its own query rows; equal to the
    same rows of the full attention."""
    gen = torch.Generator().manual_seed(n + nq)
    q, k, v, g = (torch.randn(1, n, heads, d, generator=gen).cuda() for _ in range(4))
    bias = torch.randn(1, heads, n, n, generator=gen).cuda()
    mask = _mask(1, n, gen)
    with torch.inference_mode():
        full = kernels.token_attention(q, k, v, bias, mask, 1e6, gate=g)
        bias_rows = bias[:, :, r0:r0 + nq].contiguous()
        out = torch.empty(1, nq, heads, d, device="cuda")
        row = q.stride(1) * 4
        kernels.launch_token_attention(q.data_ptr() + r0 * row, k.data_ptr(), v.data_ptr(), g.data_ptr() + r0 * row,
                                       (q.stride(0), q.stride(1), q.stride(2)), bias_rows, mask, 1e6, 1, heads, n, d,
                                       out, torch.cuda.current_stream().cuda_stream, n_q=nq)
    expected = _reference_core(q, k, v, bias, mask, 1e6)[:, r0:r0 + nq] * torch.sigmoid(g[:, r0:r0 + nq])
    assert (out - expected).abs().max().item() <= TOL
    assert (out - full[:, r0:r0 + nq]).abs().max().item() <= 1e-5
