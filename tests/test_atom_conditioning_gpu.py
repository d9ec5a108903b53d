"""Atom-conditioning cache (the reference's atom_conditioning.py) on B200.

Inside ``atom_conditioning_cache`` the projections of the constant single
conditioning are computed once per sampling call; the sampled result must be
identical (bitwise: the same kernels run on the same inputs) to the uncached
run, and the cache must actually be hit.
"""

import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu

from boltz_lumi_b200 import adapters, atom_conditioning, layers


class _AtomLayer(nn.Module):
    def __init__(self, dim, cond):
        super().__init__()
        self.adaln = layers.AdaLN(dim, cond)
        self.output_projection_linear = nn.Linear(cond, dim)
        self.transition = layers.ConditionedTransitionBlock(dim, cond)

    def forward(self, a, s):
        b = self.adaln(a, s)
        a = a + torch.sigmoid(self.output_projection_linear(s)) * b
        return a + self.transition(a, s)


def _stack(dim, cond, depth):
    t = nn.Module()
    t.diffusion_transformer = nn.Module()
    t.diffusion_transformer.layers = nn.ModuleList([_AtomLayer(dim, cond) for _ in range(depth)])
    return t


class _ScoreModel(nn.Module):
    def __init__(self, dim=128, cond=128, depth=2):
        super().__init__()
        self.atom_attention_encoder = nn.Module()
        self.atom_attention_encoder.atom_encoder = _stack(dim, cond, depth)
        self.atom_attention_decoder = nn.Module()
        self.atom_attention_decoder.atom_decoder = _stack(dim, cond, depth)
        self.token_transformer = nn.Module()

    def step(self, a, s):
        for stack in (self.atom_attention_encoder.atom_encoder, self.atom_attention_decoder.atom_decoder):
            for layer in stack.diffusion_transformer.layers:
                a = layer(a, s)
        return a


class _AtomDiffusion(nn.Module):
    def __init__(self):
        super().__init__()
        self.score_model = _ScoreModel()

    def sample(self, atoms, diffusion_conditioning=None, multiplicity=1, steps=4):
        s = diffusion_conditioning["q"]
        for i in range(steps):
            atoms = 0.5 * self.score_model.step(atoms, s) + 0.1 * i
        return atoms


def _model():
    torch.manual_seed(0)
    model = nn.Module()
    model.structure_module = _AtomDiffusion()
    with torch.no_grad():
        for p in model.parameters():
            p.mul_(0.5)
    return model.cuda().eval()


def test_cached_sampling_equals_uncached():
    model = _model()
    g = torch.Generator().manual_seed(1)
    atoms = torch.randn(1, 96, 128, generator=g).cuda()
    cond = {"q": torch.randn(1, 96, 128, generator=g).cuda(), "c": torch.zeros(1, 96, 128).cuda(),
            "token_trans_bias": torch.zeros(1, 8, 8, 4).cuda()}
    with torch.inference_mode():
        ref = model.structure_module.sample(atoms, diffusion_conditioning=cond)
        adapters.install(model)
        seen = {}
        real = atom_conditioning.atom_conditioning_cache

        def spy(score_model):  # keep the caches for inspection after sample() returns
            ctx = real(score_model)
            seen["owners"] = atom_conditioning._targets(score_model)[1]
            return ctx

        atom_conditioning.atom_conditioning_cache = spy
        try:
            out = model.structure_module.sample(atoms, diffusion_conditioning=cond)
        finally:
            atom_conditioning.atom_conditioning_cache = real
    adapters.uninstall(model)
    assert torch.equal(out, ref)
    assert len(seen["owners"]) == 12  # 4 layers x (layer AdaLN, transition AdaLN, transition)
    for owner in seen["owners"]:
        assert atom_conditioning.CACHE_ATTR not in owner.__dict__  # closed after sampling


def test_cache_hits_inside_context():
    model = _model()
    score = model.structure_module.score_model
    layer = score.atom_attention_encoder.atom_encoder.diffusion_transformer.layers[0]
    g = torch.Generator().manual_seed(2)
    s = torch.randn(1, 40, 128, generator=g).cuda()
    a1, a2 = (torch.randn(1, 40, 128, generator=g).cuda() for _ in range(2))
    with torch.inference_mode():
        plain = [layer.adaln(a, s) for a in (a1, a2)] + [layer.transition(a, s) for a in (a1, a2)]
        with atom_conditioning.atom_conditioning_cache(score):
            gate1 = layer.output_projection_linear(s)
            gate2 = layer.output_projection_linear(s)
            assert gate1 is gate2  # wrapped sub-module: computed once
            cached = [layer.adaln(a, s) for a in (a1, a2)] + [layer.transition(a, s) for a in (a1, a2)]
            cache = layer.adaln.__dict__[atom_conditioning.CACHE_ATTR]
            assert len(cache) == 1  # one (scale, shift) entry for the one conditioning layout
            assert len(layer.transition.__dict__[atom_conditioning.CACHE_ATTR]) == 1
        assert "forward" not in layer.output_projection_linear.__dict__
    for x, y in zip(plain, cached):
        assert torch.equal(x, y)
