"""CUDA-graph replay of a repeated step (boltz_lumi_b200.graphs) on B200.

The step is a small diffusion token transformer built from this package's
layers (AdaLN, bias-consuming AttentionPairBias, ConditionedTransitionBlock),
called like the score model: new activations every call, the same
conditioning, bias and mask.  Replayed results must equal eager ones.
"""

import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu

from boltz_lumi_b200 import adapters, forwards, graphs, layers


class _TokenTransformer(nn.Module):
    def __init__(self, depth=3, c=256, heads=8):
        super().__init__()
        self.heads = heads
        self.adaln = nn.ModuleList([layers.AdaLN(c, c) for _ in range(depth)])
        self.attention = nn.ModuleList([layers.AttentionPairBias(c, num_heads=heads, compute_pair_bias=False)
                                        for _ in range(depth)])
        self.transition = nn.ModuleList([layers.ConditionedTransitionBlock(c, c) for _ in range(depth)])

    def forward(self, a, s, bias, mask):
        n = a.shape[1]
        bias = bias.view(bias.shape[0], n, n, len(self.attention), self.heads)
        for i, (norm, att, tr) in enumerate(zip(self.adaln, self.attention, self.transition)):
            b = norm(a, s)
            a = a + att(b, bias[:, :, :, i], mask, b)
            a = a + tr(a, s)
        return a


def _inputs(n, depth=3, heads=8, c=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    s = torch.randn(1, n, c, generator=g).cuda()
    bias = forwards.prepare_token_bias(torch.randn(1, n, n, depth * heads, generator=g).cuda())
    mask = torch.ones(1, n).cuda()
    mask[:, -2:] = 0
    return s, bias, mask


def _model():
    torch.manual_seed(0)
    return _TokenTransformer().cuda().eval()


def test_replay_equals_eager():
    model = _model()
    s, bias, mask = _inputs(40)
    step = graphs.GraphedStep(model)
    g = torch.Generator().manual_seed(1)
    with torch.inference_mode():
        for _ in range(6):
            a = torch.randn(1, 40, 256, generator=g).cuda()
            out = step(a, s, bias, mask)
            ref = model(a, s, bias, mask)
            assert (out - ref).abs().max().item() <= 1e-5
    assert step.stats == dict(eager=1, captures=1, replays=5)


def test_changed_constant_or_shape_recaptures():
    model = _model()
    s, bias, mask = _inputs(40)
    step = graphs.GraphedStep(model)
    g = torch.Generator().manual_seed(2)
    with torch.inference_mode():
        for _ in range(3):
            step(torch.randn(1, 40, 256, generator=g).cuda(), s, bias, mask)
        mask2 = mask.clone()
        mask2[:, :5] = 0  # a different constant tensor: eager, then a new capture
        a = torch.randn(1, 40, 256, generator=g).cuda()
        out = step(a, s, bias, mask2)
        assert (out - model(a, s, bias, mask2)).abs().max().item() <= 1e-5
        out = step(a, s, bias, mask2)
        assert (out - model(a, s, bias, mask2)).abs().max().item() <= 1e-5
        assert step.stats["eager"] == 2 and step.stats["captures"] == 2
        s3, bias3, mask3 = _inputs(24, seed=3)  # a new shape: its own signature
        a3 = torch.randn(1, 24, 256, generator=g).cuda()
        out = step(a3, s3, bias3, mask3)
        assert out.shape == (1, 24, 256) and step.stats["eager"] == 3


class _AtomDiffusion(nn.Module):
    def __init__(self):
        super().__init__()
        self.score_model = _model()
        self.seen = []

    def sample(self, a, diffusion_conditioning=None, steps=5):
        s, mask = diffusion_conditioning["s"], diffusion_conditioning["mask"]
        bias = diffusion_conditioning["token_trans_bias"]
        for i in range(steps):
            self.seen.append(type(self.score_model.forward).__name__)
            a = 0.5 * self.score_model(a, s, bias, mask) + 0.01 * i
        return a


def test_install_with_cuda_graphs():
    model = nn.Module()
    model.structure_module = _AtomDiffusion()
    model = model.cuda().eval()
    s, bias, mask = _inputs(40)
    cond = {"s": s, "mask": mask, "token_trans_bias": bias.contiguous()}
    a = torch.randn(1, 40, 256, generator=torch.Generator().manual_seed(5)).cuda()
    with torch.inference_mode():
        adapters.install(model)
        ref = model.structure_module.sample(a, diffusion_conditioning=cond)
        adapters.uninstall(model)
        adapters.install(model, cuda_graphs=True)
        out = model.structure_module.sample(a, diffusion_conditioning=cond)
        adapters.uninstall(model)
    assert model.structure_module.seen[-5:] == ["GraphedStep"] * 5
    assert "forward" not in model.structure_module.score_model.__dict__
    assert (out - ref).abs().max().item() <= 1e-5
