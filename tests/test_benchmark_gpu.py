"""The upstream-versus-optimized harness (boltz_lumi_b200.benchmark) on B200.

A stand-in model with upstream's stage names: ``pairformer_module`` runs two
Pairformer blocks' pair updates and ``structure_module.sample`` a few AdaLN /
ConditionedTransitionBlock steps, all built from the oracle's modules
(upstream's class and attribute names, eager semantics).  The upstream recipe
runs them as they are.  The optimized recipe runs them after
``adapters.install``, i.e. on this build's kernels.  The report must have
every call, round, stage timing and per-field error, within the end-to-end
tolerances, and the model must come back uninstalled.
"""

import json

import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu

import oracle
from boltz_lumi_b200 import benchmark


class _Pairformer(nn.Module):
    def __init__(self, blocks, generator):
        super().__init__()
        self.layers = nn.ModuleList(
            [oracle.randomize(oracle.PairformerLayer(), std=0.05, generator=generator) for _ in range(blocks)])

    def forward(self, z, pair_mask):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            for layer in self.layers:
                for op in (layer.tri_mul_out, layer.tri_mul_in):
                    z = z + op(z, pair_mask).float()
                for op in (layer.tri_att_start, layer.tri_att_end):
                    z = z + op(z, mask=pair_mask).float()
                z = z + layer.transition_z(z).float()
        return z


class _Structure(nn.Module):
    def __init__(self, generator):
        super().__init__()
        self.score_model = nn.Module()
        self.score_model.adaln = oracle.randomize(oracle.AdaLN(128, 128), std=0.05, generator=generator)
        self.score_model.transition = oracle.randomize(oracle.ConditionedTransitionBlock(128, 128), std=0.05,
                                                       generator=generator)

    def sample(self, a, s, steps=3):
        for _ in range(steps):
            a = a + self.score_model.transition(self.score_model.adaln(a, s), s)
        return a


class _Model(nn.Module):
    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.pairformer_module = _Pairformer(2, g)
        self.structure_module = _Structure(g)


def _predict_once(model, item):
    z, pair_mask, a, s = item
    with torch.inference_mode():
        z = model.pairformer_module(z.clone(), pair_mask)
        atoms = model.structure_module.sample(a, s)
    return {"coords": atoms[..., :3], "plddt": torch.sigmoid(z.mean(-1)).mean(-1)}


def test_compare_upstream_and_optimized(tmp_path):
    model = _Model().cuda().eval()
    inputs = []
    for name, n in (("a", 48), ("b", 70)):
        g = torch.Generator().manual_seed(n)
        z = torch.randn(1, n, n, 128, generator=g).cuda()
        pair_mask = torch.ones(1, n, n).cuda()
        pair_mask[:, -3:, :] = 0
        a = torch.randn(1, 4 * n, 128, generator=g).cuda()
        s = torch.randn(1, 4 * n, 128, generator=g).cuda()
        inputs.append((name, (z, pair_mask, a, s)))
    report = benchmark.compare(model, _predict_once, inputs, repeats=1, output=tmp_path,
                               settings=dict(case="stand-in"))
    saved = json.loads((tmp_path / "timings.json").read_text())
    assert saved["status"] == report["status"] == "complete", [e for e in report["errors"] if not e.get("within_bound", True)]
    assert len(report["model_calls"]) == 2 * 2 * 2  # recipes x rounds x inputs
    assert [r["recipe"] for r in report["rounds"]] == ["upstream", "upstream", "optimized", "optimized"]
    for call in report["model_calls"]:
        assert set(call["stages_s"]) == {"pairformer_module", "diffusion_sample"}
        assert all(t > 0 for t in call["stages_s"].values())
    optimized = [e for e in report["errors"] if e["recipe"] == "optimized"]
    assert {e["field"] for e in optimized} == {"coords", "plddt"}
    assert any(e["differing_values"] for e in optimized)  # the kernels really ran
    assert report["upstream_warm_mean_s"] > 0 and report["optimized_warm_mean_s"] > 0
    assert "speedup" in report and "optimized_warm_stages_s" in report
    # The model is handed back with the upstream forwards.
    assert not any("forward" in m.__dict__ for m in model.modules())
    assert "sample" not in model.structure_module.__dict__
