"""CPU tests of the host-side logic: adapter installation, weight caches,
input validation and the benchmark's multi-rank plumbing (gloo)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp
from torch import nn

from boltz_lumi_b200 import adapters, forwards, layers


class Transition(nn.Module):
    """A stand-in with the upstream class name and attributes."""

    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(8, 64, bias=False)

    def forward(self, x, chunk_size=None):
        return x


class AdaLN(nn.Module):
    def forward(self, a, s):
        return a


class FakeModel(nn.Module):
    def __init__(self):
        super().__init__()
        self.pairformer = nn.Module()
        self.pairformer.transition_z = Transition()
        self.pairformer.transition_s = Transition()
        self.pairformer.tri_att_start = layers.TriangleAttention(128, 32, 4)
        self.pairformer.tri_att_end = layers.TriangleAttentionEndingNode(128, 32, 4)
        self.pairformer.tri_mul_out = layers.TriangleMultiplicationOutgoing(128)
        self.pairformer.tri_mul_in = layers.TriangleMultiplicationIncoming(128)
        self.structure_module = nn.Module()
        self.structure_module.score_model = nn.Module()
        self.structure_module.score_model.adaln = AdaLN()
        self.other_adaln = AdaLN()


def test_install_rebinds_by_class_name_and_path():
    model = FakeModel()
    count = adapters.install(model, require_device=False)
    # 2 attentions + 2 multiplications + transition_z + the score-model AdaLN
    assert count == 6
    assert "forward" in model.pairformer.transition_z.__dict__
    assert "forward" not in model.pairformer.transition_s.__dict__
    assert "forward" in model.structure_module.score_model.adaln.__dict__
    assert "forward" not in model.other_adaln.__dict__
    assert adapters.install(model, require_device=False) == 0  # idempotent
    adapters.uninstall(model)
    assert "forward" not in model.pairformer.transition_z.__dict__
    assert not model._b200_optimized


def test_rebound_forward_falls_back_outside_inference():
    """With grad enabled the upstream (class) forward runs, as in the reference."""
    model = FakeModel()
    adapters.install(model, require_device=False)
    x = torch.randn(1, 2, 2, 8)
    assert model.pairformer.transition_z(x) is x  # the stand-in class forward


def test_install_requires_sm100_device():
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    assert adapters.install(FakeModel()) == 0


def test_weight_cache_invalidation():
    """Derived weights rebuild when a source parameter changes (multiplication.py:29-40)."""
    module = layers.TriangleMultiplicationOutgoing(128)
    first = forwards._multiplication_weights(module)
    again = forwards._multiplication_weights(module)
    assert first is again
    with torch.no_grad():
        module.p_in.weight.add_(0.01)
    new = forwards._multiplication_weights(module)
    assert new is not first
    assert torch.equal(new["w_in"][:256], module.p_in.weight.bfloat16())
    assert torch.equal(new["w_out"][:128, :128], module.p_out.weight.bfloat16())
    assert torch.count_nonzero(new["w_out"][:128, 128:]) == 0


def test_attention_weights_layout():
    module = layers.TriangleAttention(128, 32, 4)
    w = forwards._attention_weights(module)
    assert w["w_in"].shape == (512, 128) and w["w_heads"].shape == (4, 128)
    assert torch.equal(w["w_in"][256:384], module.mha.linear_v.weight.bfloat16())
    assert torch.equal(w["b_in"][384:], module.mha.linear_g.bias)
    assert torch.count_nonzero(w["b_in"][:384]) == 0


def test_pair_input_validation():
    with pytest.raises(RuntimeError, match="CUDA"):
        forwards._check_pair_input(torch.zeros(1, 4, 4, 128), None)
    with pytest.raises(RuntimeError, match="residual"):
        forwards._check_residual(torch.zeros(1, 4, 4, 128, dtype=torch.bfloat16), torch.zeros(1, 4, 4, 128))


def test_layers_are_inference_only():
    mod = layers.Transition(128, 512)
    with pytest.raises(RuntimeError, match="inference-only"):
        mod(torch.zeros(1, 2, 2, 128))


# ---------------------------------------------------------------------------
# Multi-rank plumbing of bench.py on gloo (world size 2)
# ---------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # Each rank "measured" a different time; everyone must report the max.
        results[rank] = bench.max_over_ranks(10.0 + rank, dist, torch.device("cpu"))
    finally:
        dist.destroy_process_group()


def test_bench_max_over_ranks_gloo():
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_rank_main, args=(2, port, results), nprocs=2, start_method="spawn", join=True)
    assert dict(results) == {0: 11.0, 1: 11.0}


def test_bench_reference_arm_rank_nonzero_exits_without_work(monkeypatch):
    import bench

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    ns = type("A", (), dict(steps=1, warmup=0, n=8, impl="reference"))()
    assert bench.run_reference(ns) == 0


class _RecordingDiffusion(nn.Module):
    """AtomDiffusion stand-in: sample() records the conditioning it receives."""

    def __init__(self):
        super().__init__()
        self.score_model = nn.Module()
        self.score_model.token_transformer = nn.Module()
        self.score_model.token_transformer.attention = layers.AttentionPairBias(64, num_heads=4,
                                                                                compute_pair_bias=False)
        self.seen = []

    def sample(self, atom_mask=None, diffusion_conditioning=None, multiplicity=1):
        self.seen.append(diffusion_conditioning["token_trans_bias"])
        return diffusion_conditioning["token_trans_bias"]


def _token_model():
    model = nn.Module()
    model.structure_module = _RecordingDiffusion()
    model.trunk_attention = layers.AttentionPairBias(64, c_z=128, num_heads=4)  # not in the token transformer
    return model


def test_install_rebinds_token_transformer_and_sample():
    model = _token_model()
    assert adapters.install(model, require_device=False) == 1
    structure = model.structure_module
    assert "forward" in structure.score_model.token_transformer.attention.__dict__
    assert "forward" not in model.trunk_attention.__dict__
    assert "sample" in structure.__dict__
    adapters.uninstall(model)
    assert "forward" not in structure.score_model.token_transformer.attention.__dict__
    assert "sample" not in structure.__dict__


def test_sample_wrapper_packs_token_bias_dense():
    """Under inference the bias reaches sample() fp32 with head-major storage and
    unchanged values (the reference's diffusion.py:16-18); with grad enabled
    the original conditioning passes through untouched."""
    model = _token_model().eval()
    adapters.install(model, require_device=False)
    raw = torch.randn(1, 6, 6, 8).to(torch.bfloat16)
    cond = {"token_trans_bias": raw, "c": torch.zeros(1)}
    with torch.inference_mode():
        out = model.structure_module.sample(atom_mask=None, diffusion_conditioning=cond, multiplicity=2)
    assert out.dtype == torch.float32 and torch.equal(out, raw.float())
    assert out.permute(0, 3, 1, 2).is_contiguous()  # layer / head slices are dense [N, N] planes
    assert cond["token_trans_bias"] is raw  # the caller's dict is not modified
    out = model.structure_module.sample(atom_mask=None, diffusion_conditioning=cond)
    assert out is raw


def test_prepared_bias_layer_slices():
    raw = torch.randn(2, 5, 5, 3 * 4)
    prepared = forwards.prepare_token_bias(raw)
    assert torch.equal(prepared, raw)
    layer = prepared.view(2, 5, 5, 3, 4)[:, :, :, 1].permute(0, 3, 1, 2)
    assert layer.stride()[-2:] == (5, 1)


def test_token_attention_forward_rejects_bad_multiplicity():
    module = layers.AttentionPairBias(64, num_heads=4, compute_pair_bias=False).eval()
    s = torch.randn(3, 5, 64)
    z = torch.randn(2, 5, 5, 4)
    with torch.inference_mode(), pytest.raises(RuntimeError, match="multiplicity"):
        forwards.token_attention_forward(module, s, z, torch.ones(3, 5), s, multiplicity=1)


def test_atom_conditioning_context_installs_and_restores():
    from boltz_lumi_b200 import atom_conditioning

    def stack():
        t = nn.Module()
        t.diffusion_transformer = nn.Module()
        layer = nn.Module()
        layer.adaln = layers.AdaLN(16, 16)
        layer.output_projection_linear = nn.Linear(16, 16)
        layer.transition = layers.ConditionedTransitionBlock(16, 16)
        t.diffusion_transformer.layers = nn.ModuleList([layer])
        return t, layer

    score = nn.Module()
    score.atom_attention_encoder = nn.Module()
    score.atom_attention_decoder = nn.Module()
    score.atom_attention_encoder.atom_encoder, enc = stack()
    score.atom_attention_decoder.atom_decoder, dec = stack()
    linear = enc.output_projection_linear
    with atom_conditioning.atom_conditioning_cache(score):
        assert "forward" in linear.__dict__ and "forward" in enc.adaln.s_scale.__dict__
        assert atom_conditioning.CACHE_ATTR in dec.transition.__dict__
        x = torch.randn(2, 16)
        with torch.no_grad():
            assert torch.equal(linear(x), nn.Linear.forward(linear, x))  # CPU input: computed, not cached
    assert "forward" not in linear.__dict__ and "forward" not in enc.adaln.s_scale.__dict__
    assert atom_conditioning.CACHE_ATTR not in dec.transition.__dict__


def test_benchmark_field_errors_and_summary():
    from boltz_lumi_b200 import benchmark

    coords = torch.zeros(1, 5, 3, dtype=torch.float64)
    moved = coords.clone()
    moved[0, 0, 0] = 0.2  # one atom 0.2 A away: RMSD = sqrt(0.04 / 5)
    rec = benchmark.field_error("coords", moved, coords)
    assert abs(rec["rmsd"] - (0.04 / 5) ** 0.5) < 1e-12 and rec["within_bound"]
    far = benchmark.field_error("coords", coords + 1.0, coords)
    assert far["rmsd"] > 0.1 and not far["within_bound"]
    pl = benchmark.field_error("plddt", torch.tensor([0.5, 0.7]), torch.tensor([0.5, 0.705]))
    assert pl["metric"] == "max_abs" and pl["within_bound"] and pl["differing_values"] == 1
    other = benchmark.field_error("ptm", torch.tensor([0.3]), torch.tensor([0.2]))
    assert "within_bound" not in other
    report = {"model_calls": [
        dict(recipe="upstream", first=True, model_s=9.0, stages_s={"pairformer_module": 5.0}),
        dict(recipe="upstream", first=False, model_s=4.0, stages_s={"pairformer_module": 2.0}),
        dict(recipe="optimized", first=True, model_s=3.0, stages_s={}),
        dict(recipe="optimized", first=False, model_s=1.0, stages_s={"pairformer_module": 0.5}),
    ], "errors": [rec, pl, other]}
    benchmark.summarize(report)
    assert report["upstream_warm_mean_s"] == 4.0 and report["optimized_warm_mean_s"] == 1.0
    assert report["saved_s"] == 3.0 and report["speedup"] == 4.0 and report["status"] == "complete"
    assert report["optimized_warm_stages_s"] == {"pairformer_module": 0.5}
    report["errors"].append(far)
    assert benchmark.summarize(report)["status"] == "outside_tolerance"


def test_benchmark_cli_needs_upstream_boltz():
    from boltz_lumi_b200 import benchmark

    try:
        import boltz  # noqa: F401
        pytest.skip("upstream boltz is installed")
    except ImportError:
        pass
    with pytest.raises(SystemExit, match="boltz"):
        benchmark.main(["predict", "input.yaml"])


def test_graph_step_argument_plumbing():
    """GraphedStep's signature and leaf order (CPU: no capture here)."""
    from boltz_lumi_b200 import graphs

    a, b, c = torch.zeros(1), torch.ones(2, 3)[:, :2], torch.full((3,), 2.0)
    obj = ((a, [b]), {"z": b, "a": c, "n": 3, "f": len})
    leaves = []
    key = graphs._flatten(obj, leaves)
    rebuilt = graphs._rebuild(obj, leaves, iter(range(len(leaves))))
    assert rebuilt[0][0] is a and rebuilt[0][1][0] is b and rebuilt[1]["a"] is c and rebuilt[1]["z"] is b
    assert rebuilt[1]["n"] == 3 and rebuilt[1]["f"] is len
    other = []
    assert graphs._flatten(((a, [b.contiguous()]), {"z": b, "a": c, "n": 3, "f": len}), other) != key  # strides
    assert graphs._flatten(((a, [b]), {"z": b, "a": c, "n": 4, "f": len}), []) != key  # a Python value
    same = []
    assert graphs._flatten(((a.clone(), [b]), {"z": b, "a": c, "n": 3, "f": len}), same) == key
