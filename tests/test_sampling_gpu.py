"""The sample-parallel diffusion sampler on B200 (boltz_lumi_b200/sampling.py).

* The score model (TokenDiffusionModel: EDM preconditioning around a token transformer of
  this package's AdaLN / AttentionPairBias / ConditionedTransitionBlock kernels) equals an
  fp32 torch restatement built from the oracle's modules with the same weights (fp32
  contract, 1e-4 relative).
* distributed_sample over thread-emulated ranks on one GPU equals the single-process run:
  every sample draws its noise from its own generator, so only the batch composition
  changes, which moves the fp32 GEMM summation order and nothing else.
"""

import math
import threading

import pytest
import torch
import torch.nn.functional as F

import oracle
from conftest import assert_close

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from boltz_lumi_b200 import sampling
    from boltz_lumi_b200.sharded import SingleComm, ThreadComm

DEPTH, C, HEADS, C_S, N = 2, 256, 8, 384, 40


def _model_and_inputs():
    model = sampling.seeded_model(depth=DEPTH, c_token=C, heads=HEADS, c_s=C_S, seed=3)
    s_trunk, bias, mask = sampling.synthetic_conditioning(N, DEPTH, HEADS, C_S, seed=4)
    mask[:, -3:] = 0  # padded tokens
    return model, s_trunk, bias, mask


def _oracle_forward(model, x, sigma, s_trunk, bias, mask):
    sd = model.sigma_data
    var = sigma * sigma + sd * sd
    c_in, c_skip, c_out = var.rsqrt(), sd * sd / var, sigma * sd * var.rsqrt()
    fourier = torch.cos(2 * math.pi * ((torch.log(sigma / sd) * 0.25)[:, None] * model.fourier_w + model.fourier_b))
    s = s_trunk @ model.s_in.weight.t() + (fourier @ model.t_in.weight.t())[:, None, :]
    a = (x * c_in[:, None, None]) @ model.r_in.weight.t() + s
    samples = x.shape[0]
    for l in range(DEPTH):
        ada = oracle.AdaLN(C, C).cuda()
        ada.load_state_dict(model.adaln[l].state_dict())
        att = oracle.AttentionPairBias(C, num_heads=HEADS, inf=1e6, compute_pair_bias=False).cuda()
        att.load_state_dict(model.attention[l].state_dict())
        tr = oracle.ConditionedTransitionBlock(C, C).cuda()
        tr.load_state_dict(model.transition[l].state_dict())
        b = ada(a, s)
        bias_l = bias[..., l * HEADS:(l + 1) * HEADS].permute(0, 3, 1, 2)
        o = att(b, bias_l, mask.expand(samples, -1), b)
        a = a + torch.sigmoid(s @ model.gate[l].weight.t() + model.gate[l].bias) * o
        a = a + tr(a, s)
    an = F.layer_norm(a, (C,), model.out_norm.weight, model.out_norm.bias, model.out_norm.eps)
    return c_skip[:, None, None] * x + c_out[:, None, None] * (an @ model.r_out.weight.t())


def test_score_model_matches_oracle_composition():
    model, s_trunk, bias, mask = _model_and_inputs()
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(3, N, 3, generator=g, device="cuda") * 20
    sigma = torch.tensor([160.0, 16.0, 0.5], device="cuda")
    with torch.inference_mode():
        s_base = model.conditioning(s_trunk)
        actual = model(x, sigma, s_base, bias, mask)
        expected = _oracle_forward(model, x, sigma, s_trunk, bias, mask)
    info = assert_close(actual, expected, atol=1e-3, rtol=1e-4)
    assert info["relative_l2_error"] < 1e-5, info


def _runner(model, s_trunk, bias, mask, steps):
    sampler = sampling.EDMSampler(steps=steps)
    s_base = model.conditioning(s_trunk)

    def run(input_index, samples, gens):
        return sampler.sample(lambda x, sig: model(x, sig, s_base, bias, mask), N, gens, "cuda")

    return run


@pytest.mark.parametrize("world", [2, 3])
def test_thread_ranks_equal_single_process(world):
    model, s_trunk, bias, mask = _model_and_inputs()
    steps, inputs, mult = 8, 2, 3
    with torch.inference_mode():
        run = _runner(model, s_trunk, bias, mask, steps)
        expected = sampling.distributed_sample(run, inputs, mult, N, 5, SingleComm(), "cuda")
        comms = ThreadComm.group(world)
        results, errors = [None] * world, []

        def worker(r):
            try:
                with torch.inference_mode():
                    results[r] = sampling.distributed_sample(run, inputs, mult, N, 5, comms[r], "cuda")
            except Exception as exc:
                errors.append(exc)

        threads = [threading.Thread(target=worker, args=(r,)) for r in range(world)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=300)
    assert not errors, errors
    assert torch.isfinite(expected).all()
    for out in results:
        assert_close(out, expected, atol=1e-3, rtol=1e-4)
    assert (expected[0, 0] - expected[0, 1]).abs().max() > 0.1  # independent samples


def _nccl_rank(rank, world, port, results):
    import datetime
    import os

    import torch.distributed as dist

    from boltz_lumi_b200 import sampling
    from boltz_lumi_b200.sharded import TorchComm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        model = sampling.seeded_model(depth=DEPTH, c_token=C, heads=HEADS, c_s=C_S, seed=3, device=device)
        s_trunk, bias, mask = sampling.synthetic_conditioning(N, DEPTH, HEADS, C_S, seed=4, device=device)
        sampler = sampling.EDMSampler(steps=6)
        with torch.inference_mode():
            s_base = model.conditioning(s_trunk)

            def run(i, samples, gens):
                return sampler.sample(lambda x, sig: model(x, sig, s_base, bias, mask), N, gens, device)

            out = sampling.distributed_sample(run, 2, 3, N, 5, TorchComm(), device)
        results[rank] = out.cpu()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sampler_nccl_two_gpus_equals_one():
    """Two ranks over NCCL (each runs its units, one all_gather) give every rank the same
    coordinates as one process running all units."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_nccl_rank, args=(2, port, results), nprocs=2, start_method="spawn", join=True)
    model, s_trunk, bias, mask = _model_and_inputs()
    mask[:, -3:] = 1  # the ranks above use the unmasked conditioning
    with torch.inference_mode():
        sampler = sampling.EDMSampler(steps=6)
        s_base = model.conditioning(s_trunk)

        def run(i, samples, gens):
            return sampler.sample(lambda x, sig: model(x, sig, s_base, bias, mask), N, gens, "cuda")

        expected = sampling.distributed_sample(run, 2, 3, N, 5, SingleComm(), "cuda").cpu()
    for rank in range(2):
        assert_close(results[rank], expected, atol=1e-3, rtol=1e-4)


def test_graphed_denoiser_equals_eager():
    """make_denoiser(cuda_graphs=True) replays the score model from a CUDA graph from its
    third call on; the sampled coordinates equal the eager denoiser's."""
    model, s_trunk, bias, mask = _model_and_inputs()
    with torch.inference_mode():
        outs = []
        for graphed in (False, True):
            gens = [torch.Generator(device="cuda").manual_seed(10 + m) for m in range(3)]
            denoise = sampling.make_denoiser(model, s_trunk, bias, mask, cuda_graphs=graphed)
            outs.append(sampling.EDMSampler(steps=6).sample(denoise, N, gens, "cuda"))
    assert_close(outs[1], outs[0], atol=1e-4, rtol=1e-5)
