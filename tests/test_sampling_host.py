"""Diffusion samples and inputs spread over ranks (boltz_lumi_b200/sampling.py), on CPU.

The partition deals (input, sample) units round robin over the ranks, seeds every sample
from (seed, input, sample) and gathers the coordinates with one all_gather.  These tests
check, with a small pure-torch denoiser on CPU tensors, that every unit runs exactly once
and that the gathered coordinates equal the single-process run for every world size:
thread-emulated ranks and real gloo ranks (world size 2).
"""

import os
import socket
import threading

import pytest
import torch
import torch.multiprocessing as mp

from boltz_lumi_b200.sampling import EDMSampler, distributed_sample, sample_seed, shard_units
from boltz_lumi_b200.sharded import SingleComm, ThreadComm, TorchComm

ATOMS = 7
STEPS = 6


def _denoise(x, sigma):
    """A smooth stand-in score model: shrink towards a fixed shape."""
    target = torch.linspace(-1, 1, x.shape[1] * 3).view(1, x.shape[1], 3)
    w = (sigma / (sigma + 4.0))[:, None, None]
    return w * 0.5 * x + (1 - w) * target


def _run_samples(input_index, samples, gens):
    x = EDMSampler(steps=STEPS).sample(_denoise, ATOMS, gens, "cpu")
    return x + input_index  # inputs differ


@pytest.mark.parametrize("n_inputs,mult,world", [(1, 5, 2), (3, 5, 4), (2, 3, 8), (4, 1, 3)])
def test_units_are_dealt_exactly_once(n_inputs, mult, world):
    seen = []
    for rank in range(world):
        for i, samples in shard_units(n_inputs, mult, world, rank).items():
            assert samples == sorted(samples)
            seen += [(i, m) for m in samples]
    assert sorted(seen) == [(i, m) for i in range(n_inputs) for m in range(mult)]


def test_seeds_differ_per_unit():
    seeds = {sample_seed(5, i, m) for i in range(4) for m in range(8)}
    assert len(seeds) == 32 and all(0 <= s < 2 ** 63 for s in seeds)


def _reference(n_inputs, mult):
    return distributed_sample(_run_samples, n_inputs, mult, ATOMS, 11, SingleComm(), "cpu")


@pytest.mark.parametrize("world", [2, 3])
def test_threads_equal_single_process(world):
    n_inputs, mult = 2, 5
    expected = _reference(n_inputs, mult)
    comms = ThreadComm.group(world)
    results, errors = [None] * world, []

    def worker(r):
        try:
            results[r] = distributed_sample(_run_samples, n_inputs, mult, ATOMS, 11, comms[r], "cpu")
        except Exception as exc:
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    assert not errors, errors
    for out in results:
        assert torch.equal(out, expected)
    # samples differ from one another (independent noise)
    assert (expected[0, 0] - expected[0, 1]).abs().max() > 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = distributed_sample(_run_samples, 2, 5, ATOMS, 11, TorchComm(), "cpu")
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_gloo_world2_equals_single_process():
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_gloo_rank, args=(2, port, results), nprocs=2, start_method="spawn", join=True)
    expected = _reference(2, 5)
    assert torch.equal(results[0], expected) and torch.equal(results[1], expected)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_one_input_per_rank_runs_as_one_batch(world):
    """With as many inputs as ranks, rank r owns exactly input r's samples (one batch)."""
    for rank in range(world):
        assert shard_units(world, 5, world, rank) == {rank: [0, 1, 2, 3, 4]}


def test_fewer_inputs_than_ranks_spread_samples():
    owned = [shard_units(1, 5, 8, r) for r in range(8)]
    assert sum(len(o.get(0, [])) for o in owned) == 5
    assert max(len(o.get(0, [])) for o in owned) == 1
