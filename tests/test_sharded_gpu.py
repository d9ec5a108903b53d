"""Row-sharded Pairformer block against the single-GPU block (B200).

P virtual ranks run as threads on one GPU (ThreadComm), and, when two GPUs are
visible, two real ranks over NCCL.  Every pair op of the sharded block runs the
same kernels on row slabs (the triangle-multiplication products on channel
slabs) with the same accumulation order per output, so the sharded z must
equal the unsharded one (checked to 1e-6 absolute).  The single
track runs on query-row slabs, where the fp32 tensor-core linears and the
token attention may split their K / key ranges differently than on all rows
(fp32 summation order only): s is checked to 2e-5 absolute on O(1) values.
"""

S_TOL = 2e-5

import os
import socket
import threading

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

import bench  # seeded_block, synthetic_inputs
from boltz_lumi_b200 import layers
from boltz_lumi_b200.sharded import ShardedPairformer, ThreadComm, TorchComm


def _inputs(n, masked_tail):
    s, z, mask, pmask = bench.synthetic_inputs(n, seed=11)
    if masked_tail:
        mask[:, n - masked_tail:] = 0
        pmask[:, n - masked_tail:, :] = 0
        pmask[:, :, n - masked_tail:] = 0
    return s, z, mask, pmask


@pytest.mark.parametrize("world,n,masked_tail", [(2, 128, 0), (4, 128, 9), (2, 192, 5), (8, 128, 3), (4, 256, 7)])
def test_sharded_block_matches_single_gpu_threads(world, n, masked_tail):
    block = bench.seeded_block(layers.PairformerLayer).cuda()
    s, z, mask, pmask = (t.cuda() for t in _inputs(n, masked_tail))
    with torch.inference_mode():
        s_ref, z_ref = block(s.clone(), z.clone(), mask, pmask)
    torch.cuda.synchronize()
    n_loc = n // world
    comms = ThreadComm.group(world)
    results, errors = [None] * world, []

    def worker(r):
        try:
            torch.cuda.set_device(0)
            with torch.inference_mode(), torch.cuda.stream(torch.cuda.Stream()):
                z_rows = z[0, r * n_loc:(r + 1) * n_loc].clone()
                s_r, z_r = ShardedPairformer(block, comms[r])(s.clone(), z_rows, mask, pmask)
                torch.cuda.synchronize()
                results[r] = (s_r, z_r)
        except Exception as exc:
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    for r, (s_r, z_r) in enumerate(results):
        dz = (z_r - z_ref[0, r * n_loc:(r + 1) * n_loc]).abs().max().item()
        ds = (s_r - s_ref).abs().max().item()
        assert dz <= 1e-6 and ds <= S_TOL, (r, dz, ds)


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _nccl_rank(rank, world, port, n, results):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        block = bench.seeded_block(layers.PairformerLayer).to(device)
        s, z, mask, pmask = (t.to(device) for t in _inputs(n, 3))
        n_loc = n // world
        with torch.inference_mode():
            s_ref, z_ref = block(s.clone(), z.clone(), mask, pmask)
            s_r, z_r = ShardedPairformer(block, TorchComm())(s.clone(), z[0, rank * n_loc:(rank + 1) * n_loc].clone(),
                                                            mask, pmask)
        torch.cuda.synchronize()
        results[rank] = ((z_r - z_ref[0, rank * n_loc:(rank + 1) * n_loc]).abs().max().item(),
                         (s_r - s_ref).abs().max().item())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_block_nccl_two_gpus():
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_nccl_rank, args=(2, port, 256, results), nprocs=2, start_method="spawn", join=True)
    for rank in range(2):
        dz, ds = results[rank]
        assert dz <= 1e-6 and ds <= S_TOL, (rank, dz, ds)
