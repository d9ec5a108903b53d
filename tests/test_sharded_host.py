"""Row-sharding layout and collectives of the sharded Pairformer (CPU).

The sharded block (boltz_lumi_b200/sharded.py) moves the pair tensor between
row and column ownership with one all_to_all, gathers plane / bias row
blocks with all_gather, and regroups the triangle-multiplication planes by
channel with all_to_all.  These tests check that plumbing on CPU tensors: with
the thread-emulated group and with real gloo ranks (world size 2), against
the single-process transpose / concatenation / einsum it must equal (the
per-channel GEMM is replaced by torch.bmm on the same strided views).
"""

import os
import socket
import threading

import pytest
import torch
import torch.multiprocessing as mp

from boltz_lumi_b200 import sharded
from boltz_lumi_b200.sharded import ThreadComm, TorchComm, _gather_rows, rows_to_columns


def _run_threads(world, fn):
    comms = ThreadComm.group(world)
    results, errors = [None] * world, []

    def worker(r):
        try:
            results[r] = fn(comms[r])
        except Exception as exc:  # surfaced below
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    assert not errors, errors
    return results


@pytest.mark.parametrize("world,n_loc", [(2, 3), (4, 2), (1, 5)])
def test_rows_to_columns_threads(world, n_loc):
    n, c = world * n_loc, 3
    x = torch.randn(n, n, c, generator=torch.Generator().manual_seed(world))

    def rank_fn(comm):
        r0 = comm.rank * n_loc
        cols = rows_to_columns(x[r0:r0 + n_loc].clone(), comm)
        back = rows_to_columns(cols.clone(), comm)
        return cols, back

    for r, (cols, back) in enumerate(_run_threads(world, rank_fn)):
        r0 = r * n_loc
        assert torch.equal(cols, x.transpose(0, 1)[r0:r0 + n_loc])  # rows of x^T = columns of x
        assert torch.equal(back, x[r0:r0 + n_loc])


def test_gather_rows_threads():
    world, n_loc = 3, 2
    full = torch.randn(4, world * n_loc, 5, generator=torch.Generator().manual_seed(9))

    def rank_fn(comm):
        r0 = comm.rank * n_loc
        return _gather_rows(full[:, r0:r0 + n_loc].contiguous(), comm)

    for out in _run_threads(world, rank_fn):
        assert torch.equal(out, full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, n_loc, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = TorchComm()
        n = world * n_loc
        x = torch.arange(n * n * 2, dtype=torch.float32).view(n, n, 2)
        r0 = rank * n_loc
        cols = rows_to_columns(x[r0:r0 + n_loc].clone(), comm)
        ok_cols = torch.equal(cols, x.transpose(0, 1)[r0:r0 + n_loc])
        ok_back = torch.equal(rows_to_columns(cols, comm), x[r0:r0 + n_loc])
        planes = torch.randn(4, n, 7, generator=torch.Generator().manual_seed(3))
        ok_gather = torch.equal(_gather_rows(planes[:, r0:r0 + n_loc].contiguous(), comm), planes)
        results[rank] = (ok_cols, ok_back, ok_gather)
    finally:
        dist.destroy_process_group()


def test_rows_to_columns_gloo_world2():
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_gloo_rank, args=(2, port, 3, results), nprocs=2, start_method="spawn", join=True)
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}


def _bmm_plane_gemm(a, a_mn, b, b_mn, out, m, n, k, stream):
    """The CPU stand-in for bl_batched_gemm on strided plane views."""
    a_mk = (a.transpose(1, 2) if a_mn else a)[:, :m, :k].float()
    b_nk = (b.transpose(1, 2) if b_mn else b)[:, :n, :k].float()
    out[:, :m, :n] = torch.bmm(a_mk, b_nk.transpose(1, 2)).to(out.dtype)


@pytest.mark.parametrize("world,incoming", [(1, True), (2, False), (2, True), (4, True), (8, False), (8, True)])
def test_channel_products_threads(world, incoming, monkeypatch):
    """Channel-sharded per-channel products equal the unsharded einsum on every rank's rows:
    outgoing O_c[i, j] = sum_k a[i, k] b[j, k], incoming O_c[i, j] = sum_k a[k, i] b[k, j]."""
    monkeypatch.setattr(sharded, "_plane_gemm", _bmm_plane_gemm)
    n_loc = 3
    n, n_pad = world * n_loc, world * n_loc + 5
    g = torch.Generator().manual_seed(world + 10 * incoming)
    # small integers: every product and sum is exact in bf16 / fp32
    a = torch.randint(-2, 3, (128, n, n_pad), generator=g).to(torch.bfloat16)
    b = torch.randint(-2, 3, (128, n, n_pad), generator=g).to(torch.bfloat16)
    af, bf = a[:, :, :n].float(), b[:, :, :n].float()
    expected = torch.einsum("cki,ckj->cij", af, bf) if incoming else torch.einsum("cik,cjk->cij", af, bf)

    def rank_fn(comm):
        rows = slice(comm.rank * n_loc, (comm.rank + 1) * n_loc)
        return sharded._channel_products(a[:, rows].contiguous(), b[:, rows].contiguous(), n, comm, incoming, None)

    for r, prod in enumerate(_run_threads(world, rank_fn)):
        assert prod.shape == (128, n_loc, n_pad)
        assert torch.equal(prod[:, :, :n].float(), expected[:, r * n_loc:(r + 1) * n_loc]), r
