"""Multi-rank host logic on CPU (gloo, world size 2): row partition, padded all-gather and reassembly, and a missing
rank ending in an error instead of a hang. The local GEMV of each rank is the oracle's (no GPU here)."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from comp_b200.dist import assemble, partition, slice_rows
from oracle import ref


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _sharded_worker(rank, world, port, fmt, n, k, m, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        W, x = ref.problem(fmt, n, k, m, seed=3)
        wq, ws = ref.split(fmt, W, n, k)
        xq, xd = ref.quantize(fmt, x)  # every rank quantizes the replicated activations itself
        row0, rows = partition(n, world)[rank]
        per = slice_rows(n, world)
        part = torch.zeros((m, per), dtype=torch.float64)
        if rows:
            r, _ = ref.gemv(fmt, wq[row0 : row0 + rows], ws[row0 : row0 + rows], xq, xd, k)
            part[:, :rows] = torch.from_numpy(r)
        gathered = torch.empty((world * m, per), dtype=torch.float64)
        dist.all_gather_into_tensor(gathered, part)
        y = assemble(gathered, world, m, per, n).numpy()
        full, _ = ref.gemv(fmt, wq, ws, xq, xd, k)
        q.put((rank, bool(np.array_equal(y.view(np.uint64), full.view(np.uint64)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt,n,k,m", [("q4_0", 37, 416, 3), ("tq2_0", 130, 768, 1), ("q4_0", 5, 96, 2)])
def test_row_sharded_allgather_reassembles_the_full_output(fmt, n, k, m):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, _port_shared[0], fmt, n, k, m, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
    _port_shared[0] = _port()


_port_shared = [_port()]


def _missing_rank_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        q.put((rank, "left"))  # this rank leaves between steps, before the exchange
        return
    t = torch.zeros(4)
    out = torch.empty(8)
    try:
        dist.all_gather_into_tensor(out, t)
        q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001 -- the point is that the survivor gets an error, not a hang
        q.put((rank, f"error: {type(e).__name__}"))


def test_missing_rank_ends_in_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_missing_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]


def _host_buffer_checks_worker(rank, world, port, q):
    """RowShardedGemv's host-buffer form refuses, on every rank and before any collective or launch, an output that is
    not a pinned CPU tensor of the full shape and a host x that is not pinned (the CPU here has no pinned memory)."""
    from comp_b200.dist import RowShardedGemv

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        n, k = 37, 416
        row0, rows = partition(n, world)[rank]
        wq = torch.zeros((rows, k // 2), dtype=torch.uint8)
        ws = torch.zeros((rows, k // 32), dtype=torch.int16)
        layer = RowShardedGemv("q4_0", wq, ws, n, k, exchange="nccl")
        x = torch.zeros((2, k), dtype=torch.float32)
        verdicts = []
        for out in (torch.zeros((2, n)), torch.zeros((2, n - 1)), torch.zeros((2, n), dtype=torch.float64)):
            try:
                layer(x, out=out)
                verdicts.append("accepted")
            except ValueError as e:
                verdicts.append("refused" if "pinned" in str(e) else f"other: {e}")
        try:
            layer(x)  # a host x must be pinned: refused in the staging step
            verdicts.append("accepted")
        except ValueError as e:
            verdicts.append("refused" if "pinned" in str(e) else f"other: {e}")
        q.put((rank, verdicts))
    finally:
        dist.destroy_process_group()


def test_row_sharded_host_buffers_refused_before_any_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_host_buffer_checks_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res == {0: ["refused"] * 4, 1: ["refused"] * 4}
