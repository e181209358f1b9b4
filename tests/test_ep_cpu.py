"""Expert-parallel exchange logic on CPU: 2, 4 and 8 gloo ranks (the scaling run's sizes) against one process.

The backend is a deterministic stand-in for the GPU kernels (routing from a fixed projection, an expert that scales
its rows by the expert id): the test checks that the dispatch, the local expert indices, the return of every
(token, rank-k) result and the rank-order combine reproduce the single-process layer exactly. The real kernels' EP
parity is tests/test_gpu_ep.py.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferenz_b200.ep import ExpertParallelMoE

E, K, H = 32, 4, 16


class FakeBackend:
    def __init__(self, rank, e_per):
        self.e_first = rank * e_per
        g = torch.Generator().manual_seed(7)
        self.P = torch.randn((H, E), generator=g)

    def route(self, layer, x, bias=None):
        # row by row: a matmul over the whole batch is not bitwise batch-invariant on the CPU
        logits = torch.stack([(x[r:r + 1] @ self.P)[0] for r in range(x.shape[0])]) if x.shape[0] else x.new_zeros((0, E))
        p = torch.softmax(logits, dim=1)
        w, sel = torch.topk(p, K, dim=1)
        return sel.to(torch.int32), (w / w.sum(1, keepdim=True)).to(torch.float32)

    def experts(self, layer, x, sel, w, n_batch):
        out = torch.full((x.shape[0], K, H), float("nan"))
        for r in range(x.shape[0]):
            for k in range(K):
                if sel[r, k] >= 0:
                    e = int(sel[r, k]) + self.e_first
                    out[r, k] = w[r, k] * (x[r] * (e + 1) + n_batch)
        return out

    def combine(self, slots):
        y = torch.zeros((slots.shape[0], H))
        for k in range(K):
            y = y + slots[:, k]
        return y


def reference(x):
    be = FakeBackend(0, E)
    sel, w = be.route(0, x)
    return be.combine(be.experts(0, x, sel, w, x.shape[0]))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, counts, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(11)
        x_all = torch.randn((sum(counts), H), generator=g)
        lo = sum(counts[:rank])
        x = x_all[lo:lo + counts[rank]]
        ep = ExpertParallelMoE(FakeBackend(rank, E // world), E, K, H)
        y = ep.moe_block(0, x)
        yf = ep.moe_block_fixed(0, x, n_batch=sum(counts), capacity=max(counts))
        q.put((rank, y.numpy(), yf.numpy(), ep.last["dispatch_rows"], ep.last["results"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,counts", [(2, [5, 7]), (2, [1, 0]), (4, [3, 1, 4, 2]),
                                          (8, [4, 0, 2, 5, 1, 3, 0, 6])])
def test_ep_exchange_matches_single_process(world, counts):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, counts, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(11)
    x_all = torch.randn((sum(counts), H), generator=g)
    want = reference(x_all).numpy()
    total_results = 0
    for rank, y, yf, _, nres in sorted(res, key=lambda r: r[0]):
        lo = sum(counts[:rank])
        assert np.array_equal(y.view(np.uint32), want[lo:lo + counts[rank]].view(np.uint32))
        assert np.array_equal(yf.view(np.uint32), want[lo:lo + counts[rank]].view(np.uint32))
        total_results += nres
    assert total_results == sum(counts) * K  # every (token, rank-k) result came home exactly once


def _dead_peer_worker(rank, world, port, q):
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:  # leaves before its side of the exchange: no collective posted, the process exits
        q.put((rank, "left", 0.0))
        return
    x = torch.randn((3, H), generator=torch.Generator().manual_seed(1))
    ep = ExpertParallelMoE(FakeBackend(rank, E // world), E, K, H)
    t0 = time.time()
    try:
        ep.moe_block(0, x)
        q.put((rank, "no error", time.time() - t0))
    except Exception as e:  # the exchange reports the missing peer instead of waiting for it
        q.put((rank, type(e).__name__, time.time() - t0))


def test_ep_peer_that_never_posts_fails_instead_of_hanging():
    """A rank that leaves before the dispatch exchange: the other rank's exchange ends with an error (the peer's
    closed connection, at the latest the process group's 5 s timeout), not a hang -- the host-side detection of a
    lost rank between steps."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(2)])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1][1] == "left"
    assert res[0][1] != "no error" and res[0][2] < 60.0, res[0]
