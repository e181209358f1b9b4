"""The expert-parallel exchange driven from one process, one context per GPU (inzg_ep_connect_local) -- the wiring a C
engine that owns all its GPUs uses -- and experts loaded from device memory (inzg_pool_add_layer_device).

Outputs must equal inzg_moe_forward over the whole batch on one GPU bit for bit."""
import numpy as np
import pytest
import torch

from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


def _reference(n, bias):
    x = synth.hidden(n, H)
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E)
    with MoePool(H, FF, E, K, max_tokens=n, n_layers=1, device=0) as one:
        one.set_router(0, synth.router(0, E, H))
        one.add_layer(0, synth.T_Q4L, blobs, bb)
        y = one.moe_block(0, x, bias=bias)
    return x, blobs, bb, y


def test_pool_from_device_blobs_equals_pool_from_host_blobs():
    """The same blobs loaded from device memory give the same layer outputs as when loaded from host memory."""
    n = 20
    bias = np.zeros(E, np.float32)
    bias[[7, 300]] = 9.0  # two experts take every token: both numeric paths run
    x, blobs, bb, y_host = _reference(n, bias)
    dev = torch.device("cuda", 0)
    with MoePool(H, FF, E, K, max_tokens=n, n_layers=1, device=0) as pool:
        pool.set_router(0, synth.router(0, E, H))
        bd = torch.from_numpy(blobs).to(dev)
        pool.add_layer_device(0, synth.T_Q4L, bd.data_ptr(), bb, 0, E)
        y_dev = pool.moe_block(0, x, bias=bias)
        # a blob whose header is damaged is refused before anything is re-laid out
        bd[3 * bb] ^= 0xFF
        with pytest.raises(Exception, match="corrupt"):
            pool.add_layer_device(0, synth.T_Q4L, bd.data_ptr(), bb, 0, E)
    assert np.array_equal(y_dev.view(np.uint32), y_host.view(np.uint32))


def _run_local(world, n_total, steps=2):
    bias = np.zeros(E, np.float32)
    bias[[3, 200, 300, 511]] = 9.0
    x, blobs, bb, y_one = _reference(n_total, bias)
    per = n_total // world
    pools, xs, ys, bds = [], [], [], []
    try:
        for g in range(world):
            dev = torch.device("cuda", g)
            e0, nl = g * (E // world), E // world
            pool = MoePool(H, FF, E, K, max_tokens=n_total, n_layers=1, device=g)
            pools.append(pool)
            pool.set_router(0, synth.router(0, E, H))
            pool.add_layer_range(0, synth.T_Q4L, blobs[e0 * bb:(e0 + nl) * bb], bb, e0, nl)
            pool.ep_attach(g, world, per)
            xs.append(torch.from_numpy(x[g * per:(g + 1) * per].copy()).to(dev))
            ys.append(torch.empty_like(xs[-1]))
            bds.append(torch.from_numpy(bias).to(dev))
        MoePool.ep_connect_local(pools)
        outs = []
        for _ in range(steps):
            # one host thread enqueues every rank's step; the ranks meet on the devices (epoch flags)
            for g in range(world):
                pools[g].ep_forward_device(0, per, xs[g].data_ptr(), ys[g].data_ptr(), n_total, bds[g].data_ptr())
            for g in range(world):
                pools[g].device_status()
            outs.append(np.concatenate([y.cpu().numpy() for y in ys]))
    finally:
        for p in pools:
            p.close()
    return outs, y_one


def test_ep_connect_local_single_rank():
    outs, y_one = _run_local(1, 20)
    for y in outs:
        assert np.array_equal(y.view(np.uint32), y_one.view(np.uint32))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_connect_local_two_gpus_equals_single_gpu():
    outs, y_one = _run_local(2, 48)
    for y in outs:
        assert np.array_equal(y.view(np.uint32), y_one.view(np.uint32))
