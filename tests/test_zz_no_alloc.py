"""inzg_route_topk_noalloc -- the allocation-free routing entry point -- against the existing entry point.

Callers that cannot allocate device memory while they run a layer (a fixed device-memory plan, or a decode loop that
must not let cudaMalloc synchronise the device) use inzg_route_topk_noalloc: it keeps its scratch in a static device
array of the library. Its top-k and weights must equal, bit for bit (routing is bit-exact everywhere in this
library), what inzg_moe_forward computes for the same inputs; two calls in a row check that the shared array's
leftover contents never leak into a result. The file sorts last so a failure here comes after every other test.
"""
import ctypes

import numpy as np
import pytest

import oracle
from inferenz_b200 import MoePool, lib, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


def _existing(pool, x, bias):
    pool.moe_block(0, x, bias=bias, dump=True)
    d = pool.route_dump(x.shape[0])
    return d["sel"], d["w"]


def test_noalloc_routing_matches_moe_forward_twice():
    """Token counts that take every router kernel variant: 8 and 5 (one block of tokens), then 1, then the full 64
    (several token blocks filling the whole static array) after the small calls, then 2 and 3 again; each call's
    result must not carry anything the previous call left in the shared array."""
    import torch
    orc = oracle.Oracle()
    R = synth.router(0, E, H)
    xs = [synth.hidden(n, H, seed=31 + i) for i, n in enumerate((8, 5, 1, 64, 2, 3))]
    bias = synth.normal_bias(E)
    used = np.unique(np.concatenate([oracle.routing(orc, R, x, bias=bias).ravel() for x in xs]))
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=used)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with MoePool(H, FF, E, K, max_tokens=64, n_layers=1, device=0) as pool:
        pool.set_router(0, R)
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        want = [_existing(pool, x, bias) for x in xs]
        bd = torch.from_numpy(bias).to(dev)
        got = []
        for x in xs:  # calls in a row on the shared static scratch
            xd = torch.from_numpy(x).to(dev)
            sel = torch.full((x.shape[0], K), -1, dtype=torch.int32, device=dev)
            w = torch.full((x.shape[0], K), -1.0, dtype=torch.float32, device=dev)
            torch.cuda.synchronize(dev)  # inputs ready: the call runs on the context's own stream (NULL)
            st = lib.inzg_route_topk_noalloc(pool._ctx, 0, x.shape[0], xd.data_ptr(), bd.data_ptr(), sel.data_ptr(),
                                             w.data_ptr(), None)
            assert st == 0, lib.inzg_last_error(pool._ctx).decode()
            torch.cuda.synchronize(dev)
            assert torch.cuda.current_device() == 0
            pool.device_status()
            got.append((sel.cpu().numpy(), w.cpu().numpy()))
        # sizes beyond the static array are refused with a clear error, not run
        big = torch.zeros((65, H), dtype=torch.float32, device=dev)
        st = lib.inzg_route_topk_noalloc(pool._ctx, 0, 65, big.data_ptr(), None, sel.data_ptr(), w.data_ptr(), None)
        assert st == 1 and b"64" in lib.inzg_last_error(pool._ctx)
    assert len(got) == len(want) == 6
    for (gs, gw), (ws, ww) in zip(got, want):
        assert np.array_equal(gs, ws)
        assert np.array_equal(gw.view(np.uint32), ww.view(np.uint32))
