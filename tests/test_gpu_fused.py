"""The fused decode launch (k_fused.cu: the whole routed layer in one persistent kernel for calls of 1-2 tokens)
against the separate-kernel path of the same library (INZG_NO_FUSED) and against the CPU oracle.

Both paths run the reference's arithmetic in the same order, so the fused outputs must be the same bits as the
separate kernels' (routing, logits, probabilities, weights and every output element), and within the north-star
tolerance of the oracle. Calls are repeated through the cached CUDA graph with changing inputs, since the fused
kernel's hand-off counters and barrier are reused from call to call.
"""
import numpy as np
import pytest

import oracle
from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

FF, E, K = 640, 512, 10


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _layer(orc, H, typ, xs, bias=None, ovs=None, layer=0):
    R = synth.router(layer, E, H)
    used = set()
    for i, x in enumerate(xs):
        ov = None if ovs is None else ovs[i]
        used |= set(np.unique(oracle.routing(orc, R, x, bias=bias, override=ov)).tolist())
    blobs, bb = synth.layer_blobs(layer, typ, H, FF, E, experts=sorted(used))
    return R, blobs, bb


def _same(a, b, what):
    for k in ("sel", "units"):
        assert np.array_equal(np.sort(a[k]) if k == "units" else a[k], np.sort(b[k]) if k == "units" else b[k]), \
            f"{what}: {k}"
    for k in ("w", "logits", "probs"):
        assert np.array_equal(_bits(a[k]), _bits(b[k])), f"{what}: {k}"
    assert np.array_equal(_bits(a["y"]), _bits(b["y"])), f"{what}: y differs from the separate-kernel path"


def _call(pool, x, bias=None, ov=None, fused=True, graph=True):
    y = pool.moe_block(0, x, bias=bias, logits_override=ov, dump=True, fused=fused, graph=graph)
    d = pool.route_dump(x.shape[0])
    d["y"] = y
    d["stats"] = pool.stats()
    return d


@pytest.mark.parametrize("H,typ,ns", [(2048, synth.T_Q4L, (1, 2)), (2048, synth.T_Q8G, (1, 2)),
                                      (2560, synth.T_Q4L, (1, 2))])
def test_fused_equals_separate_kernels_and_oracle(orc, H, typ, ns):
    bias = synth.normal_bias(E)
    xs = [synth.hidden(n, H, seed=60 + n) for n in ns]
    R, blobs, bb = _layer(orc, H, typ, xs, bias=bias)
    gu_bytes = int(synth.lib.inzg_qmat_bytes(typ, 2 * FF, H))
    with MoePool(H, FF, E, K, max_tokens=16, n_layers=1, device=0) as pool:
        pool.set_router(0, R)
        pool.add_layer(0, typ, blobs, bb)
        for rep in range(2):  # twice through the cached graphs: counters and barrier carried across calls
            for x in xs:
                a = _call(pool, x, bias=bias)
                assert a["stats"]["last_launches"] == 1, "the call did not take the fused launch"
                b = _call(pool, x, bias=bias, fused=False)
                _same(a, b, f"H={H} type={typ} n={x.shape[0]}")
        c = _call(pool, xs[-1], bias=bias, graph=False)  # direct launch (no graph)
        _same(c, b, "no graph")
    for x in xs[:2]:
        want = orc.moe_routed(R, blobs, bb, gu_bytes, x, bias=bias, H=H, FF=FF, E=E)
        with MoePool(H, FF, E, K, max_tokens=16, n_layers=1, device=0) as pool:
            pool.set_router(0, R)
            pool.add_layer(0, typ, blobs, bb)
            got = _call(pool, x, bias=bias)
        assert np.array_equal(got["sel"], want["sel"]) and np.array_equal(_bits(got["w"]), _bits(want["w"]))
        err = oracle.rel_l2(got["y"], want["y"])
        print(f"fused H={H} type={typ} n={x.shape[0]}: rel_l2 max {err.max():.3e}")
        assert err.max() <= 1e-3


def test_fused_logits_override_host_and_device(orc):
    import torch
    H, n = 2048, 2
    x = synth.hidden(n, H, seed=71)
    ov = synth.normal_logits(n, E, seed=72)
    ov[:, 5] += 4.0
    R, blobs, bb = _layer(orc, H, synth.T_Q4L, [x], ovs=[ov])
    with MoePool(H, FF, E, K, max_tokens=8, n_layers=1, device=0) as pool:
        pool.add_layer(0, synth.T_Q4L, blobs, bb)  # no router: the override replaces it
        a = _call(pool, x, ov=ov)
        b = _call(pool, x, ov=ov, fused=False)
        _same(a, b, "host override")
        dev = torch.device("cuda", 0)
        xd, od = torch.from_numpy(x).to(dev), torch.from_numpy(ov).to(dev)
        yd = torch.empty_like(xd)
        torch.cuda.synchronize(dev)
        pool.moe_block_device(0, n, xd.data_ptr(), yd.data_ptr(), override_ptr=od.data_ptr(), dump=True)
        pool.device_status()
        d = pool.route_dump(n)
        assert np.array_equal(d["sel"], b["sel"]) and np.array_equal(_bits(yd.cpu().numpy()), _bits(b["y"]))


def test_fused_with_shared_expert(orc):
    H, n = 2048, 2
    x = synth.hidden(n, H, seed=81)
    bias = synth.normal_bias(E)
    R, blobs, bb = _layer(orc, H, synth.T_Q4L, [x], bias=bias)
    sh_blob, sh_bb = synth.layer_blobs_range(777, synth.T_Q8G, H, FF, 0, 1)
    gate = synth.randn(91, H, 0.05)
    with MoePool(H, FF, E, K, max_tokens=8, n_layers=1, device=0) as pool:
        pool.set_router(0, R)
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        pool.set_shared(0, synth.T_Q8G, sh_blob, sh_bb, gate)
        a = _call(pool, x, bias=bias)
        b = _call(pool, x, bias=bias, fused=False)
    _same(a, b, "shared expert after the fused launch")
