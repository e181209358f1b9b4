"""GPU parity of the hyper-connection steps either side of the layer (hc_in / hc_out, src/model_fwd.c:404-450) and of
q_forward's whole MoE step (hc_in -> layer -> hc_out, :1264-1267) through the C ABI, against the oracle (pinned to the
reference's own functions by tests/test_hc_oracle.py).

Bars: hc_out bit-exact. hc_in bit-exact except where glibc's expf enters (the SiLU of the 320-wide bottleneck and the
inject sigmoid, evaluated on the device in double and rounded once, one ulp apart on ~1e-4 of inputs): xin within
1e-6 relative L2 per token with at least 99% of values bit-identical, inj within 4e-7. The whole step: the layer's
own bar (1e-3 relative L2 per token, north_star) on the updated residual.
"""
import numpy as np
import pytest
import torch

import oracle
from inferenz_b200 import MoePool, synth
from inferenz_b200.ep import stream_handle

pytestmark = pytest.mark.gpu

XIN_TOL, INJ_TOL, LAYER_TOL = 1e-6, 4e-7, 1e-3


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _st():
    return stream_handle(torch.cuda.current_stream())


@pytest.mark.parametrize("H,n", [(2048, 1), (2048, 2), (2048, 5), (2048, 40), (2048, 333), (2560, 1), (2560, 2),
                                 (2560, 70)])
def test_hc_in_matches_oracle(orc, H, n):
    hc = oracle.synth_hc(0, H=H)
    X = oracle.synth_residual(n, H=H, seed=7 + n)
    want_xin, want_inj = orc.hc_in(hc, X)
    with MoePool(H, 640, 512, 10, max_tokens=max(n, 16), n_layers=1, device=0) as pool:
        pool.set_hc(0, hc["norm"], hc["down"], hc["up"], hc["inject"])
        Xd = _dev(X)
        xin = torch.full((n, H), float("nan"), device="cuda")
        inj = torch.full((n, 4), float("nan"), device="cuda")
        for _ in range(2):  # the second call reuses the scratch of the first
            pool.hc_in_device(0, n, Xd.data_ptr(), xin.data_ptr(), inj.data_ptr(), stream=_st())
        pool.device_status(_st())
        got_xin, got_inj = xin.cpu().numpy(), inj.cpu().numpy()
    assert np.array_equal(Xd.cpu().numpy(), X), "hc_in wrote to its input"
    err = oracle.rel_l2(got_xin, want_xin)
    exact = np.mean(got_xin.view(np.uint32) == want_xin.view(np.uint32))
    dinj = np.abs(got_inj - want_inj).max()
    print(f"hc_in H={H} n={n}: xin rel_l2 max {err.max():.2e}, bit-identical {exact:.5f}; inj max diff {dinj:.2e}, "
          f"bit-identical {np.mean(got_inj == want_inj):.4f}")
    assert err.max() <= XIN_TOL and exact >= 0.99
    assert dinj <= INJ_TOL


def test_hc_in_without_inject(orc):
    H, n = 2048, 3
    hc = dict(oracle.synth_hc(2, H=H), inject=None)
    X = oracle.synth_residual(n, H=H, seed=31)
    want_xin, _ = orc.hc_in(hc, X)
    with MoePool(H, 640, 512, 10, max_tokens=16, n_layers=1, device=0) as pool:
        pool.set_hc(0, hc["norm"], hc["down"], hc["up"], None)
        Xd = _dev(X)
        xin = torch.empty((n, H), device="cuda")
        pool.hc_in_device(0, n, Xd.data_ptr(), xin.data_ptr(), None, stream=_st())
        got = xin.cpu().numpy()
    assert oracle.rel_l2(got, want_xin).max() <= XIN_TOL


@pytest.mark.parametrize("H,n", [(2048, 1), (2048, 37), (2560, 5)])
def test_hc_out_bit_exact(orc, H, n):
    X = oracle.synth_residual(n, H=H, seed=40 + n)
    inj = (1.0 + 0.3 * oracle.synth_randn(50 + n, n * 4)).reshape(n, 4).astype(np.float32)
    y = oracle.synth_hidden(n, H=H, seed=60 + n)
    want = orc.hc_out(X, inj, y)
    with MoePool(H, 640, 512, 10, max_tokens=max(n, 16), n_layers=1, device=0) as pool:
        Xd, injd, yd = _dev(X), _dev(inj), _dev(y)
        pool.hc_out_device(n, Xd.data_ptr(), injd.data_ptr(), yd.data_ptr(), stream=_st())
        got = Xd.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n", [4, 40])
def test_moe_block_with_hyper_connections(orc, n):
    """q_forward's MoE step on the device (inzg_moe_block_hc) against hc_in -> moe_routed -> hc_out on the oracle."""
    H, FF, E = 2048, 640, 512
    hc = oracle.synth_hc(3, H=H)
    X = oracle.synth_residual(n, H=H, seed=70 + n)
    R = synth.router(0, E, H)
    xin, inj = orc.hc_in(hc, X)
    sel = oracle.routing(orc, R, xin)
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=np.unique(sel))
    gu_bytes = int(synth.lib.inzg_qmat_bytes(synth.T_Q4L, 2 * FF, H))
    y = orc.moe_routed(R, blobs, bb, gu_bytes, xin, H=H, FF=FF, E=E)["y"]
    want = orc.hc_out(X, inj, y)
    with MoePool(H, FF, E, 10, max_tokens=max(n, 16), n_layers=1, device=0) as pool:
        pool.set_router(0, R)
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        pool.set_hc(0, hc["norm"], hc["down"], hc["up"], hc["inject"])
        Xd = _dev(X)
        pool.moe_block_hc_device(0, n, Xd.data_ptr(), stream=_st())
        pool.device_status(_st())
        got = Xd.cpu().numpy()
    err = oracle.rel_l2(got - X, want - X)  # the layer's contribution inj * y, per token
    exact = np.mean(got.view(np.uint32) == want.view(np.uint32))
    print(f"moe_block_hc n={n}: rel_l2 of the update max {err.max():.2e}; bit-identical residual {exact:.4f}")
    assert err.max() <= LAYER_TOL


def test_hc_in_timing():
    """Device time of hc_in at the benchmark's token counts (printed, not asserted): L2 flushed before every call,
    CUDA events on the launching stream. Algorithmic bytes: both F16 matrices, norm and inject once, X read, xin
    written; FMAs: the two 320 x 4H products."""
    H, W, R = 2048, 8192, 320
    hc = oracle.synth_hc(4, H=H)
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB > L2
    with MoePool(H, 640, 512, 10, max_tokens=4096, n_layers=1, device=0) as pool:
        pool.set_hc(0, hc["norm"], hc["down"], hc["up"], hc["inject"])
        for n in (1, 32, 4096):
            Xd = torch.randn(n, W, device="cuda")
            xin = torch.empty((n, H), device="cuda")
            inj = torch.empty((n, 4), device="cuda")
            ts = []
            for it in range(13):
                flush.fill_(float(it))
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                pool.hc_in_device(0, n, Xd.data_ptr(), xin.data_ptr(), inj.data_ptr(), stream=_st())
                b.record()
                torch.cuda.synchronize()
                if it >= 3:
                    ts.append(a.elapsed_time(b) * 1e3)
            pool.device_status(_st())
            us = float(np.median(ts))
            byts = 2 * R * W * 2 + W * 4 + 4 * W * 4 + n * W * 4 + n * H * 4
            print(f"hc_in timing H={H} n={n}: {us:.1f} us median of {len(ts)}; {byts / us / 1e3:.0f} GB/s algorithmic; "
                  f"{2 * 2 * n * R * W / us / 1e6:.2f} TFLOP/s (fp32 FMA chains)")
