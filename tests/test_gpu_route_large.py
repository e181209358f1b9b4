"""Dispatch lists on the large-call path (more than 64 tokens: chunk masks, scan, scatter).

700 tokens = 11 chunks of 64, the last one ragged (60 tokens). The override logits carry a falling per-expert
offset, so one call has decode-path experts (1-11 tokens), GEMM-path experts and experts spanning several
128-token tiles. Routing must be the oracle's bits, the unit list its first-touch order, and the layer output within
the north-star tolerance (an entry placed at a wrong position would give another token's row).
"""
import numpy as np
import pytest

import oracle
from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


def test_large_call_dispatch_matches_oracle(orc):
    n = 700
    ov = synth.normal_logits(n, E, seed=51)
    ov += (-1.5 * np.log(np.arange(1, E + 1)))[None, :].astype(np.float32)
    R = synth.router(0, E, H)
    x = synth.hidden(n, H, seed=52)
    sel = oracle.routing(orc, R, x, override=ov)
    cnt = np.bincount(sel.ravel(), minlength=E)
    assert cnt.max() > 256 and ((cnt > 0) & (cnt < 12)).sum() >= 8 and (cnt >= 12).sum() >= 8
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=np.unique(sel))
    gu_bytes = int(synth.lib.inzg_qmat_bytes(synth.T_Q4L, 2 * FF, H))
    want = orc.moe_routed(R, blobs, bb, gu_bytes, x, override=ov)
    with MoePool(H, FF, E, K, max_tokens=n, n_layers=1, device=0) as pool:
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        y = pool.moe_block(0, x, logits_override=ov, dump=True)
        d = pool.route_dump(n)
        st = pool.stats()
    assert np.array_equal(d["sel"], want["sel"])
    assert np.array_equal(d["w"].view(np.uint32), want["w"].view(np.uint32))
    assert np.array_equal(d["units"], want["units"]), "unit list is not the reference's first-touch order"
    assert st["units"] == len(want["units"]) and st["dec_units"] >= 8 and st["gemm_units"] >= 8
    err = oracle.rel_l2(y, want["y"])
    print(f"large-call dispatch n={n}: units {st['units']} (decode {st['dec_units']}, gemm {st['gemm_units']}), "
          f"rel_l2 max {err.max():.3e}")
    assert err.max() <= 1e-3
