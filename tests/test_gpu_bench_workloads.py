"""Parity on the exact workloads bench.py times (BASELINE configs[0]-[3]): one layer call of the CUDA path per
workload against the reference's own output on the same inputs -- the fixture tests/golden/bench_<name>.npz made by the
compiled reference (make_golden.py), and, where the compiled reference travels with the repository, the reference
run live on every token.

Bar: routing bit for bit (logits, probabilities, top-k, renormalised weights, first-touch unit order); per token,
relative L2 of the output <= 1e-3 (north_star).
"""
import numpy as np
import pytest

import bench
import oracle
from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10
WORKLOADS = {"decode1": (1, synth.T_Q4L), "decode32": (32, synth.T_Q4L), "prefill4096": (4096, synth.T_Q4L),
             "q8g2048": (2048, synth.T_Q8G)}


@pytest.mark.parametrize("name", list(WORKLOADS))
def test_bench_workload_matches_reference(name):
    n, typ = WORKLOADS[name]
    x, bias, ov = bench.make_inputs(name, n)
    g = np.load(f"{bench.ROOT}/tests/golden/bench_{name}.npz")
    R = synth.router(0, E, H)
    blobs, bb = synth.layer_blobs(0, typ, H, FF, E, experts=g["experts"])
    with MoePool(H, FF, E, K, max_tokens=max(n, 16), n_layers=1, device=0) as pool:
        if ov is None:
            pool.set_router(0, R)
        pool.add_layer(0, typ, blobs, bb)
        y = pool.moe_block(0, x, bias=bias, logits_override=ov, dump=True)
        d = pool.route_dump(n)
        st = pool.stats()
    rep = bench.check_parity(name, d, y)
    print(f"{name}: units {st['units']} (decode {st['dec_units']}, gemm {st['gemm_units']}) {rep}")
    assert rep["routing_bit_exact"], rep
    assert rep["ok"], rep
    try:
        ref = oracle.Ref(H, threads=0, expert_type=typ)
    except (FileNotFoundError, OSError):
        return
    want = ref.moe_routed(R, blobs, bb, x, bias=bias, override=ov, dumps=False)["y"]
    ref.close()
    err = oracle.rel_l2(y, want)
    exact = float(np.mean(y.view(np.uint32) == want.view(np.uint32)))
    print(f"{name}: live reference, every token: rel_l2 max {err.max():.3e}, bit-identical outputs {exact:.4f}")
    assert err.max() <= 1e-3
