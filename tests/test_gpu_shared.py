"""The shared expert on B200 against the reference's own shared-expert step (oracle/_ref: lin_mm, siluf, sigmoidf,
dot_f32 of src/model_fwd.c:1041-1069, 1141-1148), after the reference's routed layer.

Q4L routed experts with a Q8G shared expert (the converter's recommended recipe) and with a Q4L one; 4 tokens take
lin_mm's decode numerics, 20 tokens its GEMM numerics. The expected differences are only the SiLU/sigmoid exponential
(double exp rounded once vs glibc expf), so the bar here is far below the 1e-3 of the routed path."""
import numpy as np
import pytest

import oracle
from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


@pytest.mark.parametrize("sh_type,n", [(synth.T_Q8G, 4), (synth.T_Q8G, 20), (synth.T_Q4L, 4), (synth.T_Q4L, 20)])
def test_shared_expert_matches_reference(ref, sh_type, n):
    R = synth.router(0, E, H)
    x = synth.hidden(n, H)
    bias = synth.normal_bias(E)
    orc = oracle.Oracle()
    sel = oracle.routing(orc, R, x, bias=bias)
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=np.unique(sel))
    sh_blob, sh_bb = synth.layer_blobs_range(777, sh_type, H, FF, 0, 1)
    gate = (np.random.default_rng(5).standard_normal(H) * 0.05).astype(np.float32)
    y_routed = ref.moe_routed(R, blobs, bb, x, bias=bias, dumps=False)["y"]
    gu_bytes = int(synth.lib.inzg_qmat_bytes(sh_type, 2 * FF, H))
    want, _ = ref.shared(sh_blob, gu_bytes, sh_type, gate, x, y_routed)
    with MoePool(H, FF, E, K, max_tokens=32, n_layers=1, device=0) as pool:
        pool.set_router(0, R)
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        y_no = pool.moe_block(0, x, bias=bias)
        pool.set_shared(0, sh_type, sh_blob, sh_bb, gate)
        y = pool.moe_block(0, x, bias=bias)
        y2 = pool.moe_block(0, x, bias=bias, graph=False)
    err = oracle.rel_l2(y, want)
    same = np.mean(y.view(np.uint32) == want.view(np.uint32))
    print(f"shared expert type={sh_type} n={n}: rel_l2 max {err.max():.3e}, bit-identical outputs {same:.4f}")
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32)), "graph and direct launches differ"
    assert not np.array_equal(y, y_no), "the shared expert changed nothing"
    assert err.max() <= 1e-5
