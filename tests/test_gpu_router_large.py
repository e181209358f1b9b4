"""Router logits on the many-token kernels (fp32 router copy in 64-token tiles; 64 experts x 2-8 tokens per block).

600 tokens = 9 full tiles and a ragged one of 24. The logits must be the oracle's bits (the reference's 8-lane FMA
chains and add tree, then the per-expert bias), and the top-k the oracle's selection.
"""
import numpy as np
import pytest

import oracle
from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


@pytest.mark.parametrize("n", [600, 3, 17, 32, 33, 64])
def test_many_token_router_bit_exact(orc, n):
    """600: the fp32-copy tiles; 3-64 (decode-sized calls): 64 experts x 2 or 4 tokens per block, odd counts leaving a
    partial token block"""
    R = synth.router(0, E, H)
    x = synth.hidden(n, H, seed=61)
    bias = synth.zipf_bias(E)  # concentrates the selection (the layer then needs few experts' blobs)
    lg = (orc.router_logits(R, x) + bias[None, :]).astype(np.float32)
    want_sel = oracle.routing(orc, R, x, bias=bias)
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=np.unique(want_sel))
    with MoePool(H, FF, E, K, max_tokens=n, n_layers=1, device=0) as pool:
        pool.set_router(0, R)
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        pool.moe_block(0, x, bias=bias, dump=True)
        d = pool.route_dump(n)
    got = d["logits"]
    bad = np.flatnonzero(got.view(np.uint32) != lg.view(np.uint32))
    print(f"many-token router n={n}: {bad.size} logits differ")
    assert bad.size == 0, f"first differing logit at flat index {bad[:4]}"
    assert np.array_equal(d["sel"], want_sel)
