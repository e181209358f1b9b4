"""GPU edge cases of the MoE layer against the CPU oracle.

* Collisions: every token of the batch picks the same ten experts (a logits override with those ten far above the
  rest). At 11 tokens each expert runs the decode numerics with the most tokens a decode expert can have; at 12 it
  crosses the reference's path rule (GEMM_MIN_T = 12, src/model_fwd.c:126, 229-249) onto the GEMM numerics; at 300
  each expert spans three token tiles of the tcgen05 GEMM, the last one ragged.
* Ragged batch sizes (not multiples of 8, 32 or 64) with a skewed N(0,1) logit bias.
* Exact ties in the router probabilities: the top-k follows the reference's order (lower index first).
* Sizes the context refuses: 0 tokens and more than its max_tokens (INZG_BAD_ARG, nothing launched).

Bar: routing bit-exact, outputs within 1e-3 relative L2 per token (north_star).
"""
import numpy as np
import pytest

import oracle
from inferenz_b200 import InzgError, MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10
TOL = 1e-3
HOT = np.array([3, 77, 140, 141, 256, 300, 301, 402, 450, 511])


def _collide(n):
    ov = synth.normal_logits(n)
    ov[:, HOT] += 40.0
    return ov


def _run_case(orc, n, bias=None, override=None):
    R = synth.router(0, E, H)
    x = synth.hidden(n, H)
    sel = oracle.routing(orc, R, x, bias=bias, override=override)
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=np.unique(sel))
    gu_bytes = int(synth.lib.inzg_qmat_bytes(synth.T_Q4L, 2 * FF, H))
    want = orc.moe_routed(R, blobs, bb, gu_bytes, x, bias=bias, override=override)
    with MoePool(H, FF, E, K, max_tokens=max(n, 16), n_layers=1, device=0) as pool:
        if override is None:
            pool.set_router(0, R)
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        y = pool.moe_block(0, x, bias=bias, logits_override=override, dump=True)
        got = pool.route_dump(n)
        stats = pool.stats()
    assert np.array_equal(got["sel"], want["sel"]), "top-k differs"
    assert np.array_equal(got["w"].view(np.uint32), want["w"].view(np.uint32)), "routing weights differ"
    assert np.array_equal(got["units"], want["units"]), "unit (first-touch) order differs"
    err = oracle.rel_l2(y, want["y"])
    print(f"n={n}: rel_l2 max {err.max():.3e}; units {stats['units']} (decode {stats['dec_units']}, "
          f"gemm {stats['gemm_units']})")
    assert err.max() <= TOL, f"rel L2 {err.max()}"
    return stats


@pytest.mark.parametrize("n,path", [(11, "decode"), (12, "gemm"), (300, "gemm")])
def test_all_tokens_on_the_same_ten_experts(orc, n, path):
    ov = _collide(n)
    assert (np.sort(oracle.routing(orc, synth.router(0, E, H), synth.hidden(n, H), override=ov), axis=1) == HOT).all()
    stats = _run_case(orc, n, override=ov)
    assert stats["units"] == 10
    if path == "decode":
        assert stats["dec_units"] == 10 and stats["gemm_units"] == 0
    else:
        assert stats["gemm_units"] == 10 and stats["dec_units"] == 0


@pytest.mark.parametrize("n", [5, 13, 67])
def test_ragged_batches(orc, n):
    _run_case(orc, n, bias=synth.normal_bias(E))


def test_refused_sizes():
    x = synth.hidden(17, H)
    with MoePool(H, FF, E, K, max_tokens=16, n_layers=1, device=0) as pool:
        pool.set_router(0, synth.router(0, E, H))
        blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=np.arange(2))
        pool.add_layer(0, synth.T_Q4L, blobs, bb)
        for bad in (x[:0], x):  # 0 tokens; 17 > max_tokens
            with pytest.raises(InzgError) as ei:
                pool.moe_block(0, bad)
            assert ei.value.status == 1  # INZG_BAD_ARG


def test_exact_ties_pick_the_lower_index(orc):
    # integer-valued logits: most probabilities tie exactly, and the top-k must follow the reference's total order
    # (probability descending, then index ascending: src/sampler.c:95-127, tests/test_regressions.py:17-31)
    n = 32
    ov = np.round(synth.normal_logits(n) * 1.5).astype(np.float32)
    sel = oracle.routing(orc, synth.router(0, E, H), synth.hidden(n, H), override=ov)
    p = np.take_along_axis(ov, sel, axis=1)
    assert (np.diff(p, axis=1) == 0).any()  # the case has ties inside the top-10
    _run_case(orc, n, override=ov)
