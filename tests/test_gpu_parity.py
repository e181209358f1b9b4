"""GPU parity: the CUDA MoE layer (through the C ABI) against the CPU oracle on seeded synthetic layers.

Bar: routing, top-k and permutation bit-exact; expert outputs within 1e-3 relative L2 per
token. The kernels reproduce the reference's integer quantization and accumulation orders, so most outputs are
bit-identical as well; the fraction is printed.
"""
import numpy as np
import pytest

import oracle
from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

TOL = 1e-3  # relative L2 per token (north_star)


def _case(orc, H, n, expert_type=synth.T_Q4L, bias=None, override=None, layer=0):
    FF, E = 640, 512
    R = synth.router(layer, E, H)
    x = synth.hidden(n, H)
    sel = oracle.routing(orc, R, x, bias=bias, override=override)
    blobs, bb = synth.layer_blobs(layer, expert_type, H, FF, E, experts=np.unique(sel))
    gu_bytes = int(synth.lib.inzg_qmat_bytes(expert_type, 2 * FF, H))
    want = orc.moe_routed(R, blobs, bb, gu_bytes, x, bias=bias, override=override, H=H, FF=FF, E=E)
    return R, x, blobs, bb, want


def _run(H, R, x, blobs, bb, expert_type, bias=None, override=None):
    n = x.shape[0]
    with MoePool(H, 640, 512, 10, max_tokens=max(n, 16), n_layers=1, device=0) as pool:
        if override is None:
            pool.set_router(0, R)
        pool.add_layer(0, expert_type, blobs, bb)
        y = pool.moe_block(0, x, bias=bias, logits_override=override, dump=True)
        d = pool.route_dump(n)
        d["stats"] = pool.stats()
    d["y"] = y
    return d


def _check(got, want, name):
    assert np.array_equal(got["logits"].view(np.uint32), want["logits"].view(np.uint32)), f"{name}: logits differ"
    assert np.array_equal(got["probs"].view(np.uint32), want["probs"].view(np.uint32)), f"{name}: probs differ"
    assert np.array_equal(got["sel"], want["sel"]), f"{name}: top-k differs"
    assert np.array_equal(got["w"].view(np.uint32), want["w"].view(np.uint32)), f"{name}: routing weights differ"
    assert np.array_equal(got["units"], want["units"]), f"{name}: unit (first-touch) order differs"
    err = oracle.rel_l2(got["y"], want["y"])
    exact = np.mean(got["y"].view(np.uint32) == want["y"].view(np.uint32))
    print(f"{name}: rel_l2 max {err.max():.3e} mean {err.mean():.3e}; bit-identical outputs {exact:.4f}; "
          f"units {got['stats']['units']} (decode {got['stats']['dec_units']}, gemm {got['stats']['gemm_units']})")
    assert err.max() <= TOL, f"{name}: rel L2 {err.max()}"
    return err, exact


def test_decode_1_token(orc):
    R, x, blobs, bb, want = _case(orc, 2048, 1)
    got = _run(2048, R, x, blobs, bb, synth.T_Q4L)
    _check(got, want, "decode n=1 Q4L")


def test_decode_batch_4_tokens_bias(orc):
    b = synth.normal_bias()
    R, x, blobs, bb, want = _case(orc, 2048, 4, bias=b)
    got = _run(2048, R, x, blobs, bb, synth.T_Q4L, bias=b)
    _check(got, want, "decode n=4 Q4L bias")


def test_decode_32_tokens_skewed(orc):
    b = synth.normal_bias()
    R, x, blobs, bb, want = _case(orc, 2048, 32, bias=b)
    got = _run(2048, R, x, blobs, bb, synth.T_Q4L, bias=b)
    _check(got, want, "decode n=32 Q4L bias")


def _gemm_override(n, hot=3, boost=6.0):
    ov = synth.normal_logits(n)
    ov[:, :hot] += boost
    return ov


def test_prefill_gemm_path_q4l(orc):
    ov = _gemm_override(48)
    R, x, blobs, bb, want = _case(orc, 2048, 48, override=ov)
    got = _run(2048, R, x, blobs, bb, synth.T_Q4L, override=ov)
    assert got["stats"]["gemm_units"] >= 3
    _check(got, want, "prefill n=48 Q4L (GEMM path)")


def test_q8g_decode_and_gemm(orc):
    b = synth.normal_bias()
    R, x, blobs, bb, want = _case(orc, 2048, 4, expert_type=synth.T_Q8G, bias=b)
    _check(_run(2048, R, x, blobs, bb, synth.T_Q8G, bias=b), want, "decode n=4 Q8G")
    ov = _gemm_override(40)
    R, x, blobs, bb, want = _case(orc, 2048, 40, expert_type=synth.T_Q8G, override=ov)
    _check(_run(2048, R, x, blobs, bb, synth.T_Q8G, override=ov), want, "prefill n=40 Q8G (GEMM path)")


def test_reference_model_hidden_2560(orc):
    R, x, blobs, bb, want = _case(orc, 2560, 2)
    _check(_run(2560, R, x, blobs, bb, synth.T_Q4L), want, "decode n=2 Q4L H=2560")


def test_reference_model_hidden_2560_gemm_path(orc):
    ov = _gemm_override(24)
    R, x, blobs, bb, want = _case(orc, 2560, 24, override=ov)
    got = _run(2560, R, x, blobs, bb, synth.T_Q4L, override=ov)
    assert got["stats"]["gemm_units"] >= 3
    _check(got, want, "prefill n=24 Q4L H=2560 (GEMM path)")


@pytest.mark.parametrize("name", ["decode_n1_q4l", "decode_n4_q4l_bias", "decode_n4_q8g_bias",
                                  "prefill_n48_q4l_override", "prefill_n40_q8g_override",
                                  "prefill_n24_q4l_h2560_override"])
def test_golden_cases(name):
    """the reference's own outputs (tests/golden, made by the compiled reference): routing bit for bit, outputs within
    the tolerance; the blobs (host draws, GPU encoder) hash to the ones the reference encoded"""
    import hashlib
    import importlib.util
    import os
    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(here, "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    n, typ, Hc, R, x, bias, ov = mg.case_inputs(name)
    g = np.load(os.path.join(here, "golden", f"{name}.npz"))
    blobs, bb = synth.layer_blobs(0, typ, Hc, 640, 512, experts=g["experts"])
    for e, h in zip(g["experts"], g["blob_sha256"]):
        assert hashlib.sha256(blobs[e * bb:(e + 1) * bb].tobytes()).hexdigest() == h, "encoder bytes differ"
    got = _run(Hc, R, x, blobs, bb, typ, bias=bias, override=ov)
    want = {k: g[k] for k in ("logits", "probs", "sel", "w", "units", "y")}
    _check(got, want, f"golden {name}")
