"""The oracle's C restatement is pinned to the reference: bit-exact against the golden fixtures generated from the
reference's compiled MoE path (tests/golden/make_golden.py), and against the live compiled reference where it can
load, function by function."""
import hashlib
import os

import numpy as np
import pytest

import oracle
from inferenz_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
H, FF, E, K = 2048, 640, 512, 10

GOLDEN = ["decode_n1_q4l", "decode_n4_q4l_bias", "decode_n4_q8g_bias", "prefill_n48_q4l_override",
          "prefill_n40_q8g_override", "prefill_n24_q4l_h2560_override"]


def gu_bytes(typ, H=H):
    return int(synth.lib.inzg_qmat_bytes(typ, 2 * FF, H))


def golden_inputs(name):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(HERE, "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.case_inputs(name)


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("name", GOLDEN)
def test_restatement_matches_golden(orc, name):
    g = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    n, typ, Hc, R, x, bias, ov = golden_inputs(name)
    blobs, bb = oracle.ref_layer_blobs(0, typ, Hc, FF, E, experts=g["experts"])
    for e, h in zip(g["experts"], g["blob_sha256"]):
        assert hashlib.sha256(blobs[e * bb:(e + 1) * bb].tobytes()).hexdigest() == h, "inputs differ from golden"
    d = orc.moe_routed(R, blobs, bb, gu_bytes(typ, Hc), x, bias=bias, override=ov, H=Hc)
    for k in ("logits", "probs", "w", "y"):
        assert np.array_equal(bits(d[k]), bits(g[k])), k
    assert np.array_equal(d["sel"], g["sel"])
    assert np.array_equal(d["units"], g["units"])


def test_router_logits_live(orc, ref):
    R = synth.router(3, E, H)
    x = synth.hidden(5, H, seed=11)
    want = np.zeros((5, E), np.float32)
    ref.lib.ref_router_logits(oracle._p(R), 5, oracle._p(x), oracle._p(want))
    assert np.array_equal(bits(orc.router_logits(R, x)), bits(want))


def test_softmax_and_topk_live_with_ties(orc, ref):
    rng = np.random.default_rng(1)
    for trial in range(20):
        s = rng.standard_normal(E).astype(np.float32) * (1 + trial)
        if trial % 2:
            s = np.round(s).astype(np.float32)  # many exact ties
        a, b = orc.softmax(s), s.copy()
        ref.lib.ref_softmax(oracle._p(b), E)
        assert np.array_equal(bits(a), bits(b))
        for k in (1, 10, 64):
            want = np.zeros(k, np.int32)
            ref.lib.ref_topk(oracle._p(a), E, k, oracle._p(want))
            assert np.array_equal(orc.topk(a, k), want)


def test_topk_order_is_value_desc_index_asc(orc):
    """the total order of src/sampler.c:95-103 (tests/test_regressions.py:17-31): ties by lower index"""
    rng = np.random.default_rng(2)
    for _ in range(20):
        v = (rng.integers(0, 17, 257) - 8).astype(np.float32)
        want = sorted(range(257), key=lambda i: (-v[i], i))[:10]
        assert list(orc.topk(v, 10)) == want


@pytest.mark.parametrize("n,rot", [(2048, 256), (640, 128), (2048, 0), (320, 64)])
def test_activation_quantization_live(orc, ref, n, rot):
    x = synth.randn(n, n, 1.0)
    x[::97] *= 9
    q, s, b = orc.act_quantize(x, rot, 0x5EED)
    q2, s2, b2 = np.zeros(n, np.int8), np.zeros(n // 64, np.float32), np.zeros(n // 64, np.float32)
    ref.lib.ref_act_quantize(oracle._p(x), n, rot, 0x5EED, oracle._p(q2), oracle._p(s2), oracle._p(b2))
    assert np.array_equal(q, q2) and np.array_equal(bits(s), bits(s2)) and np.array_equal(bits(b), bits(b2))


@pytest.mark.parametrize("K,rot", [(2048, 256), (640, 128)])
def test_prefill_activation_blocks_live(orc, ref, K, rot):
    X = synth.randn(K + 1, 3 * K, 1.0).reshape(3, K)
    nkb = (K + 255) // 256
    q2, s2, m2 = np.zeros(3 * K, np.int8), np.zeros(3 * nkb, np.float32), np.zeros(3 * nkb, np.int32)
    ref.lib.ref_xq(oracle._p(X), 3, K, rot, 0x5EED, oracle._p(q2), oracle._p(s2), oracle._p(m2))
    for t in range(3):
        q, s, m = orc.xq(X[t], rot, 0x5EED)
        assert np.array_equal(q, q2[t * K:(t + 1) * K])
        assert np.array_equal(bits(s), bits(s2[t * nkb:(t + 1) * nkb]))
        assert np.array_equal(m, m2[t * nkb:(t + 1) * nkb])


@pytest.mark.slow
@pytest.mark.parametrize("n,hook,typ", [(2, "bias", synth.T_Q4L), (20, "override", synth.T_Q4L),
                                        (20, "override", synth.T_Q8G), (3, "bias", synth.T_Q8G)])
def test_whole_layer_live(orc, n, hook, typ):
    """restated layer == compiled reference layer on fresh inputs (decode batch path and GEMM path, Q4L and Q8G)"""
    R = synth.router(5, E, H)
    x = synth.hidden(n, H, seed=21)
    bias = synth.normal_bias(E, seed=22) if hook == "bias" else None
    ov = None
    if hook == "override":
        ov = synth.normal_logits(n, E, seed=23)
        ov[:, 7] += 8.0
    sel = oracle.routing(orc, R, x, bias=bias, override=ov)
    try:
        ref = oracle.Ref(H, threads=0, expert_type=typ)
    except (FileNotFoundError, OSError) as e:
        pytest.skip(str(e))
    blobs, bb = oracle.ref_layer_blobs(5, typ, H, FF, E, experts=np.unique(sel))
    b = ref.moe_routed(R, blobs, bb, x, bias=bias, override=ov)
    ref.close()
    a = orc.moe_routed(R, blobs, bb, gu_bytes(typ), x, bias=bias, override=ov)
    for k in ("logits", "probs", "w", "moe_out", "y"):
        assert np.array_equal(bits(a[k]), bits(b[k])), k
    assert np.array_equal(a["sel"], b["sel"]) and np.array_equal(a["units"], b["units"])
