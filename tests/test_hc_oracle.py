"""The oracle's hyper-connection steps (hc_in / hc_out, src/model_fwd.c:404-450) against the reference's own functions
compiled from its tree (oracle/_ref): bit for bit, both hidden sizes, decode and GEMM-sized token counts (lin_mm's
F16 path has one numeric recipe for every n)."""
import numpy as np
import pytest

import oracle


def _ref(H):
    try:
        return oracle.Ref(H, threads=0)
    except (FileNotFoundError, OSError) as e:
        pytest.skip(f"reference harness not available: {e}")


@pytest.mark.parametrize("H", [2048, 2560])
def test_hc_in_and_hc_out_bit_exact_with_reference(orc, H):
    ref = _ref(H)
    try:
        hc = oracle.synth_hc(1, H=H)
        for n in (1, 3, 13):
            X = oracle.synth_residual(n, H=H, seed=100 + n)
            rx, ri = ref.hc_in(hc, X)
            ox, oi = orc.hc_in(hc, X)
            assert np.array_equal(rx.view(np.uint32), ox.view(np.uint32)), f"H={H} n={n}: xin differs"
            assert np.array_equal(ri.view(np.uint32), oi.view(np.uint32)), f"H={H} n={n}: inj differs"
            assert np.all(np.isfinite(rx)) and 0.1 < np.sqrt(np.mean(rx ** 2)) < 10
            y = oracle.synth_hidden(n, H=H, seed=200 + n)
            assert np.array_equal(ref.hc_out(X, ri, y).view(np.uint32), orc.hc_out(X, oi, y).view(np.uint32))
        # the final mixer has no inject vectors: xin alone
        X = oracle.synth_residual(2, H=H, seed=5)
        no_inj = dict(hc, inject=None)
        assert np.array_equal(ref.hc_in(no_inj, X)[0].view(np.uint32), orc.hc_in(no_inj, X)[0].view(np.uint32))
    finally:
        ref.close()


def test_hc_out_is_one_fma_per_element(orc):
    """A planted mistake in the checker: an unfused multiply-add must NOT match the oracle (so the fma is pinned)."""
    H, n = 2048, 2
    X = oracle.synth_residual(n, H=H, seed=9)
    inj = np.full((n, 4), 0.7368421, np.float32)
    y = oracle.synth_hidden(n, H=H, seed=10)
    unfused = (X.reshape(n, 4, H) + (inj[:, :, None] * y[:, None, :]).astype(np.float32)).reshape(n, 4 * H)
    assert not np.array_equal(orc.hc_out(X, inj, y), unfused)


def _golden():
    import importlib.util
    import os
    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(here, "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg, np.load(os.path.join(here, "golden", "hc.npz"))


@pytest.mark.parametrize("H", [2048, 2560])
def test_hc_restatement_matches_golden(orc, H):
    """The restatement against the reference's outputs stored in tests/golden/hc.npz (no compiled reference needed)."""
    mg, g = _golden()
    hc, X, y = mg.hc_inputs(H)
    want_sha = list(g[f"h{H}_sha"])
    assert [mg.sha(hc[k]) for k in ("norm", "down", "up", "inject")] + [mg.sha(X), mg.sha(y)] == want_sha, \
        "regenerated inputs differ from the fixture's"
    xin, inj = orc.hc_in(hc, X)
    assert np.array_equal(xin.view(np.uint32), g[f"h{H}_xin"].view(np.uint32))
    assert np.array_equal(inj.view(np.uint32), g[f"h{H}_inj"].view(np.uint32))
    assert np.array_equal(orc.hc_out(X, inj, y).view(np.uint32), g[f"h{H}_xout"].view(np.uint32))
