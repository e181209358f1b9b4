"""The oracle's restatement of the Q4N (NVFP4 repacked) expert numerics (src/quant.c:956-1164, 1476-1530) against the
reference's own kernels compiled from its tree (oracle/_ref): payloads made by the reference quantizer
(quantize_q4n, src/quant.c:1038-1063), products bit for bit through lin_mm's three numeric paths -- mv_q4n (one
token), mm_q4n (2-11 tokens; a different rounding order from mv_q4n) and the prefill GEMM's Q4N tile requantization
(12 tokens and more)."""
import numpy as np
import pytest

import oracle


def _ref(H=2048):
    try:
        return oracle.Ref(H, threads=0)
    except (FileNotFoundError, OSError) as e:
        pytest.skip(f"reference harness not available: {e}")


# the expert shapes at H = 2048 (gate|up 1280 x 2048, down 2048 x 640) cut to fewer rows, and a 2560-wide one
SHAPES = [(64, 2048), (96, 640), (32, 2560)]


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_q4n_products_bit_exact_with_reference(orc, rows, cols):
    ref = _ref()
    try:
        W = oracle.synth_randn(700 + rows, rows * cols, (1.0 / cols) ** 0.5).reshape(rows, cols)
        payload = ref.quantize(W, oracle.T_Q4N)
        assert payload.size == orc.lib.orc_qmat_bytes(oracle.T_Q4N, rows, cols)
        for n, gemm in [(1, False), (2, False), (5, False), (11, False), (12, True), (20, True)]:
            X = oracle.synth_hidden(n, cols, seed=800 + n)
            want = ref.matmul(payload, X, gemm=gemm)
            got = orc.matmul(payload, X, gemm=gemm)
            assert np.all(np.isfinite(want)) and np.abs(want).max() > 0
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"{rows}x{cols} n={n} gemm={gemm}"
    finally:
        ref.close()


def test_q4n_one_token_paths_round_differently(orc):
    """mv_q4n (one token) and mm_q4n (several) fold the block scales in different orders; the restatement keeps both
    (a planted equality of the two would hide which one a device kernel follows)."""
    rows, cols = 64, 2048
    W = oracle.synth_randn(901, rows * cols, (1.0 / cols) ** 0.5).reshape(rows, cols)
    ref = _ref()
    try:
        payload = ref.quantize(W, oracle.T_Q4N)
    finally:
        ref.close()
    x = oracle.synth_hidden(1, cols, seed=902)
    mv = orc.matmul(payload, x)[0]
    mm = orc.matmul(payload, np.concatenate([x, x]))[0]
    assert not np.array_equal(mv, mm)
    assert np.abs(mv - mm).max() <= 1e-5 * np.abs(mv).max()


def test_q4n_restatement_matches_golden(orc):
    """The restatement against the reference's Q4N products stored in tests/golden/q4n.npz (no compiled reference
    needed)."""
    import importlib.util
    import os
    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(here, "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    g = np.load(os.path.join(here, "golden", "q4n.npz"))
    for i, (rows, cols) in enumerate(mg.Q4N_SHAPES):
        pl = g[f"m{i}_payload"]
        for n, gemm in mg.Q4N_CALLS:
            got = orc.matmul(pl, oracle.synth_hidden(n, cols, seed=800 + n), gemm=gemm)
            assert np.array_equal(got.view(np.uint32), g[f"m{i}_n{n}"].view(np.uint32)), f"{rows}x{cols} n={n}"
