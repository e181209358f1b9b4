"""The engine's quantizer in libinzg (include/inzg_tools.h) writes the reference quantizer's bytes, and the synthetic
generator is deterministic across threads and jump-ahead."""
import ctypes
import hashlib
import os

import numpy as np
import pytest

import oracle
from inferenz_b200 import lib, synth

HERE = os.path.dirname(os.path.abspath(__file__))


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def quantize(W, typ, rot=0, seed=0, threads=1):
    rows, cols = W.shape
    out = np.zeros(lib.inzg_qmat_bytes(typ, rows, cols), np.uint8)
    assert lib.inzg_quantize(_p(np.ascontiguousarray(W, np.float32)), rows, cols, typ, rot, seed, threads, _p(out)) == 0
    return out


def test_matches_golden_reference_bytes():
    g = np.load(os.path.join(HERE, "golden", "quantizer.npz"))
    for i in range(4):
        rows, cols, typ, rot = (int(v) for v in g[f"q{i}_shape"])
        w = synth.randn(100 + i, rows * cols, 0.03).reshape(rows, cols)
        assert np.array_equal(quantize(w, typ, rot), g[f"q{i}_bytes"]), f"case {i}"


@pytest.mark.parametrize("rows,cols,typ,rot", [(1280, 2048, 102, 0), (2048, 640, 102, 0), (128, 2048, 103, 256),
                                                (256, 640, 103, 128), (33, 320, 102, 64), (9, 320, 103, -1)])
def test_matches_live_reference(rows, cols, typ, rot):
    try:
        ref = oracle.Ref(2048, threads=1)
    except (FileNotFoundError, OSError) as e:
        pytest.skip(str(e))
    w = synth.randn(rows + cols, rows * cols, 1.0 / np.sqrt(2048)).reshape(rows, cols)
    a = ref.quantize(w, typ, rot_block=rot)
    ref.close()
    assert np.array_equal(quantize(w, typ, rot), a)


def test_threads_do_not_change_bytes():
    w = synth.randn(7, 256 * 640, 0.02).reshape(256, 640)
    assert np.array_equal(quantize(w, 102, 0, threads=1), quantize(w, 102, 0, threads=4))


def test_expert_blobs_match_golden_hashes():
    """Regenerating the golden cases' experts gives the reference's bytes (inputs of every parity fixture)."""
    g = np.load(os.path.join(HERE, "golden", "decode_n1_q4l.npz"))
    experts = g["experts"][:3]
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, experts=experts)
    for e, h in zip(experts, g["blob_sha256"][:3]):
        assert hashlib.sha256(blobs[e * bb:(e + 1) * bb].tobytes()).hexdigest() == h


def test_jump_ahead_equals_sequential_draws():
    seq = synth.randn(5, 1000)
    st = lib.inzg_synth_jump(5, 600)
    tail = np.empty(400, np.float32)
    lib.inzg_synth_randn(st, 400, 1.0, _p(tail))
    assert np.array_equal(seq[600:], tail)


def test_expert_draw_order():
    """expert e's gate|up and down are the normals right after expert e-1's (per-layer stream)."""
    H, FF = 256, 64
    gu0, dn0 = synth.expert_fp32(3, 0, H, FF)
    gu1, _ = synth.expert_fp32(3, 1, H, FF)
    flat = synth.randn(3, 3 * FF * H * 2, np.float32(np.sqrt(1.0 / H)))
    assert np.array_equal(np.concatenate([gu0.ravel(), dn0.ravel()]), flat[:3 * FF * H])
    assert np.array_equal(gu1.ravel(), flat[3 * FF * H:3 * FF * H + 2 * FF * H])


def test_f16_conversion_rounds_to_nearest_even():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    got = np.array([lib.inzg_f32_to_f16(float(v)) for v in x[:20000]], np.uint16)
    want = x[:20000].astype(np.float16).view(np.uint16)
    nan = np.isnan(x[:20000])
    assert np.array_equal(got[~nan], want[~nan])
