"""The GPU expert encoder (k_quant.cu) writes the reference quantizer's bytes (inz_quantize, src/quant.c:422-556):
against the golden fixture made by the reference (tests/golden/quantizer.npz), against the compiled reference live
(oracle/_ref), and through the synthetic layers every parity test is built from (blob hashes of the golden cases).
The device generator draws the host generator's stream."""
import ctypes
import hashlib
import os

import numpy as np
import pytest

import oracle
from inferenz_b200 import lib, synth

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def quantize(W, typ, rot=0, seed=0):
    rows, cols = W.shape
    out = np.zeros(lib.inzg_qmat_bytes(typ, rows, cols), np.uint8)
    assert lib.inzg_quantize(_p(np.ascontiguousarray(W, np.float32)), rows, cols, typ, rot, seed, _p(out)) == 0
    return out


def test_matches_golden_reference_bytes():
    g = np.load(os.path.join(HERE, "golden", "quantizer.npz"))
    for i in range(4):
        rows, cols, typ, rot = (int(v) for v in g[f"q{i}_shape"])
        w = synth.randn(100 + i, rows * cols, 0.03).reshape(rows, cols)
        assert np.array_equal(quantize(w, typ, rot), g[f"q{i}_bytes"]), f"case {i}"


@pytest.mark.parametrize("rows,cols,typ,rot,seed", [(1280, 2048, 102, 0, 0), (2048, 640, 102, 0, 0),
                                                    (128, 2048, 103, 256, 0), (256, 640, 103, 128, 0),
                                                    (33, 320, 102, 64, 0), (9, 320, 103, -1, 0),
                                                    (300, 2560, 102, 0, 77), (2560, 640, 103, 128, 5),
                                                    (40, 256, 102, -1, 0), (7, 192, 102, 64, 3)])
def test_matches_live_reference(rows, cols, typ, rot, seed):
    try:
        ref = oracle.Ref(2048, threads=1)
    except (FileNotFoundError, OSError) as e:
        pytest.skip(str(e))
    w = synth.randn(rows + cols, rows * cols, 1.0 / np.sqrt(2048)).reshape(rows, cols)
    a = ref.quantize(w, typ, rot_block=rot, seed=seed)
    ref.close()
    assert np.array_equal(quantize(w, typ, rot, seed), a)


def test_degenerate_groups_match_live_reference():
    """all-zero groups, a lone spike and constant groups take the reference's degenerate branches"""
    try:
        ref = oracle.Ref(2048, threads=1)
    except (FileNotFoundError, OSError) as e:
        pytest.skip(str(e))
    w = synth.randn(3, 64 * 512, 0.02).reshape(64, 512)
    w[0] = 0.0
    w[1, :64] = 0.0
    w[2] = 0.0
    w[2, 5] = 1.0
    w[3] = 0.25
    w[4, ::2] = -1e-30
    for typ, rot in ((102, -1), (102, 0), (103, -1), (103, 128)):
        assert np.array_equal(quantize(w, typ, rot), ref.quantize(w, typ, rot_block=rot)), (typ, rot)
    ref.close()


def test_expert_blobs_match_golden_hashes():
    """the golden cases' experts, drawn on the host and encoded on the GPU, are the reference converter's bytes"""
    g = np.load(os.path.join(HERE, "golden", "decode_n1_q4l.npz"))
    experts = g["experts"]
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, experts=experts)
    for e, h in zip(experts, g["blob_sha256"]):
        assert hashlib.sha256(blobs[e * bb:(e + 1) * bb].tobytes()).hexdigest() == h
    g8 = np.load(os.path.join(HERE, "golden", "decode_n4_q8g_bias.npz"))
    blobs, bb = synth.layer_blobs(0, synth.T_Q8G, experts=g8["experts"][:6])
    for e, h in zip(g8["experts"][:6], g8["blob_sha256"][:6]):
        assert hashlib.sha256(blobs[e * bb:(e + 1) * bb].tobytes()).hexdigest() == h


def test_device_generator_draws_the_host_stream():
    """Experts drawn on the GPU equal the host draws (the LCG is exact; the Box-Muller step uses CUDA's double
    log/cos, so a float may differ where the double result sits within an ulp or two of a float rounding boundary:
    allowed at most 2 of the 15.7 M draws here, expected none)."""
    import torch
    H, FF, e0, n = 2048, 640, 37, 4
    gu = torch.empty((n, 2 * FF, H), dtype=torch.float32, device="cuda")
    dn = torch.empty((n, H, FF), dtype=torch.float32, device="cuda")
    assert lib.inzg_synth_experts_device(5, H, FF, e0, n, gu.data_ptr(), dn.data_ptr(), None) == 0
    gu, dn = gu.cpu().numpy(), dn.cpu().numpy()
    bad = 0
    for i in range(n):
        a, b = synth.expert_fp32(5, e0 + i, H, FF)
        bad += int((a.view(np.uint32) != gu[i].view(np.uint32)).sum() + (b.view(np.uint32) != dn[i].view(np.uint32)).sum())
    assert bad <= 2, bad


def test_device_layer_blobs_equal_host_layer_blobs():
    """inzg_synth_layer_blobs_device (drawn and encoded on the GPU) against host draws encoded on the GPU"""
    import torch
    H, FF, e0, e1 = 2048, 640, 10, 14
    for typ in (synth.T_Q4L, synth.T_Q8G):
        bb = synth.blob_bytes(typ, H, FF)
        d = torch.empty(((e1 - e0) * bb,), dtype=torch.uint8, device="cuda")
        assert lib.inzg_synth_layer_blobs_device(0, typ, H, FF, e0, e1, d.data_ptr(), None) == 0
        h, _ = synth.layer_blobs_range(0, typ, H, FF, e0, e1)
        assert np.array_equal(d.cpu().numpy(), h), typ
