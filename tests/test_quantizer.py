"""The synthetic generators: the product's host generator (inferenz_b200.synth, libinzg) and the oracle's copy of it
(the reference tests' LCG + Box-Muller) draw the same streams, deterministically across jump-ahead and threads. The
expert quantizer itself runs on the GPU: tests/test_gpu_quantizer.py pins its bytes to the reference quantizer."""
import ctypes

import numpy as np

import oracle
from inferenz_b200 import lib, synth


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


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


def test_oracle_generator_draws_the_product_streams():
    """the benchmark's reference arm draws its inputs with the oracle's generator: same bytes as the product's"""
    assert np.array_equal(oracle.synth_router(2, 64, 512), synth.router(2, 64, 512))
    assert np.array_equal(oracle.synth_hidden(5, 512, seed=9), synth.hidden(5, 512, seed=9))
    assert np.array_equal(oracle.normal_bias(512), synth.normal_bias(512))
    assert np.array_equal(oracle.normal_logits(3, 512), synth.normal_logits(3, 512))
    assert np.array_equal(oracle.zipf_bias(512), synth.zipf_bias(512))
    for a, b in zip(oracle.synth_expert(4, 7, 256, 64), synth.expert_fp32(4, 7, 256, 64)):
        assert np.array_equal(a, b)


def test_f16_conversion_rounds_to_nearest_even():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)][:20000]
    got = np.array([lib.inzg_f32_to_f16(float(v)) for v in x], np.uint16)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
