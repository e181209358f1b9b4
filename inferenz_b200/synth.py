"""Seeded synthetic inputs of the benchmark configurations (no dataset or checkpoint is involved).

Generator: the LCG + Box-Muller normal of the reference's own tests (tests/test_quant.c:10-17), in C
(``inzg_synth_*``, include/inzg_tools.h). Seeds: experts of layer l from seed l (per expert: gate, up, down,
row-major, N(0, 1/H)); router of layer l from seed 1000 + l, N(0, 0.02^2) rounded to F16; hidden states from seed 1,
N(0, 1) then RMS-normalised; per-expert logit bias N(0, 1) from seed 2 (decode-32 configuration); Zipf(1.1) bias
ln p_e (prefill-4096 configuration); logits N(0, 1) from seed 4 (Q8G exact-recipe configuration).
"""
import ctypes

import numpy as np

from ._lib import T_Q4L, T_Q8G, lib

ROUTER_SEED_BASE = 1000
HIDDEN_SEED, BIAS_SEED, OVERRIDE_SEED = 1, 2, 4


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def randn(seed, n, scale=1.0):
    out = np.empty(n, np.float32)
    lib.inzg_synth_randn(seed, n, scale, _p(out))
    return out


def router(layer, E=512, H=2048):
    w = np.empty((E, H), np.uint16)
    lib.inzg_synth_router(ROUTER_SEED_BASE + layer, E, H, _p(w))
    return w


def hidden(n, H=2048, seed=HIDDEN_SEED):
    x = np.empty((n, H), np.float32)
    lib.inzg_synth_hidden(seed, n, H, _p(x))
    return x


def normal_bias(E=512, seed=BIAS_SEED):
    return randn(seed, E)


def zipf_bias(E=512, s=1.1):
    """ln of the Zipf(s) pmf over expert index: experts with low index attract most tokens."""
    p = (np.arange(1, E + 1, dtype=np.float64)) ** (-s)
    return np.log(p / p.sum()).astype(np.float32)


def normal_logits(n, E=512, seed=OVERRIDE_SEED):
    return randn(seed, n * E).reshape(n, E)


def blob_bytes(expert_type, H=2048, FF=640):
    return int(lib.inzg_blob_bytes(expert_type, H, FF))


def expert_fp32(layer, e, H=2048, FF=640):
    gu = np.empty((2 * FF, H), np.float32)
    dn = np.empty((H, FF), np.float32)
    lib.inzg_synth_expert(layer, H, FF, e, _p(gu), _p(dn))
    return gu, dn


def layer_blobs(layer, expert_type=T_Q4L, H=2048, FF=640, E=512, experts=None):
    """Blobs of one synthetic layer, [E * blob_bytes] uint8 (the GGUF `blk.%d.experts` tensor).

    ``experts``: if given, only these experts are generated and quantized; the others get a valid header with a zero
    payload (they must not be routed to). Used by tests, which know the routing in advance.
    """
    bb = blob_bytes(expert_type, H, FF)
    out = np.zeros(E * bb, np.uint8)
    if experts is None:
        rc = lib.inzg_synth_layer_blobs(layer, expert_type, H, FF, 0, E, _p(out))
        if rc != 0:
            raise RuntimeError("inzg_synth_layer_blobs failed")
        return out, bb
    ex = np.array(sorted(set(int(e) for e in experts)), np.int32)
    if lib.inzg_synth_layer_blobs_subset(layer, expert_type, H, FF, E, _p(ex), ex.size, _p(out)) != 0:
        raise RuntimeError("inzg_synth_layer_blobs_subset failed")
    return out, bb


def layer_blobs_range(layer, expert_type, H, FF, e0, e1):
    """Blobs of experts [e0, e1) of a synthetic layer (the same bytes as layer_blobs), [(e1 - e0) * blob_bytes]."""
    bb = blob_bytes(expert_type, H, FF)
    out = np.zeros((e1 - e0) * bb, np.uint8)
    if lib.inzg_synth_layer_blobs(layer, expert_type, H, FF, e0, e1, _p(out)) != 0:
        raise RuntimeError("inzg_synth_layer_blobs failed")
    return out, bb


def layer_blobs_device(layer, expert_type, H, FF, e0, e1, blobs_ptr, stream=None):
    """Experts [e0, e1) of a synthetic layer drawn and encoded on the current GPU into device memory at blobs_ptr
    ([(e1 - e0) * blob_bytes] bytes): the same stream as layer_blobs up to CUDA's double log/cos/sqrt in Box-Muller."""
    if lib.inzg_synth_layer_blobs_device(layer, expert_type, H, FF, e0, e1, ctypes.c_void_p(blobs_ptr),
                                         stream and ctypes.c_void_p(stream)) != 0:
        raise RuntimeError("inzg_synth_layer_blobs_device failed")


__all__ = ["router", "hidden", "normal_bias", "zipf_bias", "normal_logits", "layer_blobs", "layer_blobs_range",
           "layer_blobs_device", "blob_bytes", "expert_fp32", "T_Q4L", "T_Q8G"]
