"""Generate the golden fixtures of tests/golden/ from the reference's own compiled MoE path (oracle/_ref).

Run here, where the reference tree was present when oracle/_ref was built:
    python tests/golden/make_golden.py
Inputs are not stored: they are regenerated from seeds by inferenz_b200.synth (deterministic), and the fixture keeps
a SHA-256 of every expert blob it used so a test can prove the regenerated inputs are the same bytes. Outputs are the
reference's: logits, probabilities, top-k, renormalised weights, first-touch unit order, y.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from inferenz_b200 import synth  # noqa: E402

H, FF, E, K = 2048, 640, 512, 10

# name: (n tokens, expert type, routing hook)
CASES = {
    "decode_n1_q4l": (1, synth.T_Q4L, None),
    "decode_n4_q4l_bias": (4, synth.T_Q4L, "bias"),
    "prefill_n48_q4l_override": (48, synth.T_Q4L, "override"),
    "decode_n4_q8g_bias": (4, synth.T_Q8G, "bias"),
}


def case_inputs(name):
    n, typ, hook = CASES[name]
    R = synth.router(0, E, H)
    x = synth.hidden(n, H)
    bias = synth.normal_bias(E) if hook == "bias" else None
    ov = None
    if hook == "override":
        ov = synth.normal_logits(n, E)
        ov[:, :3] += 6.0
    return n, typ, R, x, bias, ov


def blob_hashes(blobs, bb, experts):
    return np.array([hashlib.sha256(blobs[e * bb:(e + 1) * bb].tobytes()).hexdigest() for e in experts])


def quant_fixture(ref):
    """Small matrices quantized by the reference quantizer (bytes kept whole)."""
    out = {}
    for i, (rows, cols, typ, rot) in enumerate([(64, 320, 102, 64), (16, 640, 102, 0), (9, 320, 103, -1),
                                                (32, 256, 103, 128)]):
        w = synth.randn(100 + i, rows * cols, 0.03).reshape(rows, cols)
        out[f"q{i}_shape"] = np.array([rows, cols, typ, rot])
        out[f"q{i}_bytes"] = ref.quantize(w, typ, rot_block=rot, seed=0, threads=1)
    return out


def main():
    orc = oracle.Oracle()
    for name in CASES:
        n, typ, R, x, bias, ov = case_inputs(name)
        ref = oracle.Ref(H, threads=0, expert_type=typ)
        sel = oracle.routing(orc, R, x, bias=bias, override=ov)
        experts = np.unique(sel)
        blobs, bb = synth.layer_blobs(0, typ, H, FF, E, experts=experts)
        d = ref.moe_routed(R, blobs, bb, x, bias=bias, override=ov)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), logits=d["logits"], probs=d["probs"], sel=d["sel"],
                            w=d["w"], units=d["units"], y=d["y"], experts=experts,
                            blob_sha256=blob_hashes(blobs, bb, experts), isa=np.array(ref.isa))
        print(name, "units", len(d["units"]), "isa", ref.isa)
        ref.close()
    ref = oracle.Ref(H, threads=0)
    np.savez_compressed(os.path.join(HERE, "quantizer.npz"), **quant_fixture(ref))
    ref.close()


if __name__ == "__main__":
    main()
