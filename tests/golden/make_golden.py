"""Generate the golden fixtures of tests/golden/ from the reference's own compiled MoE path (oracle/_ref).

Run here, where the reference tree was present when oracle/_ref was built:
    python tests/golden/make_golden.py
Inputs are not stored: they are regenerated from seeds by the oracle's copy of the reference tests' generator (the
streams inferenz_b200.synth draws too), the experts encoded by the reference's own quantizer (oracle.ref_layer_blobs);
the fixture keeps a SHA-256 of every expert blob it used so a test can prove regenerated inputs are the same bytes.
Outputs are the reference's: logits, probabilities, top-k, renormalised weights, first-touch unit order, y; and for the
hyper-connection steps around the layer (hc.npz), hc_in's xin and inj and hc_out's updated residual; and Q4N payloads
with their products (q4n.npz).
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

FF, E, K = 640, 512, 10
T_Q4L, T_Q8G = oracle.T_Q4L, oracle.T_Q8G

# name: (n tokens, expert type, routing hook, hidden size). The override cases put 3 experts in every token's top-10
# (they get the prefill GEMM numerics: >= 12 tokens) next to a long tail of decode experts.
CASES = {
    "decode_n1_q4l": (1, T_Q4L, None, 2048),
    "decode_n4_q4l_bias": (4, T_Q4L, "bias", 2048),
    "prefill_n48_q4l_override": (48, T_Q4L, "override", 2048),
    "decode_n4_q8g_bias": (4, T_Q8G, "bias", 2048),
    "prefill_n40_q8g_override": (40, T_Q8G, "override", 2048),
    "prefill_n24_q4l_h2560_override": (24, T_Q4L, "override", 2560),
}


def case_inputs(name):
    """(n, expert type, H, router, x, bias, logits override) of a golden case"""
    n, typ, hook, H = CASES[name]
    R = oracle.synth_router(0, E, H)
    x = oracle.synth_hidden(n, H)
    bias = oracle.normal_bias(E) if hook == "bias" else None
    ov = None
    if hook == "override":
        ov = oracle.normal_logits(n, E)
        ov[:, :3] += 6.0
    return n, typ, H, R, x, bias, ov


# The benchmark's timed workloads (bench.py make_inputs), as the reference computes them: name -> (n, type, hook).
BENCH_CASES = {
    "decode1": (1, T_Q4L, None),
    "decode32": (32, T_Q4L, "bias"),
    "prefill4096": (4096, T_Q4L, "zipf"),
    "q8g2048": (2048, T_Q8G, "logits"),
}
BENCH_SAMPLE_ROWS = 24  # full output rows kept per large workload (evenly spaced tokens, first and last included)


def bench_inputs(name):
    """(n, type, router, x, bias, logits override) of a benchmark workload; layer 0, H = 2048"""
    n, typ, hook = BENCH_CASES[name]
    R = oracle.synth_router(0, E, 2048)
    x = oracle.synth_hidden(n, 2048)
    bias = oracle.normal_bias(E) if hook == "bias" else oracle.zipf_bias(E) if hook == "zipf" else None
    ov = oracle.normal_logits(n, E) if hook == "logits" else None
    return n, typ, R, x, bias, ov


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bench_fixture(name, threads=0):
    """Compact record of the reference's output on a benchmark workload: routing as hashes of its exact bits (logits,
    probabilities, renormalised weights) plus top-k and unit order, per-token output norms, and full output rows of
    sampled tokens (all rows for small n)."""
    n, typ, R, x, bias, ov = bench_inputs(name)
    orc = oracle.Oracle()
    sel = oracle.routing(orc, R, x, bias=bias, override=ov)
    blobs, bb = oracle.ref_layer_blobs(0, typ, 2048, FF, E, experts=np.unique(sel))
    ref = oracle.Ref(2048, threads=threads, expert_type=typ)
    d = ref.moe_routed(R, blobs, bb, x, bias=bias, override=ov)
    isa = ref.isa
    ref.close()
    rows = np.arange(n) if n <= 64 else np.unique(np.linspace(0, n - 1, BENCH_SAMPLE_ROWS).round().astype(np.int64))
    return dict(sel=d["sel"], units=d["units"], w_sha=sha(d["w"]), logits_sha=sha(d["logits"]),
                probs_sha=sha(d["probs"]), y_norm=np.linalg.norm(d["y"].astype(np.float64), axis=1),
                y_rows=rows, y_sample=d["y"][rows], experts=np.unique(sel), isa=np.array(isa))


def blob_hashes(blobs, bb, experts):
    return np.array([hashlib.sha256(blobs[e * bb:(e + 1) * bb].tobytes()).hexdigest() for e in experts])


def quant_fixture(ref):
    """Small matrices quantized by the reference quantizer (bytes kept whole)."""
    out = {}
    for i, (rows, cols, typ, rot) in enumerate([(64, 320, 102, 64), (16, 640, 102, 0), (9, 320, 103, -1),
                                                (32, 256, 103, 128)]):
        w = oracle.synth_randn(100 + i, rows * cols, 0.03).reshape(rows, cols)
        out[f"q{i}_shape"] = np.array([rows, cols, typ, rot])
        out[f"q{i}_bytes"] = ref.quantize(w, typ, rot_block=rot, seed=0, threads=1)
    return out


HC_CASES = {2048: 2, 2560: 2}  # hidden size -> tokens of the hyper-connection fixture


def hc_inputs(H):
    """(hc weights, X, y) of the hyper-connection fixture at hidden size H"""
    n = HC_CASES[H]
    return oracle.synth_hc(1, H=H), oracle.synth_residual(n, H=H, seed=300), oracle.synth_hidden(n, H=H, seed=301)


def hc_fixture():
    """The reference's own hc_in (xin, inj) and hc_out (the updated residual) on seeded inputs, both widths; the
    inputs' SHA-256 so a test can prove the regenerated inputs are the same bytes."""
    out = {}
    for H in HC_CASES:
        hc, X, y = hc_inputs(H)
        ref = oracle.Ref(H, threads=0)
        xin, inj = ref.hc_in(hc, X)
        out[f"h{H}_xin"], out[f"h{H}_inj"] = xin, inj
        out[f"h{H}_xout"] = ref.hc_out(X, inj, y)
        out[f"h{H}_sha"] = np.array([sha(hc[k]) for k in ("norm", "down", "up", "inject")] + [sha(X), sha(y)])
        ref.close()
    return out


Q4N_SHAPES = [(64, 2048), (96, 640)]
Q4N_CALLS = [(1, False), (5, False), (12, True)]  # (tokens, GEMM numerics): mv_q4n, mm_q4n, the Q4N GEMM tile


def q4n_fixture():
    """Q4N payloads written by the reference quantizer (bytes kept whole: the oracle has no Q4N quantizer) and the
    reference's products through lin_mm's three numeric paths on seeded tokens."""
    out = {}
    ref = oracle.Ref(2048, threads=0)
    for i, (rows, cols) in enumerate(Q4N_SHAPES):
        W = oracle.synth_randn(700 + rows, rows * cols, (1.0 / cols) ** 0.5).reshape(rows, cols)
        pl = ref.quantize(W, oracle.T_Q4N)
        out[f"m{i}_payload"] = pl
        for n, gemm in Q4N_CALLS:
            out[f"m{i}_n{n}"] = ref.matmul(pl, oracle.synth_hidden(n, cols, seed=800 + n), gemm=gemm)
    ref.close()
    return out


def main():
    orc = oracle.Oracle()
    only = sys.argv[1:]
    for name in CASES:
        if only and name not in only:
            continue
        n, typ, H, R, x, bias, ov = case_inputs(name)
        ref = oracle.Ref(H, threads=0, expert_type=typ)
        sel = oracle.routing(orc, R, x, bias=bias, override=ov)
        experts = np.unique(sel)
        blobs, bb = oracle.ref_layer_blobs(0, typ, H, FF, E, experts=experts)
        d = ref.moe_routed(R, blobs, bb, x, bias=bias, override=ov)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), logits=d["logits"], probs=d["probs"], sel=d["sel"],
                            w=d["w"], units=d["units"], y=d["y"], experts=experts,
                            blob_sha256=blob_hashes(blobs, bb, experts), isa=np.array(ref.isa))
        print(name, "units", len(d["units"]), "isa", ref.isa)
        ref.close()
    for name in BENCH_CASES:
        if only and f"bench_{name}" not in only:
            continue
        np.savez_compressed(os.path.join(HERE, f"bench_{name}.npz"), **bench_fixture(name))
        print("bench", name)
    if not only or "hc" in only:
        np.savez_compressed(os.path.join(HERE, "hc.npz"), **hc_fixture())
        print("hc")
    if not only or "q4n" in only:
        np.savez_compressed(os.path.join(HERE, "q4n.npz"), **q4n_fixture())
        print("q4n")
    if not only or "quantizer" in only:
        ref = oracle.Ref(2048, threads=0)
        np.savez_compressed(os.path.join(HERE, "quantizer.npz"), **quant_fixture(ref))
        ref.close()


if __name__ == "__main__":
    main()
