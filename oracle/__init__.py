"""TEST INFRASTRUCTURE ONLY -- the checker of the CUDA path. Never imported by the product (inferenz_b200/).

Two legs, both CPU:
  * ``Oracle``: liboracle.so, the plain-C restatement of the reference's MoE arithmetic (moe_oracle.c), built from
    this repository alone;
  * ``Ref``: oracle/_ref/libinzref_<isa>_h<H>.so, the reference's own MoE sources compiled from the reference tree
    with ref_harness.c (only where the reference tree was present at build time; the built library travels with the
    repository snapshot). ``<isa>`` is picked from the host CPU: AVX512-VNNI when available, else AVX2.
Allowed users: tests/, __graft_entry__.smoke(), and bench.py's CPU-baseline / reference arm.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
# the reference checkout to compile oracle/_ref from: $INZ_REFERENCE_TREE, else a `reference` directory beside the
# repository
REFERENCE_TREE = os.environ.get("INZ_REFERENCE_TREE",
                                os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

P, I, U32, U64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float
T_Q4L, T_Q8G, T_Q4N = 102, 103, 107


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def build(jobs=8):
    """Build liboracle.so, and the reference harness libraries when the reference tree is present."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", HERE, "oracle"], check=True)
    if os.path.exists(os.path.join(REFERENCE_TREE, "src", "model_fwd.c")):
        subprocess.run(["make", "-s", f"-j{jobs}", "-C", HERE, "ref", f"REF={REFERENCE_TREE}"], check=True)


def host_isa():
    try:
        flags = open("/proc/cpuinfo").read().split("flags")[1].split("\n")[0].split()
    except Exception:
        return "avx2"
    return "avx512vnni" if ("avx512_vnni" in flags and "avx512vl" in flags) else "avx2"


_ORC = None


def _orc():
    """liboracle.so with the signatures of its synthetic-input generator."""
    global _ORC
    if _ORC is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        for name, res, args in [("orc_synth_jump", U64, [U64, U64]), ("orc_synth_randn", U64, [U64, ctypes.c_int64, F, P]),
                                ("orc_synth_expert", None, [U64, I, I, I, P, P]), ("orc_synth_router", None, [U64, I, I, P]),
                                ("orc_synth_hidden", None, [U64, I, I, P])]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _ORC = L
    return _ORC


# Seeded synthetic inputs of the benchmark configurations, drawn by the oracle's copy of the reference tests'
# generator (the same streams and seeds as the product's inferenz_b200.synth): experts of layer l from seed l, router
# of layer l from seed 1000 + l, hidden states from seed 1, N(0, 1) logit bias from seed 2, N(0, 1) logits from seed 4.
ROUTER_SEED_BASE, HIDDEN_SEED, BIAS_SEED, OVERRIDE_SEED = 1000, 1, 2, 4


def synth_randn(seed, n, scale=1.0):
    out = np.empty(n, np.float32)
    _orc().orc_synth_randn(seed, n, scale, _p(out))
    return out


def synth_router(layer, E=512, H=2048):
    w = np.empty((E, H), np.uint16)
    _orc().orc_synth_router(ROUTER_SEED_BASE + layer, E, H, _p(w))
    return w


def synth_hidden(n, H=2048, seed=HIDDEN_SEED):
    x = np.empty((n, H), np.float32)
    _orc().orc_synth_hidden(seed, n, H, _p(x))
    return x


def synth_expert(layer, e, H=2048, FF=640):
    gu = np.empty((2 * FF, H), np.float32)
    dn = np.empty((H, FF), np.float32)
    _orc().orc_synth_expert(layer, H, FF, e, _p(gu), _p(dn))
    return gu, dn


def synth_hc(layer, H=2048, rank=320, seed=0x4843):
    """Hyper-connection weights of one block (the hcw of src/engine_internal.h:27-32) with magnitudes like a trained
    model's: norm = 1 + w (folded, small w), down [rank][4H] and up [4H][rank] as f16 bits, inject [4][4H]."""
    W = 4 * H
    st = seed * 1000003 + layer
    norm = 1.0 + 0.1 * synth_randn(st, W)
    down = _f16_bits(synth_randn(st + 1, rank * W, (1.0 / W) ** 0.5).reshape(rank, W))
    up = _f16_bits(synth_randn(st + 2, W * rank, (1.0 / rank) ** 0.5).reshape(W, rank))
    inject = synth_randn(st + 3, 4 * W, (1.0 / W) ** 0.5).reshape(4, W)
    return {"norm": np.ascontiguousarray(norm, np.float32), "down": down, "up": up,
            "inject": np.ascontiguousarray(inject, np.float32)}


def synth_residual(n, H=2048, seed=0x5245):
    """The residual stream X [n][4H] entering hc_in: four streams of hidden-state scale."""
    return np.ascontiguousarray(synth_randn(seed, n * 4 * H).reshape(n, 4 * H), np.float32)


def _f16_bits(a):
    return np.ascontiguousarray(np.asarray(a, np.float32).astype(np.float16).view(np.uint16))


def normal_bias(E=512, seed=BIAS_SEED):
    return synth_randn(seed, E)


def zipf_bias(E=512, s=1.1):
    p = (np.arange(1, E + 1, dtype=np.float64)) ** (-s)
    return np.log(p / p.sum()).astype(np.float32)


def normal_logits(n, E=512, seed=OVERRIDE_SEED):
    return synth_randn(seed, n * E).reshape(n, E)


def ref_layer_blobs(layer, typ, H=2048, FF=640, E=512, experts=None, threads=None, isa=None):
    """Blobs [E * blob_bytes] of a synthetic layer, encoded by the reference's own quantizer (oracle/_ref:
    ref_encode_expert, the converter's recipe) from the oracle generator's draws, experts in parallel. ``experts``:
    only these are generated; the others get the first listed expert's two headers and a zero payload (valid blobs
    that must not be routed to). Returns (blobs, blob_bytes)."""
    from concurrent.futures import ThreadPoolExecutor
    isa = isa or host_isa()
    path = os.path.join(REF_DIR, f"libinzref_{isa}_h{H}.so")
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    L = ctypes.CDLL(path)
    L.ref_blob_bytes.restype, L.ref_blob_bytes.argtypes = U64, [I]
    L.ref_qmat_bytes.restype, L.ref_qmat_bytes.argtypes = ctypes.c_size_t, [I, I, I]
    L.ref_encode_expert.restype, L.ref_encode_expert.argtypes = None, [P, P, I, I, P]
    bb = int(L.ref_blob_bytes(typ))
    gub = int(L.ref_qmat_bytes(typ, 2 * FF, H))
    out = np.zeros(E * bb, np.uint8)
    ex = list(range(E)) if experts is None else sorted(set(int(e) for e in experts))

    def one(e):
        gu, dn = synth_expert(layer, e, H, FF)
        L.ref_encode_expert(_p(gu), _p(dn), typ, 1, ctypes.c_void_p(out.ctypes.data + e * bb))

    with ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1) as pool:
        list(pool.map(one, ex))
    for e in range(E):
        if e not in ex:
            out[e * bb:e * bb + 64] = out[ex[0] * bb:ex[0] * bb + 64]
            out[e * bb + gub:e * bb + gub + 64] = out[ex[0] * bb + gub:ex[0] * bb + gub + 64]
    return out, bb


class Oracle:
    """The C restatement. q8_vnni=1 follows the VNNI form of the Q8G decode kernel (src/quant.c:909-915)."""

    def __init__(self, q8_vnni=1):
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        self.lib = ctypes.CDLL(path)
        L = self.lib
        for name, res, args in [
            ("orc_qmat_bytes", ctypes.c_size_t, [I, I, I]),
            ("orc_f16_to_f32", F, [ctypes.c_uint16]),
            ("orc_router_logits", None, [P, I, I, P, I, P]),
            ("orc_softmax", None, [P, I]),
            ("orc_topk", I, [P, I, I, P]),
            ("orc_rotate", None, [P, I, I, U32]),
            ("orc_act_quantize", None, [P, I, I, U32, P, P, P]),
            ("orc_xq", None, [P, I, I, U32, P, P, P]),
            ("orc_moe_routed", I, [I, I, I, I, P, P, U64, U64, I, P, P, P, P, P, P, P, P, P, P, I]),
            ("orc_hc_in", None, [I, I, P, P, P, P, I, P, P, P]),
            ("orc_matmul_payload", I, [P, I, P, P, I, I]),
            ("orc_hc_out", None, [I, I, P, P, P]),
        ]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        self.q8_vnni = q8_vnni

    def router_logits(self, W, X):
        E, H = W.shape
        n = X.shape[0]
        Y = np.zeros((n, E), np.float32)
        self.lib.orc_router_logits(_p(W), E, H, _p(np.ascontiguousarray(X, np.float32)), n, _p(Y))
        return Y

    def softmax(self, s):
        s = np.array(s, np.float32)
        self.lib.orc_softmax(_p(s), s.size)
        return s

    def topk(self, x, k):
        idx = np.zeros(k, np.int32)
        self.lib.orc_topk(_p(np.ascontiguousarray(x, np.float32)), x.size, k, _p(idx))
        return idx

    def act_quantize(self, x, rot, seed):
        x = np.ascontiguousarray(x, np.float32)
        n = x.size
        q = np.zeros(n, np.int8)
        s = np.zeros(n // 64, np.float32)
        b = np.zeros(n // 64, np.float32)
        self.lib.orc_act_quantize(_p(x), n, rot, seed, _p(q), _p(s), _p(b))
        return q, s, b

    def xq(self, x, rot, seed):
        x = np.ascontiguousarray(x, np.float32)
        K = x.size
        nkb = (K + 255) // 256
        q = np.zeros(K, np.int8)
        s = np.zeros(nkb, np.float32)
        sm = np.zeros(nkb, np.int32)
        self.lib.orc_xq(_p(x), K, rot, seed, _p(q), _p(s), _p(sm))
        return q, s, sm

    def matmul(self, payload, X, gemm=False):
        """Y [n][rows] = one quantized matrix (any of Q4L / Q8G / Q4N) times n tokens with lin_mm's numerics: decode
        (gemm=False) or prefill GEMM (gemm=True)."""
        X = np.ascontiguousarray(X, np.float32)
        n = X.shape[0]
        rows = int(np.frombuffer(np.ascontiguousarray(payload, np.uint8)[8:12].tobytes(), np.uint32)[0])
        Y = np.zeros((n, rows), np.float32)
        if self.lib.orc_matmul_payload(_p(np.ascontiguousarray(payload, np.uint8)), n, _p(X), _p(Y), int(gemm),
                                       self.q8_vnni) != 0:
            raise ValueError("oracle: payload or shape not covered")
        return Y

    def hc_in(self, hc, X):
        """hc_in (src/model_fwd.c:404-439): X [n][4H] -> (xin [n][H], inj [n][4]); hc: dict from synth_hc."""
        n, W = X.shape
        H, rank = W // 4, hc["down"].shape[0]
        xin = np.zeros((n, H), np.float32)
        inj = np.zeros((n, 4), np.float32)
        inject = hc.get("inject")
        self.lib.orc_hc_in(H, rank, _p(hc["norm"]), _p(hc["down"]), _p(hc["up"]), _p(inject), n,
                           _p(np.ascontiguousarray(X, np.float32)), _p(xin), _p(inj if inject is not None else None))
        return xin, inj

    def hc_out(self, X, inj, y):
        """hc_out (src/model_fwd.c:442-450): returns X + inj_s * y per stream (one fma per element)."""
        n, W = X.shape
        Xo = np.ascontiguousarray(X, np.float32).copy()
        self.lib.orc_hc_out(W // 4, n, _p(Xo), _p(np.ascontiguousarray(inj, np.float32)),
                            _p(np.ascontiguousarray(y, np.float32)))
        return Xo

    def moe_routed(self, router, blobs, blob_bytes, gu_bytes, xin, bias=None, override=None, H=2048, FF=640, E=512,
                   topk=10, dumps=True):
        n = xin.shape[0]
        y = np.zeros((n, H), np.float32)
        d = {}
        if dumps:
            d = {"logits": np.zeros((n, E), np.float32), "probs": np.zeros((n, E), np.float32),
                 "sel": np.zeros((n, topk), np.int32), "w": np.zeros((n, topk), np.float32),
                 "units": np.zeros(E, np.int32), "moe_out": np.zeros((n, topk, H), np.float32)}
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        o = None if override is None else np.ascontiguousarray(override, np.float32)
        nu = self.lib.orc_moe_routed(H, FF, E, topk, _p(router), _p(blobs), blob_bytes, gu_bytes, n,
                                     _p(np.ascontiguousarray(xin, np.float32)), _p(b), _p(o), _p(y),
                                     _p(d.get("logits")), _p(d.get("probs")), _p(d.get("sel")), _p(d.get("w")),
                                     _p(d.get("units")), _p(d.get("moe_out")), self.q8_vnni)
        if nu < 0:
            raise RuntimeError("oracle: corrupt blob")
        if dumps:
            d["units"] = d["units"][:nu]
        d["y"] = y
        return d


class Ref:
    """The reference's own MoE path (compiled from the reference tree). Raises FileNotFoundError if not built."""

    def __init__(self, hidden=2048, threads=0, expert_type=T_Q4L, isa=None):
        isa = isa or host_isa()
        path = os.path.join(REF_DIR, f"libinzref_{isa}_h{hidden}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path, self.isa_variant = path, isa
        self.lib = ctypes.CDLL(path)
        L = self.lib
        for name, res, args in [
            ("ref_hidden", I, []), ("ref_isa", ctypes.c_char_p, []), ("ref_ctx_create", P, [I, I]),
            ("ref_ctx_destroy", None, [P]), ("ref_tp_size", I, [P]), ("ref_qmat_bytes", ctypes.c_size_t, [I, I, I]),
            ("ref_quantize", ctypes.c_double, [P, I, I, I, I, U32, I, P]), ("ref_blob_bytes", U64, [I]),
            ("ref_encode_expert", None, [P, P, I, I, P]), ("ref_router_logits", None, [P, I, P, P]),
            ("ref_softmax", None, [P, I]), ("ref_topk", I, [P, I, I, P]),
            ("ref_act_quantize", None, [P, I, I, U32, P, P, P]), ("ref_matmul_decode", None, [P, I, P, P]),
            ("ref_matmul_gemm", None, [P, I, P, P]), ("ref_xq", None, [P, I, I, I, U32, P, P, P]),
            ("ref_moe_routed", I, [P, P, P, U64, I, P, P, P, P, P, P, P, P, P, P]),
            ("ref_shared", I, [P, P, U64, I, P, I, P, P, P]),
            ("ref_hc_rank", I, []), ("ref_hc_in", I, [P, P, P, P, P, I, P, P, P]), ("ref_hc_out", None, [I, P, P, P]),
        ]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        self.H = L.ref_hidden()
        self.ctx = L.ref_ctx_create(threads, expert_type)
        self.threads = L.ref_tp_size(self.ctx)
        self.isa = L.ref_isa().decode()

    def close(self):
        if self.ctx:
            self.lib.ref_ctx_destroy(self.ctx)
            self.ctx = None

    def quantize(self, W, typ, rot_block=0, seed=0, threads=1):
        rows, cols = W.shape
        out = np.zeros(self.lib.ref_qmat_bytes(typ, rows, cols), np.uint8)
        self.lib.ref_quantize(_p(np.ascontiguousarray(W, np.float32)), rows, cols, typ, rot_block, seed, threads,
                              _p(out))
        return out

    def moe_routed(self, router, blobs, blob_bytes, xin, bias=None, override=None, E=512, topk=10, dumps=True):
        n, H = xin.shape
        y = np.zeros((n, H), np.float32)
        d = {}
        if dumps:
            d = {"logits": np.zeros((n, E), np.float32), "probs": np.zeros((n, E), np.float32),
                 "sel": np.zeros((n, topk), np.int32), "w": np.zeros((n, topk), np.float32),
                 "units": np.zeros(E, np.int32), "moe_out": np.zeros((n, topk, H), np.float32)}
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        o = None if override is None else np.ascontiguousarray(override, np.float32)
        nu = self.lib.ref_moe_routed(self.ctx, _p(router), _p(blobs), blob_bytes, n,
                                     _p(np.ascontiguousarray(xin, np.float32)), _p(b), _p(o), _p(y),
                                     _p(d.get("logits")), _p(d.get("probs")), _p(d.get("sel")), _p(d.get("w")),
                                     _p(d.get("units")), _p(d.get("moe_out")))
        if nu < 0:
            raise RuntimeError("reference: corrupt blob")
        if dumps:
            d["units"] = d["units"][:nu]
        d["y"] = y
        return d


    def shared(self, blob, gu_bytes, typ, gate, xin, y):
        """y + sigmoid(gate . x) * shared_expert(x), the reference's own shared-expert step; returns (y_new, D)."""
        n, H = xin.shape
        yo = np.ascontiguousarray(y, np.float32).copy()
        D = np.zeros((n, H), np.float32)
        rc = self.lib.ref_shared(self.ctx, _p(np.ascontiguousarray(blob, np.uint8)), gu_bytes, typ,
                                 _p(np.ascontiguousarray(gate, np.float32)), n,
                                 _p(np.ascontiguousarray(xin, np.float32)), _p(yo), _p(D))
        if rc != 0:
            raise RuntimeError("reference: shared expert matrices do not match")
        return yo, D


    def matmul(self, payload, X, gemm=False):
        """The reference's own lin_mm numerics for one quantized matrix: inz_matvec_rows / inz_matmul_rows after
        per-token activation quantization (gemm=False), or inz_gemm_rows (gemm=True)."""
        X = np.ascontiguousarray(X, np.float32)
        n = X.shape[0]
        pl = np.ascontiguousarray(payload, np.uint8)
        rows = int(np.frombuffer(pl[8:12].tobytes(), np.uint32)[0])
        Y = np.zeros((n, rows), np.float32)
        (self.lib.ref_matmul_gemm if gemm else self.lib.ref_matmul_decode)(_p(pl), n, _p(X), _p(Y))
        return Y

    def hc_in(self, hc, X):
        """The reference's own hc_in; same arguments and results as Oracle.hc_in."""
        n, W = X.shape
        assert W == 4 * self.H and hc["down"].shape == (self.lib.ref_hc_rank(), W)
        xin = np.zeros((n, self.H), np.float32)
        inj = np.zeros((n, 4), np.float32)
        inject = hc.get("inject")
        rc = self.lib.ref_hc_in(self.ctx, _p(hc["norm"]), _p(hc["down"]), _p(hc["up"]), _p(inject), n,
                                _p(np.ascontiguousarray(X, np.float32)), _p(xin),
                                _p(inj if inject is not None else None))
        if rc != 0:
            raise RuntimeError("reference: bad hc_in call")
        return xin, inj

    def hc_out(self, X, inj, y):
        """The reference's own hc_out; returns the updated copy of X."""
        n = X.shape[0]
        Xo = np.ascontiguousarray(X, np.float32).copy()
        self.lib.ref_hc_out(n, _p(Xo), _p(np.ascontiguousarray(inj, np.float32)),
                            _p(np.ascontiguousarray(y, np.float32)))
        return Xo


class RefGguf:
    """The reference's own GGUF reader and writer (src/gguf.c) through _ref/libinzref_gguf.so (ref_gguf.c)."""

    def __init__(self):
        path = os.path.join(REF_DIR, "libinzref_gguf.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = ctypes.CDLL(path)
        self.lib.ref_gguf_tensor.restype = I
        self.lib.ref_gguf_tensor.argtypes = [ctypes.c_char_p, ctypes.c_char_p, P, P, P, P, P, ctypes.c_char_p,
                                             ctypes.c_size_t]
        self.lib.ref_gguf_write.restype = I
        self.lib.ref_gguf_write.argtypes = [ctypes.c_char_p, U64, I, I, U32, U64, I, P, U64]

    def tensor(self, path, name):
        """setup_experts' view of tensor `name` (src/engine.c:337-350): None when gguf_open fails or the tensor is
        absent, else a dict of its absolute offset and size, the expert type, blob size and alignment."""
        off, nb, al = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        et, bb = ctypes.c_int64(), ctypes.c_int64()
        err = ctypes.create_string_buffer(256)
        rc = self.lib.ref_gguf_tensor(str(path).encode(), name.encode(), ctypes.byref(off), ctypes.byref(nb),
                                      ctypes.byref(et), ctypes.byref(bb), ctypes.byref(al), err, len(err))
        if rc != 0:
            return None
        return {"offset": off.value, "nbytes": nb.value, "expert_type": et.value, "blob_bytes": bb.value,
                "alignment": al.value}

    def write(self, path, blobs, blob_bytes, n_expert, n_layers, mtp=False, expert_type=T_Q4L, alignment=32,
              extra_floats=0):
        """A model-shaped GGUF written by the reference's writer (ref_gguf.c). blobs: the expert tensors of the
        n_layers layers (then mtp.experts when mtp), n_expert * blob_bytes bytes each, back to back."""
        b = np.ascontiguousarray(blobs, dtype=np.uint8)
        assert b.size == blob_bytes * n_expert * (n_layers + int(mtp))
        rc = self.lib.ref_gguf_write(str(path).encode(), alignment, n_layers, int(mtp), expert_type, blob_bytes,
                                     n_expert, _p(b), extra_floats)
        assert rc == 0, "reference GGUF writer failed"


def routing(orc, router, xin, bias=None, override=None, topk=10):
    """Experts selected per token (oracle arithmetic), to know which experts a test must quantize."""
    lg = override.copy() if override is not None else orc.router_logits(router, xin)
    if override is None and bias is not None:
        lg = (lg + bias[None, :]).astype(np.float32)
    sel = np.zeros((xin.shape[0], topk), np.int32)
    for t in range(xin.shape[0]):
        sel[t] = orc.topk(orc.softmax(lg[t]), topk)
    return sel


def rel_l2(a, b):
    """per-row ||a - b|| / ||b|| (rows = tokens)"""
    a = a.reshape(a.shape[0], -1).astype(np.float64)
    b = b.reshape(b.shape[0], -1).astype(np.float64)
    return np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-30)
