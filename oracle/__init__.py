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
REFERENCE_TREE = "/root/reference"

P, I, U32, U64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float
T_Q4L, T_Q8G = 102, 103


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
