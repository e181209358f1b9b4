"""Host-side mirror of the reference's MoE operator over the libinzg C ABI.

The reference engine calls ``moe_block(e, L, l, n, xin, y)`` (src/model_fwd.c:992) with the layer's router and the
expert cache behind it. :class:`MoePool` holds the same inputs on the device -- one router per layer
(``inzg_set_router``) and one HBM pool of expert blobs per layer (``inzg_pool_add_layer``, replacing the expert
cache) -- and :meth:`MoePool.moe_block` runs the routed layer, overwriting ``y`` like the reference (:1033).
Errors raise :class:`InzgError` carrying the C status (the reference exits through ``inz_die``).
"""
import ctypes

import numpy as np

from ._lib import (DUMP_ROUTE, EP_HANDLE_BYTES, GEMM_SIMT, IO_DEVICE, N_STAGES, NO_FUSED, NO_GRAPH, PROFILE, Config, InzgError, MoeOpts, Stats, T_Q4L,
                   T_Q8G, lib)


HC_RANK = 320  # INZG_HC_RANK: the hyper-connection bottleneck (src/model.h:14)


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class MoePool:
    def __init__(self, hidden=2048, ff=640, n_expert=512, topk=10, max_tokens=512, n_layers=1, device=0):
        cfg = Config(hidden, ff, n_expert, topk, max_tokens, n_layers, device)
        st = ctypes.c_int(0)
        self._ctx = lib.inzg_create(ctypes.byref(cfg), ctypes.byref(st))
        if not self._ctx:
            raise InzgError(st.value, "inzg_create failed")
        self.hidden, self.ff, self.n_expert, self.topk = hidden, ff, n_expert, topk
        self.max_tokens, self.n_layers, self.device = max_tokens, n_layers, device

    # -- lifetime --
    def close(self):
        if self._ctx:
            lib.inzg_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _check(self, status, what):
        if status != 0:
            raise InzgError(status, f"{what}: {lib.inzg_last_error(self._ctx).decode()}")

    # -- weights --
    def set_router(self, layer, w_f16):
        w = np.ascontiguousarray(w_f16, dtype=np.uint16)
        assert w.shape == (self.n_expert, self.hidden)
        self._check(lib.inzg_set_router(self._ctx, layer, _ptr(w), w.shape[0], w.shape[1]), "set_router")

    def add_layer(self, layer, expert_type, blobs, blob_bytes):
        b = np.ascontiguousarray(blobs, dtype=np.uint8)
        assert b.size >= blob_bytes * self.n_expert
        self._check(lib.inzg_pool_add_layer(self._ctx, layer, expert_type, _ptr(b), blob_bytes, self.n_expert),
                    "pool_add_layer")

    def add_layer_gguf(self, layer, gguf, gguf_layer=None):
        """Pool slot `layer` from an open :class:`inferenz_b200.gguf.GgufExperts` file (its layer `gguf_layer`,
        default `layer`), with the engine's checks on the file; uploads straight from the file mapping."""
        self._check(lib.inzg_pool_add_layer_gguf(self._ctx, layer, gguf.handle, layer if gguf_layer is None else gguf_layer),
                    "pool_add_layer_gguf")

    def add_layer_range(self, layer, expert_type, blobs, blob_bytes, e_first, n_local):
        """Experts [e_first, e_first + n_local) only (expert parallelism); blobs holds those n_local blobs."""
        b = np.ascontiguousarray(blobs, dtype=np.uint8)
        assert b.size >= blob_bytes * n_local
        self._check(lib.inzg_pool_add_layer_range(self._ctx, layer, expert_type, _ptr(b), blob_bytes, e_first, n_local),
                    "pool_add_layer_range")

    def add_layer_device(self, layer, expert_type, blobs_ptr, blob_bytes, e_first, n_local):
        """Experts [e_first, e_first + n_local) from blobs already in this pool's device memory (a device pointer)."""
        self._check(lib.inzg_pool_add_layer_device(self._ctx, layer, expert_type, ctypes.c_void_p(blobs_ptr), blob_bytes,
                                                   e_first, n_local), "pool_add_layer_device")

    def set_shared(self, layer, expert_type, blob, blob_bytes, gate):
        """The layer's shared expert: blob = gate|up then down (one expert blob's layout), gate [H] float32."""
        b = np.ascontiguousarray(blob, dtype=np.uint8)
        g = np.ascontiguousarray(gate, dtype=np.float32)
        assert g.shape == (self.hidden,) and b.size >= blob_bytes
        self._check(lib.inzg_set_shared(self._ctx, layer, expert_type, _ptr(b), blob_bytes, _ptr(g)), "set_shared")

    # -- hyper-connections around the layer (src/model_fwd.c:404-450, 1264-1267) --
    def set_hc(self, layer, norm, down, up, inject=None):
        """The layer's hyper-connection weights: norm [4H] f32, down [320][4H] and up [4H][320] as f16 bits (uint16),
        inject [4][4H] f32 or None."""
        W = 4 * self.hidden
        nm = np.ascontiguousarray(norm, dtype=np.float32)
        dn = np.ascontiguousarray(down, dtype=np.uint16)
        upm = np.ascontiguousarray(up, dtype=np.uint16)
        ij = None if inject is None else np.ascontiguousarray(inject, dtype=np.float32)
        assert nm.shape == (W,) and dn.shape == (HC_RANK, W) and upm.shape == (W, HC_RANK)
        assert ij is None or ij.shape == (4, W)
        self._check(lib.inzg_set_hc(self._ctx, layer, _ptr(nm), _ptr(dn), _ptr(upm), _ptr(ij)), "set_hc")

    def hc_in_device(self, layer, n, X_ptr, xin_ptr, inj_ptr=None, stream=None):
        self._check(lib.inzg_hc_in(self._ctx, layer, n, ctypes.c_void_p(X_ptr), ctypes.c_void_p(xin_ptr),
                                   inj_ptr and ctypes.c_void_p(inj_ptr), stream and ctypes.c_void_p(stream)), "hc_in")

    def hc_out_device(self, n, X_ptr, inj_ptr, y_ptr, stream=None):
        self._check(lib.inzg_hc_out(self._ctx, n, ctypes.c_void_p(X_ptr), ctypes.c_void_p(inj_ptr),
                                    ctypes.c_void_p(y_ptr), stream and ctypes.c_void_p(stream)), "hc_out")

    def moe_block_hc_device(self, layer, n, X_ptr, bias_ptr=None, override_ptr=None, stream=None, graph=True):
        """q_forward's MoE step on device pointers: X [n][4H] updated in place (hc_in, the layer, hc_out)."""
        opts = MoeOpts(IO_DEVICE | (0 if graph else NO_GRAPH), bias_ptr, override_ptr, stream)
        self._check(lib.inzg_moe_block_hc(self._ctx, layer, n, ctypes.c_void_p(X_ptr), ctypes.byref(opts)),
                    "moe_block_hc")

    # -- expert-parallel building blocks (device pointers as ints; stream-ordered, no synchronisation) --
    def route_device(self, layer, n, x_ptr, sel_ptr, w_ptr, bias_ptr=None, stream=None):
        self._check(lib.inzg_route(self._ctx, layer, n, ctypes.c_void_p(x_ptr), bias_ptr and ctypes.c_void_p(bias_ptr),
                                   ctypes.c_void_p(sel_ptr), ctypes.c_void_p(w_ptr), stream and ctypes.c_void_p(stream)),
                    "route")

    def experts_device(self, layer, m, x_ptr, sel_ptr, w_ptr, n_batch, out_ptr, stream=None):
        self._check(lib.inzg_moe_experts(self._ctx, layer, m, ctypes.c_void_p(x_ptr), ctypes.c_void_p(sel_ptr),
                                         ctypes.c_void_p(w_ptr), n_batch, ctypes.c_void_p(out_ptr),
                                         stream and ctypes.c_void_p(stream)), "moe_experts")

    def combine_device(self, n, slots_ptr, y_ptr, stream=None):
        self._check(lib.inzg_combine(self._ctx, n, ctypes.c_void_p(slots_ptr), ctypes.c_void_p(y_ptr),
                                     stream and ctypes.c_void_p(stream)), "combine")

    def shared_device(self, layer, n, x_ptr, y_ptr, n_batch, stream=None):
        self._check(lib.inzg_shared_expert(self._ctx, layer, n, ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr), n_batch,
                                           stream and ctypes.c_void_p(stream)), "shared_expert")

    # expert parallelism with the exchange in the library (peer memory; include/inzg.h inzg_ep_*)
    def ep_attach(self, rank, world, capacity):
        """This rank's exchange buffer; returns its handle (bytes) for the other ranks."""
        h = ctypes.create_string_buffer(EP_HANDLE_BYTES)
        self._check(lib.inzg_ep_attach(self._ctx, rank, world, capacity, h), "ep_attach")
        return h.raw

    def ep_connect(self, handles):
        """handles: every rank's ep_attach bytes, in rank order."""
        buf = ctypes.create_string_buffer(b"".join(handles), EP_HANDLE_BYTES * len(handles))
        self._check(lib.inzg_ep_connect(self._ctx, buf), "ep_connect")

    @staticmethod
    def ep_connect_local(pools):
        """Connects the exchange of pools living in this process (one per GPU, each attached, in rank order) through
        peer access between their devices."""
        arr = (ctypes.c_void_p * len(pools))(*[p._ctx for p in pools])
        st = lib.inzg_ep_connect_local(arr, len(pools))
        if st != 0:
            pools[0]._check(st, "ep_connect_local")

    def ep_forward_device(self, layer, n, x_ptr, y_ptr, n_batch, bias_ptr=None, stream=None):
        self._check(lib.inzg_ep_forward(self._ctx, layer, n, ctypes.c_void_p(x_ptr), bias_ptr and ctypes.c_void_p(bias_ptr),
                                        ctypes.c_void_p(y_ptr), n_batch, stream and ctypes.c_void_p(stream)), "ep_forward")

    def ep_barrier(self, stream=None):
        self._check(lib.inzg_ep_barrier(self._ctx, stream and ctypes.c_void_p(stream)), "ep_barrier")

    def ep_detach(self):
        self._check(lib.inzg_ep_detach(self._ctx), "ep_detach")

    def device_status(self, stream=None):
        self._check(lib.inzg_device_status(self._ctx, stream and ctypes.c_void_p(stream)), "device_status")

    # -- forward --
    def moe_block(self, layer, xin, bias=None, logits_override=None, dump=False, y=None, graph=True, simt_gemm=False,
                  fused=True):
        """y [n][H] = routed MoE layer of xin [n][H] (host arrays; copies in and out inside the call). fused=False runs
        calls of 1-2 tokens through the separate kernels instead of the single fused launch (a cross-check)."""
        x = np.ascontiguousarray(xin, dtype=np.float32)
        n = x.shape[0]
        y = np.empty_like(x) if y is None else y
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        o = None if logits_override is None else np.ascontiguousarray(logits_override, dtype=np.float32)
        flags = (DUMP_ROUTE if dump else 0) | (0 if graph else NO_GRAPH) | (GEMM_SIMT if simt_gemm else 0) | \
            (0 if fused else NO_FUSED)
        opts = MoeOpts(flags, None if b is None else b.ctypes.data,
                       None if o is None else o.ctypes.data, None)
        self._check(lib.inzg_moe_forward(self._ctx, layer, n, _ptr(x), _ptr(y), ctypes.byref(opts)), "moe_forward")
        return y

    def moe_block_device(self, layer, n, x_ptr, y_ptr, bias_ptr=None, override_ptr=None, stream=None, dump=False,
                         profile=False, graph=True, fused=True):
        """Stream-ordered call on device pointers (ints); returns immediately (profile=True: after the call)."""
        flags = IO_DEVICE | (DUMP_ROUTE if dump else 0) | (PROFILE if profile else 0) | (0 if graph else NO_GRAPH) | \
            (0 if fused else NO_FUSED)
        opts = MoeOpts(flags, bias_ptr, override_ptr, stream)
        self._check(lib.inzg_moe_forward(self._ctx, layer, n, ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr),
                                         ctypes.byref(opts)), "moe_forward")

    def route_dump(self, n):
        K, E = self.topk, self.n_expert
        sel = np.zeros((n, K), np.int32)
        w = np.zeros((n, K), np.float32)
        logits = np.zeros((n, E), np.float32)
        probs = np.zeros((n, E), np.float32)
        units = np.zeros(E, np.int32)
        nu = ctypes.c_int(0)
        self._check(lib.inzg_moe_route_dump(self._ctx, n, _ptr(sel), _ptr(w), _ptr(logits), _ptr(probs), _ptr(units),
                                            ctypes.byref(nu)), "route_dump")
        return {"sel": sel, "w": w, "logits": logits, "probs": probs, "units": units[:nu.value]}

    def stage_times(self, reset=True):
        """{stage name: ms summed over profiled calls}, number of profiled calls"""
        ms = (ctypes.c_double * N_STAGES)()
        calls = ctypes.c_uint64(0)
        self._check(lib.inzg_stage_times(self._ctx, ms, ctypes.byref(calls), 1 if reset else 0), "stage_times")
        return {lib.inzg_stage_name(i).decode(): ms[i] for i in range(N_STAGES)}, calls.value

    def stats(self):
        s = Stats()
        self._check(lib.inzg_get_stats(self._ctx, ctypes.byref(s)), "get_stats")
        return {f: getattr(s, f) for f, _ in Stats._fields_}


__all__ = ["MoePool", "InzgError", "T_Q4L", "T_Q8G"]
