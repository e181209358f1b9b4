"""The routed-expert tensors of the engine's GGUF model file (include/inzg.h, inzg_gguf_*).

:class:`GgufExperts` opens the file the way the reference engine's setup_experts sees it (src/engine.c:336-351):
the expert type and blob size from its key/values, and one ``blk.%d.experts`` tensor per layer (``mtp.experts`` as
layer ``n_layers``). The file stays mapped until :meth:`close`; :meth:`MoePool.add_layer_gguf` uploads a layer from it.
"""
import ctypes

import numpy as np

from ._lib import GgufInfo, InzgError, lib


class GgufExperts:
    def __init__(self, path):
        info = GgufInfo()
        err = ctypes.create_string_buffer(512)
        h = lib.inzg_gguf_open(str(path).encode(), ctypes.byref(info), err, len(err))
        self._h = None
        if not h:
            raise InzgError(1, err.value.decode())
        self._h = h
        self.path = str(path)
        self.expert_type = info.expert_type
        self.blob_bytes = info.blob_bytes
        self.n_layers = info.n_layers
        self.has_mtp = bool(info.has_mtp)
        self.alignment = info.alignment
        self.data_offset = info.data_offset

    def locate(self, layer):
        """(absolute file offset, size in bytes) of layer `layer`'s expert tensor."""
        off, nb = ctypes.c_uint64(), ctypes.c_uint64()
        st = lib.inzg_gguf_experts(self._h, layer, None, ctypes.byref(nb), ctypes.byref(off))
        if st != 0:
            raise InzgError(st, f"no expert tensor for layer {layer} in {self.path}")
        return off.value, nb.value

    def blobs(self, layer):
        """The layer's expert tensor as a read-only uint8 view of the mapping (valid until close)."""
        p, nb = ctypes.c_void_p(), ctypes.c_uint64()
        st = lib.inzg_gguf_experts(self._h, layer, ctypes.byref(p), ctypes.byref(nb), None)
        if st != 0:
            raise InzgError(st, f"no expert tensor for layer {layer} in {self.path}")
        a = np.ctypeslib.as_array((ctypes.c_uint8 * nb.value).from_address(p.value))
        a.flags.writeable = False
        return a

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            lib.inzg_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
