"""ctypes binding of libinzg.so (include/inzg.h, include/inzg_tools.h).

The library is built in-tree (``inferenz_b200/libinzg.so``). There is no fallback: if the shared object is missing or
cannot be loaded, importing this module raises, so nothing can silently run another implementation.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libinzg.so")

T_F16, T_Q4L, T_Q8G = 1, 102, 103
IO_DEVICE, DUMP_ROUTE, PROFILE, NO_GRAPH, GEMM_SIMT, NO_FUSED = 1, 2, 4, 8, 16, 32
EP_HANDLE_BYTES = 128  # INZG_EP_HANDLE_BYTES
N_STAGES = 12

STATUS = {0: "INZG_OK", 1: "INZG_BAD_ARG", 2: "INZG_CORRUPT_BLOB", 3: "INZG_OOM", 4: "INZG_CUDA", 5: "INZG_NCCL",
          6: "INZG_TIMEOUT", 7: "INZG_DEVICE_CHECK", 8: "INZG_UNSUPPORTED", 9: "INZG_NOT_READY"}


class Config(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("ff", ctypes.c_int), ("n_expert", ctypes.c_int), ("topk", ctypes.c_int),
                ("max_tokens", ctypes.c_int), ("n_layers", ctypes.c_int), ("device", ctypes.c_int)]


class MoeOpts(ctypes.Structure):
    _fields_ = [("flags", ctypes.c_uint), ("logit_bias", ctypes.c_void_p), ("logits_override", ctypes.c_void_p),
                ("stream", ctypes.c_void_p)]


class GgufInfo(ctypes.Structure):
    _fields_ = [("expert_type", ctypes.c_int), ("blob_bytes", ctypes.c_uint64), ("n_layers", ctypes.c_int),
                ("has_mtp", ctypes.c_int), ("alignment", ctypes.c_uint64), ("data_offset", ctypes.c_uint64)]


class Stats(ctypes.Structure):
    _fields_ = [("calls", ctypes.c_uint64), ("tokens", ctypes.c_uint64), ("units", ctypes.c_uint64),
                ("dec_units", ctypes.c_uint64), ("gemm_units", ctypes.c_uint64), ("pool_bytes", ctypes.c_uint64),
                ("last_launches", ctypes.c_int)]


P, I, U32, U64, I64, F = (ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64,
                          ctypes.c_float)

# name: (restype, argtypes) -- every symbol the two public headers declare
SIGNATURES = {
    # inzg.h
    "inzg_create": (P, [ctypes.POINTER(Config), ctypes.POINTER(ctypes.c_int)]),
    "inzg_destroy": (None, [P]),
    "inzg_last_error": (ctypes.c_char_p, [P]),
    "inzg_status_str": (ctypes.c_char_p, [I]),
    "inzg_set_router": (I, [P, I, P, I, I]),
    "inzg_pool_add_layer": (I, [P, I, I, P, U64, I]),
    "inzg_moe_forward": (I, [P, I, I, P, P, ctypes.POINTER(MoeOpts)]),
    "inzg_moe_route_dump": (I, [P, I, P, P, P, P, P, P]),
    "inzg_get_stats": (I, [P, ctypes.POINTER(Stats)]),
    "inzg_stage_times": (I, [P, P, P, I]),
    "inzg_stage_name": (ctypes.c_char_p, [I]),
    "inzg_route_topk_noalloc": (I, [P, I, I, P, P, P, P, P]),
    "inzg_pool_add_layer_range": (I, [P, I, I, P, U64, I, I]),
    "inzg_route": (I, [P, I, I, P, P, P, P, P]),
    "inzg_moe_experts": (I, [P, I, I, P, P, P, I, P, P]),
    "inzg_combine": (I, [P, I, P, P, P]),
    "inzg_device_status": (I, [P, P]),
    "inzg_set_shared": (I, [P, I, I, P, U64, P]),
    "inzg_shared_expert": (I, [P, I, I, P, P, I, P]),
    "inzg_ep_attach": (I, [P, I, I, I, P]),
    "inzg_ep_connect": (I, [P, P]),
    "inzg_ep_connect_local": (I, [P, I]),
    "inzg_ep_forward": (I, [P, I, I, P, P, P, I, P]),
    "inzg_ep_detach": (I, [P]),
    "inzg_ep_barrier": (I, [P, P]),
    "inzg_pool_add_layer_device": (I, [P, I, I, P, U64, I, I]),
    "inzg_set_hc": (I, [P, I, P, P, P, P]),
    "inzg_hc_in": (I, [P, I, I, P, P, P, P]),
    "inzg_hc_out": (I, [P, I, P, P, P, P]),
    "inzg_moe_block_hc": (I, [P, I, I, P, ctypes.POINTER(MoeOpts)]),
    "inzg_gguf_open": (P, [ctypes.c_char_p, ctypes.POINTER(GgufInfo), ctypes.c_char_p, ctypes.c_size_t]),
    "inzg_gguf_get_info": (I, [P, ctypes.POINTER(GgufInfo)]),
    "inzg_gguf_experts": (I, [P, I, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "inzg_pool_add_layer_gguf": (I, [P, I, P, I]),
    "inzg_gguf_close": (None, [P]),
    # inzg_tools.h
    "inzg_synth_jump": (U64, [U64, U64]),
    "inzg_synth_randn": (U64, [U64, I64, F, P]),
    "inzg_f32_to_f16": (ctypes.c_uint16, [F]),
    "inzg_synth_expert": (None, [U64, I, I, I, P, P]),
    "inzg_synth_router": (None, [U64, I, I, P]),
    "inzg_synth_hidden": (None, [U64, I, I, P]),
    "inzg_qmat_bytes": (ctypes.c_size_t, [I, I, I]),
    "inzg_auto_rot_block": (I, [I]),
    "inzg_blob_bytes": (U64, [I, I, I]),
    "inzg_quantize_device": (I, [P, I, I, I, I, U32, P, P]),
    "inzg_quantize": (I, [P, I, I, I, I, U32, P]),
    "inzg_encode_experts_device": (I, [P, P, I, I, I, I, P, P]),
    "inzg_encode_expert": (I, [P, P, I, I, I, P]),
    "inzg_synth_layer_blobs": (I, [U64, I, I, I, I, I, P]),
    "inzg_synth_layer_blobs_subset": (I, [U64, I, I, I, I, P, I, P]),
    "inzg_synth_layer_blobs_device": (I, [U64, I, I, I, I, I, P, P]),
    "inzg_synth_experts_device": (I, [U64, I, I, I, I, P, P, P]),
    "inzg_probe_tensor_i8": (I, [I, I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
    "inzg_kernel_arch": (I, [I, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libinzg.so not built ({LIB_PATH}); run `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class InzgError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status
