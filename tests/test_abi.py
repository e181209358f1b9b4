"""The C ABI library loads and exports every symbol the public headers declare (no compute without a GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("inzg.h", "inzg_tools.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        for m in re.finditer(r"(?:INZG_EXPORT|INZG_API)\s+[\w\s\*]+?\b(inzg_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_headers_declare_the_abi():
    names = declared_symbols()
    for must in ("inzg_create", "inzg_destroy", "inzg_set_router", "inzg_pool_add_layer", "inzg_moe_forward",
                 "inzg_moe_route_dump", "inzg_last_error", "inzg_quantize", "inzg_synth_layer_blobs"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from inferenz_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    # the Python binding types every declared symbol
    assert declared_symbols() <= set(_lib.SIGNATURES), set(declared_symbols()) - set(_lib.SIGNATURES)


@pytest.mark.gpu
def test_library_kernels_run_as_sm100_code():
    """the kernels load as sm_100 machine code (cudaFuncGetAttributes at run time), not a PTX recompilation"""
    from inferenz_b200 import lib
    bv, pv = ctypes.c_int(0), ctypes.c_int(0)
    assert lib.inzg_kernel_arch(0, ctypes.byref(bv), ctypes.byref(pv)) == 0
    assert bv.value == 100, bv.value


def test_kernel_arch_query_fails_cleanly_without_a_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    from inferenz_b200 import lib
    bv = ctypes.c_int(0)
    assert lib.inzg_kernel_arch(0, ctypes.byref(bv), None) == -1


def test_status_strings():
    from inferenz_b200 import lib
    assert lib.inzg_status_str(0) == b"ok"
    assert lib.inzg_status_str(2) == b"corrupt expert blob"
    assert lib.inzg_status_str(99) == b"unknown status"


def test_create_rejects_bad_config_without_touching_a_device():
    from inferenz_b200._lib import Config, lib
    st = ctypes.c_int(-1)
    bad = Config(2000, 640, 512, 10, 16, 1, 0)  # hidden not a multiple of 256
    assert not lib.inzg_create(ctypes.byref(bad), ctypes.byref(st))
    assert st.value == 1  # INZG_BAD_ARG
    bad = Config(2048, 640, 512, 20, 16, 1, 0)  # top-k above the kernel limit
    assert not lib.inzg_create(ctypes.byref(bad), ctypes.byref(st))
    assert st.value == 1


def test_null_context_calls_fail_cleanly():
    from inferenz_b200 import lib
    assert lib.inzg_moe_forward(None, 0, 1, None, None, None) == 1
    assert lib.inzg_set_router(None, 0, None, 512, 2048) == 1
    assert lib.inzg_last_error(None) == b"no context"


def test_no_gpu_create_reports_cuda():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from inferenz_b200._lib import Config, lib
    st = ctypes.c_int(-1)
    assert not lib.inzg_create(ctypes.byref(Config(2048, 640, 512, 10, 16, 1, 0)), ctypes.byref(st))
    assert st.value == 4  # INZG_CUDA


def test_c_host_compiles_links_and_runs(tmp_path):
    """The public header is plain C: tests/c_host/moe_host.c (the engine's wiring, in C11) compiles with -Werror,
    links against libinzg.so and reads a GGUF; without a GPU it stops at inzg_create with INZG_CUDA (exit 2)."""
    import shutil
    import subprocess
    import sys
    gcc = shutil.which("gcc", path="/usr/bin") or shutil.which("gcc")
    if not gcc:
        pytest.skip("no C compiler")
    from inferenz_b200 import _lib
    exe = str(tmp_path / "moe_host")
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run([gcc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c_host", "moe_host.c"), "-L", libdir, "-linzg",
                    f"-Wl,-rpath,{libdir}", "-o", exe], check=True)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import gguf_file as gf
    model = str(tmp_path / "m.gguf")
    gf.write(model, [("inz.expert_type", gf.U32, 102), ("inz.expert_blob_bytes", gf.U64, 4096)],
             [("blk.0.experts", b"\0" * 8192), ("mtp.experts", b"\0" * 8192)])
    p = subprocess.run([exe, model], capture_output=True, text=True, timeout=120)
    assert "gguf: expert_type 102 blob_bytes 4096 layers 1 mtp 1" in p.stdout
    import torch
    if not torch.cuda.is_available():
        assert p.returncode == 2 and "inzg_create: CUDA error" in p.stdout
    bad = subprocess.run([exe, str(tmp_path / "missing.gguf")], capture_output=True, text=True, timeout=60)
    assert bad.returncode == 1 and "open" in bad.stderr
