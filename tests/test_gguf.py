"""The product's GGUF expert reader (inzg_gguf_*, inferenz_b200/csrc/host/gguf.c) on the CPU.

Pinned against the reference's own reader and writer (src/gguf.c through oracle/_ref/libinzref_gguf.so, when the
reference tree was present at build time): files written by the reference's writer read the same in both readers,
and so do the Python-written files below, which cover what that writer never produces (GGUF v2, tensor infos out of
data order, every key/value type, nested arrays, missing expert keys). Broken files fail in both readers.
"""
import os

import numpy as np
import pytest

import gguf_file as gf
import oracle
from inferenz_b200 import GgufExperts, InzgError


@pytest.fixture(scope="module")
def ref():
    try:
        return oracle.RefGguf()
    except (FileNotFoundError, OSError) as e:
        pytest.skip(f"reference GGUF harness not built: {e}")


def _name(g, layer):
    return f"blk.{layer}.experts" if layer < g.n_layers else "mtp.experts"


def _same_as_reference(ref, path, g):
    for layer in range(g.n_layers + int(g.has_mtp)):
        want = ref.tensor(path, _name(g, layer))
        assert want is not None
        assert g.locate(layer) == (want["offset"], want["nbytes"]), layer
        assert g.expert_type == want["expert_type"] and g.blob_bytes == want["blob_bytes"]
        assert g.alignment == want["alignment"]


@pytest.mark.parametrize("alignment,n_layers,mtp,extra", [(32, 1, False, 0), (32, 3, True, 100), (4096, 2, True, 7)])
def test_reference_written_files(tmp_path, ref, alignment, n_layers, mtp, extra):
    blob, ne = 4096, 4
    rng = np.random.default_rng(n_layers)
    data = rng.integers(0, 256, blob * ne * (n_layers + int(mtp)), dtype=np.uint8)
    path = str(tmp_path / "m.gguf")
    ref.write(path, data, blob, ne, n_layers, mtp=mtp, expert_type=103, alignment=alignment, extra_floats=extra)
    with GgufExperts(path) as g:
        assert (g.expert_type, g.blob_bytes, g.n_layers, g.has_mtp) == (103, blob, n_layers, mtp)
        _same_as_reference(ref, path, g)
        for layer in range(n_layers + int(mtp)):
            got = g.blobs(layer)
            assert got.size == blob * ne  # the writer pads each tensor to the alignment; blob*ne is aligned here
            assert np.array_equal(got, data[layer * blob * ne:(layer + 1) * blob * ne])


def _kvs(expert=True):
    kvs = [("general.name", gf.STR, "synthetic"),
           ("a.u8", gf.U8, 200), ("a.i8", gf.I8, -3), ("a.u16", gf.U16, 60000), ("a.i16", gf.I16, -300),
           ("a.f32", gf.F32, 1.5), ("a.bool", gf.BOOL, True), ("a.i64", gf.I64, -(1 << 40)), ("a.f64", gf.F64, 2.5),
           ("a.nested", gf.ARR, (gf.ARR, [(gf.STR, ["x", "yy"]), (gf.I32, [1, 2, 3])])),
           ("a.strs", gf.ARR, (gf.STR, ["", "tok", "é"]))]
    if expert:
        kvs += [("inz.expert_type", gf.U32, 102), ("inz.expert_blob_bytes", gf.U64, 8192)]
    return kvs


def test_python_written_file_out_of_order(tmp_path, ref):
    blob = 8192
    t = [("token_embd.weight", b"\x01" * 100), ("blk.1.experts", b"\x11" * (2 * blob)),
         ("blk.0.experts", b"\x10" * (2 * blob)), ("output.weight", b"\x02" * 33), ("mtp.experts", b"\x12" * (2 * blob))]
    path = str(tmp_path / "o.gguf")
    start, offs = gf.write(path, _kvs(), t, alignment=64, version=2, order=[4, 2, 0, 3, 1])
    with GgufExperts(path) as g:
        assert (g.expert_type, g.blob_bytes, g.n_layers, g.has_mtp, g.alignment) == (102, blob, 2, True, 64)
        assert g.data_offset == start
        assert g.locate(0) == (start + offs[2], offs[3] - offs[2])  # up to the next tensor in data order
        assert g.locate(2) == (start + offs[4], os.path.getsize(path) - start - offs[4])  # the last: to end of file
        assert set(g.blobs(1)[:2 * blob].tolist()) == {0x11}
        _same_as_reference(ref, path, g)


def test_defaults_gaps_and_names(tmp_path, ref):
    # no expert keys: the engine's defaults (Q8G, blob size 0); blk.2 without blk.1 ends the run of layers at 1;
    # names that only resemble an expert tensor are not one
    t = [("blk.0.experts", b"a" * 64), ("blk.2.experts", b"b" * 64), ("blk.01.experts", b"c" * 64),
         ("blk.1.experts.bias", b"d" * 64), ("xblk.1.experts", b"e" * 64)]
    path = str(tmp_path / "d.gguf")
    gf.write(path, _kvs(expert=False), t)
    with GgufExperts(path) as g:
        assert (g.expert_type, g.blob_bytes, g.n_layers, g.has_mtp, g.alignment) == (103, 0, 1, False, 32)
        with pytest.raises(InzgError):
            g.locate(1)
        with pytest.raises(InzgError):
            g.locate(-1)
        _same_as_reference(ref, path, g)


def _broken(tmp_path):
    good, _, offs = gf.gguf_bytes(_kvs(), [("blk.0.experts", b"z" * 8192)])
    cases = {"magic": b"GGUX" + good[4:], "version 1": good[:4] + b"\x01\x00\x00\x00" + good[8:],
             "version 4": good[:4] + b"\x04\x00\x00\x00" + good[8:], "short": good[:20]}
    for cut in (40, 200, len(good) - 8192 - 40):  # inside the key/values, inside the tensor info
        cases[f"cut {cut}"] = good[:cut]
    # a tensor offset far past the end of the file
    far, _, _ = gf.gguf_bytes(_kvs(), [("blk.0.experts", b"z" * 64)])
    i = far.find(b"blk.0.experts") + len(b"blk.0.experts") + 4 + 8 + 4
    cases["beyond EOF"] = far[:i] + (1 << 40).to_bytes(8, "little") + far[i + 8:]
    out = {}
    for k, b in cases.items():
        p = str(tmp_path / (k.replace(" ", "_") + ".gguf"))
        open(p, "wb").write(b)
        out[k] = p
    return out


def test_broken_files_fail_in_both_readers(tmp_path, ref):
    for what, path in _broken(tmp_path).items():
        with pytest.raises(InzgError) as ei:
            GgufExperts(path)
        assert "gguf" in str(ei.value), what
        assert ref.tensor(path, "blk.0.experts") is None, what


def test_missing_file():
    with pytest.raises(InzgError) as ei:
        GgufExperts("/nonexistent/model.gguf")
    assert "open" in str(ei.value)
