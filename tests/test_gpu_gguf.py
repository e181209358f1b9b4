"""Pool layers uploaded straight from a GGUF model file (inzg_pool_add_layer_gguf) against the same blobs uploaded
with inzg_pool_add_layer: identical routing and bit-identical outputs on the decode and the GEMM numerics, for a
"blk.%d.experts" layer and the MTP layer's "mtp.experts"; and the engine's refusals (src/engine.c:340-350): a blob size
that is not a multiple of 4096, a tensor shorter than n_expert blobs, a layer the file does not have."""
import numpy as np
import pytest

import gguf_file as gf
import oracle
from inferenz_b200 import GgufExperts, InzgError, MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


def _kvs(blob_bytes, expert_type=synth.T_Q4L):
    return [("general.architecture", gf.STR, "qwen38flash"), ("inz.expert_type", gf.U32, expert_type),
            ("inz.expert_blob_bytes", gf.U64, blob_bytes)]


def _forward(pool, layer, x, override=None):
    y = pool.moe_block(layer, x, logits_override=override, dump=True)
    return y, pool.route_dump(x.shape[0])


def test_pool_from_gguf_equals_pool_from_blobs(tmp_path, orc):
    R = [synth.router(0, E, H), synth.router(1, E, H)]
    x8, x40 = synth.hidden(8, H), synth.hidden(40, H, seed=5)
    ov = synth.normal_logits(40, E)
    ov[:, :3] += 6.0  # three experts well above 12 tokens: the GEMM numerics
    # payloads for the experts layer 0's calls route to (the others keep a valid header, zero weights), as the parity
    # tests do; the MTP tensor carries the same blobs under its own router, so its calls mix both kinds
    used = np.unique(np.concatenate([oracle.routing(orc, R[0], x8).ravel(),
                                     oracle.routing(orc, R[0], x40, override=ov).ravel()]))
    blobs0, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=used)
    blobs1 = blobs0
    path = str(tmp_path / "model.gguf")
    gf.write(path, _kvs(bb), [("token_embd.weight", b"\0" * 1000), ("blk.0.experts", blobs0), ("mtp.experts", blobs1)])
    with GgufExperts(path) as g, MoePool(H, FF, E, K, max_tokens=64, n_layers=2, device=0) as a, \
            MoePool(H, FF, E, K, max_tokens=64, n_layers=2, device=0) as b:
        assert (g.n_layers, g.has_mtp, g.blob_bytes, g.expert_type) == (1, True, bb, synth.T_Q4L)
        for layer, blobs in ((0, blobs0), (1, blobs1)):
            a.set_router(layer, R[layer])
            b.set_router(layer, R[layer])
            a.add_layer(layer, synth.T_Q4L, blobs, bb)
            b.add_layer_gguf(layer, g, layer)  # layer 1 of the file is its mtp.experts
        for layer in (0, 1):
            for x, o in ((x8, None), (x40, ov)):
                ya, da = _forward(a, layer, x, o)
                yb, db = _forward(b, layer, x, o)
                assert np.array_equal(da["sel"], db["sel"]) and np.array_equal(da["units"], db["units"])
                assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32)), (layer, x.shape[0])
        assert b.stats()["gemm_units"] >= 3  # the last call ran the GEMM numerics


def test_refused_files(tmp_path):
    bb = synth.blob_bytes(synth.T_Q4L, H, FF)
    blobs, _ = synth.layer_blobs_range(0, synth.T_Q4L, H, FF, 0, 2)
    cases = {  # each refused before anything is uploaded
        "odd blob size": ([("blk.0.experts", b"\0" * 64)], _kvs(bb - 16), 2),
        "short tensor": ([("blk.0.experts", blobs)], _kvs(bb), 2),  # 2 blobs of the 512 the context holds
        "no such layer": ([("blk.0.experts", b"\0" * 64)], _kvs(bb), 1),
    }
    with MoePool(H, FF, E, K, max_tokens=16, n_layers=2, device=0) as pool:
        for what, (tensors, kvs, status) in cases.items():
            path = str(tmp_path / (what.replace(" ", "_") + ".gguf"))
            gf.write(path, kvs, tensors)
            with GgufExperts(path) as g, pytest.raises(InzgError) as ei:
                pool.add_layer_gguf(0, g, 3 if what == "no such layer" else 0)
            assert ei.value.status == status, (what, str(ei.value))
