"""Prefill path on tcgen05 (kind::i8): experts with >= 12 tokens.

The tensor-core GEMM and the CUDA-core int8 GEMM compute the same exact int32 block dots and the reference's
per-256-block FMA sequence, so their layer outputs must be identical bit for bit; both must match the CPU oracle
within the north-star tolerance. Token counts span several 128-token tiles and a partial tile (calls above 256 rows: smaller ones run the same
numerics as GEMM items inside the decode GEMV, tested below).
"""
import numpy as np
import pytest

import oracle
from inferenz_b200 import MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


@pytest.mark.parametrize("expert_type", [synth.T_Q4L, synth.T_Q8G])
def test_tcgen05_gemm_equals_simt_gemm_and_oracle(orc, expert_type):
    n = 300  # above 256 rows: the prefill-numerics experts take the tcgen05 GEMM (smaller calls run them as GEMM items)
    ov = synth.normal_logits(n, E, seed=41)
    ov[:, :4] += 9.0          # experts 0-3 take nearly every token: 300 tokens = two full tiles and a partial one
    ov[:40, 100:104] += 12.0  # experts 100-103 get 40 tokens: one partial tile
    R = synth.router(0, E, H)
    x = synth.hidden(n, H, seed=42)
    sel = oracle.routing(orc, R, x, override=ov)
    cnt = np.bincount(sel.ravel(), minlength=E)
    assert cnt.max() > 128 and (cnt >= 12).sum() >= 8
    blobs, bb = synth.layer_blobs(0, expert_type, H, FF, E, experts=np.unique(sel))
    gu_bytes = int(synth.lib.inzg_qmat_bytes(expert_type, 2 * FF, H))
    want = orc.moe_routed(R, blobs, bb, gu_bytes, x, override=ov, dumps=False)["y"]
    with MoePool(H, FF, E, K, max_tokens=n, n_layers=1, device=0) as pool:
        pool.add_layer(0, expert_type, blobs, bb)
        y_tc = pool.moe_block(0, x, logits_override=ov, dump=True)
        st = pool.stats()
        pool.route_dump(n)
        st = pool.stats()
        y_simt = pool.moe_block(0, x, logits_override=ov, simt_gemm=True)
    assert st["gemm_units"] >= 8
    assert np.array_equal(y_tc.view(np.uint32), y_simt.view(np.uint32)), "tcgen05 GEMM differs from the int8 SIMT GEMM"
    err = oracle.rel_l2(y_tc, want)
    print(f"tcgen05 prefill n={n} type={expert_type}: rel_l2 max {err.max():.3e}, gemm experts {st['gemm_units']}")
    assert err.max() <= 1e-3


@pytest.mark.parametrize("expert_type", [synth.T_Q4L, synth.T_Q8G])
@pytest.mark.parametrize("n", [12, 20, 32, 70])
def test_decode_gemv_gemm_items_equal_simt_gemm(orc, expert_type, n):
    """Calls of 9-256 tokens run their prefill-numerics experts (>= 12 tokens) inside the decode GEMV launches as GEMM
    items (ldmatrix + s8 x s8 MMA over tensor-copied int8 tiles, 32 tokens per item: at 70 tokens the busiest experts
    take three token tiles, the last one partial): bit-identical to the CUDA-core int8 GEMM, within the north-star
    tolerance of the oracle, and without the separate gather / GEMM launches."""
    ov = synth.normal_logits(n, E, seed=50 + n)
    ov[:, :3] += 9.0           # experts 0-2 take every token
    ov[:12, 300:302] += 12.0   # experts 300-301 take exactly the first 12 (the smallest prefill-numerics expert)
    R = synth.router(0, E, H)
    x = synth.hidden(n, H, seed=60 + n)
    sel = oracle.routing(orc, R, x, override=ov)
    cnt = np.bincount(sel.ravel(), minlength=E)
    assert (cnt >= 12).sum() >= 5 and cnt.max() == n
    blobs, bb = synth.layer_blobs(0, expert_type, H, FF, E, experts=np.unique(sel))
    gu_bytes = int(synth.lib.inzg_qmat_bytes(expert_type, 2 * FF, H))
    want = orc.moe_routed(R, blobs, bb, gu_bytes, x, override=ov, dumps=False)["y"]
    with MoePool(H, FF, E, K, max_tokens=max(n, 64), n_layers=1, device=0) as pool:
        pool.add_layer(0, expert_type, blobs, bb)
        y = pool.moe_block(0, x, logits_override=ov, dump=True)
        pool.route_dump(n)
        st = pool.stats()
        y_simt = pool.moe_block(0, x, logits_override=ov, simt_gemm=True)
        st_simt = pool.stats()
    assert st["gemm_units"] == (cnt >= 12).sum()
    assert st["last_launches"] < st_simt["last_launches"], (st["last_launches"], st_simt["last_launches"])
    assert np.array_equal(y.view(np.uint32), y_simt.view(np.uint32)), "GEMM items differ from the int8 SIMT GEMM"
    err = oracle.rel_l2(y, want)
    print(f"decode GEMV GEMM items n={n} type={expert_type}: rel_l2 max {err.max():.3e}, gemm experts {st['gemm_units']}")
    assert err.max() <= 1e-3
