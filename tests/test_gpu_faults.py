"""Host-side fault detection of the pool upload (a context needs a device; nothing faulting runs on it).

The reference stops with "expert blob is corrupt (expert %d)" when an expert's INZQ header does not match its layer
(magic, type, rows, cols; src/model_fwd.c:853-855, 958-960). inzg_pool_add_layer returns INZG_CORRUPT_BLOB with the
same message for each such blob -- gate|up and down headers alike -- before it touches the device, and the context
stays usable: the same layer uploads cleanly afterwards.
"""
import struct

import numpy as np
import pytest

from inferenz_b200 import InzgError, MoePool, synth

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


def test_corrupt_expert_blobs_are_refused_and_the_context_survives():
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E, experts=np.arange(2))
    gu_bytes = int(synth.lib.inzg_qmat_bytes(synth.T_Q4L, 2 * FF, H))
    # header: magic u32 | type u16 | rot_block u16 | rows u32 | cols u32 (src/quant.h:40-50)
    cases = [("magic", 7, 0, "<I", 0x0BADF00D),
             ("type", 33, 4, "<H", synth.T_Q8G),
             ("rows", 100, 8, "<I", 2 * FF + 16),
             ("down cols", 511, gu_bytes + 12, "<I", FF + 64)]
    with MoePool(H, FF, E, K, max_tokens=16, n_layers=1, device=0) as pool:
        for what, e, off, fmt, value in cases:
            bad = blobs.copy()
            struct.pack_into(fmt, bad, e * bb + off, value)
            with pytest.raises(InzgError) as ei:
                pool.add_layer(0, synth.T_Q4L, bad, bb)
            assert ei.value.status == 2, (what, str(ei.value))  # INZG_CORRUPT_BLOB
            assert f"expert blob is corrupt (expert {e})" in str(ei.value), (what, str(ei.value))
        pool.add_layer(0, synth.T_Q4L, blobs, bb)  # the context is unharmed
        assert pool.stats()["pool_bytes"] > 0
