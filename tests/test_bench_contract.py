"""bench.py's reference arm on the CPU: one JSON line with the keys the benchmark contract asks for, and under
torchrun only rank 0 prints it (the other ranks exit 0 without work). The arm times the reference's own compiled
MoE layer (oracle/_ref), or the oracle's C restatement when the reference could not be built here. Also the
NVLink byte count the expert-parallel line reports its link fraction from."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.slow


def _bench(env_extra):
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env.update(env_extra)
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "3",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    return [l for l in p.stdout.splitlines() if l.strip()]


def test_reference_arm_prints_one_contract_line():
    lines = _bench({"RANK": "0"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["config"]["global_batch"] == 32
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_never_loads_the_product_library():
    """the reference arm draws its inputs with the oracle's generator and encodes experts with the reference's own
    quantizer: libinzg.so must not be mapped in its process"""
    code = ("import sys; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '2', '--warmup', '3']; "
            "import bench; bench.main(); maps = open('/proc/self/maps').read(); "
            "print('MAPPED' if 'libinzg' in maps else 'CLEAN')")
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    p = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.strip()]
    assert lines[-1] == "CLEAN" and json.loads(lines[0])["impl"] == "reference"


def test_arms_describe_the_same_workload():
    sys.path.insert(0, ROOT)
    import bench
    src = open(os.path.join(ROOT, "bench.py")).read()
    assert src.count('"config": {"workload": WORKLOAD') == 3  # single GPU, expert parallel, reference


def test_reference_arm_other_ranks_exit_quietly():
    assert _bench({"RANK": "1", "WORLD_SIZE": "2"}) == []


def test_ep_exchange_bytes():
    sys.path.insert(0, ROOT)
    import numpy as np
    import bench
    rng = np.random.default_rng(0)
    sel = np.stack([rng.permutation(512)[:10] for _ in range(32)])[None]  # one rank, 32 tokens
    assert bench.ep_exchange_bytes(sel, 0, 1) == (0, 0, 0)  # one GPU: nothing crosses a link
    # 2 ranks, one token each: rank 0's token picks experts 0 (own) and 300 (rank 1's); rank 1's token picks 1 and 2
    # (both rank 0's) -> rank 0 sends its row once to rank 1 with the row's (expert, weight) metadata and returns
    # both slots of rank 1's token
    sel2 = np.array([[[0, 300]], [[1, 2]]])
    assert bench.ep_exchange_bytes(sel2, 0, 2, topk=2) == (8192 + 1 * 1 * 2 * 8 + 2 * 8192, 1, 2)
    # rank 1 sends its row to rank 0 (both its experts live there) and returns the one slot of rank 0's token it owns
    assert bench.ep_exchange_bytes(sel2, 1, 2, topk=2) == (8192 + 16 + 8192, 1, 1)
