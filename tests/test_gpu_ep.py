"""Expert parallelism on 2 GPUs (NCCL): each rank owns half of the experts and half of the tokens; its outputs must
equal a single-GPU call over the whole batch bit for bit. Four experts get a large logit bias so that both numeric
paths run: they collect every token (prefill GEMM numerics, >= 12 tokens) while the rest stay on the decode GEMV.
Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, FF, E, K = 2048, 640, 512, 10


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_total, q):
    import datetime

    import torch.distributed as dist

    from inferenz_b200 import MoePool, synth
    from inferenz_b200.ep import DeviceBackend, ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        x_all = synth.hidden(n_total, H)
        bias = np.zeros(E, np.float32)
        bias[[3, 200, 300, 511]] = 9.0
        e0, nl = rank * (E // world), E // world
        blobs, bb = synth.layer_blobs_range(0, synth.T_Q4L, H, FF, e0, e0 + nl)
        R = synth.router(0, E, H)
        per = n_total // world
        dev = torch.device("cuda", rank)
        with MoePool(H, FF, E, K, max_tokens=n_total, n_layers=1, device=rank) as pool:
            pool.set_router(0, R)
            pool.add_layer_range(0, synth.T_Q4L, blobs, bb, e0, nl)
            ep = ExpertParallelMoE(DeviceBackend(pool), E, K, H)
            x = torch.from_numpy(x_all[rank * per:(rank + 1) * per]).to(dev)
            y = ep.moe_block(0, x, bias=torch.from_numpy(bias).to(dev))
            torch.cuda.synchronize(dev)
            pool.device_status()
            ys = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(ys, y)
            y_ep = torch.cat(ys).cpu().numpy()
        if rank == 0:
            full, _ = synth.layer_blobs(0, synth.T_Q4L, H, FF, E)
            with MoePool(H, FF, E, K, max_tokens=n_total, n_layers=1, device=0) as one:
                one.set_router(0, R)
                one.add_layer(0, synth.T_Q4L, full, bb)
                y_one = one.moe_block(0, x_all, bias=bias)
                one.moe_block(0, x_all, bias=bias, dump=True)
                one.route_dump(n_total)
                st = one.stats()
            q.put((y_ep, y_one, st["gemm_units"], st["dec_units"]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_equals_single_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n_total = 48
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_total, q)) for r in range(2)]
    for p in procs:
        p.start()
    y_ep, y_one, gemm_units, dec_units = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert gemm_units >= 4 and dec_units > 0
    print(f"EP 2 GPUs, {n_total} tokens: gemm experts {gemm_units}, decode experts {dec_units}, "
          f"bit-identical {np.mean(y_ep.view(np.uint32) == y_one.view(np.uint32)):.4f}")
    assert np.array_equal(y_ep.view(np.uint32), y_one.view(np.uint32))


def _single_rank(port, q):
    import datetime

    import torch.distributed as dist

    from inferenz_b200 import MoePool, synth
    from inferenz_b200.ep import DeviceBackend, ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120))
    try:
        n = 20
        x_all = synth.hidden(n, H)
        bias = synth.normal_bias(E)
        bias[[5, 77]] += 9.0
        blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E)
        sh_blob, sh_bb = synth.layer_blobs_range(777, synth.T_Q8G, H, FF, 0, 1)
        gate = (np.random.default_rng(5).standard_normal(H) * 0.05).astype(np.float32)
        with MoePool(H, FF, E, K, max_tokens=n, n_layers=1, device=0) as pool:
            pool.set_router(0, synth.router(0, E, H))
            pool.add_layer(0, synth.T_Q4L, blobs, bb)
            pool.set_shared(0, synth.T_Q8G, sh_blob, sh_bb, gate)
            ep = ExpertParallelMoE(DeviceBackend(pool), E, K, H, shared_layers={0})
            y = ep.moe_block(0, torch.from_numpy(x_all).cuda(), bias=torch.from_numpy(bias).cuda()).cpu().numpy()
            y_one = pool.moe_block(0, x_all, bias=bias)
        q.put((y, y_one))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_building_blocks_single_rank():
    """inzg_route + inzg_moe_experts + inzg_combine + inzg_shared_expert on one rank equal inzg_moe_forward (with the
    layer's shared expert) bit for bit."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_single_rank, args=(_free_port(), q))
    p.start()
    y, y_one = q.get(timeout=600)
    p.join(timeout=120)
    assert p.exitcode == 0
    assert np.array_equal(y.view(np.uint32), y_one.view(np.uint32))


# ---- the exchange inside libinzg (inzg_ep_*: peer memory, device-side epoch flags) ----

def _peer_worker(rank, world, port, n_total, steps, q, absent_rank=-1):
    import datetime

    import torch.distributed as dist

    from inferenz_b200 import InzgError, MoePool, synth
    from inferenz_b200.ep import PeerExchangeMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    # the handles travel over gloo: no collective library touches the exchange
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        x_all = synth.hidden(n_total, H)
        bias = np.zeros(E, np.float32)
        bias[[3, 200, 300, 511]] = 9.0  # four experts take every token: both numeric paths run
        e0, nl = rank * (E // world), E // world
        blobs, bb = synth.layer_blobs_range(0, synth.T_Q4L, H, FF, e0, e0 + nl)
        R = synth.router(0, E, H)
        per = n_total // world
        dev = torch.device("cuda", rank)
        with MoePool(H, FF, E, K, max_tokens=per * world, n_layers=1, device=rank) as pool:
            pool.set_router(0, R)
            pool.add_layer_range(0, synth.T_Q4L, blobs, bb, e0, nl)
            ep = PeerExchangeMoE(pool, capacity=per)
            x = torch.from_numpy(x_all[rank * per:(rank + 1) * per]).to(dev)
            bd = torch.from_numpy(bias).to(dev)
            status = "ok"
            ys = []
            if rank != absent_rank:
                for _ in range(steps):
                    if absent_rank < 0:
                        ep.barrier()  # device-side rendezvous between steps
                    ys.append(ep.moe_block(0, x, bias=bd, n_batch=n_total).clone())
                torch.cuda.synchronize(dev)
                try:
                    pool.device_status()
                except InzgError as err:
                    status = str(err)
                    pool.device_status()  # reported once: the context is usable again
            dist.barrier()  # the absent rank keeps its memory mapped until the others are done
            ep.close()
            out = [y.cpu().numpy() for y in ys]
        q.put((rank, status, out))
        if rank == 0 and absent_rank < 0:
            full, _ = synth.layer_blobs(0, synth.T_Q4L, H, FF, E)
            with MoePool(H, FF, E, K, max_tokens=n_total, n_layers=1, device=0) as one:
                one.set_router(0, R)
                one.add_layer(0, synth.T_Q4L, full, bb)
                q.put(("one", one.moe_block(0, x_all, bias=bias)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_peer(world, n_total, steps, absent_rank=-1):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, n_total, steps, q, absent_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world + (1 if absent_rank < 0 else 0)):
        item = q.get(timeout=600)
        got[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


def test_peer_exchange_single_rank():
    """One rank: the whole step (route, dispatch into its own buffer, experts, return, combine) through the exchange's
    kernels and flags equals inzg_moe_forward bit for bit, at every step (the epochs advance)."""
    got = _run_peer(1, 20, 3)
    status, ys = got[0]
    (y_one,) = got["one"]
    assert status == "ok"
    for step, y in enumerate(ys):
        same = (y.view(np.uint32) == y_one.view(np.uint32)).mean(axis=1)
        print(f"step {step}: bit-identical fraction per token {np.round(same, 3).tolist()}")
        assert np.array_equal(y.view(np.uint32), y_one.view(np.uint32)), f"step {step}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_two_gpus_equals_single_gpu():
    got = _run_peer(2, 48, 3)
    (y_one,) = got["one"]
    for step in range(3):
        y_ep = np.concatenate([got[r][1][step] for r in range(2)])
        assert got[0][0] == "ok" and got[1][0] == "ok"
        assert np.array_equal(y_ep.view(np.uint32), y_one.view(np.uint32)), f"step {step}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_absent_peer_times_out():
    """Rank 1 connects and then never runs a step (it stays out between steps, nothing in flight): rank 0's waits run
    out after about a second each, inzg_device_status reports INZG_TIMEOUT once, and the next status check is clean."""
    got = _run_peer(2, 16, 1, absent_rank=1)
    status, _ = got[0]
    assert "INZG_TIMEOUT" in status, status
