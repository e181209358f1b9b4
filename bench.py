"""MoE-layer benchmark (the metric of BASELINE.json) on B200.

Workload (headline, N=1): BASELINE configs[1] -- one MoE layer, d=2048, 512 experts, top-10, FF 640, Q4L experts
(synthetic, seeded, encoded by the engine's quantizer -- byte-identical to the reference's), F16 router, decode batch
of 32 tokens with a per-expert N(0,1) logit bias. Sub-results under "extra": configs[0] shape (1 token), configs[2]
(4096-token prefill, Zipf(1.1) bias) and configs[3] (Q8G experts, 2048 tokens, router logits replaced by N(0,1)).
Every timed workload is checked once against the reference's own output on the same inputs (tests/golden/bench_*.npz,
made by the compiled reference): routing bit for bit, outputs within 1e-3 relative L2 per token ("parity").

value  = tokens/s with inputs resident in HBM; each timed step is one layer call timed with CUDA events on the
         launching stream; the L2 is flushed (512 MB write) before every step, outside the timed events.
e2e    = the same through the public host API (MoePool.moe_block on pinned host buffers): H2D of the step's input and
         D2H of its output inside the timed region (host wall clock around the synchronous call).
--impl reference: the reference's own CPU implementation of the layer (oracle/_ref, all host cores), on inputs drawn by
         the oracle's generator and experts encoded by the reference's quantizer: this arm never loads libinzg.
Multi-GPU (--gpus N under torchrun, one process per GPU): expert parallelism. Rank g holds
experts [g*512/N, (g+1)*512/N) and decodes its own 32 tokens (weak scaling: 32*N tokens per step); a step
(inzg_ep_forward) routes the rank's tokens, writes each token row once into every GPU owning one of its experts, runs
the local experts, writes each owned (token, rank-k) output back into the token's GPU and combines in rank order -- the
library's own kernels over peer memory (NVLink), no collective library. value = all ranks' tokens / the max over ranks
of the summed per-step CUDA-event times.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE-layer tokens/s at 1/32/4096 tok; % of HBM or tensor roofline, 1–8 GPU"
H, FF, E, K = 2048, 640, 512, 10
GU_PAYLOAD = 2 * FF * (H // 64) * 34        # gate|up indices + fp16 scales, Q4L (header excluded)
DN_PAYLOAD = H * (FF // 64) * 34
EXPERT_BYTES_Q4L = 2089088                   # both matrices incl. their 64-byte headers (inz_qmat_bytes)
GU_PAYLOAD_Q8G = 2 * FF * (H // 64) * 66    # Q8G: 64 index bytes + fp16 scale per 64-group
DN_PAYLOAD_Q8G = H * (FF // 64) * 66
EXPERT_BYTES_Q8G = 4055168
ROUTER_BYTES = E * H * 2
# prefill-numerics experts read the requantized int8 weights and their per-(row, 256-block) fp32 scales
GEMM_GU_BYTES = 2 * FF * H + 2 * FF * (H // 256) * 4
GEMM_DN_BYTES = H * FF + H * (-(-FF // 256)) * 4
GEMV_GEMM_MAX_TOKENS = 256  # calls up to this size run those experts inside the decode GEMV launches


NVLINK_GBS = 770.0  # NVLink 5 peer copy per direction per GPU, the pool's published measurement (900 GB/s nominal)

# the headline workload, worded identically by both arms at every N
WORKLOAD = ("BASELINE configs[1]: MoE layer, decode batch of 32 tokens per GPU (32*N in all), d=2048, 512 experts, "
            "top-10, FF 640, Q4L experts, F16 router, N(0,1) per-expert logit bias")


def ep_exchange_bytes(sel_all, rank, world, n_expert=E, hidden=H, topk=K):
    """(bytes rank `rank` writes into its peers per expert-parallel step, rows sent, slots returned) for the step's
    selections sel_all [world][n_loc][topk]: each of its tokens' fp32 rows once to every other rank owning one of the
    token's experts, the (local expert, weight) metadata of all n_loc rows to every peer, and every slot it owns of a
    token living on another rank (fp32 [hidden]) back to that rank. What a rank keeps for itself crosses no link."""
    sel_all = np.asarray(sel_all)
    owner = sel_all // (n_expert // world)
    n_loc = sel_all.shape[1]
    rows = int(sum(len(set(owner[rank, t].tolist()) - {rank}) for t in range(n_loc)))
    slots = int(sum((owner[s] == rank).sum() for s in range(world) if s != rank))
    return rows * hidden * 4 + (world - 1) * n_loc * topk * 8 + slots * hidden * 4, rows, slots


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        p = json.load(open(path))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampler over the timed region (SM clock, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.p:
            time.sleep(0.25)
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
                self.lines = [l for l in out.splitlines() if l.strip()]
            except Exception:
                self.p.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_inputs(cfg, n):
    from inferenz_b200 import synth
    x = synth.hidden(n, H)
    bias = override = None
    if cfg == "decode32":
        bias = synth.normal_bias(E)
    elif cfg == "prefill4096":
        bias = synth.zipf_bias(E)
    elif cfg == "q8g2048":
        override = synth.normal_logits(n, E)  # router logits replaced by N(0,1), seed 4
    return x, bias, override


def check_parity(name, route, y):
    """One call's routing dump and output against the reference's output on the same workload
    (tests/golden/bench_<name>.npz, made by the compiled reference): top-k, unit order and the exact bits of the
    logits, probabilities and weights; per token, output norms and (for sampled tokens) whole rows within 1e-3
    relative L2."""
    import hashlib
    path = os.path.join(ROOT, "tests", "golden", f"bench_{name}.npz")
    if not os.path.exists(path):
        return {"ok": False, "why": f"no fixture {os.path.basename(path)}"}
    g = np.load(path)

    def sha(a):
        return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()

    routing = {"sel": bool(np.array_equal(route["sel"], g["sel"])), "units": bool(np.array_equal(route["units"], g["units"])),
               "w": sha(route["w"]) == str(g["w_sha"]), "logits": sha(route["logits"]) == str(g["logits_sha"]),
               "probs": sha(route["probs"]) == str(g["probs_sha"])}
    rows = g["y_rows"]
    got, want = y[rows].astype(np.float64), g["y_sample"].astype(np.float64)
    rel = np.linalg.norm(got - want, axis=1) / np.maximum(np.linalg.norm(want, axis=1), 1e-30)
    nrm = np.linalg.norm(y.astype(np.float64), axis=1)
    nrel = np.abs(nrm - g["y_norm"]) / np.maximum(g["y_norm"], 1e-30)
    exact = float(np.mean(y[rows].view(np.uint32) == g["y_sample"].view(np.uint32)))
    ok = all(routing.values()) and float(rel.max()) <= 1e-3 and float(nrel.max()) <= 1e-3
    return {"ok": bool(ok), "routing_bit_exact": all(routing.values()), "routing": routing,
            "rows_checked": int(len(rows)), "y_rel_l2_max": float(rel.max()), "y_norm_rel_max": float(nrel.max()),
            "bit_identical_fraction": round(exact, 4), "reference_isa": str(g["isa"])}


def time_device(pool, torch, x, bias, steps, warmup, flush, layer=0, override=None):
    """Per-step CUDA-event time (ms) of the layer on HBM-resident inputs."""
    n = x.shape[0]
    dev = torch.device("cuda", pool.device)
    xd = torch.from_numpy(x).to(dev)
    yd = torch.empty_like(xd)
    bd = None if bias is None else torch.from_numpy(bias).to(dev)
    od = None if override is None else torch.from_numpy(override).to(dev)
    # a dedicated (non-default) stream: the flush, the events and the layer all run on it
    stream = torch.cuda.Stream(dev)
    sh = stream.cuda_stream
    assert sh != 0

    def call():
        pool.moe_block_device(layer, n, xd.data_ptr(), yd.data_ptr(), None if bd is None else bd.data_ptr(),
                              None if od is None else od.data_ptr(), stream=sh)

    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            flush.zero_()
            call()
        stream.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            call()
            b.record(stream)
    torch.cuda.synchronize(dev)
    return [a.elapsed_time(b) for a, b in evs], yd


def profile_stages(pool, torch, x, bias, reps, flush, layer=0, override=None):
    n = x.shape[0]
    dev = torch.device("cuda", pool.device)
    xd = torch.from_numpy(x).to(dev)
    yd = torch.empty_like(xd)
    bd = None if bias is None else torch.from_numpy(bias).to(dev)
    od = None if override is None else torch.from_numpy(override).to(dev)
    stream = torch.cuda.Stream(dev)
    sh = stream.cuda_stream
    torch.cuda.synchronize(dev)
    pool.stage_times(reset=True)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            flush.zero_()
            pool.moe_block_device(layer, n, xd.data_ptr(), yd.data_ptr(), None if bd is None else bd.data_ptr(),
                                  None if od is None else od.data_ptr(), stream=sh, profile=True)
    torch.cuda.synchronize(dev)
    st, calls = pool.stage_times(reset=True)
    # routing summary and parity of this input (one dumped call through the host API)
    y = pool.moe_block(layer, x, bias=bias, logits_override=override, dump=True)
    route = pool.route_dump(n)
    s = pool.stats()
    s["route"], s["y"] = route, y
    return {k: v / max(calls, 1) for k, v in st.items()}, s


def time_e2e(pool, torch, x, bias, steps, warmup, flush):
    n = x.shape[0]
    xp = torch.from_numpy(x).pin_memory().numpy()
    yp = torch.empty(x.shape, dtype=torch.float32).pin_memory().numpy()
    bp = None if bias is None else torch.from_numpy(bias).pin_memory().numpy()
    for _ in range(warmup):
        pool.moe_block(0, xp, bias=bp, y=yp)
    ts = []
    for _ in range(steps):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        pool.moe_block(0, xp, bias=bp, y=yp)
        ts.append((time.perf_counter() - t0) * 1e3)
    h2d = x.nbytes + (0 if bias is None else bias.nbytes)
    d2h = x.nbytes + 64
    return ts, h2d, d2h, yp


def gemm_tokens(route, n, E=E):
    """Token-expert pairs on the prefill GEMM path: experts with >= 12 tokens, when the call has more than 8 tokens
    (the reference's path rule, src/model_fwd.c:126, 229-249, 1071)."""
    if n <= 8:
        return 0
    cnt = np.bincount(route["sel"].ravel(), minlength=E)
    return int(cnt[cnt >= 12].sum())


def stage_roofline(stage_ms, stats, n, hbm, q8g=False, i8_peak=None):
    """Algorithmic bytes per launch of each stage; the dominant stage's achieved GB/s. GEMM stages also get their
    int8 tensor-pipe fraction: ops = GEMM-path token-expert pairs x 2 x rows x K, against the measured int8 peak."""
    dec, gemm = stats["dec_units"], stats["gemm_units"]
    gu, dn = (GU_PAYLOAD_Q8G, DN_PAYLOAD_Q8G) if q8g else (GU_PAYLOAD, DN_PAYLOAD)
    expert_bytes = EXPERT_BYTES_Q8G if q8g else EXPERT_BYTES_Q4L
    algo = {
        "fused_decode": ROUTER_BYTES + stats["units"] * expert_bytes + 2 * n * H * 4,  # the whole layer, one launch
        "router_logits": ROUTER_BYTES + n * H * 4 + n * E * 4,
        # calls of <= 32 tokens: the decode GEMV launches also run the prefill-numerics experts (GEMM items)
        "gate_up_gemv": dec * gu + (gemm * GEMM_GU_BYTES if n <= GEMV_GEMM_MAX_TOKENS else 0),
        "down_gemv": dec * dn + (gemm * GEMM_DN_BYTES if n <= GEMV_GEMM_MAX_TOKENS else 0),
        "gate_up_gemm": gemm * gu,
        "down_gemm": gemm * dn,
    }
    total = sum(stage_ms.values())
    if total <= 0:
        return {"dominant": None, "stage_ms": {}, "share": {}}
    dom = max(stage_ms, key=lambda k: stage_ms[k])
    share = {k: round(v / total, 4) for k, v in stage_ms.items() if v > 0}
    out = {"dominant": dom, "stage_ms": {k: round(v, 5) for k, v in stage_ms.items()}, "share": share}
    if dom in algo and stage_ms[dom] > 0:
        ach = algo[dom] / (stage_ms[dom] * 1e-3) / 1e9
        out["roofline"] = {"bound": "hbm", "kernel": dom, "algorithmic_bytes": algo[dom], "achieved": round(ach, 1),
                           "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4)}
    tg = gemm_tokens(stats["route"], n) if "route" in stats else 0
    if tg and i8_peak:
        tens = {}
        for st, per in (("gate_up_gemm", 2 * (2 * FF) * H), ("down_gemm", 2 * H * FF)):
            if stage_ms.get(st, 0) > 0:
                tops = tg * per / (stage_ms[st] * 1e-3) / 1e12
                tens[st] = {"ops": tg * per, "achieved": round(tops, 1), "peak": round(i8_peak, 1), "unit": "TOPS",
                            "frac": round(tops / i8_peak, 4)}
        out["tensor_roofline"] = {"bound": "tensor", "gemm_token_expert_pairs": tg, "stages": tens,
                                  "peak_kind": "measured int8 tcgen05 probe (inzg_probe_tensor_i8)"}
    return out


def run_mine(args):
    import torch

    from inferenz_b200 import MoePool, synth

    rank, world, local = 0, 1, 0  # one GPU (--gpus N > 1 runs run_ep)
    dev = torch.device("cuda", local)
    hbm, bf16, peak_kind = peaks()
    i8_peak = probe_i8(local)
    t0 = time.time()
    blobs, bb = synth.layer_blobs(0, synth.T_Q4L, H, FF, E)
    gen_s = time.time() - t0
    R = synth.router(0, E, H)
    pool = MoePool(H, FF, E, K, max_tokens=4096, n_layers=2, device=local)
    pool.set_router(0, R)
    pool.add_layer(0, synth.T_Q4L, blobs, bb)
    q8 = not args.headline_only and args.only in (None, "q8g2048")
    if q8:  # the same layer with Q8G experts (slot 1; its router logits come from the override)
        t1 = time.time()
        b8, bb8 = synth.layer_blobs(0, synth.T_Q8G, H, FF, E)
        pool.add_layer(1, synth.T_Q8G, b8, bb8)
        del b8
        gen_s += time.time() - t1
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    results = {}
    plan = [("decode32", 32, args.steps, args.warmup)]
    if not args.headline_only:
        plan += [("decode1", 1, max(args.steps // 2, 10), args.warmup),
                 ("prefill4096", args.prefill_tokens, max(args.steps // 50, 5), 3),
                 ("q8g2048", 2048, max(args.steps // 50, 5), 3)]
    if args.only:
        plan = [p for p in plan if p[0] == args.only] or [(args.only, {"decode1": 1, "decode32": 32, "prefill4096": 4096,
                                                                       "q8g2048": 2048}[args.only], args.steps, args.warmup)]
        plan = [(nm, args.prefill_tokens if nm == "prefill4096" else n, st, w) for nm, n, st, w in plan]
    clocks_summary = None
    for name, n, steps, warm in plan:
        x, bias, ovr = make_inputs(name, n)
        layer = 1 if name == "q8g2048" else 0
        torch.cuda.synchronize(dev)
        if name == "decode32":
            with Clocks(local) as ck:
                ts, yd = time_device(pool, torch, x, bias, steps, warm, flush, layer, ovr)
            clocks_summary = ck.summary()
        else:
            ts, yd = time_device(pool, torch, x, bias, steps, warm, flush, layer, ovr)
        torch.cuda.synchronize(dev)
        total_ms = sum(ts)
        stage_ms, stats = profile_stages(pool, torch, x, bias, 0 if args.only else max(3, min(20, steps)), flush,
                                         layer, ovr)
        roof = stage_roofline(stage_ms, stats, n, hbm, q8g=layer == 1, i8_peak=i8_peak)
        route_dump, y_dump = stats.pop("route"), stats.pop("y")
        parity = check_parity(name, route_dump, y_dump) if n == {"decode1": 1, "decode32": 32, "prefill4096": 4096,
                                                                  "q8g2048": 2048}[name] else {"ok": None}
        U = stats["units"]
        # the override replaces the router in configs[3]: no router bytes there
        layer_bytes = (0 if ovr is not None else ROUTER_BYTES) + U * (EXPERT_BYTES_Q8G if layer == 1 else
                                                                      EXPERT_BYTES_Q4L) + 2 * n * H * 4
        ms_step = total_ms / steps
        results[name] = {
            "n_tokens": n, "steps": steps, "ms_per_step": round(ms_step, 5),
            "tokens_per_s": round(n * steps * world / (total_ms * 1e-3), 1),
            "units": U, "decode_units": stats["dec_units"], "gemm_units": stats["gemm_units"],
            "launches_per_step": stats["last_launches"], "parity": parity,
            "layer_roofline": {"bound": "hbm", "algorithmic_bytes": layer_bytes,
                               "achieved": round(layer_bytes / (ms_step * 1e-3) / 1e9, 1), "peak": hbm,
                               "unit": "GB/s", "frac": round(layer_bytes / (ms_step * 1e-3) / 1e9 / hbm, 4)},
            "stages": roof,
        }
        if name == "decode32" and not args.only:
            e2e_ts, h2d, d2h, _ = time_e2e(pool, torch, x, bias, max(steps // 4, 5), 3, flush)
            results[name]["e2e"] = {"value": round(n * len(e2e_ts) / (sum(e2e_ts) * 1e-3), 1), "unit": "tokens/s",
                                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                                    "ms_per_step": round(sum(e2e_ts) / len(e2e_ts), 5)}
    head = results.get("decode32") or next(iter(results.values()))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference("decode32", 32, budget_s=args.cpu_seconds, blobs=blobs, bb=bb, R=R)
    if rank == 0:
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            try:
                traffic = json.load(open(tp)).get(head["stages"].get("dominant"))
            except Exception:
                traffic = None
        roof = head["stages"].get("roofline", {})
        if roof:
            roof = dict(roof)
            roof["peak_kind"] = peak_kind + " (MEASURED_PEAKS.json hbm_gbs, copy burst)"
            roof["traffic"] = traffic
        line = {
            "metric": METRIC, "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 x Q4L (fp32 accumulate)", "data": "synthetic (seeded; no dataset)",
            "config": {"workload": WORKLOAD, "global_batch": 32 * world, "seq_len": 1},
            "arm": {"parallelism": "single GPU", "l2": "flushed (512 MB write) before every timed step",
                    "int8_tensor_peak_tops": i8_peak},
            "parity": {k: v["parity"]["ok"] for k, v in results.items()},
            "roofline": roof or None,
            "layer_roofline": head["layer_roofline"],
            "cpu_baseline": cpu,
            "e2e": head.get("e2e"),
            "clocks": clocks_summary,
            "gpu_launches": head["launches_per_step"] * args.steps,
            "extra": {k: v for k, v in results.items() if k != "decode32"},
            "detail": {"decode32": head, "layer_gen_s": round(gen_s, 1)},
        }
        print(json.dumps(line))
    pool.close()


def probe_i8(device):
    """int8 tensor-pipe peak (TOPS) of this GPU, measured by the library's tcgen05 probe; None if it fails"""
    import ctypes
    from inferenz_b200 import lib
    tops, ms = ctypes.c_double(0), ctypes.c_double(0)
    if lib.inzg_probe_tensor_i8(device, 20000, ctypes.byref(tops), ctypes.byref(ms)) != 0:
        return None
    return round(tops.value, 1)


def run_ep(args):
    """--gpus N > 1: the expert-parallel decode step with the exchange in libinzg (inzg_ep_forward): each rank routes
    its 32 tokens, writes every (token, owning rank) row straight into the owner's buffer, runs its 512/N experts on
    what it received, writes each owned slot straight back into the token's home and combines in rank order -- peer
    memory over NVLink, device-side epoch flags, one CUDA graph per step. torch.distributed (gloo) only carries the
    buffer handles, barriers and the per-rank timings."""
    import datetime

    # the ranks share the host's cores for the synthetic layer's generation: give each its share (torchrun sets
    # OMP_NUM_THREADS=1; the generator reads it when the library loads, below)
    lw = int(os.environ.get("LOCAL_WORLD_SIZE", os.environ.get("WORLD_SIZE", "1")))
    os.environ["OMP_NUM_THREADS"] = str(max(1, (os.cpu_count() or 1) // max(lw, 1)))
    import torch
    import torch.distributed as dist

    from inferenz_b200 import MoePool, synth
    from inferenz_b200.ep import PeerExchangeMoE

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local)
    hbm, _, peak_kind = peaks()
    n_loc = 32
    nb = n_loc * world
    e0, nl = rank * E // world, E // world
    t0 = time.time()
    blobs, bb = synth.layer_blobs_range(0, synth.T_Q4L, H, FF, e0, e0 + nl)
    gen_s = time.time() - t0
    pool = MoePool(H, FF, E, K, max_tokens=nb, n_layers=1, device=local)
    pool.set_router(0, synth.router(0, E, H))
    pool.add_layer_range(0, synth.T_Q4L, blobs, bb, e0, nl)
    del blobs
    stream = torch.cuda.Stream(dev)
    x_all = synth.hidden(nb, H)
    bias = synth.normal_bias(E)
    xd = torch.from_numpy(x_all[rank * n_loc:(rank + 1) * n_loc].copy()).to(dev)
    yd = torch.empty_like(xd)
    bd = torch.from_numpy(bias).to(dev)
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    ep = PeerExchangeMoE(pool, capacity=n_loc)
    # the step's routing on every rank (for the byte counts): this rank's selections, gathered over gloo
    sel = torch.empty((n_loc, K), dtype=torch.int32, device=dev)
    wts = torch.empty((n_loc, K), dtype=torch.float32, device=dev)
    pool.route_device(0, n_loc, xd.data_ptr(), sel.data_ptr(), wts.data_ptr(), bd.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    sels = [torch.zeros((n_loc, K), dtype=torch.int32) for _ in range(world)]
    dist.all_gather(sels, sel.cpu())
    sel_all = torch.stack(sels).numpy()                      # [world][n_loc][K]
    local_units = int(np.unique(sel_all[sel_all // (E // world) == rank]).size)
    xb, rows_out, slots_back = ep_exchange_bytes(sel_all, rank, world)

    def step():
        ep.moe_block(0, xd, bias=bd, n_batch=nb, y=yd, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            flush.zero_()
            ep.barrier(stream)
            step()
        stream.synchronize()
        pool.device_status(stream.cuda_stream)
        dist.barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        with Clocks(local) as ck:
            for a, b in evs:
                flush.zero_()
                ep.barrier(stream)  # every rank's timed step starts together (device-side rendezvous)
                a.record(stream)
                step()
                b.record(stream)
            stream.synchronize()
        pool.device_status(stream.cuda_stream)
        my_total = sum(a.elapsed_time(b) for a, b in evs)
        launches = pool.stats()["last_launches"]
        # end to end: the step's tokens from pinned host memory and its output back to the host, wall clock
        xp = torch.from_numpy(x_all[rank * n_loc:(rank + 1) * n_loc].copy()).pin_memory()
        yp = torch.empty((n_loc, H), dtype=torch.float32).pin_memory()
        e2e_steps = max(args.steps // 4, 5)
        dist.barrier()
        ts = []
        for _ in range(e2e_steps):
            flush.zero_()
            ep.barrier(stream)
            stream.synchronize()
            t1 = time.perf_counter()
            xd.copy_(xp, non_blocking=True)
            step()
            yp.copy_(yd, non_blocking=True)
            stream.synchronize()
            ts.append(time.perf_counter() - t1)
        pool.device_status(stream.cuda_stream)
    # per rank: device ms over the timed steps, end-to-end seconds, local experts touched
    mine = torch.tensor([my_total, sum(ts), float(local_units)], dtype=torch.float64)
    every = [torch.zeros(3, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(every, mine)
    per_rank = [[round(float(v), 4) for v in t.tolist()] for t in every]
    total_ms = max(r[0] for r in per_rank)
    e2e_s = max(r[1] for r in per_rank)
    ms_step = total_ms / args.steps
    value = nb * args.steps / (total_ms * 1e-3)
    units_all = int(sum(r[2] for r in per_rank))
    # per GPU: router + its experts' weights + the rows it received and returned
    bytes_gpu = ROUTER_BYTES + local_units * EXPERT_BYTES_Q4L + 2 * n_loc * H * 4
    if rank == 0:
        ach = bytes_gpu / (ms_step * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 x Q4L (fp32 accumulate)", "data": "synthetic (seeded; no dataset)",
            "config": {"workload": WORKLOAD, "global_batch": nb, "seq_len": 1},
            "arm": {"parallelism": f"ep{world}: 512/N experts per GPU; dispatch and return written by the library's "
                                   "kernels straight into the peers' memory (NVLink), device-side epoch flags",
                    "l2": "flushed (512 MB write) before every step"},
            "roofline": {"bound": "hbm", "kernel": "layer step per GPU (router + local experts, incl. the exchange)",
                         "algorithmic_bytes": bytes_gpu, "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 4), "peak_kind": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": None},
            "nvlink": {"bytes_out_rank0": xb, "achieved": round(xb / (ms_step * 1e-3) / 1e9, 1),
                       "peak": NVLINK_GBS, "unit": "GB/s", "frac": round(xb / (ms_step * 1e-3) / 1e9 / NVLINK_GBS, 4),
                       "peak_kind": "measured peer copy per direction (900 nominal)"},
            "cpu_baseline": None,
            "e2e": {"value": round(nb * e2e_steps / e2e_s, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": n_loc * H * 4 * world, "d2h_bytes_per_step": n_loc * H * 4 * world},
            "clocks": ck.summary(),
            "gpu_launches": launches * args.steps,
            "detail": {"experts_touched_all_gpus": units_all, "experts_touched_rank0": local_units,
                       "rows_sent_rank0": rows_out, "slots_returned_rank0": slots_back,
                       "launches_per_step": launches, "layer_gen_s_rank0": round(gen_s, 1),
                       "per_rank_device_ms_e2e_s_units": per_rank},
        }
        print(json.dumps(line))
    dist.barrier()
    torch.cuda.synchronize(dev)
    ep.close()
    pool.close()
    dist.destroy_process_group()


STACK_WORKLOAD = ("BASELINE configs[4]: stack of 48 MoE layers (random Q4L experts and F16 router per layer, d=2048, "
                  "512 experts, top-10, FF 640), 16384 tokens N(0,1) RMS-normalised per step, expert parallel over N GPUs")


def run_stack(args):
    """--stack: BASELINE configs[4]. Every rank draws and encodes its experts of each layer on its GPU (512/N per layer)
    and loads them without a host round trip; one step is the 48 layers on the batch's 16384 tokens (each layer on the
    same input: the benchmark measures the layer, not a model), on one GPU through inzg_moe_forward, on N GPUs through
    inzg_ep_forward with 16384/N tokens per rank. The pool (about 3.1 GB per layer on one GPU with the prefill copy)
    exceeds the L2 by far, so no flush is needed between steps."""
    import datetime

    import torch

    from inferenz_b200 import MoePool, synth
    from inferenz_b200.ep import PeerExchangeMoE

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    dev = torch.device("cuda", local)
    hbm, _, peak_kind = peaks()
    i8_peak = probe_i8(local)
    layers, n_total = args.stack_layers, args.stack_tokens
    n_loc = n_total // world
    e0, nl = rank * E // world, E // world
    bb = synth.blob_bytes(synth.T_Q4L, H, FF)
    t0 = time.time()
    pool = MoePool(H, FF, E, K, max_tokens=n_total, n_layers=layers, device=local)
    buf = torch.empty(nl * bb, dtype=torch.uint8, device=dev)
    for l in range(layers):
        synth.layer_blobs_device(l, synth.T_Q4L, H, FF, e0, e0 + nl, buf.data_ptr())
        pool.add_layer_device(l, synth.T_Q4L, buf.data_ptr(), bb, e0, nl)
        pool.set_router(l, synth.router(l, E, H))
    del buf
    setup_s = time.time() - t0
    x_all = synth.hidden(n_total, H)
    xd = torch.from_numpy(x_all[rank * n_loc:(rank + 1) * n_loc].copy()).to(dev)
    yd = torch.empty_like(xd)
    stream = torch.cuda.Stream(dev)
    ep = PeerExchangeMoE(pool, capacity=n_loc) if world > 1 else None

    def step():
        for l in range(layers):
            if ep is None:
                pool.moe_block_device(l, n_loc, xd.data_ptr(), yd.data_ptr(), stream=stream.cuda_stream)
            else:
                ep.moe_block(l, xd, n_batch=n_total, y=yd, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            if ep is not None:
                ep.barrier(stream)
            step()
        stream.synchronize()
        pool.device_status(stream.cuda_stream)
        if dist is not None:
            dist.barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        with Clocks(local) as ck:
            for a, b in evs:
                if ep is not None:
                    ep.barrier(stream)
                a.record(stream)
                step()
                b.record(stream)
            stream.synchronize()
        pool.device_status(stream.cuda_stream)
    my_ms = sum(a.elapsed_time(b) for a, b in evs)
    total_ms = my_ms
    if dist is not None:
        every = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(every, torch.tensor([my_ms], dtype=torch.float64))
        total_ms = max(float(t.item()) for t in every)
    ms_step = total_ms / args.steps
    # every expert of every layer is routed at 16384 tokens: the whole router and pool per layer, over all ranks
    bytes_step = layers * (ROUTER_BYTES * world + E * EXPERT_BYTES_Q4L + 2 * n_total * H * 4)
    ops_step = layers * n_total * (2 * E * H + K * 2 * (2 * FF * H + H * FF))
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(n_total * args.steps / (total_ms * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 x Q4L (fp32 accumulate)", "data": "synthetic (seeded; no dataset)",
            "config": {"workload": STACK_WORKLOAD, "layers": layers, "global_batch": n_total, "seq_len": 1},
            "arm": {"parallelism": "single GPU" if world == 1 else f"ep{world}: 512/N experts per GPU, in-library "
                                                                   "exchange over peer memory",
                    "l2": "inputs larger than L2 (the pool)"},
            "roofline": {"bound": "hbm", "kernel": "whole stack step, all GPUs", "algorithmic_bytes": bytes_step,
                         "achieved": round(bytes_step / (ms_step * 1e-3) / 1e9, 1), "peak": hbm * world,
                         "unit": "GB/s", "frac": round(bytes_step / (ms_step * 1e-3) / 1e9 / (hbm * world), 4),
                         "peak_kind": peak_kind + " (MEASURED_PEAKS.json hbm_gbs) x GPUs", "traffic": None},
            "tensor_roofline": {"ops": ops_step, "achieved_tops": round(ops_step / (ms_step * 1e-3) / 1e12, 1),
                                "peak_tops": round(i8_peak * world, 1) if i8_peak else None,
                                "frac": round(ops_step / (ms_step * 1e-3) / 1e12 / (i8_peak * world), 4) if i8_peak
                                else None},
            "clocks": ck.summary(), "gpu_launches": pool.stats()["last_launches"] * layers * args.steps,
            "detail": {"setup_s_rank0": round(setup_s, 1), "pool_bytes_rank0": pool.stats()["pool_bytes"]},
        }
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if ep is not None:
        ep.close()
    pool.close()
    if dist is not None:
        dist.destroy_process_group()


def oracle_inputs(cfg, n):
    """The same workload inputs as make_inputs, drawn by the oracle's generator (no product library)"""
    import oracle
    x = oracle.synth_hidden(n, H)
    bias = override = None
    if cfg == "decode32":
        bias = oracle.normal_bias(E)
    elif cfg == "prefill4096":
        bias = oracle.zipf_bias(E)
    elif cfg == "q8g2048":
        override = oracle.normal_logits(n, E)
    return x, bias, override


def cpu_reference(cfg, n, budget_s=12.0, blobs=None, bb=None, R=None, steps=None, warmup=3):
    """The reference's own CPU layer (oracle/_ref, all host threads) on a bounded sample of the workload. Without
    blobs, the layer is built on the CPU side alone: the oracle's generator and the reference's own quantizer."""
    import oracle
    if blobs is None:
        blobs, bb = oracle.ref_layer_blobs(0, oracle.T_Q4L, H, FF, E)
        R = oracle.synth_router(0, E, H)
    x, bias, _ = oracle_inputs(cfg, n)
    try:
        ref = oracle.Ref(H, threads=0)
        kind, cores, call = "reference", ref.threads, (lambda: ref.moe_routed(R, blobs, bb, x, bias=bias, dumps=False))
        isa = ref.isa
    except (FileNotFoundError, OSError):
        orc = oracle.Oracle()
        gu_bytes = 1392704  # inz_qmat_bytes(Q4L, 2*FF, H)
        kind, cores, isa = "port", 1, "scalar C restatement"
        call = (lambda: orc.moe_routed(R, blobs, bb, gu_bytes, x, bias=bias, dumps=False))
    for _ in range(warmup):
        call()
    ts = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        call()
        ts.append(time.perf_counter() - t0)
        if len(ts) >= (steps if steps is not None else 2000) or time.perf_counter() - t_start > budget_s:
            break
    med = statistics.median(ts)
    return {"value": round(n / med, 1), "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{len(ts)} calls of the {n}-token layer (median {med * 1e3:.3f} ms), {isa}",
            "ms_median": round(med * 1e3, 4)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # the same global batch as this arm at N GPUs (32 decode tokens per GPU), as one CPU call; at most about 90 s of
    # timed calls, so the run ends within minutes whatever --steps asks
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n = 32 * world
    cpu = cpu_reference("decode32", n, budget_s=90.0, steps=args.steps, warmup=max(args.warmup, 1))
    line = {"metric": METRIC, "value": cpu["value"], "unit": "tokens/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cpu["ms_median"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 x Q4L (fp32 accumulate)", "data": "synthetic (seeded; no dataset)",
            "config": {"workload": WORKLOAD, "global_batch": n, "seq_len": 1},
            "arm": {"parallelism": "CPU threads (the reference's thread pool), the whole batch as one layer call",
                    "inputs": "oracle generator + the reference's own quantizer (no product library loaded)"},
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--headline-only", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--only", choices=["decode1", "decode32", "prefill4096", "q8g2048"], default=None,
                    help="time a single workload (profiling runs); the JSON line then reports that workload")
    ap.add_argument("--prefill-tokens", type=int, default=4096,
                    help="tokens of the prefill workload (smaller only for profiler captures; parity is then skipped)")
    ap.add_argument("--stack", action="store_true", help="BASELINE configs[4]: the 48-layer stack, 16384 tokens")
    ap.add_argument("--stack-layers", type=int, default=48)
    ap.add_argument("--stack-tokens", type=int, default=16384)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.stack:
        run_stack(args)
    elif int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_ep(args)
    else:
        run_mine(args)


if __name__ == "__main__":
    main()
