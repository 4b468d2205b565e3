"""Benchmark of the B200 MoE-layer hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c0..c4]
                    [--impl ours|reference] [--path auto|gemv|tensor]

A step is one MoE layer (router -> softmax -> top-k -> permutation -> INT8
SwiGLU experts -> slot-ordered combine) over one batch of synthetic tokens.
The default workload is the OLMoE-shaped prefill layer (H=2048, I=1024, E=64,
K=8, T=512 tokens).  Inputs are larger than L2: each step uses a different
layer's weights out of a rotation (every layer is 403 MB), so nothing is
reused from L2 between steps.

value      = tokens processed by all ranks / device time (CUDA events on the
             launching stream, max over ranks), inputs already in HBM.
e2e        = the same metric through the host-buffer C-ABI call
             (moe_layer_forward_host: H2D of the step's hidden states, the
             layer, D2H of the outputs, inside the timed region).
roofline   = the dominant kernel's algorithmic bytes per launch / its mean
             CUDA-event duration, against MEASURED_PEAKS.json hbm_gbs.
cpu_baseline = the CPU restatement of the reference path (oracle/, test
             infrastructure) timed on this host on a bounded token sample.
--impl reference: the reference's CPU path (the same restatement, all host
             threads) on the same workload/metric; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (H, I, E, K, norm_topk, T, layers_in_step, description)
    "c0": dict(H=2048, I=1024, E=64, K=8, norm=False, T=1, stack=1,
               workload="olmoe_layer_decode_T1"),
    "c1": dict(H=2048, I=1024, E=64, K=8, norm=False, T=512, stack=1,
               workload="olmoe_layer_prefill_T512"),
    "c2": dict(H=2048, I=1024, E=64, K=8, norm=False, T=8, stack=16,
               workload="olmoe_16layer_decode_T8"),
    "c3": dict(H=2048, I=768, E=128, K=8, norm=True, T=64, stack=48,
               workload="qwen3_48layer_decode_T64"),
    "c4": dict(H=2048, I=768, E=128, K=8, norm=True, T=4096, stack=1, zipf=True,
               strong=True, workload="qwen3_layer_prefill_T4096_zipf1.1"),
}
SEED = 20261201


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1630.8)), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def algorithmic_bytes(cfg, D: float, T: int, wdiv: int = 1) -> dict:
    """Per-layer algorithmic bytes: active expert weights + scales once, the
    router once, the hidden states in and the outputs out.  wdiv = 2 for INT4
    experts (two weights per byte)."""
    H, I, E, K = cfg["H"], cfg["I"], cfg["E"], cfg["K"]
    R = T * K
    layer = D * (3 * I * H // wdiv + 4 * (2 * I + H)) + 4 * E * H + 8 * T * H
    gate_up = D * (2 * I * H // wdiv + 8 * I) + 4 * T * H + 4 * R * I
    down = D * (I * H // wdiv + 4 * H) + 4 * R * I + 4 * R * H
    return {"layer": layer, "gate_up_gemv": gate_up, "down_gemv": down,
            "gate_up_tc": gate_up, "down_tc": down}


def int4_from_int8(w8):
    """Synthetic INT4 experts from the INT8 generator: each weight keeps its
    top four bits (w >> 4, in [-8, 7]); element 2i goes to the low nibble of
    byte i (src/int8_expert.rs:473-516).  numpy or torch, any leading shape."""
    lo, hi = (w8[..., 0::2] >> 4) & 0xF, (w8[..., 1::2] >> 4) & 0xF
    packed = lo | (hi << 4)  # int8 bit patterns
    if isinstance(packed, np.ndarray):
        return packed.view(np.uint8)
    import torch
    return packed.contiguous().view(torch.uint8)


def oracle_layer(cfg, quant):
    from oracle import oracle as O
    H, I, E, K = cfg["H"], cfg["I"], cfg["E"], cfg["K"]
    L = O.synth_layer(SEED, 0, H, I, E, K, cfg["norm"])
    if quant == "int4":
        L = O.LayerWeights(H, I, E, K, cfg["norm"], L.router, int4_from_int8(L.experts),
                           (L.scales * 16.0).astype(np.float32), int4=True)
    return L


def run_reference(args, cfg, rank, world):
    """The reference's CPU path (C restatement), all host threads, rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    H, I, E, K, T = cfg["H"], cfg["I"], cfg["E"], cfg["K"], cfg["T"]
    L = oracle_layer(cfg, args.quant)
    sample = min(T, 32)
    h = O.synth_hidden(SEED, sample, H)
    for _ in range(max(1, args.warmup)):
        O.layer_forward(L, h[: min(sample, 2)], nthreads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(cfg["stack"]):
            O.layer_forward(L, h, nthreads=threads,
                            decode_schedule=cfg["T"] <= 64)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    v = sample / sec
    line = {"impl": "reference", "metric": "moe_layer_tokens_per_s", "value": v,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload_name(cfg, args.quant), "hidden": H,
                       "intermediate": I, "experts": E, "top_k": K, "tokens": T,
                       "layers": cfg["stack"], "weights": args.quant},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"{sample} of {T} tokens per step, "
                                       f"{cfg['stack']} layer(s)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_name(cfg, quant):
    return cfg["workload"] + ("_int4" if quant == "int4" else "")


def cpu_baseline(cfg, quant="int8") -> dict:
    """Oracle (C restatement of the reference CPU path) on a bounded sample."""
    from oracle import oracle as O
    threads = min(8, os.cpu_count() or 1)  # the reference's default pool, src/backend.rs:21-24
    H, I, E, K, T = cfg["H"], cfg["I"], cfg["E"], cfg["K"], cfg["T"]
    L = oracle_layer(cfg, quant)
    sample = min(T, 32)
    h = O.synth_hidden(SEED, sample, H)
    O.layer_forward(L, h[:1], nthreads=threads)
    reps, t_total = 0, 0.0
    t_start = time.perf_counter()
    while reps < 1 or (time.perf_counter() - t_start < 10.0 and reps < 20):
        t0 = time.perf_counter()
        O.layer_forward(L, h, nthreads=threads, decode_schedule=T <= 64)
        t_total += time.perf_counter() - t0
        reps += 1
    per_token = t_total / (reps * sample)
    return {"value": 1.0 / (per_token * cfg["stack"]), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": f"{reps} x {sample} of {T} tokens, one layer, {threads} threads; "
                      f"scaled to {cfg['stack']} layer(s)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c1", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--path", default="auto", choices=["auto", "gemv", "tensor", "gemv_fused",
                                                          "gemv_stream"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quant", default="int8", choices=["int8", "int4"],
                    help="expert weight format (int4: two signed nibbles per byte)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return

    import torch
    import torch.distributed as dist
    import doantotnghiepmoe_b200 as M
    from doantotnghiepmoe_b200 import synthetic

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if world > 1:
        return run_ep(args, cfg, rank, world, local)
    H, I, E, K, T = cfg["H"], cfg["I"], cfg["E"], cfg["K"], cfg["T"]
    n_stack = cfg["stack"]
    wdiv = 2 if args.quant == "int4" else 1
    if wdiv == 2 and args.path in ("tensor", "gemv_stream"):
        raise SystemExit("--quant int4 runs on the exact GEMV paths only")
    layer_bytes = E * (3 * I * H // wdiv + 4 * (2 * I + H))
    # Rotation of distinct layers so that consecutive steps never hit L2.
    n_layers = max(n_stack, int(np.ceil(3 * 126e6 / layer_bytes)) + 1)
    if n_stack > 1:
        n_layers = n_stack
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, cfg["norm"], T, n_layers), device=local)
    stream = torch.cuda.Stream()
    eng.set_stream(stream)
    eng.set_path({"auto": 0, "gemv": 1, "tensor": 2, "gemv_fused": 4,
                  "gemv_stream": 5}[args.path])
    keep = []
    with torch.cuda.stream(stream):
        for l in range(n_layers):
            ex = torch.empty((E, 3 * I * H), dtype=torch.int8, device="cuda")
            sc = torch.empty((E, 2 * I + H), dtype=torch.float32, device="cuda")
            for e in range(E):
                M.synth_expert(SEED, l, e, H, I, ex[e], sc[e], stream=stream)
            if wdiv == 2:
                ex, sc = int4_from_int8(ex), sc * 16.0
            rt = torch.from_numpy(synthetic.router(SEED, l, E, H, cfg.get("zipf", False))).cuda()
            eng.set_layer_packed(l, ex, sc, rt)
            keep.append((ex, sc, rt))
        n_inputs = n_layers if n_stack == 1 else 2
        hs = [torch.from_numpy(synthetic.hidden(SEED, i, T, H, cfg.get("zipf", False))).cuda()
              for i in range(n_inputs)]
        outs = [torch.empty((T, H), dtype=torch.float32, device="cuda") for _ in range(2)]
        ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    stream.synchronize()

    def step(i):
        if n_stack == 1:
            eng.forward(i % n_layers, hs[i % n_inputs], outs[i % 2], ids=ids, stream=stream)
        else:
            x = outs[i % 2]
            x.copy_(hs[i % n_inputs])
            eng.stack_forward(0, n_stack, x, 1e-5, stream=stream)

    # distinct experts touched per step (D), from the routing of each input
    Ds = []
    with torch.cuda.stream(stream):
        for i in range(n_inputs if n_stack == 1 else 1):
            eng.forward(i % n_layers, hs[i % n_inputs], outs[0], ids=ids, stream=stream)
            stream.synchronize()
            Ds.append(len(np.unique(ids.cpu().numpy())))
    D = float(np.mean(Ds))
    shares = np.bincount(ids.cpu().numpy().ravel(), minlength=E) / ids.numel()
    eng.sync_status(stream)

    # warm-up: W steps, then one untimed pass over the timed steps' inputs so
    # that every (layer, buffers) combination has its launch graph captured
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
        for i in range(args.steps):
            step(i)
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    eng.profile(False)
    launches = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
            launches += eng.last_launch_count()
        ev1.record(stream)
    ev1.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    # kernel breakdown: the same steps again with CUDA events between the
    # kernels (direct launches), for kernel_share and the roofline
    eng.profile_read()
    eng.profile(True)
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            step(i)
    stream.synchronize()
    eng.profile(False)
    prof = eng.profile_read()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    tokens_per_step = T * world
    value = tokens_per_step / (ms_max / 1e3)
    eng.sync_status(stream)

    # ---- e2e through the host-buffer C-ABI call --------------------------
    e2e = None
    if n_stack == 1:
        # pinned host buffers from the library (moe_host_alloc), kept across
        # steps as a serving loop keeps them; the library DMAs straight from
        # and into them
        h_host = []
        for i in range(min(2, n_inputs)):
            buf = M.host_empty((T, H), np.float32)
            buf[:] = hs[i].cpu().numpy()
            h_host.append(buf)
        o_host = [M.host_empty((T, H), np.float32) for _ in range(2)]
        i_host = M.host_empty((T, K), np.uint32)
        g_host = M.host_empty((T, K), np.float32)

        def host_step(i):
            eng.forward_host(i % n_layers, h_host[i % len(h_host)], out=o_host[i % 2],
                             ids=i_host, gates=g_host)

        for i in range(2):
            host_step(i)
        e_ev0, e_ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_ev0.record(stream)
        for i in range(args.steps):
            host_step(i)
        e_ev1.record(stream)
        e_ev1.synchronize()
        e_ms = e_ev0.elapsed_time(e_ev1) / args.steps
        e_t = torch.tensor([e_ms], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
        e2e = {"value": tokens_per_step / (float(e_t.item()) / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4 + 2 * T * K * 4}

    # ---- roofline of the dominant kernel --------------------------------
    hbm_peak, _, peak_kind = measured_peaks()
    alg = algorithmic_bytes(cfg, D, T, wdiv)
    alg["fused_decode"] = alg["layer"] * n_stack  # one launch runs the whole step
    alg["stream_decode"] = alg["layer"] * n_stack
    phases = {k: v for k, v in prof.items() if ":" in k}
    prof = {k: v for k, v in prof.items() if ":" not in k}
    top = max(prof.items(), key=lambda kv: kv[1][1]) if prof else ("none", (1, 0.0))
    kname, (klaunch, kms) = top
    k_avg_ms = kms / max(1, klaunch)
    kbytes = alg.get(kname, alg["layer"])
    achieved = kbytes / (k_avg_ms / 1e3) / 1e9 if k_avg_ms > 0 else 0.0
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            tj = json.load(f)
        ent = tj.get(workload_name(cfg, args.quant), {}).get(kname)
        if ent:
            traffic = ent.get("bytes_per_launch")
    roofline = {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm_peak,
                "unit": "GB/s", "frac": achieved / hbm_peak, "traffic": traffic,
                "peak_kind": peak_kind, "alg_bytes_per_launch": kbytes,
                "mean_launch_ms": k_avg_ms,
                "kernel_share": {k: round(v[1] / max(1e-9, sum(x[1] for x in prof.values())), 4)
                                 for k, v in prof.items()},
                "fused_phases_us": {k: round(v[1] * 1e3, 2) for k, v in phases.items()}}
    layer_gbs = alg["layer"] * n_stack / (ms_max / 1e3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(cfg, args.quant)
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "port",
                   "sample": f"failed: {exc}"}

    if rank == 0:
        line = {"metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": workload_name(cfg, args.quant), "hidden": H,
                           "intermediate": I, "weights": args.quant,
                           "experts": E, "top_k": K, "norm_topk_prob": cfg["norm"],
                           "tokens_per_rank": T, "layers_per_step": n_stack,
                           "distinct_experts_per_layer": D,
                           "l2": f"weights rotate over {n_layers} layers "
                                 f"({layer_bytes * n_layers / 1e9:.1f} GB) > 126 MB L2",
                           "parallelism": "single",
                           "path": args.path,
                           "expert_share_top5": [round(float(x), 4) for x in
                                                 np.sort(shares)[::-1][:5]],
                           "expert_share_max_over_mean": round(float(shares.max() * E), 2)},
                "layer_hbm_gbs": layer_gbs,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches, "clocks": clk}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ep(args, cfg, rank, world, local):
    """Expert parallelism over `world` GPUs (one process each): experts are
    split evenly (balanced by expected load), every rank routes its own
    tokens; NCCL dispatch/combine inside the library.  Tokens per rank: the
    config's T (weak scaling), or T / world for the strong-scaling config."""
    import torch
    import torch.distributed as dist

    import doantotnghiepmoe_b200 as M
    from doantotnghiepmoe_b200 import placement, synthetic

    H, I, E, K = cfg["H"], cfg["I"], cfg["E"], cfg["K"]
    strong = cfg.get("strong", False)
    T = cfg["T"] // world if strong else cfg["T"]
    zipf = cfg.get("zipf", False)
    if zipf:
        w, _ = synthetic.zipf_weights(E, SEED)
        owner = placement.balanced_owner(np.minimum(w, 1.0 / K), world)
    else:
        owner = placement.contiguous_owner(E, world)
    loc = placement.local_experts(owner, rank)
    EL = len(loc)
    layer_bytes_local = EL * (3 * I * H + 4 * (2 * I + H))
    n_layers = max(2, int(np.ceil(3 * 126e6 / max(1, layer_bytes_local))) + 1)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, cfg["norm"], T, n_layers), device=local)
    stream = torch.cuda.Stream()
    eng.set_stream(stream)
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid = torch.tensor(list(M.layer.ep_unique_id()), dtype=torch.uint8, device="cuda")
    dist.broadcast(uid, 0)
    eng.ep_init(rank, world, bytes(uid.cpu().tolist()), owner)
    keep = []
    with torch.cuda.stream(stream):
        for l in range(n_layers):
            ex = torch.empty((max(EL, 1), 3 * I * H), dtype=torch.int8, device="cuda")
            sc = torch.empty((max(EL, 1), 2 * I + H), dtype=torch.float32, device="cuda")
            for j, e in enumerate(loc):
                M.synth_expert(SEED, l, int(e), H, I, ex[j], sc[j], stream=stream)
            rt = torch.from_numpy(synthetic.router(SEED, l, E, H, zipf)).cuda()
            eng.ep_set_layer(l, ex, sc, rt)
            keep.append((ex, sc, rt))
        hs = [torch.from_numpy(synthetic.hidden(SEED, 1000 * rank + i, T, H, zipf)).cuda()
              for i in range(2)]
        outs = [torch.empty((T, H), dtype=torch.float32, device="cuda") for _ in range(2)]
    stream.synchronize()

    def step(i):
        eng.ep_forward(i % n_layers, hs[i % 2], outs[i % 2], stream=stream)

    # warm-up, plus one untimed pass over the timed steps (launch graphs)
    for i in range(args.warmup):
        step(i)
    for i in range(args.steps):
        step(i)
    stream.synchronize()
    eng.sync_status(stream)
    dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    eng.profile(False)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
        launches += eng.last_launch_count()
    ev1.record(stream)
    ev1.synchronize()
    dist.barrier()
    clk = clocks.stop()
    # kernel breakdown: the same steps with CUDA events between the kernels
    # (all ranks start together, so no rank's first wait absorbs the skew)
    torch.cuda.synchronize()
    dist.barrier()
    eng.profile_read()
    eng.profile(True)
    for i in range(args.steps):
        step(i)
    stream.synchronize()
    eng.profile(False)
    prof = eng.profile_read()
    dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    tokens = T * world
    value = tokens / (ms_max / 1e3)
    # e2e: host hidden states in (pinned), layer, host outputs back, per step
    h_host = []
    for i in range(2):
        buf = M.host_empty((T, H), np.float32)
        buf[:] = hs[i].cpu().numpy()
        h_host.append(torch.from_numpy(buf))
    o_host = [torch.from_numpy(M.host_empty((T, H), np.float32)) for _ in range(2)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    e0.record(stream)
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            hs[i % 2].copy_(h_host[i % 2], non_blocking=True)
            step(i)
            o_host[i % 2].copy_(outs[i % 2], non_blocking=True)
    e1.record(stream)
    e1.synchronize()
    e_t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device="cuda")
    dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e2e = {"value": tokens / (float(e_t.item()) / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4}
    eng.sync_status(stream)
    hbm_peak, _, peak_kind = measured_peaks()
    top = max(prof.items(), key=lambda kv: kv[1][1]) if prof else ("none", (1, 0.0))
    kname, (klaunch, kms) = top
    tot = max(1e-9, sum(v[1] for v in prof.values()))
    # local weight bytes streamed per step (every local expert is active)
    local_gbs = layer_bytes_local / (ms_max / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": "ep_layer", "achieved": local_gbs, "peak": hbm_peak,
                "unit": "GB/s", "frac": local_gbs / hbm_peak, "traffic": None,
                "peak_kind": peak_kind, "alg_bytes_per_launch": layer_bytes_local,
                "mean_launch_ms": ms_max, "top_kernel": kname,
                "kernel_share": {k: round(v[1] / tot, 4) for k, v in prof.items()}}
    if rank == 0:
        line = {"metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_max, "higher_is_better": True,
                "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic",
                "config": {"workload": cfg["workload"], "hidden": H, "intermediate": I,
                           "experts": E, "top_k": K, "norm_topk_prob": cfg["norm"],
                           "tokens_per_rank": T, "experts_per_rank": EL,
                           "parallelism": f"ep{world}",
                           "transport": eng.ep_transport(),
                           "placement": "balanced" if zipf else "contiguous",
                           "l2": f"weights rotate over {n_layers} layers > 126 MB L2"},
                "roofline": roofline, "cpu_baseline": None, "e2e": e2e,
                "gpu_launches": launches, "clocks": clk}
        print(json.dumps(line), flush=True)
    eng.ep_finalize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
