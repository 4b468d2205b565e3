"""Benchmark of the B200 MoE-layer hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c0..c4]
                    [--impl ours|reference] [--path auto|gemv|tensor|digits]

A step is one MoE layer (router -> softmax -> top-k -> permutation -> INT8
SwiGLU experts -> slot-ordered combine) over one batch of synthetic tokens,
or the whole stack for the stacked decode configs.  The default workload is
the Qwen3-30B-A3B-shaped prefill layer (H=2048, I=768, E=128,
K=8, normalized gates), 4096 tokens with Zipf(1.1) expert popularity, strong
scaling: at N GPUs each rank routes 4096/N tokens and owns E/N experts
(expert parallelism over NVLink).  Inputs are larger than L2: each step uses
a different layer's weights out of a rotation, so nothing is reused from L2
between steps.

value      = tokens processed by all ranks / device time (CUDA events on the
             launching stream, max over ranks), inputs already in HBM.
e2e        = the same metric with the step's hidden states copied in from
             pinned host memory and the outputs copied back inside the timed
             region (N=1: the host-buffer C-ABI call moe_layer_forward_host).
roofline   = the dominant kernel's algorithmic bytes (HBM) or int8 tensor
             operations per launch / its mean CUDA-event duration, against
             MEASURED_PEAKS.json; the limiting resource is the larger fraction.
parity     = routing ids and outputs of a token sample against the CPU
             restatement of the reference path (oracle/, test infrastructure),
             checked after the timed region.
decode_c0  = (N=1) configs[0], the OLMoE layer at batch-1 decode, timed in the
             same run, beside a plain read of its algorithmic bytes
             (moe_debug_stream_read): the single-launch ceiling on this GPU.
cpu_baseline = the CPU restatement timed on this host on a bounded sample.
--impl reference: the reference's CPU path (the same restatement, all host
             threads) on the same workload/metric/config; rank 0 only.
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
    "c0": dict(H=2048, I=1024, E=64, K=8, norm=False, T=1, stack=1,
               workload="olmoe_layer_decode_T1"),
    "c1": dict(H=2048, I=1024, E=64, K=8, norm=False, T=512, stack=1,
               workload="olmoe_layer_prefill_T512"),
    "c2": dict(H=2048, I=1024, E=64, K=8, norm=False, T=8, stack=16,
               workload="olmoe_16layer_decode_T8"),
    "c2t1": dict(H=2048, I=1024, E=64, K=8, norm=False, T=1, stack=16,
                 workload="olmoe_16layer_decode_T1"),
    "c2t32": dict(H=2048, I=1024, E=64, K=8, norm=False, T=32, stack=16,
                  workload="olmoe_16layer_decode_T32"),
    "c3": dict(H=2048, I=768, E=128, K=8, norm=True, T=64, stack=48,
               workload="qwen3_48layer_decode_T64"),
    "c4": dict(H=2048, I=768, E=128, K=8, norm=True, T=4096, stack=1, zipf=True,
               strong=True, workload="qwen3_layer_prefill_T4096_zipf1.1"),
}
DEFAULT_CONFIG = "c4"
SEED = 20261201
PATHS = {"auto": 0, "gemv": 1, "tensor": 2, "gemv_fused": 4, "digits": 5}
L2_NOTE = "every step uses another layer's weights (rotation larger than the 126 MB L2)"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks():
    """(HBM GB/s, int8 tensor TOP/s, kind).  The int8 dense peak is taken as
    twice the measured bf16 GEMM rate (the nominal int8:bf16 ratio is 2:1)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), 2.0 * float(d.get("bf16_tflops", 1630.8)), "measured"
    return 6650.0, 2.0 * 1590.0, "fallback"


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


def tokens_per_step(cfg, world):
    return cfg["T"] if cfg.get("strong") else cfg["T"] * world


def config_dict(cfg, quant, world):
    """The `config` object, identical in both arms."""
    total = tokens_per_step(cfg, world)
    return {"workload": workload_name(cfg, quant), "hidden": cfg["H"],
            "intermediate": cfg["I"], "experts": cfg["E"], "top_k": cfg["K"],
            "norm_topk_prob": cfg["norm"], "weights": quant, "tokens_per_step": total,
            "tokens_per_rank": total // world, "layers_per_step": cfg["stack"],
            "router_bias": "zipf1.1" if cfg.get("zipf") else "none",
            "parallelism": "single" if world == 1 else f"ep{world}", "l2": L2_NOTE}


def kernel_work(cfg, kname, D, T, wdiv=1):
    """(algorithmic HBM bytes, int8 tensor ops) of one launch of a kernel of a
    layer step over T tokens touching D distinct experts.  Tensor-core GEMMs
    multiply both activation digit planes: 2 ops per MAC per plane."""
    H, I, E, K = cfg["H"], cfg["I"], cfg["E"], cfg["K"]
    R = T * K
    layer = D * (3 * I * H // wdiv + 4 * (2 * I + H)) + 4 * E * H + 8 * T * H
    gate_up = D * (2 * I * H // wdiv + 8 * I) + 4 * T * H + 4 * R * I
    down = D * (I * H // wdiv + 4 * H) + 4 * R * I + 4 * R * H
    table = {"layer": (layer, 0), "gate_up_gemv": (gate_up, 0), "down_gemv": (down, 0),
             "gate_up_tc": (gate_up, 2 * 2 * R * 2 * I * H),
             "down_tc": (down, 2 * 2 * R * H * I)}
    return table.get(kname, (layer, 0))


def roofline_of(cfg, prof, D, T, n_stack, wdiv=1):
    """Roofline of the dominant kernel of a profiled pass (name -> (launches, ms))."""
    hbm_peak, tops_peak, kind = measured_peaks()
    phases = {k: v for k, v in prof.items() if ":" in k}
    prof = {k: v for k, v in prof.items() if ":" not in k}
    top = max(prof.items(), key=lambda kv: kv[1][1]) if prof else ("none", (1, 0.0))
    kname, (klaunch, kms) = top
    avg_ms = kms / max(1, klaunch)
    nbytes, ops = kernel_work(cfg, kname, D, T, wdiv)
    if kname in ("fused_decode", "digit_decode"):  # one launch runs the whole step
        nbytes = kernel_work(cfg, "layer", D, T, wdiv)[0] * n_stack
    gbs = nbytes / (avg_ms / 1e3) / 1e9 if avg_ms > 0 else 0.0
    tops = ops / (avg_ms / 1e3) / 1e12 if avg_ms > 0 else 0.0
    f_hbm, f_tc = gbs / hbm_peak, (tops / tops_peak if ops else 0.0)
    tot = max(1e-9, sum(v[1] for v in prof.values()))
    r = {"bound": "hbm", "kernel": kname, "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
         "frac": f_hbm, "traffic": None, "peak_kind": kind, "alg_bytes_per_launch": nbytes,
         "mean_launch_ms": avg_ms,
         "kernel_share": {k: round(v[1] / tot, 4) for k, v in prof.items()},
         "fused_phases_us": {k: round(v[1] * 1e3, 2) for k, v in phases.items()}}
    if ops:
        r["tensor"] = {"achieved_tops": tops, "peak_tops": tops_peak, "frac": f_tc,
                       "ops_per_launch": ops,
                       "peak_note": "int8 dense peak = 2 x measured bf16 GEMM rate"}
        if f_tc > f_hbm:
            r.update(bound="tensor", achieved=tops, peak=tops_peak, unit="TOP/s", frac=f_tc)
    return r


def traffic_of(cfg, quant, kname):
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(tp):
        return None
    with open(tp) as f:
        ent = json.load(f).get(workload_name(cfg, quant), {}).get(kname)
    return ent.get("bytes_per_launch") if ent else None


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


def oracle_layer(cfg, quant, layer=0):
    """Host copy of a synthetic layer (bit-identical to the device generator)."""
    from oracle import oracle as O

    from doantotnghiepmoe_b200 import synthetic
    H, I, E, K = cfg["H"], cfg["I"], cfg["E"], cfg["K"]
    L = O.synth_layer(SEED, layer, H, I, E, K, cfg["norm"])
    router = synthetic.router(SEED, layer, E, H, cfg.get("zipf", False))
    L = O.LayerWeights(H, I, E, K, cfg["norm"], router, L.experts, L.scales)
    if quant == "int4":
        L = O.LayerWeights(H, I, E, K, cfg["norm"], L.router, int4_from_int8(L.experts),
                           (L.scales * 16.0).astype(np.float32), int4=True)
    return L


def workload_name(cfg, quant):
    return cfg["workload"] + ("_int4" if quant == "int4" else "")


def run_reference(args, cfg, rank, world):
    """The reference's CPU path (C restatement), all host threads, rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as O

    from doantotnghiepmoe_b200 import synthetic
    threads = os.cpu_count() or 1
    H, T = cfg["H"], cfg["T"]
    L = oracle_layer(cfg, args.quant)
    sample = min(T, 64)
    h = synthetic.hidden(SEED, 0, sample, H, cfg.get("zipf", False))
    for _ in range(max(1, args.warmup)):
        O.layer_forward(L, h[: min(sample, 2)], nthreads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(cfg["stack"]):
            O.layer_forward(L, h, nthreads=threads, decode_schedule=T <= 64)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    v = sample / sec
    line = {"impl": "reference", "metric": "moe_layer_tokens_per_s", "value": v,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sec * 1e3 * tokens_per_step(cfg, world) / sample,
            "higher_is_better": True, "scaling": "strong" if cfg.get("strong") else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(cfg, args.quant, world),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"{sample} of {tokens_per_step(cfg, world)} tokens per "
                                       f"step ({cfg['stack']} layer(s)); ms_per_step scaled "
                                       f"to the whole step"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline(cfg, quant="int8") -> dict:
    """Oracle (C restatement of the reference CPU path) on a bounded sample."""
    from oracle import oracle as O

    from doantotnghiepmoe_b200 import synthetic
    threads = min(8, os.cpu_count() or 1)  # the reference's default pool, src/backend.rs:21-24
    H, T = cfg["H"], cfg["T"]
    L = oracle_layer(cfg, quant)
    sample = min(T, 32)
    h = synthetic.hidden(SEED, 0, sample, H, cfg.get("zipf", False))
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


def parity_check(L, h_np, ids_np, out_np, rows) -> dict:
    """Routing ids (bit-exact) and outputs (max rel err) of the sampled token
    rows against the oracle on the same inputs."""
    from oracle import oracle as O
    ref = O.layer_forward(L, h_np[rows], nthreads=min(8, os.cpu_count() or 1))
    ids_ok = bool(np.array_equal(ids_np[rows].astype(np.uint32), ref.ids))
    err = float(np.abs(out_np[rows].astype(np.float64) - ref.out).max() /
                max(np.abs(ref.out).max(), 1e-6))
    return {"ids_exact": ids_ok, "max_rel_err": err, "tokens_checked": int(len(rows)),
            "tolerance": 1e-3}


def make_layers(M, eng, cfg, n_layers, quant, stream, local_ids=None, ep=False):
    """Synthetic layers on the device (weights from the seeded generator)."""
    import torch

    from doantotnghiepmoe_b200 import synthetic
    H, I, E = cfg["H"], cfg["I"], cfg["E"]
    ids = list(range(E)) if local_ids is None else [int(e) for e in local_ids]
    keep = []
    with torch.cuda.stream(stream):
        for l in range(n_layers):
            n = max(len(ids), 1)
            ex = torch.empty((n, 3 * I * H), dtype=torch.int8, device="cuda")
            sc = torch.empty((n, 2 * I + H), dtype=torch.float32, device="cuda")
            for j, e in enumerate(ids):
                M.synth_expert(SEED, l, e, H, I, ex[j], sc[j], stream=stream)
            if quant == "int4":
                ex, sc = int4_from_int8(ex), sc * 16.0
            rt = torch.from_numpy(synthetic.router(SEED, l, E, H, cfg.get("zipf", False))).cuda()
            if ep:
                eng.ep_set_layer(l, ex, sc, rt)
            else:
                eng.set_layer_packed(l, ex, sc, rt)
            keep.append((ex, sc, rt))
    stream.synchronize()
    return keep


def rotation(cfg, quant, local_experts=None):
    wdiv = 2 if quant == "int4" else 1
    E = cfg["E"] if local_experts is None else max(1, local_experts)
    layer_bytes = E * (3 * cfg["I"] * cfg["H"] // wdiv + 4 * (2 * cfg["I"] + cfg["H"]))
    if cfg["stack"] > 1:
        return cfg["stack"], layer_bytes
    return max(2, int(np.ceil(3 * 126e6 / layer_bytes)) + 1), layer_bytes


def time_steps(step, n, stream):
    import torch
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(n):
        step(i)
    ev1.record(stream)
    ev1.synchronize()
    return ev0.elapsed_time(ev1) / n


def measure_decode_c0(M, args, local) -> dict:
    """configs[0] in the same run: one OLMoE layer at batch 1 through the
    default path, beside a plain read of the layer's algorithmic bytes."""
    import torch

    from doantotnghiepmoe_b200 import synthetic
    cfg = CONFIGS["c0"]
    H, I, E, K = cfg["H"], cfg["I"], cfg["E"], cfg["K"]
    n_layers, _ = rotation(cfg, "int8")
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, cfg["norm"], 1, n_layers), device=local)
    stream = torch.cuda.Stream()
    eng.set_stream(stream)
    eng.set_path(PATHS[args.path])
    keep = make_layers(M, eng, cfg, n_layers, "int8", stream)
    hs = [torch.from_numpy(synthetic.hidden(SEED, 50 + i, 1, H)).cuda() for i in range(n_layers)]
    outs = [torch.empty((1, H), dtype=torch.float32, device="cuda") for _ in range(2)]
    ids = torch.empty((1, K), dtype=torch.int32, device="cuda")
    stream.synchronize()
    steps = max(args.steps, 50)

    def step(i):
        eng.forward(i % n_layers, hs[i % n_layers], outs[i % 2], ids=ids, stream=stream)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3) + steps):
            step(i)
        stream.synchronize()
        eng.sync_status(stream)
        ms = time_steps(step, steps, stream)
        eng.sync_status(stream)
        eng.profile_read()
        eng.profile(True)
        for i in range(steps):
            step(i)
        stream.synchronize()
        eng.profile(False)
        prof = eng.profile_read()
    D = float(K)
    roof = roofline_of(cfg, prof, D, 1, 1)
    alg = kernel_work(cfg, "layer", D, 1)[0]
    # the ceiling: the same byte count read by one plain launch, rotating over
    # buffers that together exceed L2 (back to back, like the layer steps)
    nbuf = 8
    nb = (int(alg) + 15) // 16 * 16
    bufs = [torch.empty(nb, dtype=torch.uint8, device="cuda") for _ in range(nbuf)]
    sink = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = M.lib()

    def read(i):
        st = L.moe_debug_stream_read(bufs[i % nbuf].data_ptr(), nb, sink.data_ptr(),
                                     stream.cuda_stream)
        assert st == 0, st

    with torch.cuda.stream(stream):
        for i in range(10):
            read(i)
        stream.synchronize()
        read_ms = time_steps(read, steps, stream)
    hbm_peak, _, _ = measured_peaks()
    del bufs, keep
    eng.close()
    return {"workload": cfg["workload"], "path": args.path, "ms_per_layer": ms,
            "tokens_per_s": 1.0 / (ms / 1e3), "alg_bytes": alg,
            "layer_gbs": alg / (ms / 1e3) / 1e9, "layer_frac": alg / (ms / 1e3) / 1e9 / hbm_peak,
            "roofline": roof,
            "ceiling": {"what": "moe_debug_stream_read of the layer's algorithmic bytes, "
                                "one launch per step, rotating over 8 buffers",
                        "ms": read_ms, "gbs": alg / (read_ms / 1e3) / 1e9,
                        "frac": alg / (read_ms / 1e3) / 1e9 / hbm_peak,
                        "layer_vs_ceiling": read_ms / ms}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--path", default="auto", choices=sorted(PATHS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the same-run configs[0] decode measurement")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--quant", default="int8", choices=["int8", "int4"],
                    help="expert weight format (int4: two signed nibbles per byte)")
    ap.add_argument("--tokens", type=int, default=0,
                    help="override the config's token count (the workload name says so)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    if args.tokens > 0 and args.tokens != cfg["T"]:
        cfg = dict(cfg, T=args.tokens, workload=f"{cfg['workload']}_as_T{args.tokens}")
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return

    import torch
    import torch.distributed as dist

    import doantotnghiepmoe_b200 as M

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        try:
            return run_ep(args, cfg, rank, world, local)
        finally:
            dist.destroy_process_group()
    run_single(args, cfg, local)


def run_single(args, cfg, local):
    import torch

    import doantotnghiepmoe_b200 as M
    from doantotnghiepmoe_b200 import synthetic

    H, I, E, K, T = cfg["H"], cfg["I"], cfg["E"], cfg["K"], cfg["T"]
    n_stack = cfg["stack"]
    wdiv = 2 if args.quant == "int4" else 1
    if wdiv == 2 and args.path in ("tensor", "digits"):
        raise SystemExit("--quant int4 runs on the exact GEMV paths only")
    n_layers, layer_bytes = rotation(cfg, args.quant)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, cfg["norm"], T, n_layers), device=local)
    stream = torch.cuda.Stream()
    eng.set_stream(stream)
    eng.set_path(PATHS[args.path])
    keep = make_layers(M, eng, cfg, n_layers, args.quant, stream)
    zipf = cfg.get("zipf", False)
    n_inputs = n_layers if n_stack == 1 else 2
    hs = [torch.from_numpy(synthetic.hidden(SEED, i, T, H, zipf)).cuda() for i in range(n_inputs)]
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
    clk = clocks.stop()
    eng.sync_status(stream)
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
    ms = ev0.elapsed_time(ev1) / args.steps
    value = T / (ms / 1e3)
    eng.sync_status(stream)

    # ---- parity of a token sample against the oracle (untimed) -----------
    parity = None
    if not args.no_parity and n_stack == 1:
        with torch.cuda.stream(stream):
            eng.forward(0, hs[0], outs[0], ids=ids, stream=stream)
        stream.synchronize()
        eng.sync_status(stream)
        rows = np.unique(np.linspace(0, T - 1, min(T, 256)).astype(np.int64))
        parity = parity_check(oracle_layer(cfg, args.quant, 0), hs[0].cpu().numpy(),
                              ids.cpu().numpy(), outs[0].cpu().numpy(), rows)
        parity["path"] = args.path

    # ---- e2e through the host-buffer C-ABI call --------------------------
    e2e = None
    if n_stack == 1:
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
        e_ms = time_steps(host_step, args.steps, stream)
        e2e = {"value": T / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4 + 2 * T * K * 4}

    roofline = roofline_of(cfg, prof, D, T, n_stack, wdiv)
    roofline["traffic"] = traffic_of(cfg, args.quant, roofline["kernel"])
    layer_gbs = kernel_work(cfg, "layer", D, T, wdiv)[0] * n_stack / (ms / 1e3) / 1e9
    del keep
    eng.close()

    decode = None
    if not args.no_decode and args.config != "c0":
        decode = measure_decode_c0(M, args, local)

    cpu = None
    if not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(cfg, args.quant)
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "port",
                   "sample": f"failed: {exc}"}

    line = {"metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if cfg.get("strong") else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(cfg, args.quant, 1),
            "detail": {"path": args.path, "distinct_experts_per_layer": D,
                       "rotation_layers": n_layers,
                       "rotation_gb": round(layer_bytes * n_layers / 1e9, 2),
                       "expert_share_top5": [round(float(x), 4)
                                             for x in np.sort(shares)[::-1][:5]],
                       "expert_share_max_over_mean": round(float(shares.max() * E), 2)},
            "layer_hbm_gbs": layer_gbs, "roofline": roofline, "parity": parity,
            "decode_c0": decode, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches, "clocks": clk}
    print(json.dumps(line), flush=True)


def run_ep(args, cfg, rank, world, local):
    """Expert parallelism over `world` GPUs (one process each): experts split
    evenly (balanced by expected load), every rank routes its own tokens;
    dispatch and combine inside the library."""
    import torch
    import torch.distributed as dist

    import doantotnghiepmoe_b200 as M
    from doantotnghiepmoe_b200 import ep_group, placement, synthetic

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
    n_layers, layer_bytes_local = rotation(cfg, "int8", EL)
    n_layers = max(2, n_layers)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, cfg["norm"], T, n_layers), device=local)
    stream = torch.cuda.Stream()
    eng.set_stream(stream)
    ep_group.join(eng, rank, world, owner)
    keep = make_layers(M, eng, cfg, n_layers, "int8", stream, local_ids=loc, ep=True)
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
    launches = 0

    def counted(i):
        nonlocal launches
        step(i)
        launches += eng.last_launch_count()

    ms = time_steps(counted, args.steps, stream)
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

    def host_step(i):
        with torch.cuda.stream(stream):
            hs[i % 2].copy_(h_host[i % 2], non_blocking=True)
            step(i)
            o_host[i % 2].copy_(outs[i % 2], non_blocking=True)

    dist.barrier()
    e_t = torch.tensor([time_steps(host_step, args.steps, stream)], dtype=torch.float64,
                       device="cuda")
    dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e2e = {"value": tokens / (float(e_t.item()) / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": tokens * H * 4, "d2h_bytes_per_step": tokens * H * 4}
    eng.sync_status(stream)

    # ---- parity: every rank checks a sample of its tokens (untimed) -------
    parity = None
    if not args.no_parity:
        with torch.cuda.stream(stream):
            eng.ep_forward(0, hs[0], outs[0], stream=stream)
            ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
            gates = torch.empty((T, K), dtype=torch.float32, device="cuda")
            eng.route(0, hs[0], ids, gates, stream=stream)
        stream.synchronize()
        eng.sync_status(stream)
        rows = np.unique(np.linspace(0, T - 1, min(T, 64)).astype(np.int64))
        p = parity_check(oracle_layer(cfg, "int8", 0), hs[0].cpu().numpy(), ids.cpu().numpy(),
                         outs[0].cpu().numpy(), rows)
        agg = torch.tensor([0.0 if p["ids_exact"] else 1.0, p["max_rel_err"]],
                           dtype=torch.float64, device="cuda")
        dist.all_reduce(agg, op=dist.ReduceOp.MAX)
        parity = {"ids_exact": bool(agg[0].item() == 0.0), "max_rel_err": float(agg[1].item()),
                  "tokens_checked": int(len(rows) * world), "tolerance": 1e-3,
                  "ranks_checked": world}

    hbm_peak, _, peak_kind = measured_peaks()
    prof = {k: v for k, v in prof.items() if ":" not in k}
    tot = max(1e-9, sum(v[1] for v in prof.values()))
    top = max(prof.items(), key=lambda kv: kv[1][1]) if prof else ("none", (1, 0.0))
    phase_us = {k: round(v[1] * 1e3 / max(1, args.steps), 2) for k, v in prof.items()}
    # limiting phase on this rank, and the local weight bytes streamed per step
    local_gbs = layer_bytes_local / (ms_max / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": "ep_layer", "achieved": local_gbs, "peak": hbm_peak,
                "unit": "GB/s", "frac": local_gbs / hbm_peak, "traffic": None,
                "peak_kind": peak_kind, "alg_bytes_per_launch": layer_bytes_local,
                "mean_launch_ms": ms_max, "limiting_phase": top[0],
                "phase_us_per_step": phase_us,
                "kernel_share": {k: round(v[1] / tot, 4) for k, v in prof.items()}}
    del keep
    if rank == 0:
        line = {"metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_max, "higher_is_better": True,
                "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config_dict(cfg, "int8", world),
                "detail": {"experts_per_rank": EL, "transport": eng.ep_transport(),
                           "placement": "balanced" if zipf else "contiguous",
                           "rotation_layers": n_layers},
                "roofline": roofline, "parity": parity, "cpu_baseline": None, "e2e": e2e,
                "gpu_launches": launches, "clocks": clk}
        print(json.dumps(line), flush=True)
    eng.ep_finalize()
    dist.barrier()


if __name__ == "__main__":
    main()
