#!/usr/bin/env python3
"""Benchmark of the sparse stream-editing attention frame (one FLUX.2 double-stream attention slice
under a spatial KV cache) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--active 0.25]
    python bench.py --impl reference ...      # CPU fp32 evaluation of the same plugin math

A step is one frame: mask compaction -> gather + QK-RMSNorm + RoPE + cache write -> tcgen05
attention with the scatter fused into its epilogue -> restore of execute-only cache rows.
Default workload: 1024x1024 frame = 4096 image + 512 text tokens, 24 heads x 128, bf16,
Bernoulli(0.25) image mask (text always executed), i.e. the metric's configuration.
At N GPUs every rank runs its own independent edit stream (weak scaling, no collective in the
data path); value = attention FLOP of all ranks / max-over-ranks time.
Prints one JSON line (rank 0).
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

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(HERE, "fluxrt-cpp_b200")
sys.path.insert(0, PKG)

import numpy as np  # noqa: E402

METRIC = "active-token attn TFLOP/s + plugin µs/frame @1024², 25% active; % of peak"
HEAD_DIM = 128
L2_BYTES = 126 * 1024 * 1024


def whole_job(max_vals, sum_vals, world: int, device):
    """Whole-job figures of a multi-rank run: the max over ranks of each of `max_vals` (times) and
    the sum over ranks of each of `sum_vals` (work, bytes), as two lists of floats. Every rank must
    call it at the same point (two all-reduces). With one rank the inputs come back unchanged."""
    if world <= 1:
        return [float(x) for x in max_vals], [float(x) for x in sum_vals]
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x) for x in max_vals], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    f = torch.tensor([float(x) for x in sum_vals], dtype=torch.float64, device=device)
    dist.all_reduce(f, op=dist.ReduceOp.SUM)
    return [float(x) for x in t.tolist()], [float(x) for x in f.tolist()]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--active", type=float, default=None, help="override the active fraction")
    ap.add_argument("--heads", type=int, default=None, help="override the number of heads")
    ap.add_argument("--streams", type=int, default=None,
                    help="independent edit streams in total (one batched set of launches per GPU "
                         "per step; c4 default 8, spread over the GPUs)")
    ap.add_argument("--path", choices=["attention", "block", "single"], default="attention",
                    help="attention: the sparse attention frame (the metric's path); block: the whole "
                         "double-stream block on the executed rows (LayerNorm, Q/K/V, attention, MLP, "
                         "out-projection, residual); single: the single-stream block (fused "
                         "projection, attention, output projection over [attention | MLP])")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of CUDA graphs")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--no-sub", action="store_true",
                    help="default run: skip the c4 streams / c5 head-split sub-records")
    ap.add_argument("--no-ref-cuda", action="store_true",
                    help="reference arm: skip timing the reference's own CUDA kernels")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--split", choices=["replicas", "heads", "heads_nccl"], default=None,
                    help="multi-GPU mode: independent streams per GPU (default except c5) or one "
                         "frame split by heads whose O rows an exchange kernel stores into every "
                         "GPU's output over NVLink (default for c5), or the same split with the O "
                         "exchange as "
                         "one NCCL all-gather + scatter (heads_nccl)")
    a = ap.parse_args()
    if a.split is None:
        a.split = "heads" if a.config == "c5" else "replicas"
    if a.streams is None and a.config == "c4":
        a.streams = 8
    return a


def workload(args):
    import workloads as W
    w = {"c1": W.C1, "c2": W.C2, "c3": W.C3, "c4": W.C4, "c5": W.C5}[args.config]
    if args.active is not None:
        w = W.with_active(w, args.active)
    if args.heads is not None:     # one GPU's share of a head-split frame, timed alone
        w = W.Workload(f"{w.name}_h{args.heads}", w.grid_h, w.grid_w, w.n_text, args.heads, w.head_dim,
                       w.dtype, w.active, w.pattern, w.rope_axes, w.rope_theta)
    return w


def peaks():
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        j = json.load(open(path))
        p = {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]),
             "bf16_tflops_sustained": float(j.get("bf16_tflops_sustained", j["bf16_tflops"])),
             "source": "measured"}
    return p


def profile_traffic(name: str):
    """DRAM bytes per launch of a kernel from the committed ncu summary, if one exists."""
    path = os.path.join(HERE, "profiles", f"{name}.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("dram_bytes_per_launch"):
            try:
                return float(line.split("=")[1].split()[0])
            except (IndexError, ValueError):
                return None
    return None


# ---------------------------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "samples": len(sm),
                "power_w_max": max(power), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def make_device_frame(w, seed: int, device):
    """One frame's inputs, generated on the device (bf16/fp16 N(0,1)), mask from numpy."""
    import torch
    import workloads as W
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    N, C = w.n_tokens, w.n_heads * HEAD_DIM
    dt = torch.bfloat16 if w.dtype == "bf16" else torch.float16
    rnd = lambda *s: torch.randn(*s, generator=g, device=device, dtype=torch.float32).to(dt)
    rng = np.random.default_rng(seed)
    mask = W.make_mask(w, rng)
    fr = {
        "q": rnd(N, C), "k": rnd(N, C), "v": rnd(N, C),
        "cache_k": rnd(N, C), "cache_v": rnd(N, C), "out": rnd(N, C),
        "norm_q": (1.0 + 0.1 * torch.randn(HEAD_DIM, generator=g, device=device)).float(),
        "norm_k": (1.0 + 0.1 * torch.randn(HEAD_DIM, generator=g, device=device)).float(),
        "mask": torch.from_numpy(mask).to(device),
        "mask_host": mask,
        "pos": torch.from_numpy(W.positions(w)).to(device),
        "M": int((mask != 0).sum()),
    }
    return fr


def bench_config(w, M_avg: float, world: int, n_sets: int, use_graph: bool) -> dict:
    """The workload description both arms print (the same keys and values for the same run)."""
    return {"workload": w.name, "frame_px": w.grid_h * 16, "n_tokens": w.n_tokens,
            "n_text": w.n_text, "n_image": w.n_image, "active": w.active, "pattern": w.pattern,
            "M_avg": M_avg, "heads": w.n_heads, "head_dim": HEAD_DIM,
            "rope_axes": list(w.rope_axes), "rope_theta": w.rope_theta,
            "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": f"{n_sets} rotating input sets, {n_sets * 6 * w.n_tokens * w.n_heads * HEAD_DIM * 2 / 2**20:.0f} MiB > L2",
            "graph": f"{n_sets} consecutive frames per CUDA graph" if use_graph else False}


def frame_masks(w, seed: int, rank: int, n_sets: int) -> list:
    """The change masks of the rotating input sets (make_device_frame draws the same ones)."""
    import workloads as W
    return [W.make_mask(w, np.random.default_rng(seed + 7919 * rank + s)) for s in range(n_sets)]


def frame_cfg(w):
    import fxr
    return fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=w.n_heads, dtype=w.dtype,
                           rope_axes=w.rope_axes, rope_theta=w.rope_theta)


def run_frame(cfg, fr, ws):
    import fxr
    fxr.frame_forward(cfg, fr["q"], fr["k"], fr["v"], fr["mask"], None, fr["pos"], fr["norm_q"],
                      fr["norm_k"], fr["cache_k"], fr["cache_v"], fr["out"], ws)


def attention_kernel_name(heads_per_launch: int) -> str:
    """The attention kernel the library launches (launch_attention_streams in csrc/fxr_capi.cu):
    the two-tile kernel, in its stream-K capable form when the workspace holds the scratch slots
    (every bench workspace does; the kernel picks whole units or stream-K from M on the device);
    FXR_ATTENTION_TILES=1 selects the one-tile kernel, which splits key ranges for at most 8 heads."""
    if os.environ.get("FXR_ATTENTION_TILES", "") == "1":
        return "fxr::attn::attention_kernel" + (" (key-range split)" if heads_per_launch <= 8 else "")
    return "fxr::attn2::attention_kernel (stream-K capable)"


def attn_flops(w, M: int) -> float:
    return 4.0 * M * w.n_tokens * HEAD_DIM * w.n_heads


def gather_bytes(w, M: int) -> float:
    """Algorithmic bytes of the compacting gather/norm/RoPE/cache-write kernel: read Q,K,V rows,
    write compact Q' and the K', V cache rows (6 rows of C elements per executed token), the
    executed tokens' position ids, and the mask scan (read the mask, write the index list)."""
    eb = 2
    C = w.n_heads * HEAD_DIM
    return 6.0 * M * C * eb + M * (4 + 4 * len(w.rope_axes)) + 4.0 * w.n_tokens


def run_ours(args):
    import torch
    import torch.distributed as dist
    import fxr

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    fxr.load()
    w = workload(args)
    cfg = frame_cfg(w)
    pk = peaks()

    # Input sets: rotating over several independent frames keeps the per-step working set
    # (Q/K/V 3 x 28 MB + caches 56 MB + out 28 MB at 1024^2) far above the 126 MB L2.
    n_sets = 4
    frames = [make_device_frame(w, args.seed + 7919 * rank + s, device) for s in range(n_sets)]
    ws_bytes = fxr.workspace_size(cfg)
    wss = [torch.empty(ws_bytes, dtype=torch.uint8, device=device) for _ in range(n_sets)]
    stream = torch.cuda.current_stream()

    for i in range(max(args.warmup, 3)):
        run_frame(cfg, frames[i % n_sets], wss[i % n_sets])
    torch.cuda.synchronize()
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during warm-up")

    # Graphs: one per input set, and one holding the n_sets frames back to back as a stream of
    # frames is enqueued (programmatic dependent launch then also overlaps one frame's first kernel
    # with the previous frame's last); K frames = K // n_sets replays of the latter + the rest.
    graphs = []
    use_graph = not args.no_graph
    run_graph = None
    if use_graph:
        for s in range(n_sets):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                run_frame(cfg, frames[s], wss[s])
            graphs.append(g)
        run_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(run_graph):
            for s in range(n_sets):
                run_frame(cfg, frames[s], wss[s])
        for s in range(n_sets):
            graphs[s].replay()
        run_graph.replay()
        torch.cuda.synchronize()

    def step(i):
        if use_graph:
            graphs[i % n_sets].replay()
        else:
            run_frame(cfg, frames[i % n_sets], wss[i % n_sets])

    def steps(k):
        """k frames in order, n_sets per graph replay where possible."""
        i = 0
        if use_graph:
            while k - i >= n_sets:
                run_graph.replay()
                i += n_sets
        while i < k:
            step(i)
            i += 1

    clocks = Clocks(local)
    clocks.start()
    # soak for >= 1 s so the sampler sees the loaded clock even when K is small
    t_end = time.time() + 1.0
    while time.time() < t_end:
        steps(64)
        torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    t_ms = e0.elapsed_time(e1)
    flops_rank = sum(attn_flops(w, frames[i % n_sets]["M"]) for i in range(args.steps))
    (t_ms,), (flops_total,) = whole_job([t_ms], [flops_rank], world, device)
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during the timed region")
    ms_per_step = t_ms / args.steps
    value = flops_total / (t_ms * 1e-3) / 1e12

    # ---- per-kernel times (eager launches with events between the kernels, same stream) ----
    kern = per_kernel_times(cfg, w, frames, wss, stream, reps=max(20, min(200, args.steps)))
    iso = isolated_kernel_times(cfg, frames, wss, reps=40)
    M_avg = statistics.mean(fr["M"] for fr in frames)
    attn_us = kern["attention_us"]
    achieved = attn_flops(w, M_avg) / (attn_us * 1e-6) / 1e12
    traffic = profile_traffic(f"attention_{w.name}")
    roof = {"bound": "tensor", "kernel": attention_kernel_name(w.n_heads), "achieved": round(achieved, 1),
            "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4),
            "peak_kind": f"{pk['source']} burst bf16 (cuBLAS)",
            "frac_of_nominal_2250": round(achieved / 2250.0, 4),
            # the kernel is timed inside a stream of frames that has run for over a second, under
            # the same power cap as the sustained GEMM figure
            "frac_of_sustained": round(achieved / pk["bf16_tflops_sustained"], 4),
            "peak_sustained": pk["bf16_tflops_sustained"],
            "traffic": traffic, "algorithmic_flop_per_launch": attn_flops(w, M_avg)}
    g_us = iso["gather_us"]      # back-to-back launches: no event-record gap around the launch
    gb = gather_bytes(w, M_avg)
    mem = {"kernel": "fxr::gather_bulk_kernel (compacting)", "bound": "hbm", "us": round(g_us, 2),
           "achieved": round(gb / (g_us * 1e-6) / 1e9, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
           "frac": round(gb / (g_us * 1e-6) / 1e9 / pk["hbm_gbs"], 4),
           "algorithmic_bytes_per_launch": gb, "traffic": profile_traffic(f"gather_{w.name}")}

    # ---- end to end through the C ABI with host buffers ----
    # PCIe throughput varies between runs of the same frames by up to ~15 %: three rounds, the
    # median one reported with all three
    rounds = [e2e_measure(cfg, w, frames, wss, stream, reps=max(5, min(100, args.steps)), world=world)
              for _ in range(3)]
    rounds_us = [r["us_per_frame"] for r in rounds]
    e2e = sorted(rounds, key=lambda r: r["us_per_frame"])[1]
    e2e["rounds_us_per_frame"] = rounds_us

    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "us_per_frame": round(ms_per_step * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": w.dtype, "impl": "ours",
        "data": "synthetic: N(0,1) Q/K/V/cache, N(1,0.1) norm weights, Bernoulli mask (seeded)",
        "config": bench_config(w, M_avg, world, n_sets, use_graph),
        "roofline": roof,
        "kernels": {"gather": mem,
                    "in_frame_us": {k[:-3]: round(v, 2) for k, v in kern.items()},
                    "isolated_us": {k[:-3]: round(v, 2) for k, v in iso.items()},
                    "timing": "the frame's launches (compacting gather, attention, which restores "
                              "mask==1 rows itself; the one-tile attention adds a restore launch) through "
                              "fxr_frame_step on the frame's workspace; in_frame: event records between "
                              "them in a CUDA graph, mean over frames (each interval also holds one "
                              "launch gap); isolated: 40 back-to-back launches of one step per graph; the "
                              "attention roofline uses in_frame, the gather roofline isolated"},
        "e2e": e2e,
        "gpu_launches": len(FRAME_STEPS) * args.steps,   # compacting gather + attention (+ restore)
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            out["cpu_baseline"] = cpu_baseline(w, args.cpu_seconds, args.seed)
        except Exception as ex:  # the baseline is reported, not required
            out["cpu_baseline"] = {"value": None, "error": str(ex)[:200]}
    for g_ in graphs:
        del g_
    graphs.clear()
    del run_graph
    del frames, wss
    torch.cuda.empty_cache()
    if not args.no_sub and args.config == "c2" and args.active is None and args.heads is None:
        out["sub"] = sub_records(args, world)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def sub_records(args, world: int) -> dict:
    """The two configurations that shard over GPUs, measured on the same ranks after the main
    figure (every rank takes the same steps): 8 independent 768^2 edit streams spread over the
    GPUs (aggregate frames/s, no collective) and one 2048^2 frame split by heads (us per frame,
    exchange of O over NVLink peer stores). Each keeps the keys its own runner prints."""
    import copy
    import torch
    keep = ("value", "unit", "ms_per_step", "frames_per_s", "us_per_frame", "us_per_frame_per_gpu",
            "scaling", "config", "roofline", "clocks", "steps", "warmup")
    recs = {}
    for name, cfg_, extra in (("c4_streams8", "c4", {"streams": 8, "split": None}),
                              ("c5_heads", "c5", {"streams": None, "split": "heads"})):
        a = copy.copy(args)
        a.config, a.active, a.heads = cfg_, None, None
        a.streams, a.split = extra["streams"], extra["split"]
        a.steps = max(20, min(args.steps, 200 if cfg_ == "c4" else 100))
        a.warmup = 3
        try:
            line = run_streams(a, embedded=True) if cfg_ == "c4" else run_heads(a, embedded=True)
            recs[name] = {k: line[k] for k in keep if k in line}
        except Exception as ex:   # reported, not required
            recs[name] = {"error": str(ex)[:200]}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return recs


def run_step(cfg, fr, ws, step):
    import fxr
    fxr.frame_step(step, cfg, fr["q"], fr["k"], fr["v"], fr["mask"], None, fr["pos"], fr["norm_q"],
                   fr["norm_k"], fr["cache_k"], fr["cache_v"], fr["out"], ws)


# The frame's launches as fxr_frame_step runs them (same workspace, same schedule): the compacting
# gather and the attention, which restores the mask==1 rows itself; the one-tile attention
# (FXR_ATTENTION_TILES=1) leaves the restore to a third launch.
ONE_TILE = os.environ.get("FXR_ATTENTION_TILES", "") == "1"
FRAME_STEPS = (("gather_us", 2), ("attention_us", 3)) + ((("restore_us", 4),) if ONE_TILE else ())


def per_kernel_times(cfg, w, frames, wss, stream, reps: int):
    """Per-kernel device time inside a stream of frames: the frame's launches (FRAME_STEPS, through
    fxr_frame_step on the frame's own workspace) of `reps` frames are
    captured in one CUDA graph with event records between them (on the launching stream), so host
    launch overhead does not leak into the intervals. Mean over frames: event timestamps inside a
    graph advance in steps of about 2 us on this GPU, so a median would land on a tick; the mean
    over frames (whose phase against the tick varies) does not, and it pairs with the mean
    executed-row count."""
    import torch
    ev = lambda: torch.cuda.Event(enable_timing=True, external=True)
    names = [n for n, _ in FRAME_STEPS]
    events = [[ev() for _ in range(len(names) + 1)] for _ in range(reps)]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        s = torch.cuda.current_stream()
        for i in range(reps):
            fr, ws = frames[i % len(frames)], wss[i % len(wss)]
            e = events[i]
            e[0].record(s)
            for k, (_, step) in enumerate(FRAME_STEPS):
                run_step(cfg, fr, ws, step)
                e[k + 1].record(s)
    g.replay()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    acc = {k: [] for k in names}
    for i in range(2, reps):
        e = events[i]
        for k, name in enumerate(names):
            acc[name].append(e[k].elapsed_time(e[k + 1]) * 1e3)
    del g
    return {k: statistics.mean(v) for k, v in acc.items()}


def isolated_kernel_times(cfg, frames, wss, reps: int):
    """Per-kernel device time of `reps` back-to-back launches of one of the frame's steps alone
    (rotating input sets, one CUDA graph, CUDA events around its replay on the launching stream),
    after the frames have run once so that the index lists exist. Every step is idempotent on its
    inputs. Mean per launch, median of 5 replays."""
    import torch
    n = len(frames)
    out = {}
    for name, step in FRAME_STEPS:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(reps):
                run_step(cfg, frames[i % n], wss[i % n], step)
        g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / reps)
        out[name] = statistics.median(ts)
        del g
    return out


def e2e_measure(cfg, w, frames, wss, stream, reps: int, world: int = 1):
    """Frames through the C ABI with the frame's tensors in pinned HOST memory, the way a streaming
    host feeds them: fxr_frame_forward_host reads the mask and the executed tokens' Q, K, V rows
    from host memory and writes the executed output rows back, every frame. Frames alternate between
    two CUDA streams with their own caches and workspace, so one frame's transfers overlap the
    other's kernels. For comparison, the same frames with whole-tensor copies (Q, K, V, mask in,
    the full output back) around fxr_frame_forward. With several ranks, every rank runs its frames at
    the same time (a barrier before each timed loop) and the line reports the whole job: the slowest
    rank's time per frame, every rank's work and bytes."""
    import torch

    import fxr
    fr0 = frames[0]
    host = {k: fr0[k].cpu().pin_memory() for k in ("q", "k", "v", "mask")}
    lanes = []
    for b in range(2):
        lane = {"stream": torch.cuda.Stream(), "cache_k": fr0["cache_k"].clone(),
                "cache_v": fr0["cache_v"].clone(), "out_h": fr0["out"].cpu().pin_memory(),
                "ws": torch.empty(fxr.frame_host_workspace_size(cfg), dtype=torch.uint8, device="cuda")}
        lanes.append(lane)
    row_bytes = w.n_heads * HEAD_DIM * 2
    M = int(fr0["M"])

    def rows_frame(i):
        ln = lanes[i % 2]
        fxr.frame_forward_host(cfg, host["q"], host["k"], host["v"], host["mask"], None, fr0["pos"],
                               fr0["norm_q"], fr0["norm_k"], ln["cache_k"], ln["cache_v"], ln["out_h"],
                               ln["ws"], stream=ln["stream"])

    full_dev = []
    for b in range(2):
        dev = {k: torch.empty_like(fr0[k]) for k in ("q", "k", "v", "mask")}
        fr = dict(fr0)
        fr.update(dev)
        fr["out"] = fr0["out"].clone()
        fr["cache_k"], fr["cache_v"] = fr0["cache_k"].clone(), fr0["cache_v"].clone()
        full_dev.append((fr, wss[b], dev))

    def full_frame(i):
        st = lanes[i % 2]["stream"]
        fr, ws, dev = full_dev[i % 2]
        with torch.cuda.stream(st):
            for k in host:
                dev[k].copy_(host[k], non_blocking=True)
            run_frame(cfg, fr, ws)
            lanes[i % 2]["out_h"].copy_(fr["out"], non_blocking=True)

    def timed(one):
        for i in range(4):
            one(i)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
            torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for ln in lanes:
            ln["stream"].wait_stream(stream)
        for i in range(reps):
            one(i)
        for ln in lanes:
            stream.wait_stream(ln["stream"])
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / reps

    ms = timed(rows_frame)
    ms_full = timed(full_frame)
    full_h2d = sum(t.numel() * t.element_size() for t in host.values())
    full_d2h = fr0["out"].numel() * fr0["out"].element_size()
    tot = [attn_flops(w, M), 3 * M * row_bytes + 4 * w.n_tokens, M * row_bytes, full_h2d, full_d2h]
    (ms, ms_full), tot = whole_job([ms, ms_full], tot, world, "cuda")
    value = tot[0] / (ms * 1e-3) / 1e12
    return {"value": round(value, 2), "unit": "TFLOP/s", "us_per_frame": round(ms * 1e3, 1), "ranks": world,
            "h2d_bytes_per_step": int(tot[1]),
            "d2h_bytes_per_step": int(tot[2]),
            "path": "fxr_frame_forward_host via ctypes: pinned host Q/K/V/mask/out, only executed rows "
                    "cross PCIe (zero-copy row kernels), frames alternating over two streams",
            "full_frame_copies": {"us_per_frame": round(ms_full * 1e3, 1),
                                  "value": round(tot[0] / (ms_full * 1e-3) / 1e12, 2),
                                  "h2d_bytes_per_step": int(tot[3]),
                                  "d2h_bytes_per_step": int(tot[4]),
                                  "path": "whole-tensor copies in and out around fxr_frame_forward"}}


# ---------------------------------------------------------------------------------------------
# CPU (oracle) arm
# ---------------------------------------------------------------------------------------------
def _cpu_oracle():
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    native = True
    try:
        O.build(native=True)
    except Exception:
        native = False
    return O, native


def cpu_frame_sample(O, native, w, M_s: int, seed: int, mask=None):
    """One frame of the plugin math on the CPU: gather/norm/RoPE of the executed tokens, attention
    of their queries over all N keys, scatter, cache update. The executed tokens are those of
    `mask` when given (a whole frame of the workload), else M_s random ones (a bounded sample).
    Returns (seconds, attention FLOP)."""
    import workloads as W
    rng = np.random.default_rng(seed)
    N, C = w.n_tokens, w.n_heads * HEAD_DIM
    if not hasattr(cpu_frame_sample, "cache") or cpu_frame_sample.cache[0] != (w.name, N):
        f = lambda: W.round_storage(rng.normal(size=(N, C)).astype(np.float32), w.dtype)
        cpu_frame_sample.cache = ((w.name, N), {k: f() for k in ("q", "k", "v", "ck", "cv", "out")},
                                  W.positions(w), rng.normal(1, 0.1, 128).astype(np.float32))
    _, a, pos, nw = cpu_frame_sample.cache
    if mask is None:
        mask = np.zeros(N, dtype=np.int32)
        mask[rng.choice(N, size=M_s, replace=False)] = 2
    else:
        mask = np.array(mask, dtype=np.int32, copy=True)
    L = O.lib(native)
    fp = lambda x: x.ctypes.data_as(O._f32p)
    ip = lambda x: x.ctypes.data_as(O._i32p)
    ck, cv, out = a["ck"].copy(), a["cv"].copy(), a["out"].copy()
    qc = np.empty_like(a["q"])
    idx = np.empty(N, dtype=np.int32)
    ax = np.array(w.rope_axes, dtype=np.int32)
    t0 = time.perf_counter()
    M = L.fxo_frame_forward(fp(a["q"]), fp(a["k"]), fp(a["v"]), ip(mask), None, ip(pos), fp(nw), fp(nw),
                            fp(ck), fp(cv), fp(out), fp(qc), ip(idx), N, w.n_heads, HEAD_DIM,
                            ax.size, ip(ax), w.rope_theta, 1e-6, 0.0)
    dt = time.perf_counter() - t0
    return dt, attn_flops(w, M)


def cpu_baseline(w, budget_s: float, seed: int) -> dict:
    """Whole frames of the workload (its executed-token count, all heads, all N keys) through the
    oracle on every host core, repeated until about budget_s seconds of CPU work."""
    O, native = _cpu_oracle()
    cores = O.set_threads(os.cpu_count() or 1, native)
    M_s = int(round(w.n_text + w.active * w.n_image))
    cpu_frame_sample(O, native, w, 16, seed)                  # warms the inputs and the pool
    total, flops, frames = 0.0, 0.0, 0
    while frames == 0 or total < budget_s:
        dt, fl = cpu_frame_sample(O, native, w, M_s, seed + 1 + frames)
        total += dt
        flops += fl
        frames += 1
    return {"value": round(flops / total / 1e12, 4), "unit": "TFLOP/s", "cores": cores,
            "kind": "port", "sample": f"{frames} oracle frames of {w.name} with {M_s} executed tokens of "
            f"{w.n_tokens} (all {w.n_heads} heads, all N keys), {total:.1f} s, "
            f"-march={'native' if native else 'x86-64-v3'}",
            "seconds": round(total, 3), "us_per_frame": round(total / frames * 1e6, 1)}


def run_reference(args):
    """The reference arm: the CPU fp32 restatement of the reference math on all host cores, on the
    same frames as our arm (the masks of the rotating input sets: the same executed tokens, all
    heads, all N keys) when the whole run fits in about two minutes, else on a bounded number of
    executed tokens per step. On rank 0 only; with a GPU it also times the reference's own CUDA
    kernels on one such frame (reference_cuda)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = workload(args)
    n_sets = 4
    masks = frame_masks(w, args.seed, 0, n_sets)
    M_avg = statistics.mean(int((m != 0).sum()) for m in masks)
    O, native = _cpu_oracle()
    cores = O.set_threads(os.cpu_count() or 1, native)
    dt, _ = cpu_frame_sample(O, native, w, 16, args.seed)
    per_row = max(dt / 16, 1e-6)
    total_steps = args.steps + args.warmup
    whole = per_row * M_avg * total_steps <= 150.0
    budget_per_step = max(0.02, min(4.0, 120.0 / max(total_steps, 1)))   # whole run ~2 minutes
    M_s = int(max(16, min(w.n_tokens, budget_per_step / per_row)))
    one = (lambda i: cpu_frame_sample(O, native, w, 0, args.seed + i, mask=masks[i % n_sets])) if whole \
        else (lambda i: cpu_frame_sample(O, native, w, M_s, args.seed + 1000 + i))
    for i in range(args.warmup):
        one(i)
    tot_t, tot_f = 0.0, 0.0
    for i in range(args.steps):
        dt, fl = one(i)
        tot_t += dt
        tot_f += fl
    value = tot_f / tot_t / 1e12
    ms_per_step = tot_t / max(args.steps, 1) * 1e3
    sample = (f"per step: one whole oracle frame of {w.name} (the executed tokens of our arm's input "
              f"set i % {n_sets}, M_avg {M_avg:.1f} of {w.n_tokens}, all heads and keys)") if whole else \
        (f"per step: an oracle frame of {w.name} restricted to {M_s} executed tokens of {w.n_tokens} "
         f"(all heads and keys), bounded so that the run ends within minutes")
    out = {
        "metric": METRIC, "value": round(value, 5), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
        "us_per_frame": round(ms_per_step * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "impl": "reference", "data": "synthetic: N(0,1) Q/K/V/cache, N(1,0.1) norm weights, Bernoulli mask (seeded)",
        "config": bench_config(w, M_avg, world, n_sets, not args.no_graph),
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU implementation of this path and its GPU attention is "
                "numerically defective; this arm times the CPU fp32 restatement of the reference math",
    }
    if not args.no_ref_cuda:
        try:
            out["reference_cuda"] = reference_cuda_leg(w, masks[0], args.seed)
        except Exception as ex:      # reported, not required
            out["reference_cuda"] = {"unavailable": str(ex)[:200]}
    print(json.dumps(out), flush=True)


def reference_cuda_leg(w, mask_h, seed: int) -> dict:
    """The reference's own CUDA kernels (oracle/_ref/libfxr_refkernels.so, compiled for sm_100a from
    its sources) on one frame of the workload, as its plugins would run the slice in fp32:
    gather_tokens of the Q, K, V rows (gather_scatter_kernels.cu:15-41), launch_rms_norm of the
    gathered Q and K per head (seq_len = M*H, dim = 128; flux2_kernels.cu:58-90),
    SpatialCache::sync_kv_cache over all N rows (spatial_kv_cache.cu:55-87,175-196), attention_fwd
    of the M queries over the N merged keys ((batch, heads, len, dim) layout; the transposes around
    it are not timed; attention_kernels.cu:85-173) and scatter_tokens of the outputs
    (gather_scatter_kernels.cu:46-72). The reference has no RoPE. CUDA events on the launching
    stream, median of repetitions, nvidia-smi clocks sampled over the leg."""
    import torch
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    if not torch.cuda.is_available():
        return {"unavailable": "no GPU"}
    L = O.ref_kernels()
    if L is None:
        return {"unavailable": "oracle/_ref/libfxr_refkernels.so not built (reference sources absent where build() ran)"}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N, H, D = w.n_tokens, w.n_heads, HEAD_DIM
    C = H * D
    g = torch.Generator(device=dev).manual_seed(seed)
    M = int((mask_h != 0).sum())
    idx = torch.from_numpy(np.nonzero(mask_h)[0].astype(np.int32)).to(dev)
    mask = torch.from_numpy(np.asarray(mask_h, dtype=np.int32)).to(dev)
    q, k, v = (torch.randn(N, C, device=dev, generator=g) for _ in range(3))
    qg, kg, vg = (torch.empty(M, C, device=dev) for _ in range(3))
    wq = 1 + 0.1 * torch.randn(D, device=dev, generator=g)
    out_full = torch.zeros(N, C, device=dev)
    s = torch.cuda.current_stream()
    ss = s.cuda_stream
    cache = L.ref_cache_create(N - w.n_text, w.n_text, 64, H, D, 1, 0)
    if not cache:
        return {"unavailable": "reference SpatialCache construction failed"}

    def timed(fn, reps):
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            fn()
            e1.record(s)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts[1:] if len(ts) > 2 else ts)

    clocks = Clocks(0)
    clocks.start()
    rows = {}
    try:
        rows["gather_tokens x3 (Q, K, V)"] = timed(lambda: [L.ref_gather_tokens(
            t.data_ptr(), o.data_ptr(), idx.data_ptr(), M, C, ss) for t, o in ((q, qg), (k, kg), (v, vg))], 7)
        qn, kn = torch.empty_like(qg), torch.empty_like(kg)
        rows["launch_rms_norm x2 (Q, K per head)"] = timed(lambda: [L.ref_rms_norm(
            a.data_ptr(), b.data_ptr(), wq.data_ptr(), 1e-6, M * H, D, ss) for a, b in ((qg, qn), (kg, kn))], 7)
        kk, vv = k.clone(), v.clone()
        rows["SpatialCache::sync_kv_cache (N rows)"] = timed(lambda: L.ref_cache_sync_kv(
            cache, kk.data_ptr(), vv.data_ptr(), mask.data_ptr(), 0, 1, ss), 7)
        qh = qn.view(M, H, D).transpose(0, 1).contiguous()
        kh = kk.view(N, H, D).transpose(0, 1).contiguous()
        vh = vv.view(N, H, D).transpose(0, 1).contiguous()
        oh = torch.empty_like(qh)
        rows["attention_fwd (fp32, B=1)"] = timed(lambda: L.ref_attention_fwd(
            qh.data_ptr(), kh.data_ptr(), vh.data_ptr(), oh.data_ptr(), 1, H, M, N, D, ss), 3)
        og = oh.transpose(0, 1).reshape(M, C).contiguous()
        rows["scatter_tokens"] = timed(lambda: L.ref_scatter_tokens(
            og.data_ptr(), out_full.data_ptr(), idx.data_ptr(), M, C, ss), 7)
        torch.cuda.synchronize()
    finally:
        clk = clocks.stop()
        L.ref_cache_destroy(cache)
    total = sum(rows.values())
    return {"us_per_frame": round(total, 1), "value": round(attn_flops(w, M) / (total * 1e-6) / 1e12, 4),
            "unit": "TFLOP/s", "M": M, "kernels_us": {k_: round(v_, 1) for k_, v_ in rows.items()},
            "kind": "the reference's CUDA kernels compiled for sm_100a from its sources (fp32, no RoPE)",
            "attention_fwd": "numerically defective: it normalises with one warp's partial row maximum "
                             "and sum (attention_kernels.cu:117-139); timed, never used as an oracle",
            "clocks": clk}


# ---------------------------------------------------------------------------------------------
# one frame split by heads over the GPUs (peer stores + arrival wait)
# ---------------------------------------------------------------------------------------------
def run_heads(args, embedded: bool = False):
    """A step is one frame of all heads, split across the ranks by heads; each rank's exchange
    kernel stores its heads' O rows into every rank's output over NVLink, then each rank waits
    for all arrivals. value = whole-frame attention FLOP / max-over-ranks time (strong scaling).
    embedded: run inside an initialised process group and return the JSON object instead of
    printing it (the multi-GPU sub-records of the default run)."""
    import datetime
    import torch
    import torch.distributed as dist
    import fxr

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not embedded:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    fxr.load()
    w = workload(args)
    cfg = frame_cfg(w)
    pk = peaks()
    g = fxr.head_group(world, rank, w.n_heads, w.n_tokens)
    N, C = w.n_tokens, w.n_heads * HEAD_DIM
    c0, c1 = g.head0 * HEAD_DIM, (g.head0 + g.n_heads) * HEAD_DIM
    dt = torch.bfloat16 if w.dtype == "bf16" else torch.float16

    # rotating input sets: this rank's K/V cache shard of every set together exceeds twice the L2
    shard_bytes = 2 * N * (c1 - c0) * 2
    n_sets = int(min(12, max(2, -(-2 * L2_BYTES // max(shard_bytes, 1)))))
    frames = []
    for s_ in range(n_sets):
        fr = make_device_frame(w, args.seed + 7919 * s_, device)   # same inputs on every rank
        fr["cache_k"] = fr["cache_k"][:, c0:c1].contiguous()
        fr["cache_v"] = fr["cache_v"][:, c0:c1].contiguous()
        if s_ > 0:
            del fr["out"]
        frames.append(fr)
    nccl = args.split == "heads_nccl"
    out_bytes = N * C * 2
    mapped, buf, comm = [], None, None
    if nccl:
        uid = [fxr.nccl_unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(uid, src=0)
        comm = fxr.nccl_comm_init(world, rank, uid[0])
        out = frames[0]["out"]
        m_cap = max(fr["M"] for fr in frames)
        ws = [torch.empty(fxr.heads_nccl_workspace_size(cfg, g, m_cap), dtype=torch.uint8,
                          device=device) for _ in range(n_sets)]
    else:
        buf = fxr.IpcBuffer(out_bytes + 256)
        out = fxr.device_view(buf.ptr.value, (N, C), dt)
        out.copy_(frames[0]["out"])
        handles = [buf.handle_bytes()]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, buf.handle_bytes())
        for r in range(world):
            ptr = buf.ptr.value if r == rank else fxr.ipc_open(handles[r])
            if r != rank:
                mapped.append(ptr)
            g.out[r] = ptr
            g.arrive[r] = ptr + out_bytes
        ws = [torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device=device)
              for _ in range(n_sets)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    def frame(i):
        fr = frames[i % n_sets]
        if nccl:
            fxr.frame_forward_heads_nccl(cfg, g, comm, m_cap, fr["q"], fr["k"], fr["v"], fr["mask"],
                                         None, fr["pos"], fr["norm_q"], fr["norm_k"],
                                         fr["cache_k"], fr["cache_v"], out, ws[i % n_sets])
            return
        fxr.frame_forward_heads(cfg, g, fr["q"], fr["k"], fr["v"], fr["mask"], None, fr["pos"],
                                fr["norm_q"], fr["norm_k"], fr["cache_k"], fr["cache_v"],
                                ws[i % n_sets])
        fxr.head_group_wait(g)

    for i in range(max(args.warmup, 3)):
        frame(i)
    torch.cuda.synchronize()
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during warm-up")
    use_graph = not args.no_graph
    graphs = []
    if use_graph:
        for s_ in range(n_sets):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                frame(s_)
            graphs.append(gr)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for s_ in range(n_sets):
            graphs[s_].replay()
        torch.cuda.synchronize()

    def step(i):
        if use_graph:
            graphs[i % n_sets].replay()
        else:
            frame(i)

    stream = torch.cuda.current_stream()
    clocks = Clocks(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    n_soak = 0
    t_end = time.time() + 1.0
    while True:                      # every rank runs the same number of soak frames
        for _ in range(16):
            step(n_soak)
            n_soak += 1
        torch.cuda.synchronize()
        more = torch.tensor([1 if time.time() < t_end else 0], device=device)
        if world > 1:
            dist.all_reduce(more, op=dist.ReduceOp.MIN)
        if not int(more.item()):
            break
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    err = fxr.check_device_error()
    if world > 1:
        t = torch.tensor([t_ms, float(err != 0)], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms, bad = float(t[0].item()), bool(t[1].item())
    else:
        bad = err != 0
    if bad:
        raise RuntimeError("device error during the timed region")
    flops = sum(attn_flops(w, frames[i % n_sets]["M"]) for i in range(args.steps))
    ms_per_step = t_ms / args.steps
    value = flops / (t_ms * 1e-3) / 1e12
    M_avg = statistics.mean(fr["M"] for fr in frames)
    # roofline of the fused attention + all-gather: the slower of the tensor-core time of this
    # rank's heads and the NVLink time of the O slices it sends to the other ranks
    flop_rank = attn_flops(w, M_avg) * g.n_heads / w.n_heads
    nvlink_bytes = M_avg * (c1 - c0) * 2 * (world - 1)
    t_tensor = flop_rank / (pk["bf16_tflops"] * 1e12)
    t_link = nvlink_bytes / 770e9
    out_line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "us_per_frame": round(ms_per_step * 1e3, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": w.dtype, "impl": "ours",
        "data": "synthetic: N(0,1) Q/K/V/cache, N(1,0.1) norm weights, Bernoulli mask (seeded)",
        "config": {"workload": w.name, "frame_px": w.grid_h * 16, "n_tokens": N,
                   "n_text": w.n_text, "active": w.active, "M_avg": M_avg, "heads": w.n_heads,
                   "heads_per_gpu": [int(x) for x in _heads_split(w.n_heads, world)],
                   "parallelism": f"heads{world}" + ("-nccl" if nccl else "-p2p"),
                   "l2": f"{n_sets} rotating input sets, cache shards {n_sets * shard_bytes / 2**20:.0f} MiB > L2",
                   "graph": use_graph},
        "roofline": {"bound": "tensor" if t_tensor >= t_link else "nvlink",
                     "kernel": (attention_kernel_name(max(_heads_split(w.n_heads, world)))
                                + ("" if world == 1 else " + NCCL all-gather + heads_scatter_kernel" if nccl
                                   else " + heads_push_kernel (peer stores to every rank)")),
                     "target_us": round(max(t_tensor, t_link) * 1e6, 2),
                     "achieved_frac": round(max(t_tensor, t_link) * 1e3 / ms_per_step, 4),
                     "peak_tensor": pk["bf16_tflops"], "peak_nvlink_gbs": 770.0,
                     "nvlink_bytes_per_rank": nvlink_bytes,
                     "note": "frac = roofline time of one frame / measured frame time (the whole frame)"},
        "e2e": None,
        # the gather (which compacts the mask) and the attention (which restores mask==1 rows);
        # with peers also the exchange and the arrival wait (heads_push_kernel, arrival_wait_kernel),
        # or the scatter after NCCL's own all-gather kernel (heads_scatter_kernel)
        "gpu_launches": (3 if nccl else 2 if world == 1 else 4) * args.steps,
        "clocks": clk,
    }
    if rank == 0 and not embedded:
        print(json.dumps(out_line), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()             # no rank unmaps or frees while a peer could still store
    for gr in graphs:
        del gr
    graphs.clear()
    for p_ in mapped:
        fxr.ipc_close(p_)
    if buf is not None:
        buf.free()
    if comm is not None:
        fxr.nccl_comm_destroy(comm)
    if world > 1:
        dist.barrier()
        if not embedded:
            dist.destroy_process_group()
    return out_line


# ---------------------------------------------------------------------------------------------
# independent edit streams, batched (config 4: 8 streams of 768^2 spread over the GPUs)
# ---------------------------------------------------------------------------------------------
def run_streams(args, embedded: bool = False):
    """A step is one frame of every stream: each GPU runs its streams' frames as one batched set
    of launches (fxr_frame_forward_batch). value = attention FLOP of all streams / max-over-ranks
    time; frames_per_s = streams / step time. Strong scaling: the total of streams is fixed.
    embedded: as for run_heads."""
    import datetime
    import torch
    import torch.distributed as dist
    import fxr

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not embedded:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    fxr.load()
    w = workload(args)
    cfg = frame_cfg(w)
    total = args.streams
    mine = [s_ for s_ in range(total) if s_ % world == rank]
    # two rotating sets of every stream's inputs: 2 x streams x ~100 MB > L2
    n_sets = 2
    sets = [[make_device_frame(w, args.seed + 7919 * s_ + 104729 * k, device) for s_ in mine]
            for k in range(n_sets)]
    pos = sets[0][0]["pos"]
    nq, nk = sets[0][0]["norm_q"], sets[0][0]["norm_k"]
    ws = [torch.empty(max(1, fxr.batch_workspace_size(cfg, len(mine))), dtype=torch.uint8, device=device)
          for _ in range(n_sets)]

    def step(i):
        k = i % n_sets
        if mine:
            fxr.frame_forward_batch(cfg, sets[k], pos, nq, nk, ws[k])

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during warm-up")
    graphs = []
    if not args.no_graph:
        for k in range(n_sets):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(k)
            graphs.append(g)
    run = (lambda i: graphs[i % n_sets].replay()) if graphs else step
    stream = torch.cuda.current_stream()
    clocks = Clocks(local)
    clocks.start()
    t_end = time.time() + 1.0
    i = 0
    while time.time() < t_end:
        run(i)
        i += 1
        if i % 16 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        run(i)
    e1.record(stream)
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    flops = sum(attn_flops(w, fr["M"]) for k in range(n_sets) for fr in sets[k]) / n_sets * args.steps
    if world > 1:
        t = torch.tensor([t_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms = float(t.item())
        f = torch.tensor([flops], dtype=torch.float64, device=device)
        dist.all_reduce(f, op=dist.ReduceOp.SUM)
        flops = float(f.item())
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during the timed region")
    ms_per_step = t_ms / args.steps
    out_line = {
        "metric": METRIC, "value": round(flops / (t_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "frames_per_s": round(total / (ms_per_step * 1e-3), 1),
        "us_per_frame_per_gpu": round(ms_per_step * 1e3 / max(1, len(mine)), 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
        "impl": "ours", "data": "synthetic: N(0,1) Q/K/V/cache, N(1,0.1) norm weights, Bernoulli masks (seeded, one per stream)",
        "config": {"workload": w.name, "streams": total, "streams_per_gpu": len(mine),
                   "n_tokens": w.n_tokens, "active": w.active, "heads": w.n_heads,
                   "parallelism": f"streams{total}-over-{world}",
                   "l2": f"{n_sets} rotating sets of every stream's inputs", "graph": bool(graphs)},
        "e2e": None, "gpu_launches": 2 * args.steps, "clocks": clk,
    }
    if rank == 0 and not embedded:
        print(json.dumps(out_line), flush=True)
    for g in graphs:
        del g
    graphs.clear()
    if world > 1:
        dist.barrier()
        if not embedded:
            dist.destroy_process_group()
    return out_line


# ---------------------------------------------------------------------------------------------
# the whole double-stream block on the executed rows (--path block)
# ---------------------------------------------------------------------------------------------
BLOCK_METRIC = "double-block frames/s @1024², 25% active (executed rows only; LN+QKV+attn+MLP+out)"
SINGLE_METRIC = "single-block frames/s @1024², 25% active (executed rows only; LN+QKV/MLP+attn+out)"


def single_weights(w, H: int, device, seed: int) -> dict:
    """Random-init weights of one single-stream block, bf16 matrices."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    C = w.n_heads * HEAD_DIM
    r = lambda *shape, sd=1.0: torch.randn(*shape, generator=g, device=device) * sd
    return {"shift": r(C, sd=0.1), "scale": r(C, sd=0.1), "gate": 1.0 + r(C, sd=0.2),
            "w_qkv_mlp": r(3 * C + H, C, sd=C ** -0.5).bfloat16(), "b_qkv_mlp": r(3 * C + H, sd=0.05),
            "norm_q": 1.0 + r(HEAD_DIM, sd=0.1), "norm_k": 1.0 + r(HEAD_DIM, sd=0.1),
            "w_out": r(C, C + H, sd=(C + H) ** -0.5).bfloat16(), "b_out": r(C, sd=0.05)}


def block_weights(w, H: int, device, seed: int) -> dict:
    """Random-init weights of one double-stream block (text and image streams), bf16 matrices."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    C = w.n_heads * HEAD_DIM
    r = lambda *shape, sd=1.0: torch.randn(*shape, generator=g, device=device) * sd
    out = {}
    for name in ("txt", "img"):
        out[name] = {"shift": r(C, sd=0.1), "scale": r(C, sd=0.1), "gate": 1.0 + r(C, sd=0.2),
                     "w_qkv": r(3 * C, C, sd=C ** -0.5).bfloat16(), "b_qkv": r(3 * C, sd=0.05),
                     "norm_q": 1.0 + r(HEAD_DIM, sd=0.1), "norm_k": 1.0 + r(HEAD_DIM, sd=0.1),
                     "w_out": r(C, C, sd=C ** -0.5).bfloat16(), "b_out": r(C, sd=0.05),
                     "w_mlp0": r(H, C, sd=C ** -0.5).bfloat16(), "b_mlp0": r(H, sd=0.05),
                     "w_mlp2": r(C, H, sd=H ** -0.5).bfloat16(), "b_mlp2": r(C, sd=0.05)}
    return out


def block_gemm_flops(w, M: int, H: int) -> float:
    C = w.n_heads * HEAD_DIM
    return 2.0 * M * C * 3 * C + 2.0 * M * C * H + 2.0 * M * (C + H) * C


def block_flops(w, M: int, H: int) -> float:
    return block_gemm_flops(w, M, H) + attn_flops(w, M)


def _graph_us(fn, reps: int = 20, rounds: int = 7) -> float:
    """Median device time of one call, from CUDA graphs of `reps` back-to-back calls."""
    import torch
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(rounds):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3 / reps)
    return statistics.median(ts)


def dense_block_torch(w, H, wts, x, pos_cos_sin):
    """The same block computed densely on every token with torch bf16 (cuBLAS GEMMs, SDPA
    attention): what running the block without the spatial cache costs on this GPU."""
    import torch
    import torch.nn.functional as F
    T, C = w.n_text, w.n_heads * HEAD_DIM
    cos, sin = pos_cos_sin
    outs = []
    qkv_all, xn_all = [], []
    for name, sl in (("txt", slice(0, T)), ("img", slice(T, None))):
        s = wts[name]
        xn = (F.layer_norm(x[sl].float(), (C,), eps=1e-6) * (1 + s["scale"]) + s["shift"]).bfloat16()
        xn_all.append(xn)
        qkv_all.append(F.linear(xn, s["w_qkv"], s["b_qkv"].bfloat16()))
    qkv = torch.cat(qkv_all)
    q, k, v = qkv.split(C, dim=1)

    def norm_rope(t, wn):
        t = t.view(-1, w.n_heads, HEAD_DIM).float()
        t = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * wn
        t1, t2 = t[..., 0::2], t[..., 1::2]
        return torch.stack((t1 * cos - t2 * sin, t1 * sin + t2 * cos), -1).flatten(-2).bfloat16()
    qn = norm_rope(q, wts["img"]["norm_q"]).transpose(0, 1).unsqueeze(0)
    kn = norm_rope(k, wts["img"]["norm_k"]).transpose(0, 1).unsqueeze(0)
    vv = v.reshape(-1, w.n_heads, HEAD_DIM).transpose(0, 1).unsqueeze(0)
    o = F.scaled_dot_product_attention(qn, kn, vv).squeeze(0).transpose(0, 1).reshape(-1, C)
    for (name, sl), xn in zip((("txt", slice(0, T)), ("img", slice(T, None))), xn_all):
        s = wts[name]
        h = F.gelu(F.linear(xn, s["w_mlp0"], s["b_mlp0"].bfloat16()), approximate="tanh")
        y = F.linear(o[sl], s["w_out"], s["b_out"].bfloat16()) + F.linear(h, s["w_mlp2"], s["b_mlp2"].bfloat16())
        outs.append(x[sl] + s["gate"].bfloat16() * y)
    return torch.cat(outs)


def run_block(args):
    import torch
    import fxr
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    fxr.load()
    w = workload(args)
    cfg = frame_cfg(w)
    pk = peaks()
    N, T, C = w.n_tokens, w.n_text, w.n_heads * HEAD_DIM
    H = 3 * C
    single = args.path == "single"
    wts = (single_weights if single else block_weights)(w, H, device, args.seed + 17 * rank)
    n_sets = 2
    sets = []
    for sidx in range(n_sets):
        fr = make_device_frame(w, args.seed + 7919 * rank + sidx, device)
        sets.append({"x_in": fr["q"], "x_out": fr["out"], "mask": fr["mask"], "pos": fr["pos"],
                     "valid": torch.ones(N, dtype=torch.uint8, device=device),
                     "cache_k": fr["cache_k"], "cache_v": fr["cache_v"], "M": fr["M"],
                     "ws": torch.empty(fxr.double_block_workspace_size(cfg, H), dtype=torch.uint8,
                                       device=device)})

    def run(st):
        if single:
            fxr.single_block_forward(cfg, wts, H, st["x_in"], st["x_out"], st["mask"], st["valid"],
                                     st["pos"], st["cache_k"], st["cache_v"], st["ws"])
        else:
            fxr.double_block_forward(cfg, wts["txt"], wts["img"], H, st["x_in"], st["x_out"], st["mask"],
                                     st["valid"], st["pos"], st["cache_k"], st["cache_v"], st["ws"])

    for i in range(max(args.warmup, 3)):
        run(sets[i % n_sets])
    torch.cuda.synchronize()
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during warm-up")
    # one graph per input set, and one holding both frames back to back (a stream of frames)
    graphs = []
    for st in sets:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run(st)
        graphs.append(g)
    run_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(run_graph):
        for st in sets:
            run(st)

    def steps(k):
        i = 0
        while k - i >= n_sets:
            run_graph.replay()
            i += n_sets
        while i < k:
            graphs[i % n_sets].replay()
            i += 1
    stream = torch.cuda.current_stream()
    clocks = Clocks(local)
    clocks.start()
    t_end = time.time() + 1.0
    while time.time() < t_end:
        steps(16)
        torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    t_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([t_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms = float(t.item())
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during the timed region")
    ms = t_ms / args.steps
    M_avg = statistics.mean(st["M"] for st in sets)
    fl = block_flops(w, M_avg, H)
    if single:
        out = single_block_report(args, w, cfg, wts, sets, run, H, ms, fl, M_avg, clk, pk, world)
        if rank == 0:
            print(json.dumps(out), flush=True)
        if world > 1:
            graphs.clear()
            dist.barrier()
            dist.destroy_process_group()
        return

    # ---- the block's kernels one at a time (image rows of set 0; graphs of 20 launches) ----
    st = sets[0]
    idx = torch.empty(N, dtype=torch.int32, device=device)
    cnt = torch.empty(1, dtype=torch.int32, device=device)
    fxr.mask_compact(st["mask"], None, idx, cnt)
    xn = torch.randn(N, C, device=device).bfloat16()
    qkv = [torch.empty(N, C, device=device, dtype=torch.bfloat16) for _ in range(3)]
    hbuf = torch.randn(N, H, device=device).bfloat16() * 0.1
    attn = torch.randn(N, C, device=device).bfloat16()
    yout = torch.empty(N, C, device=device, dtype=torch.bfloat16)
    scr = fxr.rows_gemm_scratch(device)
    s_img = wts["img"]
    kern = {
        "ln_modulate": _graph_us(lambda: fxr.ln_modulate_rows(st["x_in"], idx, cnt, xn, s_img["scale"],
                                                              s_img["shift"], row0=T)),
        "qkv_gemm": _graph_us(lambda: fxr.rows_gemm([(xn, s_img["w_qkv"], False)],
                                                    [(t, C, True, 0) for t in qkv], idx, cnt, N,
                                                    bias0=s_img["b_qkv"], row0=T, scratch=scr)),
        "mlp_up_gemm": _graph_us(lambda: fxr.rows_gemm([(xn, s_img["w_mlp0"], False)],
                                                       [(hbuf, H, False, fxr.FXR_ACT_GELU_TANH)], idx, cnt, N,
                                                       bias0=s_img["b_mlp0"], row0=T, scratch=scr)),
        "out_down_gemm": _graph_us(lambda: fxr.rows_gemm([(attn, s_img["w_out"], True), (hbuf, s_img["w_mlp2"], False)],
                                                         [(yout, C, True, 0)], idx, cnt, N, bias0=s_img["b_out"],
                                                         bias1=s_img["b_mlp2"], residual=st["x_in"],
                                                         gate=s_img["gate"], row0=T, scratch=scr)),
    }
    M_img = st["M"] - T
    qkv_fl = 2.0 * M_img * C * 3 * C
    achieved = qkv_fl / (kern["qkv_gemm"] * 1e-6) / 1e12
    roof = {"bound": "tensor", "kernel": "fxr::gemm::rows_gemm_kernel (Q/K/V of the executed image rows)",
            "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["bf16_tflops"], 4), "peak_kind": f"{pk['source']} burst bf16 (cuBLAS)",
            "traffic": profile_traffic(f"rows_gemm_qkv_{w.name}"), "algorithmic_flop_per_launch": qkv_fl}

    # ---- the dense block on every token with torch (cuBLAS + SDPA), same GPU ----
    import workloads as W
    posn = torch.from_numpy(W.positions(w)).to(device)
    ax = list(w.rope_axes)
    ang = []
    for a, d in enumerate(ax):
        om = w.rope_theta ** (-torch.arange(0, d, 2, device=device, dtype=torch.float64) / d)
        ang.append(posn[:, a:a + 1].double() * om)
    ang = torch.cat(ang, dim=1).float()[:, None, :]
    cs = (torch.cos(ang), torch.sin(ang))
    dense_us = _graph_us(lambda: dense_block_torch(w, H, wts, st["x_in"], cs), reps=5, rounds=5)

    # ---- end to end through the C ABI with the hidden states in pinned host memory: the host entry
    # moves only the executed rows of x_in in and of x_out back; frames alternate between the two
    # sets on two streams. For comparison, whole-tensor copies around the device entry. ----
    host_x = st["x_in"].cpu().pin_memory()
    host_m = torch.from_numpy(W.make_mask(w, np.random.default_rng(args.seed))).pin_memory()
    host_o = [torch.empty_like(host_x).pin_memory() for _ in range(2)]
    host_ws = [torch.empty(fxr.block_host_workspace_size(cfg, H), dtype=torch.uint8, device=device)
               for _ in range(2)]
    lanes = [torch.cuda.Stream() for _ in range(2)]
    M_exec = T + int((host_m[T:] != 0).sum())

    def one_host(i):
        st_i = sets[i % 2]
        fxr.double_block_forward(cfg, wts["txt"], wts["img"], H, host_x, host_o[i % 2], host_m, st_i["valid"],
                                 st_i["pos"], st_i["cache_k"], st_i["cache_v"], host_ws[i % 2],
                                 stream=lanes[i % 2], host=True)

    def one_full(i):
        st_i = sets[i % 2]
        with torch.cuda.stream(lanes[i % 2]):
            st_i["x_in"].copy_(host_x, non_blocking=True)
            st_i["mask"].copy_(host_m, non_blocking=True)
            run(st_i)
            host_o[i % 2].copy_(st_i["x_out"], non_blocking=True)

    def timed(one):
        for i in range(4):
            one(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()
        reps = max(6, min(30, args.steps))
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for ln in lanes:
            ln.wait_stream(stream)
        for i in range(reps):
            one(i)
        for ln in lanes:
            stream.wait_stream(ln)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / reps

    e2e_ms = timed(one_host)
    full_ms = timed(one_full)
    if fxr.check_device_error() != 0:
        raise RuntimeError("device error during the end-to-end frames")
    # whole job: the slowest rank's time per frame, every rank's frames and bytes
    tot = [M_exec * C * 2 + host_m.numel() * 4, M_exec * C * 2, host_x.numel() * 2 + host_m.numel() * 4,
           host_o[0].numel() * 2]
    (e2e_ms, full_ms), tot = whole_job([e2e_ms, full_ms], tot, world, device)
    e2e = {"value": round(1e3 / e2e_ms * world, 2), "unit": "frames/s", "us_per_frame": round(e2e_ms * 1e3, 1),
           "ranks": world, "h2d_bytes_per_step": int(tot[0]), "d2h_bytes_per_step": int(tot[1]),
           "path": "fxr_double_block_forward_host via ctypes: pinned host x_in / mask / x_out, only the "
                   "executed rows cross PCIe, frames alternating over two streams",
           "full_frame_copies": {"us_per_frame": round(full_ms * 1e3, 1),
                                 "value": round(1e3 / full_ms * world, 2),
                                 "h2d_bytes_per_step": int(tot[2]),
                                 "d2h_bytes_per_step": int(tot[3]),
                                 "path": "whole-tensor copies around fxr_double_block_forward"}}
    out = {
        "metric": BLOCK_METRIC, "value": round(1e3 / ms * world, 2), "unit": "frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "us_per_frame": round(ms * 1e3, 2), "block_tflops": round(fl / (ms * 1e-3) / 1e12, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype, "impl": "ours",
        "data": "synthetic: N(0,1) hidden states and caches, random-init block weights (seeded)",
        "config": {"workload": w.name + "_double_block", "n_tokens": N, "n_text": T, "active": w.active,
                   "M_avg": M_avg, "heads": w.n_heads, "hidden": C, "mlp_hidden": H,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "weights 377 MB per step > L2", "graph": "2 consecutive frames per CUDA graph"},
        "roofline": roof,
        "kernels_isolated_us": {k: round(v, 2) for k, v in kern.items()},
        "dense_torch_same_gpu_us": round(dense_us, 1),
        "e2e": e2e,
        "gpu_launches": 12 * args.steps,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            out["cpu_baseline"] = cpu_block_baseline(w, H, args.seed)
        except Exception as ex:  # the baseline is reported, not required
            out["cpu_baseline"] = {"value": None, "error": str(ex)[:200]}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        graphs.clear()
        dist.barrier()
        dist.destroy_process_group()


def single_block_report(args, w, cfg, wts, sets, run, H, ms, fl, M_avg, clk, pk, world) -> dict:
    """JSON line of the single-stream block: the fused projection GEMM as the roofline kernel."""
    import torch
    import fxr
    device = sets[0]["x_in"].device
    N, C = w.n_tokens, w.n_heads * HEAD_DIM
    st = sets[0]
    idx = torch.empty(N, dtype=torch.int32, device=device)
    cnt = torch.empty(1, dtype=torch.int32, device=device)
    fxr.mask_compact(st["mask"], None, idx, cnt)
    M = int(cnt.item())
    xn = torch.randn(N, C, device=device).bfloat16()
    qkv = [torch.empty(N, C, device=device, dtype=torch.bfloat16) for _ in range(3)]
    hbuf = torch.empty(N, H, device=device, dtype=torch.bfloat16)
    attn = torch.randn(N, C, device=device).bfloat16()
    yout = torch.empty(N, C, device=device, dtype=torch.bfloat16)
    scr = fxr.rows_gemm_scratch(device)
    w_out = wts["w_out"]
    kern = {
        "fused_proj_gemm": _graph_us(lambda: fxr.rows_gemm([(xn, wts["w_qkv_mlp"], False)],
                                                           [(t, C, True, 0) for t in qkv] +
                                                           [(hbuf, H, False, fxr.FXR_ACT_GELU_TANH)],
                                                           idx, cnt, N, bias0=wts["b_qkv_mlp"], scratch=scr)),
        "out_gemm": _graph_us(lambda: fxr.rows_gemm([(attn, w_out[:, :C], True), (hbuf, w_out[:, C:], False)],
                                                    [(yout, C, True, 0)], idx, cnt, N, bias0=wts["b_out"],
                                                    residual=st["x_in"], gate=wts["gate"], scratch=scr)),
    }
    proj_fl = 2.0 * M * C * (3 * C + H)
    achieved = proj_fl / (kern["fused_proj_gemm"] * 1e-6) / 1e12
    roof = {"bound": "tensor", "kernel": "fxr::gemm::rows_gemm_kernel (fused Q/K/V + MLP-in projection)",
            "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["bf16_tflops"], 4), "peak_kind": f"{pk['source']} burst bf16 (cuBLAS)",
            "traffic": None, "algorithmic_flop_per_launch": proj_fl}
    return {
        "metric": SINGLE_METRIC, "value": round(1e3 / ms * world, 2), "unit": "frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "us_per_frame": round(ms * 1e3, 2), "block_tflops": round(fl / (ms * 1e-3) / 1e12, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype, "impl": "ours",
        "data": "synthetic: N(0,1) hidden states and caches, random-init block weights (seeded)",
        "config": {"workload": w.name + "_single_block", "n_tokens": N, "active": w.active, "M_avg": M_avg,
                   "heads": w.n_heads, "hidden": C, "mlp_hidden": H, "graph": True},
        "roofline": roof, "kernels_isolated_us": {k: round(v, 2) for k, v in kern.items()},
        "gpu_launches": 7 * args.steps, "clocks": clk,
        "e2e": None, "note": "e2e and the CPU arm are reported by --path block",
    }


def cpu_block_sample(w, H: int, seed: int, rows: int = 256) -> dict:
    """One dense fp32 frame of the reference block on the host cores (the oracle's
    dense_block_sample); returns seconds per frame."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    return O.dense_block_sample(w.n_tokens, w.n_heads, HEAD_DIM, H, seed, rows)


def cpu_block_baseline(w, H: int, seed: int) -> dict:
    try:
        import threadpoolctl
        cores = max(info.get("num_threads", 1) for info in threadpoolctl.threadpool_info()) or 1
    except Exception:
        cores = os.cpu_count() or 1
    s = cpu_block_sample(w, H, seed)
    spf = s["seconds_per_frame"]
    return {"value": round(1.0 / spf, 4), "unit": "frames/s", "cores": cores, "kind": "port",
            "sample": f"one dense fp32 frame of {w.name}: LayerNorm + Q/K/V of all {w.n_tokens} tokens, "
                      f"attention/MLP/out-projection of {s['rows']} sampled query tokens over all keys "
                      f"scaled to {w.n_tokens} (numpy BLAS, oracle dense_block_sample)",
            "seconds_per_frame": round(spf, 3)}


def run_block_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    w = workload(args)
    H = 3 * w.n_heads * HEAD_DIM
    cpu_block_sample(w, H, args.seed, rows=32)                 # warm the BLAS pool
    steps = max(1, min(args.steps, 5))
    t = [cpu_block_sample(w, H, args.seed + i)["seconds_per_frame"] for i in range(steps)]
    spf = statistics.mean(t)
    base = cpu_block_baseline(w, H, args.seed)
    out = {"metric": BLOCK_METRIC, "value": round(1.0 / spf, 4), "unit": "frames/s", "n_gpus": world,
           "steps": steps, "warmup": 1, "ms_per_step": round(spf * 1e3, 1), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
           "data": "synthetic (seeded)", "config": {"workload": w.name + "_double_block", "n_tokens": w.n_tokens},
           "cpu_baseline": dict(base, value=round(1.0 / spf, 4)),
           "e2e": {"value": round(1.0 / spf, 4), "unit": "frames/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0},
           "note": "the reference block runs densely in fp32 (cublasSgemm per projection); this arm "
                   "times the same dense fp32 math on the host cores with numpy BLAS"}
    print(json.dumps(out), flush=True)


def _heads_split(n_heads, world):
    return [n_heads // world + (1 if r < n_heads % world else 0) for r in range(world)]


def main():
    args = parse()
    if args.path in ("block", "single"):
        (run_block_reference if args.impl == "reference" else run_block)(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.split in ("heads", "heads_nccl"):
        run_heads(args)
    elif args.streams is not None and args.streams > 1:
        run_streams(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
