#!/usr/bin/env python3
"""Times the reference's own CUDA kernels (oracle/_ref, built from the reference sources by
oracle/build_ref.sh) on one frame of the sparse attention slice, beside this library's frame on the
same GPU. TEST/BASELINE INFRASTRUCTURE: nothing in the product imports it.

    python oracle/time_reference_cuda.py [--config c2] [--reps 5]

The reference slice (fp32, as its plugins run it): gather_tokens of Q, K, V rows
(gather_scatter_kernels.cu:15-41), launch_rms_norm on the gathered Q and K per head (seq_len =
M*H, dim = 128; flux2_kernels.cu:58-90), SpatialCache::sync_kv_cache over all N rows
(spatial_kv_cache.cu:55-87, 175-196), attention_fwd of the M queries over the N merged keys
(attention_kernels.cu:85-173, (B,H,S,D) layout: the transposes around it are not timed) and
scatter_tokens of the outputs (gather_scatter_kernels.cu:46-72). The reference has no RoPE.
Prints a markdown table (per-kernel median device time, CUDA events on the launching stream)."""
from __future__ import annotations

import argparse
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "fluxrt-cpp_b200"))

import numpy as np  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    import torch
    import oracle as O
    import workloads as W
    import fxr

    L = O.ref_kernels()
    if L is None:
        raise SystemExit("oracle/_ref/libfxr_refkernels.so missing: run oracle/build_ref.sh")
    w = {"c1": W.C1, "c2": W.C2, "c3": W.C3, "c4": W.C4, "c5": W.C5}[args.config]
    N, H, D = w.n_tokens, w.n_heads, w.head_dim
    C = H * D
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    rng = np.random.default_rng(12)
    mask_h = W.make_mask(w, rng)
    M = int((mask_h != 0).sum())
    idx = torch.from_numpy(np.nonzero(mask_h)[0].astype(np.int32)).to(dev)
    mask = torch.from_numpy(mask_h).to(dev)
    q, k, v = (torch.randn(N, C, device=dev, generator=g) for _ in range(3))
    qg, kg, vg = (torch.empty(M, C, device=dev) for _ in range(3))
    wq = (1 + 0.1 * torch.randn(D, device=dev, generator=g))
    out_full = torch.zeros(N, C, device=dev)
    s = torch.cuda.current_stream()
    cache = L.ref_cache_create(N - w.n_text, w.n_text, 64, H, D, 1, 0)
    if not cache:
        raise SystemExit("reference SpatialCache construction failed")

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

    ss = s.cuda_stream
    rows = {}
    rows["gather_tokens x3 (Q,K,V)"] = timed(lambda: [L.ref_gather_tokens(
        t.data_ptr(), o.data_ptr(), idx.data_ptr(), M, C, ss) for t, o in ((q, qg), (k, kg), (v, vg))],
        args.reps)
    qn, kn = torch.empty_like(qg), torch.empty_like(kg)
    rows["launch_rms_norm x2 (Q,K per head)"] = timed(lambda: [L.ref_rms_norm(
        a.data_ptr(), b.data_ptr(), wq.data_ptr(), 1e-6, M * H, D, ss) for a, b in ((qg, qn), (kg, kn))],
        args.reps)
    kk, vv = k.clone(), v.clone()
    rows["SpatialCache::sync_kv_cache (N rows)"] = timed(lambda: L.ref_cache_sync_kv(
        cache, kk.data_ptr(), vv.data_ptr(), mask.data_ptr(), 0, 1, ss), args.reps)
    qh = qn.view(M, H, D).transpose(0, 1).contiguous()
    kh = kk.view(N, H, D).transpose(0, 1).contiguous()
    vh = vv.view(N, H, D).transpose(0, 1).contiguous()
    oh = torch.empty_like(qh)
    rows["attention_fwd (fp32, B=1)"] = timed(lambda: L.ref_attention_fwd(
        qh.data_ptr(), kh.data_ptr(), vh.data_ptr(), oh.data_ptr(), 1, H, M, N, D, ss),
        max(2, min(args.reps, 3)))
    og = oh.transpose(0, 1).reshape(M, C).contiguous()
    rows["scatter_tokens"] = timed(lambda: L.ref_scatter_tokens(
        og.data_ptr(), out_full.data_ptr(), idx.data_ptr(), M, C, ss), args.reps)
    torch.cuda.synchronize()
    L.ref_cache_destroy(cache)
    total = sum(rows.values())

    # this library's frame on the same inputs (bf16), in a CUDA graph, median per frame
    dt = torch.bfloat16 if w.dtype == "bf16" else torch.float16
    cfg = fxr.FrameConfig(n_tokens=N, n_text=w.n_text, n_heads=H, dtype=w.dtype,
                          rope_axes=w.rope_axes, rope_theta=w.rope_theta)
    qb, kb, vb = q.to(dt), k.to(dt), v.to(dt)
    ckb, cvb, ob = k.to(dt), v.to(dt), torch.zeros(N, C, device=dev, dtype=dt)
    pos = torch.from_numpy(W.positions(w)).to(dev)
    ws = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device=dev)
    masks = mask.clone()
    frame = lambda: fxr.frame_forward(cfg, qb, kb, vb, masks, None, pos, wq, wq, ckb, cvb, ob, ws)
    for _ in range(3):
        frame()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(20):
            frame()
    ours = timed(lambda: gr.replay(), 8) / 20
    flop = 4.0 * M * N * D * H
    print(f"| kernel ({w.name}, M = {M}, N = {N}) | reference fp32, µs |")
    print("|---|---|")
    for name, us in rows.items():
        print(f"| {name} | {us:.1f} |")
    print(f"| **reference slice total** | **{total:.1f}** ({flop / (total * 1e-6) / 1e12:.2f} TFLOP/s) |")
    print(f"| this library, fxr_frame_forward ({w.dtype}, incl. RoPE) | {ours:.1f} ({flop / (ours * 1e-6) / 1e12:.1f} TFLOP/s) |")
    print(f"\nspeed-up of the frame: {total / ours:.0f}x")


if __name__ == "__main__":
    main()
