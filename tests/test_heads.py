"""One frame split by attention heads (fxr_head_group_*, fxr_frame_forward_heads).

CPU: the head split, argument checks, and — as world-size-2 gloo ranks — that per-rank head shards
of the oracle, all-gathered by head, reproduce the full-frame oracle exactly (heads are independent
in every step of the path). GPU: G ranks emulated on one GPU (every rank's frame is issued before
any rank's wait, so no wait depends on later work) against the single-GPU frame (caches bit-exact,
outputs within the attention bar, every rank's output identical); and, where the box has two GPUs,
two real ranks exchanging O over NVLink peer mappings or an NCCL all-gather (bit-exact between the
two exchanges)."""
import os
import socket

import numpy as np
import pytest

import fxr
import workloads as W


@pytest.mark.parametrize("world,heads", [(1, 24), (2, 24), (3, 24), (4, 24), (8, 24), (5, 24),
                                         (8, 3), (8, 9)])
def test_head_split_tiles_the_heads(world, heads):
    gs = [fxr.head_group(world, r, heads, 4608) for r in range(world)]
    h = 0
    for r, g in enumerate(gs):
        assert g.world == world and g.rank == r and g.epoch == 0
        assert g.head0 == h
        assert g.n_heads in (heads // world, heads // world + 1)
        h += g.n_heads
        assert list(g.ctas[:world]) == list(gs[0].ctas[:world])     # every rank agrees
        assert all(not p for p in g.out) and all(not p for p in g.arrive)
    assert h == heads
    for r, g in enumerate(gs):
        # arrivals per frame: one per exchange CTA of every GPU that has heads; none on one GPU
        assert (gs[0].ctas[r] > 0) == (world > 1 and g.n_heads > 0)


def test_head_group_rejects_bad_arguments():
    L = fxr.load()
    g = fxr.HeadGroup()
    for args in [(0, 0, 24, 16), (9, 0, 24, 16), (2, 2, 24, 16), (2, 0, 0, 16), (2, 0, 24, -1)]:
        assert L.fxr_head_group_init(g, *args) == fxr.FXR_ERR_INVALID
    # a group whose heads do not fit the frame is refused before any GPU work
    g = fxr.head_group(2, 1, 24, 1536)
    cfg = fxr.FrameConfig(n_tokens=1536, n_text=512, n_heads=4)
    st = L.fxr_frame_forward_heads(cfg.desc(), g, *([None] * 11), 0, None)
    assert st == fxr.FXR_ERR_INVALID and b"heads" in L.fxr_last_error_string()
    g = fxr.head_group(2, 0, 4, 1536)                 # out[] pointers not set
    st = L.fxr_frame_forward_heads(cfg.desc(), g, *([None] * 11), 0, None)
    assert st == fxr.FXR_ERR_INVALID and b"out[0]" in L.fxr_last_error_string()


def test_nccl_variant_workspace_and_argument_checks():
    L = fxr.load()
    cfg = fxr.FrameConfig(n_tokens=16896, n_text=512)
    g = fxr.head_group(8, 3, 24, 16896)
    frame = fxr.workspace_size(fxr.FrameConfig(n_tokens=16896, n_text=512, n_heads=3))
    ws = fxr.heads_nccl_workspace_size(cfg, g, 3000)
    # shard frame workspace + iota + compact O [3000, 3*128] + gathered [8, 3000, 3*128]
    assert ws >= frame + 16896 * 4 + 9 * 3000 * 384 * 2
    assert fxr.heads_nccl_workspace_size(cfg, g, -1) == 0
    st = L.fxr_frame_forward_heads_nccl(cfg.desc(), g, None, 16897, *([None] * 12), 0, None)
    assert st == fxr.FXR_ERR_INVALID and b"m_cap" in L.fxr_last_error_string()
    g2 = fxr.head_group(8, 3, 16, 16896)                       # split of another head count
    st = L.fxr_frame_forward_heads_nccl(cfg.desc(), g2, None, 100, *([None] * 12), 0, None)
    assert st == fxr.FXR_ERR_INVALID


def _shard_worker(rank, world, port, n_heads, result_path):
    import torch
    import torch.distributed as dist
    import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        w = W.Workload("c1_h%d" % n_heads, 32, 32, 512, n_heads, 128, "f16", 0.25, "bernoulli",
                       (16, 56, 56), 10000.0)
        fr = W.make_frame(w, seed=3)
        g = fxr.head_group(world, rank, n_heads, w.n_tokens)
        c0, c1 = g.head0 * 128, (g.head0 + g.n_heads) * 128
        cols = lambda a: np.ascontiguousarray(a[:, c0:c1])
        r = O.frame_forward(cols(fr["q"]), cols(fr["k"]), cols(fr["v"]), fr["mask"], None,
                            fr["pos"], fr["norm_q"], fr["norm_k"], cols(fr["cache_k"]),
                            cols(fr["cache_v"]), cols(fr["out"]), g.n_heads, 128, w.rope_axes,
                            w.rope_theta)
        mine = torch.from_numpy(r["out"])
        parts = [None] * world
        dist.all_gather_object(parts, (g.head0, g.n_heads, mine))
        if rank == 0:
            full = O.frame_forward(fr["q"], fr["k"], fr["v"], fr["mask"], None, fr["pos"],
                                   fr["norm_q"], fr["norm_k"], fr["cache_k"], fr["cache_v"],
                                   fr["out"], n_heads, 128, w.rope_axes, w.rope_theta)
            got = np.concatenate([p[2].numpy() for p in sorted(parts, key=lambda p: p[0])], axis=1)
            np.save(result_path, np.array([np.array_equal(got, full["out"]),
                                           sum(p[1] for p in parts) == n_heads]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_shards_reassemble_the_oracle_frame_gloo(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "ok.npy")
    mp.start_processes(_shard_worker, args=(2, _free_port(), 6, out), nprocs=2,
                       start_method="spawn")
    assert np.load(out).all()


# ---------------------------------------------------------------------------------------------
def _out_close(a, b, dtype):
    """Outputs of a head-split frame against the single-GPU frame. A rank's attention runs fewer
    (query tile, head) units than the whole frame and may split each unit's key range across CTAs
    where the single-GPU frame does not, which reorders the softmax sums: equal within the bar of
    the attention output, not bit for bit."""
    import torch
    tol = (2e-3, 2e-4)
    err = (a.float() - b.float()).abs()
    return bool(torch.isfinite(a.float()).all()) and err.max().item() <= tol[0] and \
        err.mean().item() <= tol[1]


def _frame_tensors(w, fr):
    import torch
    td = {"bf16": torch.bfloat16, "f16": torch.float16}[w.dtype]
    t = {k: torch.from_numpy(fr[k]).cuda().to(td) for k in ("q", "k", "v", "cache_k", "cache_v",
                                                           "out")}
    t["mask"] = torch.from_numpy(fr["mask"]).cuda()
    t["pos"] = torch.from_numpy(fr["pos"]).cuda()
    t["norm_q"] = torch.from_numpy(fr["norm_q"]).cuda()
    t["norm_k"] = torch.from_numpy(fr["norm_k"]).cuda()
    return t


@pytest.mark.gpu
@pytest.mark.parametrize("world,dtype,geom", [(2, "bf16", "c2_h12"), (3, "bf16", "c2_h12"), (4, "f16", "c2_h12"),
                                              (2, "bf16", "grid400_h2")])
def test_heads_emulated_on_one_gpu_match_the_frame(cuda, world, dtype, geom):
    """Every rank's share issued before any wait, on one GPU; the assembled frame equals the
    single-GPU frame within the O bar and the oracle on sampled rows. grid400_h2: 160 512 tokens,
    more per CTA than the gather's row list holds (the compaction kernel runs first)."""
    import torch
    if geom == "c2_h12":
        w = W.Workload("c2_h12", 64, 64, 512, 12, 128, dtype, 0.25, "bernoulli", (16, 56, 56), 10000.0)
    else:
        w = W.Workload("grid400_h2", 400, 400, 512, 2, 128, dtype, 0.02, "bernoulli", (16, 56, 56), 10000.0)
    cfg = fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=w.n_heads, dtype=dtype,
                          rope_axes=w.rope_axes, rope_theta=w.rope_theta)
    ws_full = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
    groups = [fxr.head_group(world, r, w.n_heads, w.n_tokens) for r in range(world)]
    outs = [None] * world
    slots = torch.zeros(world, 16, dtype=torch.int32, device="cuda")
    caches = []
    for f in range(2):
        rng = np.random.default_rng(40 + f)
        fr = W.make_frame(w, seed=50 + f)
        valid = (rng.random(w.n_tokens) < 0.8).astype(np.uint8)
        ref = _frame_tensors(w, fr)
        if f == 0:
            caches = [(ref["cache_k"][:, g.head0 * 128:(g.head0 + g.n_heads) * 128].contiguous(),
                       ref["cache_v"][:, g.head0 * 128:(g.head0 + g.n_heads) * 128].contiguous())
                      for g in groups]
            outs = [ref["out"].clone() for _ in range(world)]
        else:
            ref["cache_k"] = torch.cat([c[0] for c in caches], dim=1).contiguous()
            ref["cache_v"] = torch.cat([c[1] for c in caches], dim=1).contiguous()
            ref["out"] = outs[0].clone()
        for g in groups:
            for r in range(world):
                g.out[r] = outs[r].data_ptr()
                g.arrive[r] = slots[r].data_ptr()
        dvalid = torch.from_numpy(valid).cuda()
        pre_k, pre_v = ref["cache_k"].float().cpu().numpy(), ref["cache_v"].float().cpu().numpy()
        masks = [ref["mask"].clone() for _ in range(world)]
        ws = [torch.empty_like(ws_full) for _ in range(world)]
        for r, g in enumerate(groups):      # every rank's frame first ...
            fxr.frame_forward_heads(cfg, g, ref["q"], ref["k"], ref["v"], masks[r], dvalid,
                                    ref["pos"], ref["norm_q"], ref["norm_k"], caches[r][0],
                                    caches[r][1], ws[r])
        for g in groups:                    # ... then the waits, already satisfied
            fxr.head_group_wait(g)
        fxr.frame_forward(cfg, ref["q"], ref["k"], ref["v"], ref["mask"], dvalid, ref["pos"],
                          ref["norm_q"], ref["norm_k"], ref["cache_k"], ref["cache_v"], ref["out"],
                          ws_full)
        torch.cuda.synchronize()
        assert fxr.check_device_error() == 0
        for r, g in enumerate(groups):
            assert g.epoch == f + 1
            assert _out_close(outs[r], ref["out"], dtype), (f, r)
            assert torch.equal(outs[r], outs[0]), (f, r)        # every rank holds the same output
            c0, c1 = g.head0 * 128, (g.head0 + g.n_heads) * 128
            assert torch.equal(caches[r][0], ref["cache_k"][:, c0:c1]), (f, r)
            assert torch.equal(caches[r][1], ref["cache_v"][:, c0:c1]), (f, r)
            assert torch.equal(masks[r], ref["mask"])
            expect = [(f + 1) * groups[0].ctas[s] for s in range(world)]
            assert slots[r, :world].tolist() == expect and slots[r, 8].item() == f + 1
        # the assembled frame against the oracle on the stored operands (ranks of 4 or 6 heads run
        # the split-capable attention)
        import oracle as O
        import parity_stats
        op = O.frame_operands(fr["q"], fr["k"], fr["v"], fr["mask"], valid, fr["pos"], fr["norm_q"],
                              fr["norm_k"], pre_k, pre_v, w.n_heads, 128, w.rope_axes, w.rope_theta,
                              dtype)
        sel = np.sort(np.random.default_rng(f).choice(op["idx"].size, size=128, replace=False))
        ref_o = O.attention(op["qc"][sel], op["keys"], op["values"], w.n_heads, 128)
        got = outs[0].float().cpu().numpy()[op["idx"][sel]]
        mx, mn = parity_stats.record(f"O frame {f} vs oracle", got, ref_o, 2e-3, 2e-4)
        assert mx <= 2e-3 and mn <= 2e-4, (f, mx, mn)


@pytest.mark.gpu
@pytest.mark.parametrize("m_cap_kind", ["exact", "n_tokens"])
def test_nccl_variant_single_rank_matches_the_frame(cuda, m_cap_kind):
    import torch
    w = W.Workload("c2_h6", 64, 64, 512, 6, 128, "bf16", 0.25, "bernoulli", (16, 56, 56), 10000.0)
    cfg = fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=w.n_heads, dtype="bf16",
                          rope_axes=w.rope_axes, rope_theta=w.rope_theta)
    fr = W.make_frame(w, seed=71)
    a, b = _frame_tensors(w, fr), _frame_tensors(w, fr)
    M = int((fr["mask"] != 0).sum())
    m_cap = M if m_cap_kind == "exact" else w.n_tokens
    g = fxr.head_group(1, 0, w.n_heads, w.n_tokens)
    comm = fxr.nccl_comm_init(1, 0, fxr.nccl_unique_id())
    try:
        ws = torch.empty(fxr.heads_nccl_workspace_size(cfg, g, m_cap), dtype=torch.uint8,
                         device="cuda")
        fxr.frame_forward_heads_nccl(cfg, g, comm, m_cap, a["q"], a["k"], a["v"], a["mask"], None,
                                     a["pos"], a["norm_q"], a["norm_k"], a["cache_k"],
                                     a["cache_v"], a["out"], ws)
        wsf = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
        fxr.frame_forward(cfg, b["q"], b["k"], b["v"], b["mask"], None, b["pos"], b["norm_q"],
                          b["norm_k"], b["cache_k"], b["cache_v"], b["out"], wsf)
        torch.cuda.synchronize()
        assert fxr.check_device_error() == 0
        for key in ("out", "cache_k", "cache_v", "mask"):
            bad = (a[key] != b[key]).reshape(a[key].shape[0], -1).any(dim=1).nonzero().flatten()
            assert bad.numel() == 0, (key, bad.numel(), bad[:8].tolist(), M)
    finally:
        torch.cuda.synchronize()
        fxr.nccl_comm_destroy(comm)


def _two_gpu_worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    bufs, mapped = None, []
    try:
        w = W.Workload("c5_small", 96, 96, 512, 8, 128, "bf16", 0.15, "bernoulli", (16, 56, 56),
                       10000.0)
        cfg = fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=w.n_heads,
                              dtype="bf16", rope_axes=w.rope_axes, rope_theta=w.rope_theta)
        fr = W.make_frame(w, seed=91)
        t = _frame_tensors(w, fr)
        g = fxr.head_group(world, rank, w.n_heads, w.n_tokens)
        C = w.n_heads * 128
        out_bytes = w.n_tokens * C * 2
        bufs = fxr.IpcBuffer(out_bytes + 256)
        out = fxr.device_view(bufs.ptr.value, (w.n_tokens, C), torch.bfloat16)
        out.copy_(t["out"])
        handles = [None] * world
        dist.all_gather_object(handles, bufs.handle_bytes())
        for r in range(world):
            p = bufs.ptr.value if r == rank else fxr.ipc_open(handles[r])
            if r != rank:
                mapped.append(p)
            g.out[r] = p
            g.arrive[r] = p + out_bytes
        torch.cuda.synchronize()
        dist.barrier()                     # every rank's output holds the initial values
        c0, c1 = g.head0 * 128, (g.head0 + g.n_heads) * 128
        ck = t["cache_k"][:, c0:c1].contiguous()
        cv = t["cache_v"][:, c0:c1].contiguous()
        ws = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
        mask = t["mask"].clone()
        fxr.frame_forward_heads(cfg, g, t["q"], t["k"], t["v"], mask, None, t["pos"],
                                t["norm_q"], t["norm_k"], ck, cv, ws)
        fxr.head_group_wait(g)
        torch.cuda.synchronize()
        err = fxr.check_device_error()
        got = out.clone()
        dist.barrier()                     # nobody frees or rewrites while a peer still stores
        fxr.frame_forward(cfg, t["q"], t["k"], t["v"], t["mask"], None, t["pos"], t["norm_q"],
                          t["norm_k"], t["cache_k"], t["cache_v"], t["out"], ws)
        torch.cuda.synchronize()
        ok = (err == 0 and _out_close(got, t["out"], "bf16") and
              torch.equal(ck, t["cache_k"][:, c0:c1]) and torch.equal(cv, t["cache_v"][:, c0:c1]))
        outs = [None] * world
        dist.all_gather_object(outs, got.cpu())
        ok = ok and all(torch.equal(o, outs[0]) for o in outs)   # both ranks hold the same frame
        # the same frame with the O exchange as one NCCL all-gather
        uid = [fxr.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = fxr.nccl_comm_init(world, rank, uid[0])
        try:
            t2 = _frame_tensors(w, fr)
            ck2 = t2["cache_k"][:, c0:c1].contiguous()
            cv2 = t2["cache_v"][:, c0:c1].contiguous()
            M = int((fr["mask"] != 0).sum())
            wsn = torch.empty(fxr.heads_nccl_workspace_size(cfg, g, M), dtype=torch.uint8,
                              device="cuda")
            fxr.frame_forward_heads_nccl(cfg, g, comm, M, t2["q"], t2["k"], t2["v"], t2["mask"],
                                         None, t2["pos"], t2["norm_q"], t2["norm_k"], ck2, cv2,
                                         t2["out"], wsn)
            torch.cuda.synchronize()
            ok = ok and fxr.check_device_error() == 0 and torch.equal(t2["out"], got) and \
                torch.equal(ck2, ck)
        finally:
            torch.cuda.synchronize()
            fxr.nccl_comm_destroy(comm)
        oks = [None] * world
        dist.all_gather_object(oks, bool(ok))
        if rank == 0:
            np.save(result_path, np.array(oks))
        dist.barrier()
    finally:
        for p in mapped:
            fxr.ipc_close(p)
        if bufs is not None:
            torch.cuda.synchronize()
            bufs.free()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_heads_on_two_gpus_over_peer_memory(cuda, tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = str(tmp_path / "ok.npy")
    mp.start_processes(_two_gpu_worker, args=(2, _free_port(), out), nprocs=2,
                       start_method="spawn")
    assert np.load(out).all()
