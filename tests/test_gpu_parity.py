"""GPU parity tests: every step of the CUDA path, called through the C ABI, against the CPU oracle
on the same seeded inputs.

Bars (stated per test): compaction, gather/scatter/copies and cache bookkeeping bit-exact;
attention outputs within max-abs 2e-3 and mean-abs 2e-4, for fp16 and bf16 storage alike, both
against the oracle evaluated on the kernel's operands (Q'/K' rounded to the storage type where the
CUDA path stores them) and against the unrounded fp32 oracle. Normed + roped Q'/K' in fp16 within
2e-3 / 2e-4 of the fp32 oracle. Stored bf16 Q'/K' cannot meet an absolute 2e-3 bar: bf16 keeps 8
significant bits, so storing a value of magnitude 2-4 alone moves it by up to 2^-7 = 7.8e-3. They
are held to at most 1 bf16 ulp from the oracle rounded to bf16, with mean-abs <= 2e-4. Every
tolerance check records its measured max-abs / mean-abs (printed in pytest's summary).
"""
import os

import numpy as np
import pytest
import torch

import fxr
import oracle as O
import parity_stats
import workloads as W

pytestmark = pytest.mark.gpu

TDT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
TOL_F16 = dict(max_abs=2e-3, mean_abs=2e-4)
TOL_O = dict(max_abs=2e-3, mean_abs=2e-4)      # attention outputs, fp16 and bf16


def dev(a, dtype="f32"):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(TDT[dtype]) if dtype != "i32" else \
        torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to("cuda")


def host(t):
    return t.float().cpu().numpy() if t.is_floating_point() else t.cpu().numpy()


def assert_close(got, ref, max_abs, mean_abs, what=""):
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    mx, mn = parity_stats.record(what, got, ref, max_abs, mean_abs)
    assert mx <= max_abs, f"{what}: max-abs {mx:.3e} > {max_abs}"
    assert mn <= mean_abs, f"{what}: mean-abs {mn:.3e} > {mean_abs}"


def assert_bf16_close(got, ref_fp32, what=""):
    """|got - bf16(ref)| <= max(1 bf16 ulp of bf16(ref), 1e-5) element-wise, mean-abs <= 2e-4.
    The 1e-5 floor covers near-zero RoPE outputs (a*cos - b*sin cancelling), whose absolute error
    is set by the fp32 rotation angle pos*omega (|angle| <= ~130 rad, fp32 rounding ~1e-5 rad)."""
    r = W.round_storage(ref_fp32, "bf16").astype(np.float64)
    g = got.astype(np.float64)
    assert np.isfinite(g).all(), f"{what}: non-finite values"
    mag = np.maximum(np.abs(r), 2.0 ** -126)
    ulp = 2.0 ** (np.floor(np.log2(mag)) - 7)
    err = np.abs(g - r)
    parity_stats.record(what + " vs bf16(oracle)", g, r, float("nan"), 2e-4)
    bad = err > np.maximum(ulp * (1 + 1e-6), 1e-5)
    assert not bad.any(), f"{what}: {bad.sum()} elements > 1 bf16 ulp (worst {err[bad].max():.3e})"
    assert err.mean() <= 2e-4, f"{what}: mean-abs vs bf16(oracle) {err.mean():.3e} > 2e-4"


def check_qk(got, ref, dtype, what):
    if dtype == "bf16":
        assert_bf16_close(got, ref, what)
    else:
        assert_close(got, ref, what=what, **TOL_F16)


def cfg_of(w: W.Workload, n_heads=None) -> fxr.FrameConfig:
    return fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=n_heads or w.n_heads,
                           dtype=w.dtype, rope_axes=w.rope_axes, rope_theta=w.rope_theta)


def small(w: W.Workload, n_heads: int) -> W.Workload:
    return W.Workload(w.name + f"_h{n_heads}", w.grid_h, w.grid_w, w.n_text, n_heads, w.head_dim,
                      w.dtype, w.active, w.pattern, w.rope_axes, w.rope_theta)


def sync_ok():
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0


# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("n", [0, 1, 31, 33, 1536, 4608, 16896, 40000])
def test_mask_compact_bit_exact(cuda, n):
    rng = np.random.default_rng(n + 11)
    mask = rng.choice([0, 1, 2], size=n, p=[0.7, 0.1, 0.2]).astype(np.int32)
    valid = (rng.random(n) < 0.9).astype(np.uint8)
    m_ref, idx_ref = O.mask_compact(mask, valid)
    dm = dev(mask, "i32")
    dv = torch.from_numpy(valid).cuda()
    idx = torch.full((max(n, 1),), -7, dtype=torch.int32, device="cuda")
    cnt = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    fxr.mask_compact(dm, dv, idx, cnt)
    sync_ok()
    M = int(cnt.item())
    assert M == idx_ref.size
    assert np.array_equal(host(dm), m_ref)
    assert np.array_equal(host(idx)[:M], idx_ref)
    # without a validity array: pure compaction, mask untouched
    dm2 = dev(mask, "i32")
    fxr.mask_compact(dm2, None, idx, cnt)
    sync_ok()
    assert np.array_equal(host(dm2), mask)
    assert np.array_equal(host(idx)[: int(cnt.item())], np.nonzero(mask)[0])


def _frame_tensors(w: W.Workload, fr: dict):
    t = {k: dev(fr[k], w.dtype) for k in ("q", "k", "v", "cache_k", "cache_v", "out")}
    t["mask"] = dev(fr["mask"], "i32")
    t["pos"] = dev(fr["pos"], "i32")
    t["norm_q"] = dev(fr["norm_q"])
    t["norm_k"] = dev(fr["norm_k"])
    return t


def _with_exec_only(fr: dict, seed: int, frac: float = 0.05) -> dict:
    """Turns a fraction of the executed image rows into mask 1 (execute, keep cache)."""
    rng = np.random.default_rng(seed)
    m = fr["mask"].copy()
    cand = np.nonzero(m == 2)[0]
    pick = cand[rng.random(cand.size) < frac]
    m[pick] = 1
    fr = dict(fr)
    fr["mask"] = m
    return fr


@pytest.mark.parametrize("wl,heads", [(W.C1, 24), (W.KLEIN, 6), (W.C2, 4)])
def test_gather_norm_rope_parity(cuda, wl, heads):
    w = small(wl, heads)
    fr = _with_exec_only(W.make_frame(w, seed=5), seed=6)
    cfg = cfg_of(w)
    t = _frame_tensors(w, fr)
    N, C = w.n_tokens, heads * 128
    idx = torch.zeros(N, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    qc = torch.zeros(N, C, dtype=TDT[w.dtype], device="cuda")
    save = torch.zeros(N, 2 * C, dtype=TDT[w.dtype], device="cuda")
    fxr.mask_compact(t["mask"], None, idx, cnt)
    fxr.gather_norm_rope(cfg, t["q"], t["k"], t["v"], t["mask"], idx, cnt, t["pos"], t["norm_q"],
                         t["norm_k"], qc, t["cache_k"], t["cache_v"], save)
    sync_ok()
    M = int(cnt.item())
    idx_h = host(idx)[:M]
    mask = fr["mask"]
    assert np.array_equal(idx_h, np.nonzero(mask)[0])
    # oracle per executed row and head
    qn = O.rms_norm(fr["q"][idx_h].reshape(-1, 128), fr["norm_q"]).reshape(M, C)
    kn = O.rms_norm(fr["k"][idx_h].reshape(-1, 128), fr["norm_k"]).reshape(M, C)
    for r, i in enumerate(idx_h):
        for h in range(heads):
            sl = slice(h * 128, (h + 1) * 128)
            qn[r, sl] = O.rope_row(qn[r, sl], fr["pos"][i], w.rope_axes, w.rope_theta)
            kn[r, sl] = O.rope_row(kn[r, sl], fr["pos"][i], w.rope_axes, w.rope_theta)
    check_qk(host(qc)[:M], qn, w.dtype, "Q'")
    ck, cv = host(t["cache_k"]), host(t["cache_v"])
    check_qk(ck[idx_h], kn, w.dtype, "K'")
    assert np.array_equal(cv[idx_h], fr["v"][idx_h])                     # V copy: bit-exact
    skipped = mask == 0
    assert np.array_equal(ck[skipped], fr["cache_k"][skipped])
    assert np.array_equal(cv[skipped], fr["cache_v"][skipped])
    ones = np.nonzero(mask[idx_h] == 1)[0]
    sv = host(save)
    for r in ones:                                                         # saved old rows: bit-exact
        assert np.array_equal(sv[r, :C], fr["cache_k"][idx_h[r]])
        assert np.array_equal(sv[r, C:], fr["cache_v"][idx_h[r]])


@pytest.mark.parametrize("M,N,H,dtype", [(1, 128, 1, "f16"), (77, 300, 2, "f16"), (77, 300, 2, "bf16"),
                                         (256, 1536, 3, "bf16"), (300, 1000, 2, "bf16"),
                                         (640, 4608, 2, "f16"), (640, 4608, 2, "bf16")])
def test_attention_parity(cuda, M, N, H, dtype):
    rng = np.random.default_rng(M * 7 + N)
    C = H * 128
    f = lambda *s: W.round_storage(rng.normal(size=s).astype(np.float32), dtype)
    qc, k, v = f(N, C), f(N, C), f(N, C)
    idx = np.sort(rng.choice(N, size=M, replace=False)).astype(np.int32)
    out0 = f(N, C)
    cfg = fxr.FrameConfig(n_tokens=N, n_text=0, n_heads=H, dtype=dtype)
    d_out = dev(out0, dtype)
    cnt = torch.tensor([M], dtype=torch.int32, device="cuda")
    fxr.attention_active(cfg, dev(qc, dtype), cnt, dev(k, dtype), dev(v, dtype), dev(idx, "i32"), d_out)
    sync_ok()
    ref = O.attention(qc[:M], k, v, H, 128)
    got = host(d_out)
    assert_close(got[idx], ref, what="O", **TOL_O)
    untouched = np.ones(N, dtype=bool)
    untouched[idx] = False
    assert np.array_equal(got[untouched], out0[untouched])


@pytest.mark.parametrize("jump,dtype", [(10.0, "bf16"), (10.0, "f16"), (40.0, "bf16"), (150.0, "bf16")])
def test_attention_row_maximum_jumps(cuda, jump, dtype):
    """Rows whose score maximum jumps by `jump` (log2 units) at a key of the third 128-key step, so
    that the lazy rescale of the softmax (only when a row maximum grows by more than 2^8) runs, from
    a small jump up to one that would overflow fp32 without it, against the oracle. One key then
    carries most of each row's weight, and the rounding of its probability to the 16-bit PV operand
    (up to 2^-9 relative in bf16) goes straight into the output, so V is scaled to keep that inside
    the bar."""
    rng = np.random.default_rng(int(jump) + (1 if dtype == "f16" else 0))
    H, N, M = 1, 640, 96
    C = 128 * H
    scale_log2 = 1.4426950408889634 / np.sqrt(128.0)
    qdir = rng.normal(size=C).astype(np.float32)
    qdir /= np.linalg.norm(qdir)
    a = np.sqrt(jump / scale_log2)
    qc = (qdir[None, :] * a + rng.normal(scale=0.05, size=(N, C))).astype(np.float32)
    k = rng.normal(scale=0.3, size=(N, C)).astype(np.float32)
    k[300] = qdir * a                                   # the key that every row's maximum jumps to
    k[:128] -= (qc[:1] * 0.5 / a)                       # the first step's scores a little lower still
    v = rng.normal(scale=0.25, size=(N, C)).astype(np.float32)
    qc, k, v = (W.round_storage(x, dtype) for x in (qc, k, v))
    idx = np.sort(rng.choice(N, size=M, replace=False)).astype(np.int32)
    cfg = fxr.FrameConfig(n_tokens=N, n_text=0, n_heads=H, dtype=dtype)
    d_out = dev(np.zeros((N, C), np.float32), dtype)
    cnt = torch.tensor([M], dtype=torch.int32, device="cuda")
    fxr.attention_active(cfg, dev(qc, dtype), cnt, dev(k, dtype), dev(v, dtype), dev(idx, "i32"), d_out)
    sync_ok()
    ref = O.attention(qc[:M], k, v, H, 128)
    got = host(d_out)[idx]
    assert_close(got, ref, what=f"O jump 2^{jump:g}", **TOL_O)


def _run_frame(w: W.Workload, fr: dict, valid=None, cfg=None):
    cfg = cfg or cfg_of(w)
    t = _frame_tensors(w, fr)
    ws = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
    dvalid = None if valid is None else torch.from_numpy(valid).cuda()
    fxr.frame_forward(cfg, t["q"], t["k"], t["v"], t["mask"], dvalid, t["pos"], t["norm_q"],
                      t["norm_k"], t["cache_k"], t["cache_v"], t["out"], ws)
    sync_ok()
    return {k: host(v) for k, v in t.items()}


@pytest.mark.parametrize("split_gather", [False, True])
@pytest.mark.parametrize("active", [0.25, 0.27])
def test_frame_steps_equal_frame_forward(cuda, split_gather, active):
    """fxr_frame_step run step by step (compacting gather, attention, restore; or compaction and
    gather as two steps) on the frame's workspace gives fxr_frame_forward's outputs, cache rows and
    mask bit for bit (at 27 % active the attention runs its stream-K schedule), with a frame of
    execute-only rows so that the restore has work."""
    w = W.with_active(W.C2, active)
    fr = _with_exec_only(W.make_frame(w, seed=61), seed=62)
    cfg = cfg_of(w)
    a = _run_frame(w, fr)
    t = _frame_tensors(w, fr)
    ws = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
    steps = ([fxr.STEP_COMPACT, fxr.STEP_GATHER] if split_gather else [fxr.STEP_GATHER_COMPACT]) + \
        [fxr.STEP_ATTENTION, fxr.STEP_RESTORE]
    for st in steps:
        fxr.frame_step(st, cfg, t["q"], t["k"], t["v"], t["mask"], None, t["pos"], t["norm_q"], t["norm_k"],
                       t["cache_k"], t["cache_v"], t["out"], ws)
    sync_ok()
    for k in ("out", "cache_k", "cache_v", "mask"):
        assert np.array_equal(host(t[k]), a[k]), k


@pytest.mark.parametrize("wl,heads", [(W.C1, 24), (W.KLEIN, 24), (W.C3, 4), (W.C2, 6)])
def test_frame_forward_parity(cuda, wl, heads):
    w = small(wl, heads)
    fr = _with_exec_only(W.make_frame(w, seed=21), seed=22)
    rng = np.random.default_rng(23)
    valid = (rng.random(w.n_tokens) < 0.97).astype(np.uint8)
    g = _run_frame(w, fr, valid)
    r = O.frame_forward(fr["q"], fr["k"], fr["v"], fr["mask"], valid, fr["pos"], fr["norm_q"],
                        fr["norm_k"], fr["cache_k"], fr["cache_v"], fr["out"], heads, 128,
                        w.rope_axes, w.rope_theta)
    assert np.array_equal(g["mask"], r["mask"])                            # preprocess: bit-exact
    ex = r["idx"]
    skipped = r["mask"] == 0
    assert np.array_equal(g["out"][skipped], fr["out"][skipped])           # untouched: bit-exact
    assert np.array_equal(g["cache_k"][skipped], fr["cache_k"][skipped])
    assert np.array_equal(g["cache_v"][skipped], fr["cache_v"][skipped])
    ones = r["mask"] == 1
    assert np.array_equal(g["cache_k"][ones], fr["cache_k"][ones])         # restored: bit-exact
    assert np.array_equal(g["cache_v"][ones], fr["cache_v"][ones])
    twos = r["mask"] == 2
    assert np.array_equal(g["cache_v"][twos], fr["v"][twos])
    check_qk(g["cache_k"][twos], r["cache_k"][twos], w.dtype, "K' cache")
    assert_close(g["out"][ex], r["out"][ex], what="O vs fp32 oracle", **TOL_O)
    rows, ref = _oracle_rows(w, fr, valid, w.dtype)
    assert np.array_equal(rows, ex)
    assert_close(g["out"][ex], ref, what="O vs oracle on stored operands", **TOL_O)


@pytest.mark.parametrize("active,heads", [(0.5, 4), (0.27, 24)])
def test_frame_restores_many_execute_only_rows(cuda, active, heads):
    """Most executed rows with mask 1 (execute, keep the cache): their cache rows must come back bit
    for bit after the frame, which the attention does in its tail, eight warps per head sharing the
    listed rows (here hundreds per warp). At 27 % active with 24 heads the attention runs its
    stream-K schedule, so the restore follows cut units too. Outputs (sampled rows) against the
    oracle on the stored operands."""
    w = small(W.with_active(W.C2, active), heads)
    fr = _with_exec_only(W.make_frame(w, seed=71), seed=72, frac=0.9)
    g = _run_frame(w, fr)
    m = fr["mask"]
    ones, twos = m == 1, m == 2
    assert ones.sum() > 1000
    assert np.array_equal(g["cache_k"][ones], fr["cache_k"][ones])
    assert np.array_equal(g["cache_v"][ones], fr["cache_v"][ones])
    assert np.array_equal(g["cache_v"][twos], fr["v"][twos])
    assert np.array_equal(g["cache_k"][m == 0], fr["cache_k"][m == 0])
    rows, ref = _oracle_rows(w, fr, None, w.dtype, n_sample=128, seed=73)
    assert_close(g["out"][rows], ref, what=f"O, {int(ones.sum())} execute-only rows", **TOL_O)


def _oracle_rows(w: W.Workload, fr: dict, valid, operand_dtype: str, n_sample=None, seed=0):
    """Oracle attention outputs of the executed rows (or a seeded sample of n_sample of them) with
    every operand as the CUDA path stores it: Q' and K' rounded to `operand_dtype` after RMSNorm +
    RoPE, K/V = cache rows with the executed rows replaced (mask-1 rows included: they are
    attention operands before the restore). Returns (token rows, outputs)."""
    op = O.frame_operands(fr["q"], fr["k"], fr["v"], fr["mask"], valid, fr["pos"], fr["norm_q"],
                          fr["norm_k"], fr["cache_k"], fr["cache_v"], w.n_heads, 128, w.rope_axes,
                          w.rope_theta, operand_dtype)
    sel = np.arange(op["idx"].size)
    if n_sample is not None and n_sample < sel.size:
        sel = np.sort(np.random.default_rng(seed).choice(sel.size, size=n_sample, replace=False))
    ref = O.attention(op["qc"][sel], op["keys"], op["values"], w.n_heads, 128)
    return op["idx"][sel], ref


def _cuts_units(M: int, n_heads: int, n_tokens: int, grid: int = 148, slots: int = 4 * 148) -> bool:
    """Whether the attention of a frame cuts work units between CTAs, from the kernels' own cost
    models restated on the host (persistent grid of one CTA per SM, the split slots that
    fxr_workspace_size provides):
      two-tile kernel (fxr_attention2.cuh, choose_schedule): units of 256 query rows x all keys in
        128-key steps; stream-K (per = ceil(units x steps / grid) iterations per CTA) when
        per + 2 x items + 2 x 4.5 < ceil(units / grid) x (steps + 2), items = ceil(per / steps) + 1,
        and the workspace holds 4 slots per CTA;
      one-tile kernel (fxr_attention.cuh, choose_splits; FXR_ATTENTION_TILES=1, at most 8 heads):
        units of 128 rows, 256-key steps, 2 to 4 equal parts when
        ceil(units x parts / grid) x (steps / parts + 6) < ceil(units / grid) x (steps + 2)."""
    if os.environ.get("FXR_ATTENTION_TILES", "") == "1":
        if n_heads > 8:
            return False
        units, steps = -(-M // 128) * n_heads, -(-n_tokens // 256)
        whole = -(-units // grid) * (steps + 2.0)
        return any(sp <= steps and units * sp <= slots and -(-(units * sp) // grid) * (steps / sp + 6.0) < whole
                   for sp in range(2, 5))
    if slots < 4 * grid:
        return False
    units, steps = -(-M // 256) * n_heads, -(-n_tokens // 128)
    whole = -(-units // grid) * (steps + 2.0)
    per = -(-(units * steps) // grid)
    items = -(-per // steps) + 1
    return per + 2.0 * items + 9.0 < whole


def test_frame_forward_deterministic_and_noop(cuda):
    w = small(W.C2, 4)
    fr = W.make_frame(w, seed=31)
    a = _run_frame(w, fr)
    b = _run_frame(w, fr)
    for k in ("out", "cache_k", "cache_v", "mask"):
        assert np.array_equal(a[k], b[k]), k
    # nothing executed (all valid, mask 0): the frame is a no-op
    fr0 = dict(fr)
    fr0["mask"] = np.zeros(w.n_tokens, dtype=np.int32)
    c = _run_frame(w, fr0, valid=np.ones(w.n_tokens, dtype=np.uint8))
    assert np.array_equal(c["out"], fr["out"])
    assert np.array_equal(c["cache_k"], fr["cache_k"])


def test_full_size_c2_properties(cuda):
    """Full-size frame (1024^2, 25 %, 24 heads, bf16): untouched rows and cache bookkeeping for
    every row, and 256 sampled executed rows against the oracle, whose keys are its own normed +
    roped K' of every executed token (not the GPU's cache)."""
    w = W.C2
    fr = W.make_frame(w, seed=41)
    g = _run_frame(w, fr)
    mask = fr["mask"]
    skipped = mask == 0
    assert np.array_equal(g["out"][skipped], fr["out"][skipped])
    assert np.array_equal(g["cache_k"][skipped], fr["cache_k"][skipped])
    assert np.array_equal(g["cache_v"][mask == 2], fr["v"][mask == 2])
    rows, ref = _oracle_rows(w, fr, None, "bf16", n_sample=256, seed=42)
    assert_close(g["out"][rows], ref, what="O (256 rows) vs oracle on stored operands", **TOL_O)
    rows32, ref32 = _oracle_rows(w, fr, None, "f32", n_sample=256, seed=42)
    assert np.array_equal(rows, rows32)
    assert_close(g["out"][rows], ref32, what="O (256 rows) vs fp32 oracle", **TOL_O)


@pytest.mark.parametrize("wl,heads,active,n_sample,cut", [(W.C5, 3, None, 128, True), (W.C2, 2, 1.0, 256, True),
                                                          (W.C5, 24, None, 96, False), (W.C2, 24, 0.27, 128, True),
                                                          (W.C2, 24, 0.10, 128, True), (W.C2, 24, 1.0, 64, False)])
def test_high_resolution_and_split_attention_vs_oracle(cuda, wl, heads, active, n_sample, cut):
    """Frames whose attention cuts work units between CTAs (a GPU's 3 heads of an 8-way split
    2048^2 frame; 2 heads of a fully active 1024^2 frame; 1024^2 frames with 24 heads whose units
    fill one wave and a few SMs of a second, or fewer than the SMs) and frames that run whole units
    (the full 2048^2 frame, N = 16896, in two rounds; a fully active 1024^2 frame), sampled executed
    rows against the oracle on the stored operands and against the fp32 oracle.
    The cut frames also equal, within the bar, the same frame run with a workspace that leaves no
    split slots (whole units)."""
    w = small(wl if active is None else W.with_active(wl, active), heads)
    fr = W.make_frame(w, seed=57)
    M = int((fr["mask"] != 0).sum())
    split = _cuts_units(M, heads, w.n_tokens)
    if os.environ.get("FXR_ATTENTION_TILES", "") == "1":
        cut = cut and heads <= 8          # the one-tile kernel splits only launches of few heads
    assert split == cut, (M, split)
    g = _run_frame(w, fr)
    mask = fr["mask"]
    assert np.array_equal(g["out"][mask == 0], fr["out"][mask == 0])
    assert np.array_equal(g["cache_v"][mask == 2], fr["v"][mask == 2])
    rows, ref = _oracle_rows(w, fr, None, w.dtype, n_sample=n_sample, seed=58)
    assert_close(g["out"][rows], ref, what=f"O cut={split} vs oracle on stored operands", **TOL_O)
    _, ref32 = _oracle_rows(w, fr, None, "f32", n_sample=n_sample, seed=58)
    assert_close(g["out"][rows], ref32, what=f"O cut={split} vs fp32 oracle", **TOL_O)
    if split:
        cfg = cfg_of(w)
        t = _frame_tensors(w, fr)
        ws = torch.empty(fxr.workspace_min_size(cfg), dtype=torch.uint8, device="cuda")
        fxr.frame_forward(cfg, t["q"], t["k"], t["v"], t["mask"], None, t["pos"], t["norm_q"],
                          t["norm_k"], t["cache_k"], t["cache_v"], t["out"], ws)
        sync_ok()
        u = host(t["out"])
        assert not np.array_equal(u[rows], g["out"][rows])        # the cut schedule did run
        assert_close(g["out"][rows], u[rows], what="O cut vs whole units", **TOL_O)


def test_frame_past_the_gather_list_capacity_vs_oracle(cuda):
    """A frame of 160 512 tokens (a 400 x 400 grid and 512 text tokens), one head, 2 % of the image
    active: more tokens per CTA than the gather's shared-memory row list holds, so the frame runs
    the compaction kernel before a gather that reads the index list; its 15 units of 1254 key steps
    run stream-K with every unit cut into about ten parts that one CTA combines. Sampled executed
    rows against the oracle, the other rows and the cache bit-exact."""
    w = W.Workload("grid400_h1", 400, 400, 512, n_heads=1, dtype="bf16", active=0.02)
    n_sm = torch.cuda.get_device_properties(0).multi_processor_count
    assert -(-w.n_tokens // n_sm) > 1024          # past the gather's per-CTA list (kBulkListCap)
    fr = W.make_frame(w, seed=61)
    M = int((fr["mask"] != 0).sum())
    assert _cuts_units(M, 1, w.n_tokens, grid=n_sm, slots=4 * n_sm), M
    g = _run_frame(w, fr)
    mask = fr["mask"]
    assert np.array_equal(g["out"][mask == 0], fr["out"][mask == 0])
    assert np.array_equal(g["cache_k"][mask == 0], fr["cache_k"][mask == 0])
    assert np.array_equal(g["cache_v"][mask == 2], fr["v"][mask == 2])
    rows, ref = _oracle_rows(w, fr, None, "bf16", n_sample=64, seed=62)
    assert_close(g["out"][rows], ref, what="O 160k tokens vs oracle on stored operands", **TOL_O)
    _, ref32 = _oracle_rows(w, fr, None, "f32", n_sample=64, seed=62)
    assert_close(g["out"][rows], ref32, what="O 160k tokens vs fp32 oracle", **TOL_O)


# ---------------------------------------------------------------------------------------------
# reference known-answer tests, run through the GPU path
# ---------------------------------------------------------------------------------------------
def test_reference_gather_scatter_known_answers(cuda):
    import json, os
    kat = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")))
    g = kat["gather"]
    src = dev(np.array(g["src"], dtype=np.float32).reshape(-1, g["dim"]))
    dst = torch.zeros(len(g["indices"]), g["dim"], device="cuda")
    fxr.gather_rows(src, dev(np.array(g["indices"]), "i32"), dst, host_count=len(g["indices"]))
    sync_ok()
    assert host(dst).reshape(-1).tolist() == g["expected"]
    s = kat["scatter"]
    dst = torch.full((s["seq_len"], s["dim"]), s["dst_init"], device="cuda")
    src = dev(np.array(s["src"], dtype=np.float32).reshape(-1, s["dim"]))
    fxr.scatter_rows(src, dev(np.array(s["indices"]), "i32"), dst, host_count=len(s["indices"]))
    sync_ok()
    assert host(dst).reshape(-1).tolist() == s["expected"]


def test_reference_spatial_cache_known_answers(cuda):
    import json, os
    kat = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")))
    c = kat["cache"]
    n = c["img_len"] + c["txt_len"]
    valid = torch.zeros(n, dtype=torch.uint8, device="cuda")
    mask = dev(np.array(c["mask0"]), "i32")
    fxr.preprocess_mask(mask, valid)
    sync_ok()
    assert host(mask).tolist() == c["mask0_expected"]
    pred = dev(np.array(c["pred1"], dtype=np.float32).reshape(c["img_len"], c["out_ch"]))
    cache = torch.zeros_like(pred)
    fxr.output_cache_sync(pred, cache, mask, valid, c["txt_len"])
    sync_ok()
    assert host(pred).reshape(-1).tolist() == c["pred1_expected"]
    mask2 = dev(np.array(c["mask2"]), "i32")
    pred2 = dev(np.array(c["pred2"], dtype=np.float32).reshape(c["img_len"], c["out_ch"]))
    fxr.output_cache_sync(pred2, cache, mask2, valid, c["txt_len"])
    sync_ok()
    flat = host(pred2).reshape(-1)
    for k, v in c["pred2_checks"].items():
        assert flat[int(k)] == v
    m = kat["cache_mixed"]
    t_, i_ = m["txt_len"], m["img_len"]
    valid = torch.zeros(t_ + i_, dtype=torch.uint8, device="cuda")
    mk = torch.zeros(t_ + i_, dtype=torch.int32, device="cuda")
    fxr.preprocess_mask(mk, valid)
    sync_ok()
    assert host(mk).tolist() == m["after_reset_expected"]
    pred = torch.ones(i_, m["out_ch"], device="cuda")
    fxr.output_cache_sync(pred, torch.zeros_like(pred), dev(np.array(m["populate_mask"]), "i32"), valid, t_)
    mk = torch.zeros(t_ + i_, dtype=torch.int32, device="cuda")
    idx = torch.zeros(t_ + i_, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    fxr.mask_compact(mk, valid, idx, cnt)
    sync_ok()
    assert host(mk).tolist() == m["final_expected"]


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_kv_sync_bit_exact(cuda, dtype):
    rng = np.random.default_rng(9)
    n, e = 257, 3 * 128 + (0 if dtype != "f32" else 1)
    arrs = [W.round_storage(rng.normal(size=(n, e)).astype(np.float32), dtype) for _ in range(4)]
    mask = rng.choice([0, 1, 2], size=n).astype(np.int32)
    ref = O.kv_sync(*arrs, mask)
    d = [dev(a, dtype) for a in arrs]
    fxr.kv_sync(*d, dev(mask, "i32"))
    sync_ok()
    for got, exp in zip(d, ref):
        assert np.array_equal(host(got), exp)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_output_cache_sync_bit_exact(cuda, dtype):
    rng = np.random.default_rng(10)
    T, I, ch = 5, 300, 3072
    pred = W.round_storage(rng.normal(size=(I, ch)).astype(np.float32), dtype)
    cache = W.round_storage(rng.normal(size=(I, ch)).astype(np.float32), dtype)
    mask = rng.choice([0, 1, 2], size=T + I).astype(np.int32)
    valid = (rng.random(T + I) < 0.5).astype(np.uint8)
    rp, rc, rv = O.output_cache_sync(pred, cache, mask, valid, T)
    dp, dc, dv = dev(pred, dtype), dev(cache, dtype), torch.from_numpy(valid).cuda()
    fxr.output_cache_sync(dp, dc, dev(mask, "i32"), dv, T)
    sync_ok()
    assert np.array_equal(host(dp), rp) and np.array_equal(host(dc), rc)
    assert np.array_equal(host(dv), rv)


@pytest.mark.parametrize("dtype,dim", [("f32", 3072), ("f32", 100), ("f16", 128), ("bf16", 128)])
def test_rms_norm_standalone(cuda, dtype, dim):
    rng = np.random.default_rng(dim)
    x = W.round_storage(rng.normal(size=(37, dim)).astype(np.float32), dtype)
    w = rng.normal(1, 0.1, size=dim).astype(np.float32)
    ref = O.rms_norm(x, w, 1e-6)
    dx = dev(x, dtype)
    dy = torch.empty_like(dx)
    fxr.rms_norm(dx, dy, dev(w), 1e-6)
    sync_ok()
    if dtype == "f32":
        assert_close(host(dy), ref, what="rmsnorm", max_abs=2e-5, mean_abs=2e-6)
    else:
        check_qk(host(dy), ref, dtype, "rmsnorm")


@pytest.mark.parametrize("B,H,S,L,D", [(1, 2, 37, 300, 128), (2, 3, 64, 64, 64), (1, 1, 5, 1, 32)])
def test_attention_f32_bhsd_vs_torch(cuda, B, H, S, L, D):
    """The fp32 SIMT attention behind the reference-signature attention_fwd: joint softmax over all
    kv_len keys, checked against torch's fp32 scaled-dot-product attention."""
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + S)
    q = torch.randn(B, H, S, D, device="cuda", generator=g)
    k = torch.randn(B, H, L, D, device="cuda", generator=g)
    v = torch.randn(B, H, L, D, device="cuda", generator=g)
    out = torch.empty_like(q)
    fxr.attention_f32_bhsd(q, k, v, out)
    sync_ok()
    ref = torch.nn.functional.scaled_dot_product_attention(q.double(), k.double(), v.double())
    assert_close(host(out), ref.float().cpu().numpy(), what="attention f32", max_abs=2e-5,
                 mean_abs=2e-6)


def test_mark_updated_bit_exact(cuda):
    rng = np.random.default_rng(77)
    T, N = 17, 1000
    mask = rng.choice([0, 1, 2], size=N).astype(np.int32)
    valid = (rng.random(N) < 0.3).astype(np.uint8)
    dv = torch.from_numpy(valid).cuda()
    fxr.mark_updated(dev(mask, "i32"), dv, T)
    sync_ok()
    exp = valid.copy()
    exp[T:][mask[T:] == 2] = 1
    assert np.array_equal(host(dv), exp)


@pytest.mark.parametrize("fill", [0x00, 0x7F, 0xFF])
def test_frame_output_independent_of_stale_workspace(cuda, fill):
    """The padding rows of the last query tile read stale compact-Q rows of the workspace; they must
    not change a single bit of the stored rows (0x7F7F.. = large finite bf16, 0xFFFF.. = NaN)."""
    w = small(W.C2, 6)
    fr = W.make_frame(w, seed=91)
    cfg = cfg_of(w)
    outs = []
    for f in (0x00, fill):
        t = _frame_tensors(w, fr)
        ws = torch.full((fxr.workspace_size(cfg),), f, dtype=torch.uint8, device="cuda")
        fxr.frame_forward(cfg, t["q"], t["k"], t["v"], t["mask"], None, t["pos"], t["norm_q"],
                          t["norm_k"], t["cache_k"], t["cache_v"], t["out"], ws)
        sync_ok()
        outs.append(t)
    for k in ("out", "cache_k", "cache_v"):
        assert torch.equal(outs[0][k], outs[1][k]), k


@pytest.mark.parametrize("n_streams,wl,heads", [(3, W.C4, 24), (9, W.C1, 12), (1, W.C2, 12)])
def test_frame_forward_batch_matches_per_stream_frames(cuda, n_streams, wl, heads):
    """Streams in one set of launches equal per-stream frames bit for bit (each (query tile, head)
    unit is computed the same way whichever launch holds it); 9 streams run as groups of 8 + 1.
    The per-stream frames get a workspace without split slots, so that both paths run whole units
    (a lone small frame would otherwise take the stream-K schedule)."""
    w = small(wl, heads)
    cfg = cfg_of(w)
    pos = dev(W.positions(w), "i32")
    frs = [_with_exec_only(W.make_frame(w, seed=300 + b), seed=400 + b) for b in range(n_streams)]
    nq, nk = dev(frs[0]["norm_q"]), dev(frs[0]["norm_k"])
    rng = np.random.default_rng(5)
    valids = [torch.from_numpy((rng.random(w.n_tokens) < 0.9).astype(np.uint8)).cuda()
              for _ in range(n_streams)]
    a = [_frame_tensors(w, fr) for fr in frs]
    b = [_frame_tensors(w, fr) for fr in frs]
    ws = torch.empty(fxr.batch_workspace_size(cfg, n_streams), dtype=torch.uint8, device="cuda")
    fxr.frame_forward_batch(cfg, [dict(t, valid=valids[i]) for i, t in enumerate(a)], pos, nq, nk, ws)
    wsf = torch.empty(fxr.workspace_min_size(cfg), dtype=torch.uint8, device="cuda")
    for i, t in enumerate(b):
        fxr.frame_forward(cfg, t["q"], t["k"], t["v"], t["mask"], valids[i], pos, nq, nk,
                          t["cache_k"], t["cache_v"], t["out"], wsf)
    sync_ok()
    for i in range(n_streams):
        for k in ("out", "cache_k", "cache_v", "mask"):
            assert torch.equal(a[i][k], b[i][k]), (i, k)
