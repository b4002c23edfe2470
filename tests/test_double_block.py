"""The double-stream block on the executed rows (fxr_double_block_forward) against a CPU restatement
of the reference block (flux2_double_block_plugin.cpp:330-460: LayerNorm + modulation, Q/K/V, QK
RMSNorm, attention, out-projection, GELU MLP, residual) with joint text + image attention over the
spatial K/V cache, fp32 arithmetic rounded to bf16 where the kernels store; and the single-stream
block (fxr_single_block_forward: one fused to_qkv_mlp_proj, one to_out over [attention | MLP],
tools/export_block_weights.py:79-113) against the same kind of restatement. Every step of the
restatement is the oracle's (oracle/fxr_oracle.c): LayerNorm + modulation, linear projections, tanh
GELU, gated residual, QK-RMSNorm, RoPE and attention."""
import ctypes

import numpy as np
import pytest

import fxr
import workloads as W


def test_double_block_argument_checks():
    L = fxr.load()
    cfg = fxr.FrameConfig(n_tokens=1280, n_text=256, n_heads=6)
    d = cfg.desc()
    blk = fxr.DoubleBlock()
    blk.mlp_hidden, blk.ln_eps = 2304, 1e-6
    args = lambda b, ws_bytes=1 << 40: (ctypes.byref(d), b, *([None] * 8), ws_bytes, None)
    assert L.fxr_double_block_forward(*args(None)) == fxr.FXR_ERR_INVALID            # null block
    assert L.fxr_double_block_forward(*args(ctypes.byref(blk))) == fxr.FXR_ERR_INVALID  # null weights
    bad = fxr.DoubleBlock()
    bad.mlp_hidden, bad.ln_eps = 2300, 1e-6
    assert L.fxr_double_block_forward(*args(ctypes.byref(bad))) == fxr.FXR_ERR_UNSUPPORTED
    d5 = fxr.FrameConfig(n_tokens=1280, n_text=256, n_heads=5).desc()               # C = 640
    assert L.fxr_double_block_forward(ctypes.byref(d5), ctypes.byref(blk), *([None] * 8), 1 << 40,
                                      None) == fxr.FXR_ERR_UNSUPPORTED
    # workspace: the frame's, Q/K/V, LayerNorm and attention rows, MLP rows, GEMM scratch
    ws = fxr.double_block_workspace_size(cfg, 2304)
    rows = 1280 * 768 * 2
    assert ws >= fxr.workspace_size(cfg) + 5 * rows + 1280 * 2304 * 2 + fxr.rows_gemm_scratch_size()
    assert fxr.double_block_workspace_size(cfg, 4608) > ws


def _reference_block(w, fr, x_in, valid, streams, H):
    """fp32 restatement, rounded to the storage type where the kernels store; returns the executed
    token list, their block outputs, the caches, the preprocessed mask and the validity flags."""
    import oracle
    bf = lambda a: W.round_storage(a, w.dtype)
    N, T, C, D = w.n_tokens, w.n_text, w.n_heads * w.head_dim, w.head_dim
    mask = fr["mask"].copy()
    mask[valid == 0] = 2
    mask[:T][mask[:T] == 0] = 2
    idx = np.nonzero(mask)[0]
    M = idx.size
    xn = np.zeros((M, C), np.float32)
    q = np.zeros((N, C), np.float32); k = np.zeros((N, C), np.float32); v = np.zeros((N, C), np.float32)
    qn = np.zeros((M, C), np.float32)
    ck, cv = fr["cache_k"].copy(), fr["cache_v"].copy()
    k_att, v_att = ck.copy(), cv.copy()
    hmid = np.zeros((M, H), np.float32)
    for name, sel in (("txt", idx < T), ("img", idx >= T)):
        s = streams[name]
        rows = np.nonzero(sel)[0]
        if rows.size == 0:
            continue
        toks = idx[rows]
        xn[rows] = bf(oracle.layer_norm_modulate(x_in[toks], s["scale"], s["shift"]))
        qkv = bf(oracle.linear(xn[rows], s["w_qkv"], s["b_qkv"]))
        q[toks], k[toks], v[toks] = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
        hmid[rows] = bf(oracle.gelu_tanh(oracle.linear(xn[rows], s["w_mlp0"], s["b_mlp0"])))
        rope = lambda x, t: np.concatenate([oracle.rope_row(x[h * D:(h + 1) * D], fr["pos"][t], w.rope_axes,
                                                            w.rope_theta) for h in range(w.n_heads)])
        for r, t in zip(rows, toks):
            qh = oracle.rms_norm(q[t].reshape(-1, D), s["norm_q"]).reshape(-1)
            kh = oracle.rms_norm(k[t].reshape(-1, D), s["norm_k"]).reshape(-1)
            qn[r] = bf(rope(qh, t))
            k_att[t] = bf(rope(kh, t))
            v_att[t] = v[t]
    o = bf(oracle.attention(qn, k_att, v_att, w.n_heads, D))
    x_out = np.zeros((M, C), np.float32)
    for name, sel in (("txt", idx < T), ("img", idx >= T)):
        s = streams[name]
        rows = np.nonzero(sel)[0]
        if rows.size == 0:
            continue
        toks = idx[rows]
        proj = oracle.linear(o[rows], s["w_out"], s["b_out"]) + oracle.linear(hmid[rows], s["w_mlp2"], s["b_mlp2"])
        x_out[rows] = bf(oracle.gated_residual(x_in[toks], proj, s["gate"]))
    upd = mask == 2
    ck[upd], cv[upd] = k_att[upd], v_att[upd]
    valid_out = valid.copy()
    valid_out[T:][mask[T:] == 2] = 1
    return {"idx": idx, "x_out": x_out, "cache_k": ck, "cache_v": cv, "mask": mask, "valid": valid_out}


def _streams(w, H, rng):
    C, D = w.n_heads * w.head_dim, w.head_dim
    g = lambda *shape, sd=1.0: W.round_storage(rng.normal(0, sd, size=shape).astype(np.float32), w.dtype)
    f = lambda *shape, mu=0.0, sd=1.0: rng.normal(mu, sd, size=shape).astype(np.float32)
    out = {}
    for name in ("txt", "img"):
        out[name] = {
            "shift": f(C, sd=0.1), "scale": f(C, sd=0.1), "gate": f(C, mu=1.0, sd=0.2),
            "w_qkv": g(3 * C, C, sd=C ** -0.5), "b_qkv": f(3 * C, sd=0.05),
            "norm_q": f(D, mu=1.0, sd=0.1), "norm_k": f(D, mu=1.0, sd=0.1),
            "w_out": g(C, C, sd=C ** -0.5), "b_out": f(C, sd=0.05),
            "w_mlp0": g(H, C, sd=C ** -0.5), "b_mlp0": f(H, sd=0.05),
            "w_mlp2": g(C, H, sd=H ** -0.5), "b_mlp2": f(C, sd=0.05),
        }
    return out


def _ulp_err(got, ref, dtype="bf16"):
    """|got - ref| in storage steps (bf16 / fp16) of max(|ref|, the RMS of ref): values near zero are
    judged on the scale of the tensor, not on their own tiny step."""
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    mag = np.maximum(np.abs(ref), rms)
    ulp = 2.0 ** (np.floor(np.log2(mag)) - (7 if dtype == "bf16" else 10))
    return np.abs(got - ref) / ulp


@pytest.mark.gpu
@pytest.mark.parametrize("p,seed,dtype", [(0.3, 3, "bf16"), (0.05, 4, "bf16"), (0.3, 5, "f16")])
def test_double_block_matches_reference(cuda, p, seed, dtype):
    import torch
    w = W.Workload("blk_512px_h6", 32, 32, 256, n_heads=6, dtype=dtype)
    td = torch.bfloat16 if dtype == "bf16" else torch.float16
    H = 3 * w.n_heads * w.head_dim
    N, T, C = w.n_tokens, w.n_text, w.n_heads * w.head_dim
    rng = np.random.default_rng(seed)
    fr = W.make_frame(w, seed=seed, p=p)
    fr["mask"][T + 5] = 1                    # executed, cache row kept (restored after)
    fr["mask"][T + 9] = 1
    fr["mask"][3] = 0                        # a skipped text token still executes
    fr["mask"][7] = 1
    valid = (rng.random(N) < 0.9).astype(np.uint8)
    valid[:T] = 1
    x_in = W.round_storage(rng.normal(0, 1, size=(N, C)).astype(np.float32), dtype)
    x_prev = W.round_storage(rng.normal(0, 1, size=(N, C)).astype(np.float32), dtype)
    streams = _streams(w, H, rng)
    ref = _reference_block(w, fr, x_in, valid, streams, H)

    dev = lambda a, dt=td: torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dt)
    tw = {n: {k: dev(v, td if k.startswith("w_") else torch.float32) for k, v in s.items()}
          for n, s in streams.items()}
    cfg = fxr.FrameConfig(n_tokens=N, n_text=T, n_heads=w.n_heads, dtype=dtype, rope_axes=w.rope_axes,
                          rope_theta=w.rope_theta)
    xi, xo = dev(x_in), dev(x_prev)
    mask = torch.from_numpy(fr["mask"].copy()).cuda()
    vd = torch.from_numpy(valid.copy()).cuda()
    pos = torch.from_numpy(fr["pos"]).cuda()
    ck, cv = dev(fr["cache_k"]), dev(fr["cache_v"])
    ws = torch.empty(fxr.double_block_workspace_size(cfg, H), dtype=torch.uint8, device="cuda")
    fxr.double_block_forward(cfg, tw["txt"], tw["img"], H, xi, xo, mask, vd, pos, ck, cv, ws)
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0

    idx = ref["idx"]
    assert np.array_equal(mask.cpu().numpy(), ref["mask"])
    assert np.array_equal(vd.cpu().numpy(), ref["valid"])
    got = xo.float().cpu().numpy()
    e = _ulp_err(got[idx], ref["x_out"], dtype)
    wr, wc = np.unravel_index(int(np.argmax(e)), e.shape)
    print(f"x_out rows {idx.size}: max {e.max():.1f} steps (got {got[idx][wr, wc]:.5f} ref "
          f"{ref['x_out'][wr, wc]:.5f}), >2 steps {np.mean(e > 2):.2e}, mean {e.mean():.3f}")
    # the GPU's intermediate roundings (LayerNorm rows, Q/K/V, attention, MLP rows) may each land one
    # bf16 step away from the restatement's; measured: the block output within 1 step (mean 0.013)
    assert e.max() <= 2 and e.mean() < 0.05, (e.max(), e.mean())
    skipped = np.setdiff1d(np.arange(N), idx)
    assert np.array_equal(got[skipped], x_prev[skipped])      # the output cache rows are untouched
    for key in ("cache_k", "cache_v"):
        gc = (ck if key == "cache_k" else cv).float().cpu().numpy()
        upd = ref["mask"] == 2
        assert np.array_equal(gc[~upd], fr[key][~upd]), key      # skipped and mask-1 rows restored
        ec = _ulp_err(gc[upd], ref[key][upd], dtype)
        print(f"{key} updated rows: max {ec.max():.1f} steps, >1 step {np.mean(ec > 1):.2e}, mean {ec.mean():.3f}")
        assert ec.max() <= 2 and np.mean(ec > 1) < 1e-4, (key, ec.max(), ec.mean())


def _reference_single_block(w, fr, x_in, valid, wt, H):
    """fp32 restatement of the single-stream block, rounded to the storage type where the kernels
    store."""
    import oracle
    bf = lambda a: W.round_storage(a, w.dtype)
    N, T, C, D = w.n_tokens, w.n_text, w.n_heads * w.head_dim, w.head_dim
    mask = fr["mask"].copy()
    mask[valid == 0] = 2
    mask[:T][mask[:T] == 0] = 2
    idx = np.nonzero(mask)[0]
    xn = bf(oracle.layer_norm_modulate(x_in[idx], wt["scale"], wt["shift"]))
    proj = oracle.linear(xn, wt["w_qkv_mlp"], wt["b_qkv_mlp"])
    q, k, v = bf(proj[:, :C]), bf(proj[:, C:2 * C]), bf(proj[:, 2 * C:3 * C])
    h = bf(oracle.gelu_tanh(proj[:, 3 * C:]))
    rope = lambda x, t: np.concatenate([oracle.rope_row(x[j * D:(j + 1) * D], fr["pos"][t], w.rope_axes,
                                                        w.rope_theta) for j in range(w.n_heads)])
    ck, cv = fr["cache_k"].copy(), fr["cache_v"].copy()
    k_att, v_att = ck.copy(), cv.copy()
    qn = np.zeros_like(q)
    for r, t in enumerate(idx):
        qn[r] = bf(rope(oracle.rms_norm(q[r].reshape(-1, D), wt["norm_q"]).reshape(-1), t))
        k_att[t] = bf(rope(oracle.rms_norm(k[r].reshape(-1, D), wt["norm_k"]).reshape(-1), t))
        v_att[t] = v[r]
    o = bf(oracle.attention(qn, k_att, v_att, w.n_heads, D))
    x_out = bf(oracle.gated_residual(x_in[idx], oracle.linear(np.concatenate([o, h], axis=1), wt["w_out"],
                                                              wt["b_out"]), wt["gate"]))
    upd = mask == 2
    ck[upd], cv[upd] = k_att[upd], v_att[upd]
    return {"idx": idx, "x_out": x_out, "cache_k": ck, "cache_v": cv, "mask": mask}


@pytest.mark.gpu
@pytest.mark.parametrize("p,seed,dtype", [(0.3, 13, "bf16"), (0.02, 14, "bf16"), (0.3, 15, "f16")])
def test_single_block_matches_reference(cuda, p, seed, dtype):
    """fxr_single_block_forward against a CPU restatement built from the oracle's block-row
    functions. Parity of the MLP activation is unpinned: the reference has no single-stream block
    code (only its plan, results.md:95, and its weight export, tools/export_block_weights.py:79-113),
    so the restatement and the kernel both take the double block's tanh GELU
    (flux2_double_block_plugin.cpp:434-448); a model whose single block uses another MLP form
    (for example a gated one) is not covered by this test."""
    import torch
    w = W.Workload("sblk_512px_h6", 32, 32, 256, n_heads=6, dtype=dtype)
    td = torch.bfloat16 if dtype == "bf16" else torch.float16
    H = 3 * w.n_heads * w.head_dim
    N, T, C, D = w.n_tokens, w.n_text, w.n_heads * w.head_dim, w.head_dim
    rng = np.random.default_rng(seed)
    fr = W.make_frame(w, seed=seed, p=p)
    fr["mask"][T + 3] = 1
    valid = (rng.random(N) < 0.9).astype(np.uint8)
    valid[:T] = 1
    x_in = W.round_storage(rng.normal(0, 1, size=(N, C)).astype(np.float32), dtype)
    x_prev = W.round_storage(rng.normal(0, 1, size=(N, C)).astype(np.float32), dtype)
    g = lambda *shape, sd=1.0: W.round_storage(rng.normal(0, sd, size=shape).astype(np.float32), dtype)
    f = lambda *shape, mu=0.0, sd=1.0: rng.normal(mu, sd, size=shape).astype(np.float32)
    wt = {"shift": f(C, sd=0.1), "scale": f(C, sd=0.1), "gate": f(C, mu=1.0, sd=0.2),
          "w_qkv_mlp": g(3 * C + H, C, sd=C ** -0.5), "b_qkv_mlp": f(3 * C + H, sd=0.05),
          "norm_q": f(D, mu=1.0, sd=0.1), "norm_k": f(D, mu=1.0, sd=0.1),
          "w_out": g(C, C + H, sd=(C + H) ** -0.5), "b_out": f(C, sd=0.05)}
    ref = _reference_single_block(w, fr, x_in, valid, wt, H)

    dev = lambda a, dt=td: torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dt)
    tw = {k: dev(v, td if k.startswith("w_") else torch.float32) for k, v in wt.items()}
    cfg = fxr.FrameConfig(n_tokens=N, n_text=T, n_heads=w.n_heads, dtype=dtype, rope_axes=w.rope_axes,
                          rope_theta=w.rope_theta)
    xi, xo = dev(x_in), dev(x_prev)
    mask = torch.from_numpy(fr["mask"].copy()).cuda()
    vd = torch.from_numpy(valid.copy()).cuda()
    pos = torch.from_numpy(fr["pos"]).cuda()
    ck, cv = dev(fr["cache_k"]), dev(fr["cache_v"])
    ws = torch.empty(fxr.single_block_workspace_size(cfg, H), dtype=torch.uint8, device="cuda")
    fxr.single_block_forward(cfg, tw, H, xi, xo, mask, vd, pos, ck, cv, ws)
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0
    idx = ref["idx"]
    assert np.array_equal(mask.cpu().numpy(), ref["mask"])
    got = xo.float().cpu().numpy()
    e = _ulp_err(got[idx], ref["x_out"], dtype)
    print(f"single block x_out rows {idx.size}: max {e.max():.1f} steps, mean {e.mean():.3f}")
    assert e.max() <= 2 and e.mean() < 0.05, (e.max(), e.mean())
    skipped = np.setdiff1d(np.arange(N), idx)
    assert np.array_equal(got[skipped], x_prev[skipped])
    for key in ("cache_k", "cache_v"):
        gc = (ck if key == "cache_k" else cv).float().cpu().numpy()
        upd = ref["mask"] == 2
        assert np.array_equal(gc[~upd], fr[key][~upd]), key
        ec = _ulp_err(gc[upd], ref[key][upd], dtype)
        assert ec.max() <= 2 and np.mean(ec > 1) < 1e-4, (key, ec.max())
