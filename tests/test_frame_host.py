"""fxr_frame_forward_host: a frame whose Q, K, V, mask and output live in page-locked host memory,
moving only the executed rows across PCIe (in place of the reference's whole-tensor
Tensor::upload / Tensor::download, src/utils/tensor.cpp:50-56). It must produce exactly what
fxr_frame_forward produces on device copies of the same buffers — frame after frame, since the K/V
cache carries state — leave every non-executed output row as it was, and reject host memory the
device cannot address."""
import ctypes

import numpy as np
import pytest

import fxr
import workloads as W


def test_host_frame_argument_checks():
    L = fxr.load()
    cfg = fxr.FrameConfig(n_tokens=1280, n_text=256, n_heads=6)
    d = cfg.desc()
    # desc, q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v, out, workspace, bytes, stream
    args = lambda ws=16, ws_bytes=1 << 40, host=16: (ctypes.byref(d), host, host, host, host, None, None,
                                                     None, None, None, None, host, ws, ws_bytes, None)
    assert L.fxr_frame_forward_host(*args(ws=None)) == fxr.FXR_ERR_INVALID          # null workspace
    assert L.fxr_frame_forward_host(*args(ws=8)) == fxr.FXR_ERR_INVALID             # misaligned
    assert L.fxr_frame_forward_host(*args(ws_bytes=1 << 20)) == fxr.FXR_ERR_WORKSPACE
    assert L.fxr_frame_forward_host(*args(host=None)) == fxr.FXR_ERR_INVALID        # null host buffers
    d0 = fxr.FrameConfig(n_tokens=0, n_text=0, n_heads=6).desc()
    assert L.fxr_frame_forward_host(ctypes.byref(d0), *([None] * 11), None, 0, None) == fxr.FXR_OK
    # workspace: the staging rows (mask, Q, K, V, out) in front of the frame's own workspace
    ws = fxr.frame_host_workspace_size(cfg)
    assert ws >= fxr.workspace_size(cfg) + 1280 * 4 + 4 * 1280 * 768 * 2


def _frames(w, seed, n):
    out = []
    for i in range(n):
        fr = W.make_frame(w, seed=seed + i)
        out.append(fr)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,p", [("bf16", 0.25), ("f16", 0.3), ("bf16", 1.0)])
def test_host_frames_match_device_frames(cuda, dtype, p):
    import torch
    td = torch.bfloat16 if dtype == "bf16" else torch.float16
    w = W.Workload("host_24x24", 24, 24, 128, n_heads=4, dtype=dtype, active=p)
    cfg = fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=w.n_heads, dtype=dtype,
                          rope_axes=w.rope_axes, rope_theta=w.rope_theta)
    frames = _frames(w, 21, 3)
    f0 = frames[0]
    dev = lambda a, dt=td: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dt)
    pos = torch.from_numpy(f0["pos"]).cuda()
    nq, nk = torch.from_numpy(f0["norm_q"]).cuda(), torch.from_numpy(f0["norm_k"]).cuda()
    valid = torch.ones(w.n_tokens, dtype=torch.uint8, device="cuda")
    valid[w.n_text + 3] = 0                                   # one image row without a cached entry
    # device path state and host path state start equal
    d_ck, d_cv, d_out = dev(f0["cache_k"]), dev(f0["cache_v"]), dev(f0["out"])
    h_ck, h_cv = d_ck.clone(), d_cv.clone()
    h_out = d_out.cpu().pin_memory()
    ws_d = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
    ws_h = torch.empty(fxr.frame_host_workspace_size(cfg), dtype=torch.uint8, device="cuda")
    for i, fr in enumerate(frames):
        mask = fr["mask"].copy()
        mask[w.n_text + 5] = 1                                # executed, cache row kept
        q, k, v = dev(fr["q"]), dev(fr["k"]), dev(fr["v"])
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hmask = torch.from_numpy(mask).pin_memory()
        before = h_out.clone()
        fxr.frame_forward(cfg, q, k, v, torch.from_numpy(mask).cuda(), valid, pos, nq, nk, d_ck, d_cv,
                          d_out, ws_d)
        fxr.frame_forward_host(cfg, hq, hk, hv, hmask, valid, pos, nq, nk, h_ck, h_cv, h_out, ws_h)
        torch.cuda.synchronize()
        assert fxr.check_device_error() == 0
        assert torch.equal(h_out, d_out.cpu()), f"frame {i}: output differs"
        assert torch.equal(h_ck, d_ck) and torch.equal(h_cv, d_cv), f"frame {i}: cache differs"
        m2 = mask.copy()
        m2[valid.cpu().numpy() == 0] = 2
        skipped = torch.from_numpy(m2 == 0)
        assert torch.equal(h_out[skipped], before[skipped])   # non-executed rows untouched
        assert torch.equal(hmask, torch.from_numpy(mask))     # the host mask is read only


@pytest.mark.gpu
def test_host_frame_rejects_unmapped_memory(cuda):
    import torch
    w = W.Workload("host_16x16", 16, 16, 64, n_heads=2, dtype="bf16", active=0.3)
    cfg = fxr.FrameConfig(n_tokens=w.n_tokens, n_text=w.n_text, n_heads=w.n_heads, dtype="bf16",
                          rope_axes=w.rope_axes, rope_theta=w.rope_theta)
    C = w.n_heads * 128
    pinned = torch.zeros(w.n_tokens, C, dtype=torch.bfloat16).pin_memory()
    pageable = torch.zeros(w.n_tokens, C, dtype=torch.bfloat16)
    on_device = torch.zeros(w.n_tokens, C, dtype=torch.bfloat16, device="cuda")
    mask = torch.zeros(w.n_tokens, dtype=torch.int32).pin_memory()
    ck = torch.zeros(w.n_tokens, C, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(w.n_tokens, 3, dtype=torch.int32, device="cuda")
    nw = torch.ones(128, device="cuda")
    ws = torch.empty(fxr.frame_host_workspace_size(cfg), dtype=torch.uint8, device="cuda")
    for bad in (pageable, on_device):
        with pytest.raises(fxr.FxrError) as ei:
            fxr.frame_forward_host(cfg, pinned, bad, pinned, mask, None, pos, nw, nw, ck, ck.clone(),
                                   pinned, ws)
        assert ei.value.status == fxr.FXR_ERR_INVALID
        with pytest.raises(fxr.FxrError):
            fxr.frame_forward_host(cfg, pinned, pinned, pinned, mask, None, pos, nw, nw, ck, ck.clone(),
                                   bad, ws)
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0


def test_host_block_argument_checks():
    L = fxr.load()
    cfg = fxr.FrameConfig(n_tokens=1280, n_text=256, n_heads=6)
    d = cfg.desc()
    blk = fxr.DoubleBlock()
    blk.mlp_hidden, blk.ln_eps = 2304, 1e-6
    args = lambda ws=16, ws_bytes=1 << 40, host=16: (ctypes.byref(d), ctypes.byref(blk), host, host, host, None,
                                                     None, None, None, ws, ws_bytes, None)
    sblk = fxr.SingleBlock()
    sblk.mlp_hidden, sblk.ln_eps = 2304, 1e-6
    sargs = lambda ws=16, ws_bytes=1 << 40, host=16: (ctypes.byref(d), ctypes.byref(sblk), host, host, host,
                                                      None, None, None, None, ws, ws_bytes, None)
    for fn, a in ((L.fxr_double_block_forward_host, args), (L.fxr_single_block_forward_host, sargs)):
        assert fn(*a(ws=None)) == fxr.FXR_ERR_INVALID
        assert fn(*a(ws=8)) == fxr.FXR_ERR_INVALID
        assert fn(*a(ws_bytes=1 << 20)) == fxr.FXR_ERR_WORKSPACE
        assert fn(*a(host=None)) == fxr.FXR_ERR_INVALID
        assert fn(ctypes.byref(d), None, *([None] * 7), 16, 1 << 40, None) == fxr.FXR_ERR_INVALID  # null block
    ws = fxr.block_host_workspace_size(cfg, 2304)
    assert ws >= fxr.double_block_workspace_size(cfg, 2304) + 1280 * 4 + 2 * 1280 * 768 * 2
    assert fxr.block_host_workspace_size(cfg, 0) == 0                       # no MLP width: no size


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["double", "single"])
def test_host_blocks_match_device_blocks(cuda, kind):
    """Two consecutive block frames from host buffers against the device entry: bit for bit."""
    import torch
    w = W.Workload("hblk_512px_h6", 32, 32, 256, n_heads=6, dtype="bf16", active=0.3)
    N, T, C, D = w.n_tokens, w.n_text, w.n_heads * w.head_dim, w.head_dim
    H = 3 * C
    cfg = fxr.FrameConfig(n_tokens=N, n_text=T, n_heads=w.n_heads, dtype="bf16", rope_axes=w.rope_axes,
                          rope_theta=w.rope_theta)
    g = torch.Generator(device="cuda").manual_seed(31)
    rw = lambda *shape, sd: (torch.randn(*shape, device="cuda", generator=g) * sd).bfloat16()
    rf = lambda *shape, mu=0.0, sd=1.0: torch.randn(*shape, device="cuda", generator=g) * sd + mu
    if kind == "double":
        mk = lambda: {"shift": rf(C, sd=0.1), "scale": rf(C, sd=0.1), "gate": rf(C, mu=1.0, sd=0.2),
                      "w_qkv": rw(3 * C, C, sd=C ** -0.5), "b_qkv": rf(3 * C, sd=0.05),
                      "norm_q": rf(D, mu=1.0, sd=0.1), "norm_k": rf(D, mu=1.0, sd=0.1),
                      "w_out": rw(C, C, sd=C ** -0.5), "b_out": rf(C, sd=0.05),
                      "w_mlp0": rw(H, C, sd=C ** -0.5), "b_mlp0": rf(H, sd=0.05),
                      "w_mlp2": rw(C, H, sd=H ** -0.5), "b_mlp2": rf(C, sd=0.05)}
        txt, img = mk(), mk()
        run = lambda *a, **k: fxr.double_block_forward(cfg, txt, img, H, *a, **k)
    else:
        wts = {"shift": rf(C, sd=0.1), "scale": rf(C, sd=0.1), "gate": rf(C, mu=1.0, sd=0.2),
               "w_qkv_mlp": rw(3 * C + H, C, sd=C ** -0.5), "b_qkv_mlp": rf(3 * C + H, sd=0.05),
               "norm_q": rf(D, mu=1.0, sd=0.1), "norm_k": rf(D, mu=1.0, sd=0.1),
               "w_out": rw(C, C + H, sd=(C + H) ** -0.5), "b_out": rf(C, sd=0.05)}
        run = lambda *a, **k: fxr.single_block_forward(cfg, wts, H, *a, **k)
    f0 = W.make_frame(w, seed=41)
    pos = torch.from_numpy(f0["pos"]).cuda()
    d_ck = torch.from_numpy(f0["cache_k"]).cuda().bfloat16()
    d_cv = torch.from_numpy(f0["cache_v"]).cuda().bfloat16()
    h_ck, h_cv = d_ck.clone(), d_cv.clone()
    d_valid = (torch.rand(N, device="cuda", generator=g) < 0.9).to(torch.uint8)
    h_valid = d_valid.clone()
    d_out = torch.randn(N, C, device="cuda", generator=g).bfloat16()
    h_out = d_out.cpu().pin_memory()
    ws_d = torch.empty(fxr.double_block_workspace_size(cfg, H), dtype=torch.uint8, device="cuda")
    ws_h = torch.empty(fxr.block_host_workspace_size(cfg, H), dtype=torch.uint8, device="cuda")
    for i in range(2):
        mask = W.make_frame(w, seed=50 + i)["mask"].copy()
        mask[T + 7] = 1
        x = torch.randn(N, C, device="cuda", generator=g).bfloat16()
        hx, hmask = x.cpu().pin_memory(), torch.from_numpy(mask).pin_memory()
        before = h_out.clone()
        dmask = torch.from_numpy(mask).cuda()
        run(x, d_out, dmask, d_valid, pos, d_ck, d_cv, ws_d)
        run(hx, h_out, hmask, h_valid, pos, h_ck, h_cv, ws_h, host=True)
        torch.cuda.synchronize()
        assert fxr.check_device_error() == 0
        assert torch.equal(h_out, d_out.cpu()), f"{kind} frame {i}: block output differs"
        assert torch.equal(h_ck, d_ck) and torch.equal(h_cv, d_cv), f"{kind} frame {i}: cache differs"
        assert torch.equal(h_valid, d_valid)
        executed = dmask.cpu() != 0                       # the device mask after preprocessing
        assert torch.equal(h_out[~executed], before[~executed])
        assert torch.equal(hmask, torch.from_numpy(mask))
