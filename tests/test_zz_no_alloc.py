"""fxr_frame_forward_noalloc: the frame entry point for callers that cannot allocate device memory
when they run a frame (it uses a fixed scratch array inside the library instead of a workspace).

Checked through the C ABI against fxr_frame_forward (caller workspace) on the same inputs, for two
calls in a row, with the tolerance the parity tests use and bit for bit: the two paths run the same
kernels with the same schedule (the 6-head case also gets the same key-range split slots from the
built-in scratch as from fxr_workspace_size's workspace). This file is collected last so that a
stopping run has already run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import fxr
import workloads as W

pytestmark = pytest.mark.gpu

TOL = dict(max_abs=2e-3, mean_abs=2e-4)


def _lib():
    L = fxr.load()
    f = L.fxr_frame_forward_noalloc
    f.argtypes = [ctypes.POINTER(fxr.FrameDesc)] + [ctypes.c_void_p] * 12
    f.restype = ctypes.c_int32
    return L


def _tensors(w, fr, tdt):
    t = {k: torch.from_numpy(fr[k]).cuda().to(tdt) for k in ("q", "k", "v", "cache_k", "cache_v", "out")}
    t["mask"] = torch.from_numpy(fr["mask"]).cuda()
    t["pos"] = torch.from_numpy(fr["pos"]).cuda()
    t["norm_q"] = torch.from_numpy(fr["norm_q"]).cuda()
    t["norm_k"] = torch.from_numpy(fr["norm_k"]).cuda()
    return t


def _close(a, b, what):
    a = a.float().cpu().numpy().astype(np.float64)
    b = b.float().cpu().numpy().astype(np.float64)
    err = np.abs(a - b)
    assert np.isfinite(a).all(), what
    assert err.max() <= TOL["max_abs"] and err.mean() <= TOL["mean_abs"], (what, err.max(), err.mean())


C2_6HEADS = W.Workload("c2_1024px_p25_bf16_h6", 64, 64, 512, n_heads=6)


@pytest.mark.parametrize("wl", [W.C2, W.C1, C2_6HEADS])
def test_noalloc_matches_workspace_entry_point(cuda, wl):
    L = _lib()
    tdt = torch.bfloat16 if wl.dtype == "bf16" else torch.float16
    cfg = fxr.FrameConfig(n_tokens=wl.n_tokens, n_text=wl.n_text, n_heads=wl.n_heads, dtype=wl.dtype,
                          rope_axes=wl.rope_axes, rope_theta=wl.rope_theta)
    d = cfg.desc()
    ws = torch.empty(fxr.workspace_size(cfg), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((101, 202)):                 # two calls in a row
        fr = W.make_frame(wl, seed=seed)
        fr["mask"][wl.n_text + 3] = 1                         # one execute-only token (save/restore)
        a = _tensors(wl, fr, tdt)                             # workspace entry point
        b = _tensors(wl, fr, tdt)                             # allocation-free entry point
        fxr.frame_forward(cfg, a["q"], a["k"], a["v"], a["mask"], None, a["pos"], a["norm_q"],
                          a["norm_k"], a["cache_k"], a["cache_v"], a["out"], ws)
        st = L.fxr_frame_forward_noalloc(ctypes.byref(d), b["q"].data_ptr(), b["k"].data_ptr(),
                                         b["v"].data_ptr(), b["mask"].data_ptr(), None,
                                         b["pos"].data_ptr(), b["norm_q"].data_ptr(),
                                         b["norm_k"].data_ptr(), b["cache_k"].data_ptr(),
                                         b["cache_v"].data_ptr(), b["out"].data_ptr(), s)
        assert st == fxr.FXR_OK, L.fxr_last_error_string()
        torch.cuda.synchronize()
        assert fxr.check_device_error() == 0
        assert torch.equal(a["mask"], b["mask"])
        for k in ("out", "cache_k", "cache_v"):
            _close(b[k], a[k], f"call {call}: {k}")
            assert torch.equal(b[k], a[k]), f"call {call}: {k} differs from the workspace entry point"


def test_noalloc_rejects_frames_beyond_its_scratch(cuda):
    L = _lib()
    big = fxr.FrameConfig(n_tokens=16896, n_text=512).desc()    # 2048x2048 frame: ~311 MB scratch
    st = L.fxr_frame_forward_noalloc(ctypes.byref(big), *([None] * 11), None)
    assert st == fxr.FXR_ERR_WORKSPACE
    assert b"built-in scratch" in L.fxr_last_error_string()
