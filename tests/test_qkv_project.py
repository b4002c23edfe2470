"""QKV projection of the executed tokens (fxr_qkv_project): the tcgen05 GEMM with gathered A rows
against torch's fp32 matmul of the same gathered rows (flux2_double_block_plugin.cpp:392-398 runs
this projection as fp32 cublasSgemm on every token)."""
import ctypes

import numpy as np
import pytest

import fxr
import workloads as W


def test_qkv_project_argument_checks():
    L = fxr.load()
    d = fxr.FrameConfig(n_tokens=1536, n_text=512, n_heads=4).desc()
    rest = [None] * 8 + [0, None]        # w, bias, idx, count, q, k, v, scratch, bytes, stream
    assert L.fxr_qkv_project(ctypes.byref(d), None, 256, 100, *rest) == fxr.FXR_ERR_UNSUPPORTED
    d3 = fxr.FrameConfig(n_tokens=1536, n_text=512, n_heads=3).desc()      # C = 384, not / 256
    assert L.fxr_qkv_project(ctypes.byref(d3), None, 256, 256, *rest) == fxr.FXR_ERR_UNSUPPORTED
    assert L.fxr_qkv_project(ctypes.byref(d), None, 256, 256, *rest) == fxr.FXR_ERR_INVALID


@pytest.mark.gpu
@pytest.mark.parametrize("n,heads,k_dim,dtype,p", [(1536, 4, 256, "bf16", 0.25), (4608, 24, 3072, "bf16", 0.25),
                                                  (1536, 2, 1024, "f16", 0.6), (640, 2, 64, "bf16", 0.0)])
@pytest.mark.parametrize("stream_k", [True, False])
def test_qkv_project_matches_fp32_matmul(cuda, n, heads, k_dim, dtype, p, stream_k):
    import torch
    td = torch.bfloat16 if dtype == "bf16" else torch.float16
    C = heads * 128
    g = torch.Generator(device="cuda").manual_seed(n + k_dim)
    x = (torch.randn(n, k_dim, device="cuda", generator=g) * 0.5).to(td)
    w = (torch.randn(3 * C, k_dim, device="cuda", generator=g) / np.sqrt(k_dim)).to(td)
    bias = torch.randn(3 * C, device="cuda", generator=g) * 0.1
    rng = np.random.default_rng(n)
    mask = np.zeros(n, np.int32)
    mask[:128] = 2
    mask[128:] = np.where(rng.random(n - 128) < p, 2, 0)
    idx_h = np.nonzero(mask)[0].astype(np.int32)
    idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    idx[: idx_h.size] = torch.from_numpy(idx_h).cuda()
    count = torch.tensor([idx_h.size], dtype=torch.int32, device="cuda")
    outs = [torch.full((n, C), 7.0, device="cuda").to(td) for _ in range(3)]
    cfg = fxr.FrameConfig(n_tokens=n, n_text=128, n_heads=heads, dtype=dtype)
    scratch = fxr.rows_gemm_scratch() if stream_k else None
    fxr.qkv_project(cfg, x, w, bias, idx, count, *outs, scratch=scratch)
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0
    rows = torch.from_numpy(idx_h).long().cuda()
    ref = (x[rows].float() @ w.float().T + bias).to(td).float()
    got = torch.cat([o[rows].float() for o in outs], dim=1)
    # bf16/fp16 rounding of an fp32 sum whose order differs: within 1 unit in the last place
    mag = ref.abs().clamp_min(1e-3)
    ulp = 2.0 ** (torch.floor(torch.log2(mag)) - (7 if dtype == "bf16" else 10))
    err = (got - ref).abs()
    assert bool((err <= ulp * 1.0001 + 1e-4).all()), float(err.max())
    untouched = torch.ones(n, dtype=torch.bool, device="cuda")
    untouched[rows] = False
    for o in outs:
        assert bool((o[untouched].float() == 7.0).all())
