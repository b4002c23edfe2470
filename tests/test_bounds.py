"""Out-of-range row indices: the kernels skip the row and report it, they never read or write
outside a buffer. The reference kernels index without any check (gather_scatter_kernels.cu:15-72)
and report CUDA errors by throwing or returning -1 (src/utils/error.h:27-91,
flux2_double_block_plugin.cpp:208,230); here each kernel sets bit 1 of the device error word and
fxr_check_device_error returns FXR_ERR_BOUNDS, after which the context keeps working.

Every index passed below is either inside its buffer or caught by the kernel's own check before
the access (rows_copy_kernel, gather_bulk_kernel's producer, the attention epilogue), so nothing
reads or writes out of bounds."""
import numpy as np
import pytest
import torch

import fxr
import oracle as O
import parity_stats
import workloads as W

pytestmark = pytest.mark.gpu


def _status_after_sync():
    try:
        fxr.check_device_error()
        return fxr.FXR_OK
    except fxr.FxrError as e:
        return e.status


def test_row_gather_and_scatter_skip_bad_indices(cuda):
    assert _status_after_sync() == fxr.FXR_OK
    src = torch.arange(10 * 64, dtype=torch.float32, device="cuda").reshape(10, 64)
    idx = torch.tensor([0, 10, 3, -1, 9], dtype=torch.int32, device="cuda")
    dst = torch.full((5, 64), -5.0, device="cuda")
    fxr.gather_rows(src, idx, dst, host_count=5)
    assert _status_after_sync() == fxr.FXR_ERR_BOUNDS
    assert torch.equal(dst[[0, 2, 4]], src[[0, 3, 9]])
    assert bool((dst[[1, 3]] == -5.0).all())                   # skipped rows untouched
    assert _status_after_sync() == fxr.FXR_OK                   # reading the word cleared it

    s2 = torch.arange(5 * 64, dtype=torch.float32, device="cuda").reshape(5, 64) + 1000
    idx2 = torch.tensor([2, 12, -4, 7, 0], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([5], dtype=torch.int32, device="cuda")   # count read on the device
    d2 = torch.full((10, 64), 7.0, device="cuda")
    fxr.scatter_rows(s2, idx2, d2, count=cnt)
    assert _status_after_sync() == fxr.FXR_ERR_BOUNDS
    assert torch.equal(d2[[2, 7, 0]], s2[[0, 3, 4]])
    keep = [r for r in range(10) if r not in (2, 7, 0)]
    assert bool((d2[keep] == 7.0).all())
    # a bound smaller than the buffer: row 7 is now out of range too
    d3 = torch.full((10, 64), 7.0, device="cuda")
    fxr.scatter_rows(s2, idx2, d3, count=cnt, n_index_rows=5)
    assert _status_after_sync() == fxr.FXR_ERR_BOUNDS
    assert bool((d3[7] == 7.0).all()) and torch.equal(d3[[2, 0]], s2[[0, 4]])
    # in-range indices: no report
    fxr.gather_rows(src, torch.tensor([1, 2], dtype=torch.int32, device="cuda"), dst, host_count=2)
    assert _status_after_sync() == fxr.FXR_OK


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_frame_steps_skip_bad_indices(cuda, dtype):
    """A caller-built executed-row list with one index past the last token and one negative one,
    through the gather (+ RMSNorm + RoPE + cache write) and the attention (+ scatter): both steps
    report FXR_ERR_BOUNDS, the rows of the good indices equal the oracle, nothing else changes."""
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    w = W.Workload("bounds_16x16", 16, 16, 44, n_heads=2, dtype=dtype)
    N, C = w.n_tokens, 2 * 128
    fr = W.make_frame(w, seed=13)
    rng = np.random.default_rng(14)
    good = np.sort(rng.choice(N, size=40, replace=False)).astype(np.int32)
    idx_h = np.insert(good, [5, 17], [N, -1]).astype(np.int32)        # 42 entries, 2 bad
    bad = np.nonzero((idx_h < 0) | (idx_h >= N))[0]
    assert bad.size == 2
    mask = np.zeros(N, dtype=np.int32)
    mask[good] = 2
    cfg = fxr.FrameConfig(n_tokens=N, n_text=w.n_text, n_heads=2, dtype=dtype,
                          rope_axes=w.rope_axes, rope_theta=w.rope_theta)
    t = {k: torch.from_numpy(fr[k]).cuda().to(tdt) for k in ("q", "k", "v", "cache_k", "cache_v", "out")}
    dmask = torch.from_numpy(mask).cuda()
    pos = torch.from_numpy(fr["pos"]).cuda()
    nq, nk = torch.from_numpy(fr["norm_q"]).cuda(), torch.from_numpy(fr["norm_k"]).cuda()
    idx = torch.from_numpy(idx_h).cuda()
    cnt = torch.tensor([idx_h.size], dtype=torch.int32, device="cuda")
    qc = torch.zeros(N, C, dtype=tdt, device="cuda")
    assert _status_after_sync() == fxr.FXR_OK
    fxr.gather_norm_rope(cfg, t["q"], t["k"], t["v"], dmask, idx, cnt, pos, nq, nk, qc,
                         t["cache_k"], t["cache_v"], None)
    assert _status_after_sync() == fxr.FXR_ERR_BOUNDS
    assert bool((qc[bad.tolist()] == 0).all())                 # compact rows of bad entries untouched
    fxr.attention_active(cfg, qc, cnt, t["cache_k"], t["cache_v"], idx, t["out"])
    assert _status_after_sync() == fxr.FXR_ERR_BOUNDS
    out = t["out"].float().cpu().numpy()
    ck, cv = t["cache_k"].float().cpu().numpy(), t["cache_v"].float().cpu().numpy()
    rest = np.ones(N, dtype=bool)
    rest[good] = False
    assert np.array_equal(out[rest], fr["out"][rest])
    assert np.array_equal(ck[rest], fr["cache_k"][rest]) and np.array_equal(cv[rest], fr["cache_v"][rest])
    assert np.array_equal(cv[good], fr["v"][good])
    op = O.frame_operands(fr["q"], fr["k"], fr["v"], mask, None, fr["pos"], fr["norm_q"], fr["norm_k"],
                          fr["cache_k"], fr["cache_v"], 2, 128, w.rope_axes, w.rope_theta, dtype)
    assert np.array_equal(op["idx"], good)
    ref = O.attention(op["qc"], op["keys"], op["values"], 2, 128)
    mx, mn = parity_stats.record("O of the good rows", out[good], ref, 2e-3, 2e-4)
    assert mx <= 2e-3 and mn <= 2e-4, (mx, mn)
