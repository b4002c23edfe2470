"""The double-stream block's dense steps on the executed rows only: fxr_ln_modulate_rows (LayerNorm
+ modulation) and fxr_rows_gemm (Q/K/V, MLP up with GELU, out-projection + MLP down + residual)
against torch fp32 restatements of the reference's steps (flux2_double_block_plugin.cpp:370-458,
gather_scatter_kernels.cu:77-169, flux2_kernels.cu:14-29)."""
import ctypes

import numpy as np
import pytest

import fxr


def _desc(**kw):
    d = fxr.RowsGemmDesc()
    d.dtype, d.n_tokens, d.row0, d.row_end = fxr.FXR_BF16, 1024, 0, -1
    d.n_operands, d.n_outputs = 1, 1
    d.a[0] = fxr.RowsOperand(16, 256, 256, 1, 16)
    d.y[0] = fxr.RowsOutput(16, 256, 256, 1, 0, 0)
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def test_rows_gemm_argument_checks():
    L = fxr.load()
    idx = ctypes.c_void_p(16)

    def call(d, scratch=None, nbytes=0):
        return L.fxr_rows_gemm(ctypes.byref(d), idx, idx, scratch, nbytes, None)

    assert call(_desc(dtype=fxr.FXR_F32)) == fxr.FXR_ERR_UNSUPPORTED
    assert call(_desc(n_operands=3)) == fxr.FXR_ERR_INVALID
    assert call(_desc(n_outputs=0)) == fxr.FXR_ERR_INVALID
    assert call(_desc(n_outputs=5)) == fxr.FXR_ERR_INVALID
    d = _desc()
    d.y[0] = fxr.RowsOutput(16, 256, 128, 1, 0, 0)           # cols not a multiple of 256
    assert call(d) == fxr.FXR_ERR_UNSUPPORTED
    d = _desc()
    d.a[0] = fxr.RowsOperand(16, 256, 96, 1, 16)             # k not a multiple of 64
    assert call(d) == fxr.FXR_ERR_UNSUPPORTED
    d = _desc()
    d.a[0] = fxr.RowsOperand(16, 100, 256, 1, 16)            # ld < k
    assert call(d) == fxr.FXR_ERR_INVALID
    d = _desc()
    d.a[0] = fxr.RowsOperand(24, 256, 256, 1, 16)            # unaligned rows
    assert call(d) == fxr.FXR_ERR_INVALID
    d = _desc()
    d.a[0] = fxr.RowsOperand(16, 256, 256, 1, 16, 128)       # W row stride below k
    assert call(d) == fxr.FXR_ERR_INVALID
    d = _desc()
    d.a[0] = fxr.RowsOperand(16, 256, 256, 1, 16, 260)       # W row stride not a multiple of 8
    assert call(d) == fxr.FXR_ERR_INVALID
    d = _desc()
    d.y[0] = fxr.RowsOutput(16, 256, 256, 1, 7, 0)           # unknown activation
    assert call(d) == fxr.FXR_ERR_INVALID
    d = _desc(n_outputs=2, residual=16, ld_residual=512)     # residual with two parts
    d.y[1] = fxr.RowsOutput(16, 256, 256, 1, 0, 0)
    assert call(d) == fxr.FXR_ERR_INVALID
    assert call(_desc(row_end=2000)) == fxr.FXR_ERR_INVALID  # past n_tokens
    assert call(_desc(), scratch=16, nbytes=1024) == fxr.FXR_ERR_WORKSPACE
    assert L.fxr_rows_gemm(ctypes.byref(_desc()), None, None, None, 0, None) == fxr.FXR_ERR_INVALID
    # 148 SMs: the sync area and one 128 KB partial tile per CTA
    assert fxr.rows_gemm_scratch_size() == 32768 + 148 * 128 * 1024


def test_ln_modulate_rows_argument_checks():
    L = fxr.load()
    p = ctypes.c_void_p(16)
    args = lambda dtype=fxr.FXR_BF16, dim=3072, ldx=3072, row_end=-1, eps=1e-6: (
        dtype, p, ldx, dim, p, p, 0, row_end, 4608, None, None, ctypes.c_float(eps), p, dim, None)
    assert L.fxr_ln_modulate_rows(*args(dtype=fxr.FXR_F32)) == fxr.FXR_ERR_UNSUPPORTED
    assert L.fxr_ln_modulate_rows(*args(dim=3000, ldx=3000)) == fxr.FXR_ERR_UNSUPPORTED
    assert L.fxr_ln_modulate_rows(*args(dim=8192, ldx=8192)) == fxr.FXR_ERR_UNSUPPORTED
    assert L.fxr_ln_modulate_rows(*args(ldx=2048)) == fxr.FXR_ERR_INVALID
    assert L.fxr_ln_modulate_rows(*args(row_end=5000)) == fxr.FXR_ERR_INVALID
    assert L.fxr_ln_modulate_rows(*args(eps=-1.0)) == fxr.FXR_ERR_INVALID
    assert L.fxr_ln_modulate_rows(*args(row_end=0)) == fxr.FXR_OK     # empty range: nothing to do


# ---------------------------------------------------------------------------------------------
# GPU: against torch fp32
# ---------------------------------------------------------------------------------------------

def _mask_idx(n, n_text, p, seed):
    import torch
    rng = np.random.default_rng(seed)
    mask = np.zeros(n, np.int32)
    mask[:n_text] = 2
    mask[n_text:] = np.where(rng.random(n - n_text) < p, 2, 0)
    idx_h = np.nonzero(mask)[0].astype(np.int32)
    idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    idx[: idx_h.size] = torch.from_numpy(idx_h).cuda()
    count = torch.tensor([idx_h.size], dtype=torch.int32, device="cuda")
    return idx_h, idx, count


def _within_ulps(got, ref, dtype, ulps=1.0, floor=1e-4):
    import torch
    mag = ref.abs().clamp_min(1e-3)
    ulp = 2.0 ** (torch.floor(torch.log2(mag)) - (7 if dtype == torch.bfloat16 else 10))
    err = (got - ref).abs()
    return bool((err <= ulp * ulps * 1.0001 + floor).all()), float(err.max())


def _ref_ln_mod(x, scale, shift, eps=1e-6):
    """layer_norm_modulated_kernel (no gamma/beta) then apply_modulation_kernel, fp32."""
    import torch
    xf = x.float()
    mean = xf.mean(dim=1, keepdim=True)
    var = ((xf - mean) ** 2).mean(dim=1, keepdim=True)
    y = (xf - mean) * torch.rsqrt(var + eps)
    return (1.0 + scale) * y + shift


def _gelu_tanh(x):
    import torch
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608 * (x + 0.044715 * x * x * x)))


@pytest.mark.gpu
@pytest.mark.parametrize("n,dim,p,dtype", [(4608, 3072, 0.25, "bf16"), (1536, 1024, 0.6, "f16"),
                                           (700, 4096, 0.1, "bf16")])
def test_ln_modulate_rows_matches_fp32(cuda, n, dim, p, dtype):
    import torch
    td = torch.bfloat16 if dtype == "bf16" else torch.float16
    g = torch.Generator(device="cuda").manual_seed(dim + n)
    x = (torch.randn(n, dim, device="cuda", generator=g) * 2 + 0.5).to(td)
    scale = torch.randn(dim, device="cuda", generator=g) * 0.2
    shift = torch.randn(dim, device="cuda", generator=g) * 0.2
    idx_h, idx, count = _mask_idx(n, 128, p, n)
    y = torch.full((n, dim), 9.0, device="cuda").to(td)
    fxr.ln_modulate_rows(x, idx, count, y, scale, shift)
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0
    M = idx_h.size
    ref = _ref_ln_mod(x[torch.from_numpy(idx_h).long().cuda()], scale, shift).to(td).float()
    ok, err = _within_ulps(y[:M].float(), ref, td, ulps=1.0, floor=2e-3)
    assert ok, err
    assert bool((y[M:].float() == 9.0).all())          # rows past the count untouched


def _weights(n_out, k, td, g, scale=1.0):
    import torch
    return (torch.randn(n_out, k, device="cuda", generator=g) * scale / np.sqrt(k)).to(td)


@pytest.mark.gpu
@pytest.mark.parametrize("n,p,stream_k", [(4608, 0.25, True), (4608, 0.25, False), (1536, 0.05, True),
                                          (4608, 1.0, True), (300, 0.0, True)])
def test_rows_gemm_block_steps(cuda, n, p, stream_k):
    """The three GEMM recipes of the block on the same executed rows: Q/K/V from compact LayerNorm
    rows, MLP up with GELU into compact rows, out-projection + MLP down (two operands) + gated
    residual scattered into the block output."""
    import torch
    td = torch.bfloat16
    C, H3 = 768, 2304
    g = torch.Generator(device="cuda").manual_seed(n + int(p * 100))
    idx_h, idx, count = _mask_idx(n, min(256, n), p, n + 1)
    M = idx_h.size
    rows = torch.from_numpy(idx_h).long().cuda()
    scratch = fxr.rows_gemm_scratch() if stream_k else None
    xn = torch.zeros(n, C, device="cuda", dtype=td)
    xn[:M] = (torch.randn(M, C, device="cuda", generator=g)).to(td)
    # Q/K/V scattered
    w_qkv = _weights(3 * C, C, td, g)
    b_qkv = torch.randn(3 * C, device="cuda", generator=g) * 0.1
    qkv = [torch.full((n, C), 5.0, device="cuda").to(td) for _ in range(3)]
    fxr.rows_gemm([(xn, w_qkv, False)], [(t, C, True, fxr.FXR_ACT_NONE) for t in qkv], idx, count, n,
                  bias0=b_qkv, scratch=scratch)
    # MLP up, GELU, compact
    w_up = _weights(H3, C, td, g)
    b_up = torch.randn(H3, device="cuda", generator=g) * 0.1
    h = torch.zeros(n, H3, device="cuda", dtype=td)
    fxr.rows_gemm([(xn, w_up, False)], [(h, H3, False, fxr.FXR_ACT_GELU_TANH)], idx, count, n,
                  bias0=b_up, scratch=scratch)
    # out-projection of the (token-major) attention output + MLP down, gated residual, scattered
    o = (torch.randn(n, C, device="cuda", generator=g)).to(td)
    x_in = (torch.randn(n, C, device="cuda", generator=g)).to(td)
    w_o, w_2 = _weights(C, C, td, g), _weights(C, H3, td, g)
    b_o = torch.randn(C, device="cuda", generator=g) * 0.1
    b_2 = torch.randn(C, device="cuda", generator=g) * 0.1
    gate = torch.rand(C, device="cuda", generator=g) + 0.5
    out = torch.full((n, C), 3.0, device="cuda").to(td)
    fxr.rows_gemm([(o, w_o, True), (h, w_2, False)], [(out, C, True, fxr.FXR_ACT_NONE)], idx, count, n,
                  bias0=b_o, bias1=b_2, residual=x_in, gate=gate, scratch=scratch)
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0

    xf = xn[:M].float()
    ref_qkv = (xf @ w_qkv.float().T + b_qkv).to(td).float()
    got_qkv = torch.cat([t[rows].float() for t in qkv], dim=1)
    ok, err = _within_ulps(got_qkv, ref_qkv, td)
    assert ok, ("qkv", err)
    ref_h = _gelu_tanh(xf @ w_up.float().T + b_up).to(td).float()
    ok, err = _within_ulps(h[:M].float(), ref_h, td, floor=2e-4)
    assert ok, ("mlp up", err)
    hf = h[:M].float()                       # the kernel's own bf16 H feeds the down projection
    ref_out = (x_in[rows].float() + gate * (o[rows].float() @ w_o.float().T + b_o + hf @ w_2.float().T + b_2))
    ok, err = _within_ulps(out[rows].float(), ref_out.to(td).float(), td, floor=2e-3)
    assert ok, ("out", err)
    untouched = torch.ones(n, dtype=torch.bool, device="cuda")
    untouched[rows] = False
    for t in qkv:
        assert bool((t[untouched].float() == 5.0).all())
    assert bool((out[untouched].float() == 3.0).all())


@pytest.mark.gpu
def test_rows_gemm_row_ranges_and_determinism(cuda):
    """Text rows [0, T) and image rows [T, count) with their own weights (two launches sharing one
    scratch), and bit-identical results when repeated (the stream-K finisher adds partials in CTA
    order)."""
    import torch
    td = torch.bfloat16
    n, T, C = 4608, 512, 3072
    g = torch.Generator(device="cuda").manual_seed(11)
    idx_h, idx, count = _mask_idx(n, T, 0.25, 12)
    M = idx_h.size
    rows = torch.from_numpy(idx_h).long().cuda()
    xn = (torch.randn(n, C, device="cuda", generator=g)).to(td)
    w_txt, w_img = _weights(C, C, td, g), _weights(C, C, td, g)
    scratch = fxr.rows_gemm_scratch()
    outs = []
    for _ in range(3):
        y = torch.zeros(n, C, device="cuda", dtype=td)
        fxr.rows_gemm([(xn, w_txt, False)], [(y, C, True, 0)], idx, count, n, row0=0, row_end=T,
                      scratch=scratch)
        fxr.rows_gemm([(xn, w_img, False)], [(y, C, True, 0)], idx, count, n, row0=T, row_end=-1,
                      scratch=scratch)
        outs.append(y)
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    ref = torch.cat([xn[:T].float() @ w_txt.float().T, xn[T:M].float() @ w_img.float().T])
    ok, err = _within_ulps(outs[0][rows].float(), ref.to(td).float(), td)
    assert ok, err
