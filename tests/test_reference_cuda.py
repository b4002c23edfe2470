"""Cross-check against the reference's own CUDA kernels, compiled for sm_100a from its sources by
oracle/build_ref.sh into oracle/_ref (skipped when that library was not built).

Row gather/scatter (gather_scatter_kernels.cu:15-72) and the spatial-cache
protocol — preprocess, K/V merge + update, output merge + update + validity
(spatial_kv_cache.cu:12-87, SpatialCache methods :153-196) — over two frames, so that the second
frame runs on the state the first one left — bit-exact; the GELU, bias and modulation kernels
(flux2_kernels.cu:14-56, gather_scatter_kernels.cu:77-99) against the oracle's restatements
(oracle/fxr_oracle.c) and the GEMM's fused epilogue. The reference RMSNorm and LayerNorm (uninitialised shared
accumulators, flux2_kernels.cu:58-82, gather_scatter_kernels.cu:129-150) and attention (one warp's partial max and sum broadcast as
the block's, attention_kernels.cu:117-139) are not deterministic oracles and are only timed (the `reference_cuda` record of
`bench.py --impl reference`)."""
import numpy as np
import pytest

import fxr

O = pytest.importorskip("oracle")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref(cuda):
    L = O.ref_kernels()
    if L is None:
        pytest.skip("reference kernels not built (oracle/build_ref.sh)")
    return L


def _s():
    import torch
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("n_rows,M,dim", [(4608, 1525, 3072), (1536, 1, 128), (300, 300, 40)])
def test_row_gather_scatter_match_reference(ref, n_rows, M, dim):
    import torch
    g = torch.Generator(device="cuda").manual_seed(n_rows + M)
    src = torch.randn(n_rows, dim, device="cuda", generator=g)
    idx = torch.sort(torch.randperm(n_rows, device="cuda", generator=g)[:M]).values.int()
    a = torch.full((M, dim), 7.0, device="cuda")
    b = torch.full((M, dim), 7.0, device="cuda")
    ref.ref_gather_tokens(src.data_ptr(), a.data_ptr(), idx.data_ptr(), M, dim, _s())
    fxr.gather_rows(src, idx, b, host_count=M)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    base = torch.randn(n_rows, dim, device="cuda", generator=g)
    c, d = base.clone(), base.clone()
    ref.ref_scatter_tokens(a.data_ptr(), c.data_ptr(), idx.data_ptr(), M, dim, _s())
    fxr.scatter_rows(a, idx, d, host_count=M)
    torch.cuda.synchronize()
    assert torch.equal(c, d)


def test_spatial_cache_protocol_matches_reference_over_two_frames(ref):
    import torch
    T, I, heads, hd, out_ch = 64, 1024, 4, 128, 64
    N, C = T + I, heads * hd
    h = ref.ref_cache_create(I, T, out_ch, heads, hd, 1, 0)
    assert h
    try:
        valid = torch.zeros(N, dtype=torch.uint8, device="cuda")
        ck = torch.zeros(N, C, device="cuda")
        cv = torch.zeros(N, C, device="cuda")
        oc = torch.zeros(I, out_ch, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(5)
        rng = np.random.default_rng(6)
        for frame in range(3):
            p = [1.0, 0.3, 0.05][frame]
            m = np.zeros(N, np.int32)
            img = rng.random(I)
            m[T:] = np.where(img < p, 2, np.where(img < p + 0.05, 1, 0))
            mask_r = torch.from_numpy(m).cuda()
            mask_o = mask_r.clone()
            assert ref.ref_cache_preprocess_mask(h, mask_r.data_ptr(), _s()) == 0
            fxr.preprocess_mask(mask_o, valid)
            torch.cuda.synchronize()
            assert torch.equal(mask_r, mask_o), frame
            keys = torch.randn(N, C, device="cuda", generator=g)
            vals = torch.randn(N, C, device="cuda", generator=g)
            kr, vr, ko, vo = keys.clone(), vals.clone(), keys.clone(), vals.clone()
            assert ref.ref_cache_sync_kv(h, kr.data_ptr(), vr.data_ptr(), mask_r.data_ptr(), 0, 1,
                                         _s()) == 0
            fxr.kv_sync(ko, vo, ck, cv, mask_o)
            torch.cuda.synchronize()
            assert torch.equal(kr, ko) and torch.equal(vr, vo), frame
            pred = torch.randn(I, out_ch, device="cuda", generator=g)
            pr, po = pred.clone(), pred.clone()
            assert ref.ref_cache_sync_output(h, pr.data_ptr(), mask_r.data_ptr(), _s()) == 0
            fxr.output_cache_sync(po, oc, mask_o, valid, T)
            torch.cuda.synchronize()
            assert torch.equal(pr, po), frame
        # the validity flags the reference keeps are visible through its next preprocess
        probe_r = torch.zeros(N, dtype=torch.int32, device="cuda")
        probe_o = probe_r.clone()
        ref.ref_cache_preprocess_mask(h, probe_r.data_ptr(), _s())
        fxr.preprocess_mask(probe_o, valid)
        torch.cuda.synchronize()
        assert torch.equal(probe_r, probe_o)
        assert ref.ref_cache_reset(h, _s()) == 0
        valid.zero_()
        ref.ref_cache_preprocess_mask(h, probe_r.data_ptr(), _s())
        fxr.preprocess_mask(probe_o, valid)
        torch.cuda.synchronize()
        assert torch.equal(probe_r, probe_o) and bool((probe_o == 2).all())
    finally:
        torch.cuda.synchronize()
        ref.ref_cache_destroy(h)


def test_gelu_modulation_and_bias_restatements_match_reference(ref):
    """The oracle's tanh GELU, modulation and linear bias (fxo_gelu_tanh, fxo_layer_norm_modulate,
    fxo_linear: the restatement the block tests check against) against the reference's own
    gelu_kernel (flux2_kernels.cu:14-29), apply_modulation_kernel (gather_scatter_kernels.cu:77-99)
    and bias_add_kernel (flux2_kernels.cu:34-53), fp32 on the GPU."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(1 << 16, device="cuda", generator=g) * 3
    a = x.clone()
    ref.ref_gelu(a.data_ptr(), a.numel(), _s())
    torch.cuda.synchronize()
    mine = O.gelu_tanh(x.cpu().numpy())
    np.testing.assert_allclose(a.cpu().numpy(), mine, rtol=4e-6, atol=4e-7)
    rows, dim = 257, 3072
    # modulation of already-normalised rows: LayerNorm leaves a zero-mean, unit-variance row unchanged
    xm = torch.randn(rows, dim, device="cuda", generator=g, dtype=torch.float64)
    xm = ((xm - xm.mean(1, keepdim=True)) / xm.std(1, unbiased=False, keepdim=True)).float()
    sc = torch.randn(dim, device="cuda", generator=g) * 0.2
    sh = torch.randn(dim, device="cuda", generator=g) * 0.2
    out = torch.empty_like(xm)
    ref.ref_apply_modulation(xm.data_ptr(), sc.data_ptr(), sh.data_ptr(), out.data_ptr(), rows, dim, _s())
    torch.cuda.synchronize()
    mine = O.layer_norm_modulate(xm.cpu().numpy(), sc.cpu().numpy(), sh.cpu().numpy(), eps=0.0)
    np.testing.assert_allclose(out.cpu().numpy(), mine, rtol=2e-6, atol=2e-6)
    # bias add: a zero product leaves the bias broadcast over the rows
    bias = torch.randn(dim, device="cuda", generator=g)
    z = torch.zeros(rows, dim, device="cuda")
    ref.ref_bias_add(z.data_ptr(), bias.data_ptr(), rows, dim, _s())
    torch.cuda.synchronize()
    mine = O.linear(np.zeros((rows, 8), np.float32), np.zeros((dim, 8), np.float32), bias.cpu().numpy())
    np.testing.assert_array_equal(z.cpu().numpy(), mine)


def test_rows_gemm_gelu_epilogue_matches_reference_gelu(ref):
    """The GEMM's fused bias + GELU epilogue against the reference's bias_add + gelu kernels
    (flux2_kernels.cu:14-56): a one-hot W makes the product an exact copy of the A columns, so the
    epilogue sees the same fp32 values the reference kernels get; ours rounds to bf16 once."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(6)
    M, K, n_out = 640, 64, 256
    a = (torch.rand(M, K, device="cuda", generator=g) * 12 - 6).bfloat16()
    w = torch.zeros(n_out, K, device="cuda", dtype=torch.bfloat16)
    w[torch.arange(n_out), torch.arange(n_out) % K] = 1.0
    bias = torch.randn(n_out, device="cuda", generator=g) * 0.5
    idx = torch.arange(M, dtype=torch.int32, device="cuda")
    cnt = torch.tensor([M], dtype=torch.int32, device="cuda")
    y = torch.empty(M, n_out, device="cuda", dtype=torch.bfloat16)
    fxr.rows_gemm([(a, w, False)], [(y, n_out, False, fxr.FXR_ACT_GELU_TANH)], idx, cnt, M, bias0=bias)
    r = a.float()[:, torch.arange(n_out, device="cuda") % K].contiguous()
    ref.ref_bias_add(r.data_ptr(), bias.data_ptr(), M, n_out, _s())
    ref.ref_gelu(r.data_ptr(), r.numel(), _s())
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0
    rb = r.bfloat16().float()
    diff = (y.float() - rb).abs()
    ulp = 2.0 ** (torch.floor(torch.log2(rb.abs().clamp_min(1e-30))) - 7)
    assert bool((diff <= ulp).all()), float((diff / ulp).max())   # one bf16 rounding apart at most
    assert float((diff == 0).float().mean()) > 0.99
