"""The reference's dense fp32 block helpers as this library runs them (fxr_layer_norm_f32,
fxr_modulate_f32, fxr_gelu_tanh_f32, fxr_bias_add_f32, fxr_add_f32, fxr_scale_add_f32; the
C++ mirror's layer_norm_modulated, apply_modulation, launch_gelu, launch_bias_add, launch_elem_add,
launch_scale_add). Against the oracle's restatements and numpy in float64, and, where the reference's
own kernel is a correct oracle (gelu, bias_add, apply_modulation, elem/scale add are plain
elementwise maps), against that kernel compiled from its sources (oracle/_ref)."""
import ctypes

import numpy as np
import pytest
import torch

import fxr
import oracle as O
import parity_stats

pytestmark = pytest.mark.gpu

_vp, _i64, _i32, _f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float


def _lib():
    L = fxr.load()
    L.fxr_layer_norm_f32.argtypes = [_vp, _vp, _vp, _vp, _f, _i64, _i32, _vp]
    L.fxr_modulate_f32.argtypes = [_vp, _vp, _vp, _vp, _i64, _i32, _vp]
    L.fxr_gelu_tanh_f32.argtypes = [_vp, _i64, _vp]
    L.fxr_bias_add_f32.argtypes = [_vp, _vp, _i64, _i32, _vp]
    L.fxr_add_f32.argtypes = [_vp, _vp, _vp, _i64, _vp]
    L.fxr_scale_add_f32.argtypes = [_vp, _vp, _vp, _f, _i64, _vp]
    return L


def _ok(st):
    assert st == fxr.FXR_OK, fxr.load().fxr_last_error_string()


def _close(what, got, ref, max_abs, mean_abs):
    mx, mn = parity_stats.record(what, got, ref, max_abs, mean_abs)
    assert mx <= max_abs and mn <= mean_abs, (what, mx, mn)


@pytest.mark.parametrize("rows,dim,affine", [(37, 3072, True), (5, 100, False), (2, 4, False), (300, 257, True)])
def test_layer_norm_f32(cuda, rows, dim, affine):
    L = _lib()
    rng = np.random.default_rng(rows * dim)
    x = (rng.normal(size=(rows, dim)) * 3 + 1).astype(np.float32)
    g = rng.normal(1, 0.2, size=dim).astype(np.float32) if affine else None
    b = rng.normal(0, 0.2, size=dim).astype(np.float32) if affine else None
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    dg = None if g is None else torch.from_numpy(g).cuda()
    db = None if b is None else torch.from_numpy(b).cuda()
    s = torch.cuda.current_stream().cuda_stream
    _ok(L.fxr_layer_norm_f32(dx.data_ptr(), dy.data_ptr(), dg.data_ptr() if g is not None else None,
                             db.data_ptr() if b is not None else None, 1e-6, rows, dim, s))
    # in place (y aliases x), as the mirror's callers may do
    dz = dx.clone()
    _ok(L.fxr_layer_norm_f32(dz.data_ptr(), dz.data_ptr(), dg.data_ptr() if g is not None else None,
                             db.data_ptr() if b is not None else None, 1e-6, rows, dim, s))
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0
    xd = x.astype(np.float64)
    mean = xd.mean(1, keepdims=True)
    ref = (xd - mean) / np.sqrt(((xd - mean) ** 2).mean(1, keepdims=True) + 1e-6)
    if affine:
        ref = ref * g + b
    _close("layer norm vs float64", dy.cpu().numpy(), ref, 2e-5, 2e-6)
    assert torch.equal(dz, dy)
    if not affine:
        _close("layer norm vs oracle", dy.cpu().numpy(), O.layer_norm_modulate(x), 2e-5, 2e-6)


def test_layer_norm_f32_reference_known_answer(cuda):
    """test_gather_scatter.cpp:106-133: rows [1,2,3,4] and [5,6,7,8] normalise to +-1.3416, +-0.4472."""
    L = _lib()
    x = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8]], dtype=torch.float32, device="cuda")
    y = torch.empty_like(x)
    _ok(L.fxr_layer_norm_f32(x.data_ptr(), y.data_ptr(), None, None, 1e-6, 2, 4,
                             torch.cuda.current_stream().cuda_stream))
    exp = np.array([-1.3416407, -0.4472136, 0.4472136, 1.3416407], dtype=np.float32)
    got = y.cpu().numpy()
    assert np.abs(got - exp).max() <= 1e-4


@pytest.mark.parametrize("n,dim", [(4096 * 3, 3072), (1001, 7), (8, 4)])
def test_elementwise_f32(cuda, n, dim):
    L = _lib()
    rng = np.random.default_rng(n)
    rows = max(1, n // dim)
    n = rows * dim
    x = rng.normal(size=n).astype(np.float32) * 3
    y = rng.normal(size=n).astype(np.float32)
    bias = rng.normal(size=dim).astype(np.float32)
    sc, sh = rng.normal(0, 0.1, size=dim).astype(np.float32), rng.normal(0, 0.1, size=dim).astype(np.float32)
    s = torch.cuda.current_stream().cuda_stream
    t = lambda a: torch.from_numpy(a).cuda()
    dx, dy, db, dsc, dsh = t(x), t(y), t(bias), t(sc), t(sh)
    g = dx.clone()
    _ok(L.fxr_gelu_tanh_f32(g.data_ptr(), n, s))
    ba = dx.clone()
    _ok(L.fxr_bias_add_f32(ba.data_ptr(), db.data_ptr(), rows, dim, s))
    z = torch.empty_like(dx)
    _ok(L.fxr_add_f32(dx.data_ptr(), dy.data_ptr(), z.data_ptr(), n, s))
    sa = torch.empty_like(dx)
    _ok(L.fxr_scale_add_f32(dx.data_ptr(), dy.data_ptr(), sa.data_ptr(), 0.37, n, s))
    md = torch.empty_like(dx)
    _ok(L.fxr_modulate_f32(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), md.data_ptr(), rows, dim, s))
    torch.cuda.synchronize()
    assert fxr.check_device_error() == 0
    _close("gelu vs oracle", g.cpu().numpy(), O.gelu_tanh(x), 2e-6, 2e-7)
    xr = x.reshape(rows, dim)
    assert np.array_equal(ba.cpu().numpy().reshape(rows, dim), xr + bias)
    assert np.array_equal(z.cpu().numpy(), x + y)
    # x + gate * y: the device contracts it into one fused multiply-add (a single rounding)
    _close("scale add vs float64", sa.cpu().numpy(), x.astype(np.float64) + np.float64(np.float32(0.37)) * y,
           4e-7 * max(1.0, float(np.abs(x).max() + np.abs(y).max())), 1e-7)
    _close("modulate vs float64", md.cpu().numpy().reshape(rows, dim),
           (1.0 + sc.astype(np.float64)) * xr + sh, 2e-6, 2e-7)
    ref = O.ref_kernels()
    if ref is not None:                      # the reference's own kernels, compiled from its sources
        rg = dx.clone()
        ref.ref_gelu(rg.data_ptr(), n, s)
        rb = dx.clone()
        ref.ref_bias_add(rb.data_ptr(), db.data_ptr(), rows, dim, s)
        rm = torch.empty_like(dx)
        ref.ref_apply_modulation(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), rm.data_ptr(), rows, dim, s)
        torch.cuda.synchronize()
        _close("gelu vs reference kernel", g.cpu().numpy(), rg.cpu().numpy(), 1e-6, 1e-7)
        assert torch.equal(ba, rb)
        _close("modulate vs reference kernel", md.cpu().numpy(), rm.cpu().numpy(), 1e-6, 1e-7)
