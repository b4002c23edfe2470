"""CPU tests of the oracle: pinned against the reference's known-answer tests (tests/golden) and
against independent torch fp32 evaluations; RoPE (parity unpinned) checked by its properties."""
import json
import math
import os

import numpy as np
import pytest
import torch

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "reference_kat.json")))


# ---------------------------------------------------------------------------------------------
# reference known answers (test_gather_scatter.cpp, test_spatial_cache.cu, test_spatial_cache_trt.cpp)
# ---------------------------------------------------------------------------------------------
def test_gather_known_answer():
    c = KAT["gather"]
    src = np.array(c["src"], dtype=np.float32).reshape(-1, c["dim"])
    got = O.gather_rows(src, np.array(c["indices"], dtype=np.int32))
    assert got.reshape(-1).tolist() == c["expected"]


def test_scatter_known_answer():
    c = KAT["scatter"]
    dst = np.full((c["seq_len"], c["dim"]), c["dst_init"], dtype=np.float32)
    src = np.array(c["src"], dtype=np.float32).reshape(-1, c["dim"])
    got = O.scatter_rows(src, np.array(c["indices"], dtype=np.int32), dst)
    assert got.reshape(-1).tolist() == c["expected"]


def test_spatial_cache_known_answer():
    c = KAT["cache"]
    n = c["img_len"] + c["txt_len"]
    valid = np.zeros(n, dtype=np.uint8)
    mask, _ = O.mask_compact(np.array(c["mask0"]), valid)
    assert mask.tolist() == c["mask0_expected"]
    pred = np.array(c["pred1"], dtype=np.float32).reshape(c["img_len"], c["out_ch"])
    cache = np.zeros_like(pred)
    pred, cache, valid = O.output_cache_sync(pred, cache, mask, valid, c["txt_len"])
    assert pred.reshape(-1).tolist() == c["pred1_expected"]
    mask2 = np.array(c["mask2"], dtype=np.int32)
    pred2 = np.array(c["pred2"], dtype=np.float32).reshape(c["img_len"], c["out_ch"])
    pred2, cache, valid = O.output_cache_sync(pred2, cache, mask2, valid, c["txt_len"])
    flat = pred2.reshape(-1)
    for k, v in c["pred2_checks"].items():
        assert flat[int(k)] == v


def test_spatial_cache_mixed_validity():
    c = KAT["cache_mixed"]
    t, i = c["txt_len"], c["img_len"]
    valid = np.zeros(t + i, dtype=np.uint8)
    mask, _ = O.mask_compact(np.zeros(t + i, dtype=np.int32), valid)
    assert mask.tolist() == c["after_reset_expected"]
    pred = np.ones((i, c["out_ch"]), dtype=np.float32)
    _, _, valid = O.output_cache_sync(pred, np.zeros_like(pred), np.array(c["populate_mask"]), valid, t)
    mask, idx = O.mask_compact(np.zeros(t + i, dtype=np.int32), valid)
    assert mask.tolist() == c["final_expected"]
    assert idx.tolist() == [k for k, m in enumerate(c["final_expected"]) if m != 0]


def test_kv_sync_semantics():
    rng = np.random.default_rng(3)
    n, e = 6, 4
    k, v, ck, cv = (rng.normal(size=(n, e)).astype(np.float32) for _ in range(4))
    mask = np.array([2, 2, 0, 1, 0, 2], dtype=np.int32)
    k2, v2, ck2, cv2 = O.kv_sync(k, v, ck, cv, mask)
    for r, m in enumerate(mask):
        assert np.array_equal(k2[r], k[r] if m else ck[r])
        assert np.array_equal(v2[r], v[r] if m else cv[r])
        assert np.array_equal(ck2[r], k[r] if m == 2 else ck[r])
        assert np.array_equal(cv2[r], v[r] if m == 2 else cv[r])


# ---------------------------------------------------------------------------------------------
# compaction properties
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("n", [0, 1, 31, 32, 33, 1536, 4608, 16896, 40000])
def test_compaction_properties(n):
    rng = np.random.default_rng(n)
    mask = rng.choice([0, 1, 2], size=n, p=[0.7, 0.1, 0.2]).astype(np.int32)
    valid = (rng.random(n) < 0.9).astype(np.uint8)
    m2, idx = O.mask_compact(mask, valid)
    exp_mask = np.where(valid == 0, 2, mask)
    assert np.array_equal(m2, exp_mask)
    assert np.array_equal(idx, np.nonzero(exp_mask)[0])


# ---------------------------------------------------------------------------------------------
# RMSNorm and attention against independent torch fp32 evaluations
# ---------------------------------------------------------------------------------------------
def test_rms_norm_vs_torch():
    rng = np.random.default_rng(7)
    x = rng.normal(size=(64, 128)).astype(np.float32)
    w = rng.normal(1.0, 0.1, size=128).astype(np.float32)
    got = O.rms_norm(x, w, 1e-6)
    xt = torch.from_numpy(x)
    ref = xt * torch.rsqrt(xt.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(w)
    np.testing.assert_allclose(got, ref.numpy(), rtol=2e-6, atol=2e-6)


def test_layer_norm_known_answer():
    c = KAT["layer_norm"]
    x = np.array(c["x"], dtype=np.float32).reshape(c["seq_len"], c["dim"])
    got = O.layer_norm_modulate(x, eps=c["eps"])
    for row in got:
        assert np.abs(row - np.array(c["expected_row"], dtype=np.float32)).max() <= c["tol"]


@pytest.mark.parametrize("rows,dim", [(1, 4), (33, 256), (8, 3072)])
def test_layer_norm_modulate_vs_torch(rows, dim):
    rng = np.random.default_rng(rows + dim)
    x = rng.normal(0.3, 2.0, size=(rows, dim)).astype(np.float32)
    sc = rng.normal(0, 0.1, size=dim).astype(np.float32)
    sh = rng.normal(0, 0.1, size=dim).astype(np.float32)
    got = O.layer_norm_modulate(x, sc, sh, 1e-6)
    ln = torch.nn.functional.layer_norm(torch.from_numpy(x).double(), (dim,), eps=1e-6)
    ref = (1 + torch.from_numpy(sc).double()) * ln + torch.from_numpy(sh).double()
    np.testing.assert_allclose(got, ref.numpy(), rtol=1e-6, atol=1e-6)
    # plain LayerNorm: the reference's gamma = beta = NULL call
    np.testing.assert_allclose(O.layer_norm_modulate(x, eps=1e-6), ln.numpy(), rtol=1e-6, atol=1e-6)


def test_gelu_tanh_vs_torch():
    x = np.linspace(-8, 8, 4001, dtype=np.float32)
    ref = torch.nn.functional.gelu(torch.from_numpy(x).double(), approximate="tanh").numpy()
    np.testing.assert_allclose(O.gelu_tanh(x), ref, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("rows,k,n,bias", [(1, 64, 3, True), (37, 130, 256, True), (5, 256, 17, False)])
def test_linear_vs_numpy_f64(rows, k, n, bias):
    rng = np.random.default_rng(rows * k + n)
    x = rng.normal(size=(rows, k)).astype(np.float32)
    w = rng.normal(size=(n, k)).astype(np.float32)
    b = rng.normal(size=n).astype(np.float32) if bias else None
    ref = x.astype(np.float64) @ w.astype(np.float64).T + (b.astype(np.float64) if bias else 0.0)
    np.testing.assert_allclose(O.linear(x, w, b), ref, rtol=1e-6, atol=1e-5)


def test_gated_residual():
    rng = np.random.default_rng(11)
    x, p = rng.normal(size=(2, 9, 16)).astype(np.float32)
    g = rng.normal(size=16).astype(np.float32)
    np.testing.assert_array_equal(O.gated_residual(x, p, g), x + g * p)
    np.testing.assert_array_equal(O.gated_residual(x, p), x + p)       # the reference's gate = 1.0


@pytest.mark.parametrize("M,N,H", [(1, 1, 1), (5, 37, 2), (130, 300, 3)])
def test_attention_vs_torch_sdpa(M, N, H):
    rng = np.random.default_rng(M * 1000 + N)
    D = 128
    q = rng.normal(size=(M, H * D)).astype(np.float32)
    k = rng.normal(size=(N, H * D)).astype(np.float32)
    v = rng.normal(size=(N, H * D)).astype(np.float32)
    got = O.attention(q, k, v, H, D)
    qt = torch.from_numpy(q).view(M, H, D).transpose(0, 1)
    kt = torch.from_numpy(k).view(N, H, D).transpose(0, 1)
    vt = torch.from_numpy(v).view(N, H, D).transpose(0, 1)
    ref = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt).transpose(0, 1).reshape(M, H * D)
    np.testing.assert_allclose(got, ref.numpy(), rtol=1e-5, atol=2e-6)


# ---------------------------------------------------------------------------------------------
# RoPE: parity unpinned, properties only
# ---------------------------------------------------------------------------------------------
AXES = [((16, 56, 56), 10000.0), ((32, 32, 32, 32), 2000.0)]


@pytest.mark.parametrize("axes,theta", AXES)
def test_rope_identity_at_origin(axes, theta):
    x = np.random.default_rng(0).normal(size=128).astype(np.float32)
    y = O.rope_row(x, [0] * len(axes), axes, theta)
    assert np.array_equal(x, y)


@pytest.mark.parametrize("axes,theta", AXES)
def test_rope_preserves_pair_norms(axes, theta):
    rng = np.random.default_rng(1)
    x = rng.normal(size=128).astype(np.float32)
    pos = rng.integers(0, 128, size=len(axes))
    y = O.rope_row(x, pos, axes, theta)
    nx = np.hypot(x[0::2], x[1::2])
    ny = np.hypot(y[0::2], y[1::2])
    np.testing.assert_allclose(nx, ny, rtol=1e-5)


@pytest.mark.parametrize("axes,theta", AXES)
def test_rope_relative_position(axes, theta):
    """<R(p)q, R(p')k> depends only on p - p' (the property RoPE exists for)."""
    rng = np.random.default_rng(2)
    q = rng.normal(size=128).astype(np.float32)
    k = rng.normal(size=128).astype(np.float32)
    na = len(axes)
    p1, p2 = rng.integers(0, 60, size=na), rng.integers(0, 60, size=na)
    shift = rng.integers(0, 60, size=na)
    a = float(np.dot(O.rope_row(q, p1, axes, theta).astype(np.float64), O.rope_row(k, p2, axes, theta)))
    b = float(np.dot(O.rope_row(q, p1 + shift, axes, theta).astype(np.float64),
                     O.rope_row(k, p2 + shift, axes, theta)))
    assert abs(a - b) < 1e-3 * (1 + abs(a))


def test_rope_hand_computed_pair():
    """Pair 0 of axis 1 (FLUX 16/56/56 layout) rotates by pos_h * theta^0 = pos_h radians."""
    x = np.zeros(128, dtype=np.float32)
    x[16], x[17] = 1.0, 0.0                      # first pair of axis 1 (columns 16, 17)
    y = O.rope_row(x, [0, 3, 0], (16, 56, 56), 10000.0)
    assert abs(y[16] - math.cos(3.0)) < 1e-6 and abs(y[17] - math.sin(3.0)) < 1e-6
    x2 = np.zeros(128, dtype=np.float32)
    x2[18] = 1.0                                  # second pair of axis 1: omega = 10000^(-2/56)
    y2 = O.rope_row(x2, [0, 5, 0], (16, 56, 56), 10000.0)
    ang = 5.0 * 10000.0 ** (-2.0 / 56.0)
    assert abs(y2[18] - math.cos(ang)) < 1e-6 and abs(y2[19] - math.sin(ang)) < 1e-6


# ---------------------------------------------------------------------------------------------
# frame invariants
# ---------------------------------------------------------------------------------------------
def _small_frame(seed=0, n_text=8, grid=(6, 5), H=2):
    rng = np.random.default_rng(seed)
    N, C = n_text + grid[0] * grid[1], H * 128
    f = lambda *s: rng.normal(size=s).astype(np.float32)
    mask = np.zeros(N, dtype=np.int32)
    mask[:n_text] = 2
    mask[n_text:] = rng.choice([0, 1, 2], size=N - n_text, p=[0.6, 0.2, 0.2])
    pos = np.zeros((N, 3), dtype=np.int32)
    hh, ww = np.meshgrid(np.arange(grid[0]), np.arange(grid[1]), indexing="ij")
    pos[n_text:, 1], pos[n_text:, 2] = hh.reshape(-1), ww.reshape(-1)
    return dict(q=f(N, C), k=f(N, C), v=f(N, C), mask=mask, pos=pos,
                norm_q=rng.normal(1, 0.1, 128).astype(np.float32),
                norm_k=rng.normal(1, 0.1, 128).astype(np.float32),
                cache_k=f(N, C), cache_v=f(N, C), out=f(N, C), H=H)


def test_frame_invariants():
    fr = _small_frame()
    H = fr["H"]
    r = O.frame_forward(fr["q"], fr["k"], fr["v"], fr["mask"], None, fr["pos"], fr["norm_q"],
                        fr["norm_k"], fr["cache_k"], fr["cache_v"], fr["out"], H, 128,
                        (16, 56, 56), 10000.0)
    mask = fr["mask"]
    exec_rows = np.nonzero(mask)[0]
    assert r["M"] == exec_rows.size and np.array_equal(r["idx"], exec_rows)
    skipped = mask == 0
    # skipped rows keep their previous output and cache bytes
    assert np.array_equal(r["out"][skipped], fr["out"][skipped])
    assert np.array_equal(r["cache_k"][skipped], fr["cache_k"][skipped])
    # mask==1 rows: executed, cache unchanged
    one = mask == 1
    assert np.array_equal(r["cache_k"][one], fr["cache_k"][one])
    assert np.array_equal(r["cache_v"][one], fr["cache_v"][one])
    # mask==2 rows: V cached bit-exactly, K cached as normed+roped
    two = mask == 2
    assert np.array_equal(r["cache_v"][two], fr["v"][two])
    i = int(np.nonzero(two)[0][0])
    k_head0 = O.rope_row(O.rms_norm(fr["k"][i, :128][None], fr["norm_k"])[0], fr["pos"][i], (16, 56, 56), 10000.0)
    np.testing.assert_allclose(r["cache_k"][i, :128], k_head0, rtol=1e-6, atol=1e-6)
    # executed outputs equal a direct attention over the merged K/V
    ak = fr["cache_k"].copy()
    ak[two] = r["cache_k"][two]
    # mask==1 rows use fresh K in attention although the cache keeps the old row
    for j in np.nonzero(one)[0]:
        ak[j] = np.concatenate([
            O.rope_row(O.rms_norm(fr["k"][j, h * 128:(h + 1) * 128][None], fr["norm_k"])[0], fr["pos"][j], (16, 56, 56), 10000.0)
            for h in range(H)])
    av = np.where(mask[:, None] != 0, fr["v"], fr["cache_v"])
    o = O.attention(r["qc"], ak, av, H, 128)
    np.testing.assert_allclose(r["out"][exec_rows], o, rtol=1e-5, atol=1e-5)
