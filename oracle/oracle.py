"""ctypes bindings of the CPU oracle (oracle/fxr_oracle.c) plus numpy storage helpers.

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke check and the CPU-baseline leg of
bench.py, never by the product path. RoPE parity is unpinned (the reference has no RoPE code);
see fxr_oracle.h for what each function restates and how it is pinned.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_BUILD = os.path.join(_HERE, "_build")

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


def build(native: bool = False) -> str:
    """Compile the oracle shared library and return its path."""
    args = [os.path.join(_HERE, "build_oracle.sh")] + (["native"] if native else [])
    out = subprocess.run(args, check=True, capture_output=True, text=True)
    return out.stdout.strip().splitlines()[-1]


_libs: dict[bool, ctypes.CDLL] = {}


def lib(native: bool = False) -> ctypes.CDLL:
    """Load (building on first use) the oracle library."""
    if native in _libs:
        return _libs[native]
    name = "libfxr_oracle_native.so" if native else "libfxr_oracle.so"
    path = os.path.join(_BUILD, name)
    src = os.path.join(_HERE, "fxr_oracle.c")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        try:
            path = build(native)
        except (OSError, subprocess.CalledProcessError):
            if not os.path.exists(path):
                raise
    L = ctypes.CDLL(path)
    L.fxo_set_threads.argtypes = [ctypes.c_int]
    L.fxo_set_threads.restype = ctypes.c_int
    L.fxo_mask_compact.argtypes = [_i32p, _u8p, _i32, _i32p]
    L.fxo_mask_compact.restype = _i32
    for fn in (L.fxo_gather_rows, L.fxo_scatter_rows):
        fn.argtypes = [_vp, _i64, _i32p, _i32, _vp, _i64, _i64]
        fn.restype = None
    L.fxo_rms_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_float, _i64, _i32]
    L.fxo_rope_row.argtypes = [_f32p, _i32, _i32p, _i32, _i32p, ctypes.c_float]
    L.fxo_norm_rope_rows.argtypes = [_f32p, _i64, _i32p, _i32, _i32p, _i32, _i32p, ctypes.c_float,
                                     _f32p, ctypes.c_float, _i32, _i32, _f32p, _i64]
    L.fxo_norm_rope_rows.restype = None
    L.fxo_attention.argtypes = [_f32p, _i64, _i32, _f32p, _f32p, _i64, _i32, _i32, _i32,
                                ctypes.c_float, _f32p, _i64]
    L.fxo_kv_sync.argtypes = [_f32p, _f32p, _f32p, _f32p, _i32p, _i32, _i64]
    L.fxo_output_cache_sync.argtypes = [_f32p, _f32p, _i32p, _u8p, _i32, _i32, _i32]
    L.fxo_layer_norm_modulate.argtypes = [_f32p, _i64, _f32p, _f32p, _f32p, ctypes.c_float, _i64, _i32]
    L.fxo_gelu_tanh.argtypes = [_f32p, _i64]
    L.fxo_linear.argtypes = [_f32p, _i64, _i64, _i32, _f32p, _f32p, _f32p, _i32]
    L.fxo_gated_residual.argtypes = [_f32p, _i64, _f32p, _f32p, _f32p, _i64, _i32]
    for fn in (L.fxo_layer_norm_modulate, L.fxo_gelu_tanh, L.fxo_linear, L.fxo_gated_residual):
        fn.restype = None
    L.fxo_frame_forward.argtypes = [_f32p, _f32p, _f32p, _i32p, _u8p, _i32p, _f32p, _f32p,
                                    _f32p, _f32p, _f32p, _f32p, _i32p,
                                    _i32, _i32, _i32, _i32, _i32p, ctypes.c_float,
                                    ctypes.c_float, ctypes.c_float]
    L.fxo_frame_forward.restype = _i32
    _libs[native] = L
    return L


def _p(a: np.ndarray | None, t):
    if a is None:
        return ctypes.cast(None, t)
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(t)


def set_threads(n: int = 0, native: bool = False) -> int:
    return lib(native).fxo_set_threads(n)


# ---------------------------------------------------------------------------------------------
# numpy storage helpers: exact fp16 / bf16 round trips (round to nearest even)
# ---------------------------------------------------------------------------------------------
def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even; NaN stays NaN."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rnd = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rnd) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_storage(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to the storage dtype and back to fp32 (exactly representable)."""
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(to_bf16_bits(x))
    raise ValueError(dtype)


def storage_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 values (already representable) -> raw storage array (uint16 bits or float32)."""
    if dtype == "f32":
        return np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "f16":
        return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return to_bf16_bits(x)
    raise ValueError(dtype)


def bits_to_f32(b: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return np.asarray(b).view(np.float32)
    if dtype == "f16":
        return np.asarray(b).view(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(np.asarray(b).view(np.uint16))
    raise ValueError(dtype)


# ---------------------------------------------------------------------------------------------
# wrappers
# ---------------------------------------------------------------------------------------------
def mask_compact(mask: np.ndarray, valid: np.ndarray | None = None):
    mask = np.ascontiguousarray(mask, dtype=np.int32).copy()
    idx = np.zeros(max(1, mask.size), dtype=np.int32)
    v = None if valid is None else np.ascontiguousarray(valid, dtype=np.uint8)
    m = lib().fxo_mask_compact(_p(mask, _i32p), _p(v, _u8p), mask.size, _p(idx, _i32p))
    return mask, idx[:m].copy()


def gather_rows(src: np.ndarray, idx: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(src)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    row = src.strides[0]
    dst = np.empty((idx.size,) + src.shape[1:], dtype=src.dtype)
    lib().fxo_gather_rows(src.ctypes.data, row, _p(idx, _i32p), idx.size, dst.ctypes.data, row, row)
    return dst


def scatter_rows(src: np.ndarray, idx: np.ndarray, dst: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(src)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    out = np.ascontiguousarray(dst).copy()
    row = out.strides[0]
    lib().fxo_scatter_rows(src.ctypes.data, src.strides[0] if src.ndim > 1 else row,
                           _p(idx, _i32p), idx.size, out.ctypes.data, row, row)
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    dim = x.shape[-1]
    lib().fxo_rms_norm(_p(x, _f32p), _p(y, _f32p), _p(w, _f32p), eps, x.size // dim, dim)
    return y


def rope_row(x: np.ndarray, pos, axes_dim, theta: float) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    p = np.ascontiguousarray(pos, dtype=np.int32)
    a = np.ascontiguousarray(axes_dim, dtype=np.int32)
    lib().fxo_rope_row(_p(y, _f32p), y.size, _p(p, _i32p), a.size, _p(a, _i32p), theta)
    return y


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, n_heads: int, head_dim: int,
              scale: float = 0.0) -> np.ndarray:
    """q [M, C], k/v [N, C] fp32 -> o [M, C]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    M, C = q.shape
    o = np.zeros((M, C), dtype=np.float32)
    lib().fxo_attention(_p(q, _f32p), C, M, _p(k, _f32p), _p(v, _f32p), k.shape[1], k.shape[0],
                        n_heads, head_dim, scale, _p(o, _f32p), C)
    return o


def norm_rope_rows(x: np.ndarray, idx: np.ndarray, pos: np.ndarray, w: np.ndarray, n_heads: int,
                   head_dim: int, axes_dim, theta: float, eps: float = 1e-6) -> np.ndarray:
    """RMSNorm + RoPE of rows x[idx], every head -> [len(idx), n_heads * head_dim] fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    ax = np.ascontiguousarray(axes_dim, dtype=np.int32)
    C = n_heads * head_dim
    y = np.zeros((idx.size, C), dtype=np.float32)
    if idx.size:
        lib().fxo_norm_rope_rows(_p(x, _f32p), x.shape[1], _p(idx, _i32p), idx.size, _p(pos, _i32p),
                                 ax.size, _p(ax, _i32p), theta, _p(w, _f32p), eps, n_heads, head_dim,
                                 _p(y, _f32p), C)
    return y


def frame_operands(q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v, n_heads: int,
                   head_dim: int, axes_dim, theta: float, operand_dtype: str = "f32",
                   eps: float = 1e-6) -> dict:
    """The attention operands of one frame as the CUDA path stores them: mask protocol and
    compaction, normed + roped Q' (compact) and K' of the executed rows rounded to `operand_dtype`
    ("f32" = unrounded), attention K/V = cache rows with the executed rows replaced by K' / V
    (spatial_kv_cache.cu:64-67). Returns mask, idx, qc [M, C], keys, values [N, C] (fp32 arrays
    holding the rounded values)."""
    mask, idx = mask_compact(mask, valid)
    qc = round_storage(norm_rope_rows(q, idx, pos, norm_q, n_heads, head_dim, axes_dim, theta, eps),
                       operand_dtype)
    kn = round_storage(norm_rope_rows(k, idx, pos, norm_k, n_heads, head_dim, axes_dim, theta, eps),
                       operand_dtype)
    keys = np.array(cache_k, dtype=np.float32, copy=True)
    values = np.array(cache_v, dtype=np.float32, copy=True)
    keys[idx] = kn
    values[idx] = np.asarray(v, dtype=np.float32)[idx]
    return {"mask": mask, "idx": idx, "qc": qc, "keys": keys, "values": values}


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def layer_norm_modulate(x: np.ndarray, scale=None, shift=None, eps: float = 1e-6) -> np.ndarray:
    """LayerNorm without affine weights, then (1 + scale) * . + shift; x [rows, dim]."""
    x = _f32(x)
    rows, dim = x.shape
    sc, sh = _f32(scale), _f32(shift)
    y = np.empty_like(x)
    lib().fxo_layer_norm_modulate(_p(x, _f32p), dim, _p(y, _f32p), _p(sc, _f32p), _p(sh, _f32p),
                                  eps, rows, dim)
    return y


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    y = _f32(x).copy()
    lib().fxo_gelu_tanh(_p(y, _f32p), y.size)
    return y


def linear(x: np.ndarray, w: np.ndarray, b=None) -> np.ndarray:
    """y = x W^T + b; x [rows, k], W [n, k]."""
    x, w, b = _f32(x), _f32(w), _f32(b)
    rows, k = x.shape
    n = w.shape[0]
    assert w.shape[1] == k and (b is None or b.size == n)
    y = np.empty((rows, n), dtype=np.float32)
    lib().fxo_linear(_p(x, _f32p), k, rows, k, _p(w, _f32p), _p(b, _f32p), _p(y, _f32p), n)
    return y


def gated_residual(x: np.ndarray, proj: np.ndarray, gate=None) -> np.ndarray:
    """x + gate * proj (gate per channel, None = 1.0)."""
    x, proj, gate = _f32(x), _f32(proj), _f32(gate)
    rows, dim = x.shape
    out = np.empty_like(proj)
    lib().fxo_gated_residual(_p(x, _f32p), dim, _p(gate, _f32p), _p(proj, _f32p), _p(out, _f32p),
                             rows, dim)
    return out


def kv_sync(keys, values, cached_keys, cached_values, mask):
    keys = np.ascontiguousarray(keys, dtype=np.float32).copy()
    values = np.ascontiguousarray(values, dtype=np.float32).copy()
    ck = np.ascontiguousarray(cached_keys, dtype=np.float32).copy()
    cv = np.ascontiguousarray(cached_values, dtype=np.float32).copy()
    mask = np.ascontiguousarray(mask, dtype=np.int32)
    n = mask.size
    lib().fxo_kv_sync(_p(keys, _f32p), _p(values, _f32p), _p(ck, _f32p), _p(cv, _f32p),
                      _p(mask, _i32p), n, keys.size // n)
    return keys, values, ck, cv


def output_cache_sync(pred, cache, mask, valid, n_text: int):
    pred = np.ascontiguousarray(pred, dtype=np.float32).copy()
    cache = np.ascontiguousarray(cache, dtype=np.float32).copy()
    valid = np.ascontiguousarray(valid, dtype=np.uint8).copy()
    mask = np.ascontiguousarray(mask, dtype=np.int32)
    n_image, ch = pred.shape
    lib().fxo_output_cache_sync(_p(pred, _f32p), _p(cache, _f32p), _p(mask, _i32p),
                                _p(valid, _u8p), n_text, n_image, ch)
    return pred, cache, valid


def frame_forward(q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v, out,
                  n_heads: int, head_dim: int, axes_dim, theta: float, eps: float = 1e-6,
                  scale: float = 0.0):
    """fp32 frame of the sparse attention slice; returns a dict with every output."""
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32).copy()
    q, k, v = f(q), f(k), f(v)
    ck, cv, o = f(cache_k), f(cache_v), f(out)
    nq, nk = f(norm_q), f(norm_k)
    mask = np.ascontiguousarray(mask, dtype=np.int32).copy()
    vd = None if valid is None else np.ascontiguousarray(valid, dtype=np.uint8)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    ax = np.ascontiguousarray(axes_dim, dtype=np.int32)
    N = mask.size
    qc = np.zeros_like(q)
    idx = np.zeros(max(N, 1), dtype=np.int32)
    M = lib().fxo_frame_forward(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), _p(mask, _i32p),
                                _p(vd, _u8p), _p(pos, _i32p), _p(nq, _f32p), _p(nk, _f32p),
                                _p(ck, _f32p), _p(cv, _f32p), _p(o, _f32p), _p(qc, _f32p),
                                _p(idx, _i32p), N, n_heads, head_dim, ax.size, _p(ax, _i32p),
                                theta, eps, scale)
    return {"M": int(M), "mask": mask, "idx": idx[:M].copy(), "qc": qc[:M].copy(),
            "cache_k": ck, "cache_v": cv, "out": o}


# ---------------------------------------------------------------------------------------------
# The reference's own CUDA kernels (oracle/_ref/libfxr_refkernels.so, built from the reference
# sources by oracle/build_ref.sh). Test infrastructure: a bit-exact cross-check of the copy and
# cache steps and a timing baseline on the GPU. Arguments are device pointers (ints).
# ---------------------------------------------------------------------------------------------
REF_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libfxr_refkernels.so")
_ref_lib = None


def ref_kernels():
    """ctypes handle on the reference kernels, or None when they were not built."""
    global _ref_lib
    if _ref_lib is not None:
        return _ref_lib
    if not os.path.exists(REF_LIB_PATH):
        return None
    L = ctypes.CDLL(REF_LIB_PATH)
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    for f in (L.ref_gather_tokens, L.ref_scatter_tokens):
        f.argtypes = [vp, vp, vp, i32, i32, vp]
        f.restype = None
    L.ref_gelu.argtypes = [vp, i32, vp]
    L.ref_gelu.restype = None
    L.ref_bias_add.argtypes = [vp, vp, i32, i32, vp]
    L.ref_bias_add.restype = None
    L.ref_apply_modulation.argtypes = [vp, vp, vp, vp, i32, i32, vp]
    L.ref_apply_modulation.restype = None
    L.ref_rms_norm.argtypes = [vp, vp, vp, ctypes.c_float, i32, i32, vp]
    L.ref_rms_norm.restype = None
    L.ref_attention_fwd.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]
    L.ref_attention_fwd.restype = None
    L.ref_cache_create.argtypes = [ctypes.c_int] * 7
    L.ref_cache_create.restype = vp
    L.ref_cache_destroy.argtypes = [vp]
    L.ref_cache_destroy.restype = None
    L.ref_cache_reset.argtypes = [vp, vp]
    L.ref_cache_preprocess_mask.argtypes = [vp, vp, vp]
    L.ref_cache_sync_output.argtypes = [vp, vp, vp, vp]
    L.ref_cache_sync_kv.argtypes = [vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, vp]
    _ref_lib = L
    return L


def dense_block_sample(n_tokens: int, n_heads: int, head_dim: int, mlp_hidden: int, seed: int,
                       rows: int = 256) -> dict:
    """The reference double block's fp32 math timed on the host cores as the reference runs it,
    densely on every token (flux2_double_block_plugin.cpp:330-460): LayerNorm and Q/K/V of all N
    tokens, then QK-RMSNorm, attention, the tanh-GELU MLP and the out-projection of a sample of
    `rows` query tokens over all N keys, scaled to N rows. numpy BLAS on seeded random data; the CPU
    baseline of the block benchmark, not a checker. Returns seconds per frame."""
    import time
    rng = np.random.default_rng(seed)
    N, C, D, H = n_tokens, n_heads * head_dim, head_dim, mlp_hidden
    f = lambda *shape, sd=1.0: (rng.standard_normal(shape, dtype=np.float32) * sd)
    x = f(N, C)
    wq, wo, w0, w2 = f(3 * C, C, sd=C ** -0.5), f(C, C, sd=C ** -0.5), f(H, C, sd=C ** -0.5), f(C, H, sd=H ** -0.5)
    t0 = time.perf_counter()
    mean = x.mean(1, keepdims=True)
    xn = (x - mean) / np.sqrt(((x - mean) ** 2).mean(1, keepdims=True) + 1e-6)
    qkv = xn @ wq.T
    t_all = time.perf_counter() - t0
    sel = rng.choice(N, size=rows, replace=False)
    t1 = time.perf_counter()
    q = qkv[sel, :C].reshape(rows, n_heads, D)
    k = qkv[:, C:2 * C].reshape(N, n_heads, D)
    v = qkv[:, 2 * C:].reshape(N, n_heads, D)
    q = q / np.sqrt((q ** 2).mean(-1, keepdims=True) + 1e-6)
    k = k / np.sqrt((k ** 2).mean(-1, keepdims=True) + 1e-6)
    o = np.empty((rows, n_heads, D), np.float32)
    for h in range(n_heads):
        s = (q[:, h] @ k[:, h].T) / np.sqrt(D)
        s = np.exp(s - s.max(1, keepdims=True))
        o[:, h] = (s / s.sum(1, keepdims=True)) @ v[:, h]
    hh = xn[sel] @ w0.T
    hh = 0.5 * hh * (1 + np.tanh(0.7978845608 * (hh + 0.044715 * hh ** 3)))
    _ = x[sel] + o.reshape(rows, C) @ wo.T + hh @ w2.T
    t_rows = time.perf_counter() - t1
    return {"seconds_per_frame": t_all + t_rows * N / rows, "rows": rows}
