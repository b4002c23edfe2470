"""Python host binding of the C ABI in include/fxr.h (ctypes over lib/libfxr.so).

Tensors are torch CUDA tensors (torch is used for device memory and streams only); every call goes
through the C ABI with raw device pointers and the current torch stream. There is no CPU fallback:
if the library or a GPU is missing, the calls raise.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libfxr.so")

FXR_OK = 0
FXR_ERR_INVALID = 1
FXR_ERR_CUDA = 2
FXR_ERR_TIMEOUT = 3
FXR_ERR_UNSUPPORTED = 4
FXR_ERR_WORKSPACE = 5
FXR_ERR_NCCL = 6

FXR_F32, FXR_F16, FXR_BF16 = 0, 1, 2

# Every symbol include/fxr.h declares (checked by the CPU test suite).
EXPORTED = [
    "fxr_abi_version", "fxr_build_info", "fxr_last_error_string", "fxr_check_device_error",
    "fxr_workspace_size", "fxr_workspace_views", "fxr_mask_compact", "fxr_preprocess_mask",
    "fxr_gather_norm_rope", "fxr_attention_active", "fxr_restore_rows", "fxr_gather_rows",
    "fxr_scatter_rows", "fxr_kv_sync", "fxr_output_cache_sync", "fxr_rms_norm",
    "fxr_frame_forward",
]


class FxrError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"fxr status {status}: {msg}")
        self.status = status


class FrameDesc(ctypes.Structure):
    """Mirror of fxr_frame_desc (include/fxr.h)."""
    _fields_ = [
        ("n_tokens", ctypes.c_int32),
        ("n_text", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("rope_n_axes", ctypes.c_int32),
        ("rope_axes_dim", ctypes.c_int32 * 4),
        ("rope_theta", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("softmax_scale", ctypes.c_float),
        ("reserved0", ctypes.c_int32),
        ("ld_qkv", ctypes.c_int64),
        ("ld_cache", ctypes.c_int64),
        ("ld_out", ctypes.c_int64),
    ]


_lib = None
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


def load(path: str | None = None) -> ctypes.CDLL:
    """Load lib/libfxr.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise FxrError(FXR_ERR_UNSUPPORTED, f"{path} missing: run fluxrt-cpp_b200/build.py")
    L = ctypes.CDLL(path)
    L.fxr_abi_version.restype = _i32
    L.fxr_build_info.restype = ctypes.c_char_p
    L.fxr_last_error_string.restype = ctypes.c_char_p
    L.fxr_check_device_error.argtypes = [_vp, ctypes.POINTER(ctypes.c_uint32)]
    L.fxr_workspace_size.argtypes = [ctypes.POINTER(FrameDesc)]
    L.fxr_workspace_size.restype = ctypes.c_size_t
    L.fxr_workspace_views.argtypes = [ctypes.POINTER(FrameDesc), _vp, ctypes.POINTER(_vp),
                                      ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                      ctypes.POINTER(_i64), ctypes.POINTER(_vp)]
    L.fxr_mask_compact.argtypes = [_vp, _vp, _i32, _vp, _vp, _vp]
    L.fxr_preprocess_mask.argtypes = [_vp, _vp, _i32, _vp]
    L.fxr_gather_norm_rope.argtypes = [ctypes.POINTER(FrameDesc), _vp, _vp, _vp, _vp, _vp, _vp,
                                       _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp]
    L.fxr_attention_active.argtypes = [ctypes.POINTER(FrameDesc), _vp, _i64, _vp, _vp, _vp, _vp,
                                       _vp, _vp]
    L.fxr_restore_rows.argtypes = [ctypes.POINTER(FrameDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp]
    for fn in (L.fxr_gather_rows, L.fxr_scatter_rows):
        fn.argtypes = [_vp, _i64, _vp, _vp, _i32, _vp, _i64, _i64, _vp]
    L.fxr_kv_sync.argtypes = [_vp, _vp, _vp, _vp, _vp, _i32, _i64, _i32, _vp]
    L.fxr_output_cache_sync.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp]
    L.fxr_rms_norm.argtypes = [_vp, _vp, _vp, ctypes.c_float, _i64, _i32, _i32, _vp]
    L.fxr_frame_forward.argtypes = [ctypes.POINTER(FrameDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]
    for name in EXPORTED:
        f = getattr(L, name)
        if f.restype is ctypes.c_int:  # default
            f.restype = _i32
    _lib = L
    return L


def _check(status: int):
    if status != FXR_OK:
        raise FxrError(status, load().fxr_last_error_string().decode())


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def dtype_code(torch_dtype) -> int:
    import torch
    return {torch.float32: FXR_F32, torch.float16: FXR_F16, torch.bfloat16: FXR_BF16}[torch_dtype]


@dataclass
class FrameConfig:
    n_tokens: int
    n_text: int
    n_heads: int = 24
    head_dim: int = 128
    dtype: str = "bf16"                  # "bf16" | "f16"
    rope_axes: tuple = (16, 56, 56)
    rope_theta: float = 10000.0
    eps: float = 1e-6
    softmax_scale: float = 0.0
    ld_qkv: int = 0
    ld_cache: int = 0
    ld_out: int = 0

    def desc(self) -> FrameDesc:
        d = FrameDesc()
        C = self.n_heads * self.head_dim
        d.n_tokens, d.n_text, d.n_heads, d.head_dim = self.n_tokens, self.n_text, self.n_heads, self.head_dim
        d.dtype = {"f32": FXR_F32, "f16": FXR_F16, "bf16": FXR_BF16}[self.dtype]
        d.rope_n_axes = len(self.rope_axes)
        for i, a in enumerate(self.rope_axes):
            d.rope_axes_dim[i] = a
        d.rope_theta, d.eps, d.softmax_scale = self.rope_theta, self.eps, self.softmax_scale
        d.ld_qkv = self.ld_qkv or C
        d.ld_cache = self.ld_cache or C
        d.ld_out = self.ld_out or C
        return d


def workspace_size(cfg: FrameConfig) -> int:
    d = cfg.desc()
    return int(load().fxr_workspace_size(ctypes.byref(d)))


def workspace_views(cfg: FrameConfig, ws):
    """(idx_ptr, count_ptr, qc_ptr, ld_qc, save_ptr) device addresses inside a workspace tensor."""
    d = cfg.desc()
    idx, cnt, qc, save = _vp(), _vp(), _vp(), _vp()
    ld = _i64()
    _check(load().fxr_workspace_views(ctypes.byref(d), ws.data_ptr(), ctypes.byref(idx),
                                      ctypes.byref(cnt), ctypes.byref(qc), ctypes.byref(ld),
                                      ctypes.byref(save)))
    return idx.value, cnt.value, qc.value, ld.value, save.value


def check_device_error(stream=None) -> int:
    w = ctypes.c_uint32(0)
    _check(load().fxr_check_device_error(_stream(stream), ctypes.byref(w)))
    return w.value


def mask_compact(mask, valid, idx, count, stream=None):
    n = mask.numel()
    _check(load().fxr_mask_compact(_ptr(mask), _ptr(valid), n, _ptr(idx), _ptr(count), _stream(stream)))


def preprocess_mask(mask, valid, stream=None):
    _check(load().fxr_preprocess_mask(_ptr(mask), _ptr(valid), mask.numel(), _stream(stream)))


def gather_norm_rope(cfg: FrameConfig, q, k, v, mask, idx, count, pos, norm_q, norm_k, qc,
                     cache_k, cache_v, save=None, stream=None):
    d = cfg.desc()
    _check(load().fxr_gather_norm_rope(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(mask),
                                       _ptr(idx), _ptr(count), _ptr(pos), _ptr(norm_q),
                                       _ptr(norm_k), _ptr(qc), qc.stride(0), _ptr(cache_k),
                                       _ptr(cache_v), _ptr(save), _stream(stream)))


def attention_active(cfg: FrameConfig, qc, count, cache_k, cache_v, idx, out, stream=None):
    d = cfg.desc()
    _check(load().fxr_attention_active(ctypes.byref(d), _ptr(qc), qc.stride(0), _ptr(count),
                                       _ptr(cache_k), _ptr(cache_v), _ptr(idx), _ptr(out),
                                       _stream(stream)))


def restore_rows(cfg: FrameConfig, mask, idx, count, save, cache_k, cache_v, stream=None):
    d = cfg.desc()
    _check(load().fxr_restore_rows(ctypes.byref(d), _ptr(mask), _ptr(idx), _ptr(count), _ptr(save),
                                   _ptr(cache_k), _ptr(cache_v), _stream(stream)))


def gather_rows(src, idx, dst, count=None, host_count: int = -1, stream=None):
    eb = src.element_size()
    _check(load().fxr_gather_rows(_ptr(src), src.stride(0) * eb, _ptr(idx), _ptr(count), host_count,
                                  _ptr(dst), dst.stride(0) * eb, src[0].numel() * eb if src.dim() > 1 else eb,
                                  _stream(stream)))


def scatter_rows(src, idx, dst, count=None, host_count: int = -1, stream=None):
    eb = src.element_size()
    _check(load().fxr_scatter_rows(_ptr(src), src.stride(0) * eb, _ptr(idx), _ptr(count), host_count,
                                   _ptr(dst), dst.stride(0) * eb, dst[0].numel() * eb if dst.dim() > 1 else eb,
                                   _stream(stream)))


def kv_sync(keys, values, cached_keys, cached_values, mask, stream=None):
    n = mask.numel()
    _check(load().fxr_kv_sync(_ptr(keys), _ptr(values), _ptr(cached_keys), _ptr(cached_values),
                              _ptr(mask), n, keys.numel() // max(n, 1), dtype_code(keys.dtype),
                              _stream(stream)))


def output_cache_sync(pred, cache, mask, valid, n_text: int, stream=None):
    n_image, ch = pred.shape
    _check(load().fxr_output_cache_sync(_ptr(pred), _ptr(cache), _ptr(mask), _ptr(valid), n_text,
                                        n_image, ch, dtype_code(pred.dtype), _stream(stream)))


def rms_norm(x, y, w, eps: float = 1e-6, stream=None):
    dim = x.shape[-1]
    _check(load().fxr_rms_norm(_ptr(x), _ptr(y), _ptr(w), eps, x.numel() // dim, dim,
                               dtype_code(x.dtype), _stream(stream)))


def frame_forward(cfg: FrameConfig, q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v,
                  out, workspace, stream=None):
    d = cfg.desc()
    _check(load().fxr_frame_forward(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(mask),
                                    _ptr(valid), _ptr(pos), _ptr(norm_q), _ptr(norm_k),
                                    _ptr(cache_k), _ptr(cache_v), _ptr(out), _ptr(workspace),
                                    workspace.numel() * workspace.element_size(), _stream(stream)))
