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
FXR_ERR_BOUNDS = 7

FXR_F32, FXR_F16, FXR_BF16 = 0, 1, 2

# Every symbol include/fxr.h and include/fxr_plugin.h declare (checked by the CPU test suite).
EXPORTED = [
    "fxr_abi_version", "fxr_build_info", "fxr_last_error_string", "fxr_check_device_error",
    "fxr_workspace_size", "fxr_workspace_min_size", "fxr_workspace_views", "fxr_mask_compact", "fxr_preprocess_mask",
    "fxr_mark_updated", "fxr_gather_norm_rope", "fxr_attention_active", "fxr_restore_rows",
    "fxr_gather_rows", "fxr_scatter_rows", "fxr_kv_sync", "fxr_output_cache_sync",
    "fxr_rms_norm", "fxr_layer_norm_f32", "fxr_modulate_f32", "fxr_gelu_tanh_f32", "fxr_bias_add_f32",
    "fxr_add_f32", "fxr_scale_add_f32", "fxr_attention_f32_bhsd", "fxr_frame_forward", "fxr_frame_step", "fxr_frame_forward_noalloc",
    "fxr_frame_host_workspace_size", "fxr_frame_forward_host",
    "fxr_plugin_create", "fxr_plugin_clone", "fxr_plugin_destroy", "fxr_plugin_name",
    "fxr_plugin_version", "fxr_plugin_namespace", "fxr_plugin_fields", "fxr_plugin_output_desc",
    "fxr_plugin_supports", "fxr_plugin_configure", "fxr_plugin_workspace_size",
    "fxr_plugin_enqueue", "fxr_plugin_cache", "fxr_head_group_init", "fxr_frame_forward_heads",
    "fxr_head_group_wait", "fxr_ipc_alloc", "fxr_ipc_open", "fxr_ipc_close", "fxr_ipc_free",
    "fxr_nccl_unique_id", "fxr_nccl_comm_init", "fxr_nccl_comm_destroy",
    "fxr_heads_nccl_workspace_size", "fxr_allgather_heads", "fxr_frame_forward_heads_nccl",
    "fxr_batch_workspace_size", "fxr_frame_forward_batch", "fxr_qkv_project",
    "fxr_ln_modulate_rows", "fxr_rows_gemm_scratch_size", "fxr_rows_gemm",
    "fxr_double_block_workspace_size", "fxr_double_block_forward",
    "fxr_single_block_workspace_size", "fxr_single_block_forward",
    "fxr_block_host_workspace_size", "fxr_double_block_forward_host", "fxr_single_block_forward_host",
]

FXR_ACT_NONE, FXR_ACT_GELU_TANH = 0, 1

FXR_MAX_BATCH = 8

FXR_MAX_RANKS = 8

FXR_FIELD_FLOAT32, FXR_FIELD_INT32, FXR_FIELD_CHAR = 1, 3, 6
FXR_DTYPE_INT32 = 3


class FxrError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"fxr status {status}: {msg}")
        self.status = status


class RowsOperand(ctypes.Structure):
    """Mirror of fxr_rows_operand (include/fxr.h)."""
    _fields_ = [("rows", ctypes.c_void_p), ("ld", ctypes.c_int64), ("k", ctypes.c_int32),
                ("gathered", ctypes.c_int32), ("w", ctypes.c_void_p), ("ld_w", ctypes.c_int64)]


class RowsOutput(ctypes.Structure):
    """Mirror of fxr_rows_output (include/fxr.h)."""
    _fields_ = [("rows", ctypes.c_void_p), ("ld", ctypes.c_int64), ("cols", ctypes.c_int32),
                ("scattered", ctypes.c_int32), ("act", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class RowsGemmDesc(ctypes.Structure):
    """Mirror of fxr_rows_gemm_desc (include/fxr.h)."""
    _fields_ = [("dtype", ctypes.c_int32), ("n_tokens", ctypes.c_int32), ("row0", ctypes.c_int32),
                ("row_end", ctypes.c_int32), ("n_operands", ctypes.c_int32),
                ("n_outputs", ctypes.c_int32), ("a", RowsOperand * 2), ("y", RowsOutput * 4),
                ("bias0", ctypes.c_void_p), ("bias1", ctypes.c_void_p), ("residual", ctypes.c_void_p),
                ("ld_residual", ctypes.c_int64), ("gate", ctypes.c_void_p)]


class BlockStream(ctypes.Structure):
    """Mirror of fxr_block_stream (include/fxr.h)."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("shift", "scale", "gate", "w_qkv", "b_qkv", "norm_q",
                                                "norm_k", "w_out", "b_out", "w_mlp0", "b_mlp0",
                                                "w_mlp2", "b_mlp2")]


class DoubleBlock(ctypes.Structure):
    """Mirror of fxr_double_block (include/fxr.h)."""
    _fields_ = [("txt", BlockStream), ("img", BlockStream), ("mlp_hidden", ctypes.c_int32),
                ("ln_eps", ctypes.c_float)]


class SingleBlock(ctypes.Structure):
    """Mirror of fxr_single_block (include/fxr.h)."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("shift", "scale", "gate", "w_qkv_mlp", "b_qkv_mlp",
                                                "norm_q", "norm_k", "w_out", "b_out")] + \
        [("mlp_hidden", ctypes.c_int32), ("ln_eps", ctypes.c_float)]


class PluginField(ctypes.Structure):
    """Mirror of fxr_plugin_field (include/fxr_plugin.h)."""
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("type", ctypes.c_int32),
                ("length", ctypes.c_int32)]


class TensorDesc(ctypes.Structure):
    """Mirror of fxr_tensor_desc (include/fxr_plugin.h)."""
    _fields_ = [("nb_dims", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 8)]


class StreamFrame(ctypes.Structure):
    """Mirror of fxr_stream_frame (include/fxr.h)."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("q", "k", "v", "mask", "valid", "cache_k", "cache_v", "out")]


class HeadGroup(ctypes.Structure):
    """Mirror of fxr_head_group (include/fxr.h)."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("head0", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("ctas", ctypes.c_int32 * 8),
                ("epoch", ctypes.c_uint32), ("reserved0", ctypes.c_int32),
                ("out", ctypes.c_void_p * 8), ("arrive", ctypes.c_void_p * 8)]


class IpcHandle(ctypes.Structure):
    """Mirror of fxr_ipc_handle (include/fxr.h)."""
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


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
    L.fxr_workspace_min_size.argtypes = [ctypes.POINTER(FrameDesc)]
    L.fxr_workspace_min_size.restype = ctypes.c_size_t
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
        fn.argtypes = [_vp, _i64, _vp, _vp, _i32, _vp, _i64, _i64, _i32, _vp]
    L.fxr_kv_sync.argtypes = [_vp, _vp, _vp, _vp, _vp, _i32, _i64, _i32, _vp]
    L.fxr_output_cache_sync.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp]
    L.fxr_rms_norm.argtypes = [_vp, _vp, _vp, ctypes.c_float, _i64, _i32, _i32, _vp]
    L.fxr_frame_forward.argtypes = [ctypes.POINTER(FrameDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]
    L.fxr_frame_step.argtypes = [_i32, ctypes.POINTER(FrameDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]
    L.fxr_frame_forward_noalloc.argtypes = [ctypes.POINTER(FrameDesc)] + [_vp] * 12
    L.fxr_frame_host_workspace_size.argtypes = [ctypes.POINTER(FrameDesc)]
    L.fxr_frame_host_workspace_size.restype = ctypes.c_size_t
    L.fxr_frame_forward_host.argtypes = [ctypes.POINTER(FrameDesc)] + [_vp] * 12 + [ctypes.c_size_t, _vp]
    L.fxr_qkv_project.argtypes = [ctypes.POINTER(FrameDesc), _vp, _i64, _i32, _vp, _vp, _vp, _vp,
                                  _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]
    L.fxr_ln_modulate_rows.argtypes = [_i32, _vp, _i64, _i32, _vp, _vp, _i32, _i32, _i32, _vp, _vp,
                                       ctypes.c_float, _vp, _i64, _vp]
    L.fxr_rows_gemm_scratch_size.argtypes = []
    L.fxr_rows_gemm_scratch_size.restype = ctypes.c_size_t
    L.fxr_rows_gemm.argtypes = [ctypes.POINTER(RowsGemmDesc), _vp, _vp, _vp, ctypes.c_size_t, _vp]
    L.fxr_single_block_workspace_size.argtypes = [ctypes.POINTER(FrameDesc), _i32]
    L.fxr_single_block_workspace_size.restype = ctypes.c_size_t
    L.fxr_single_block_forward.argtypes = [ctypes.POINTER(FrameDesc), ctypes.POINTER(SingleBlock)] + \
        [_vp] * 8 + [ctypes.c_size_t, _vp]
    L.fxr_double_block_workspace_size.argtypes = [ctypes.POINTER(FrameDesc), _i32]
    L.fxr_double_block_workspace_size.restype = ctypes.c_size_t
    L.fxr_double_block_forward.argtypes = [ctypes.POINTER(FrameDesc), ctypes.POINTER(DoubleBlock)] + \
        [_vp] * 8 + [ctypes.c_size_t, _vp]
    L.fxr_double_block_forward_host.argtypes = L.fxr_double_block_forward.argtypes
    L.fxr_single_block_forward_host.argtypes = L.fxr_single_block_forward.argtypes
    L.fxr_block_host_workspace_size.argtypes = [ctypes.POINTER(FrameDesc), _i32]
    L.fxr_block_host_workspace_size.restype = ctypes.c_size_t
    L.fxr_batch_workspace_size.argtypes = [ctypes.POINTER(FrameDesc), _i32]
    L.fxr_batch_workspace_size.restype = ctypes.c_size_t
    L.fxr_frame_forward_batch.argtypes = [ctypes.POINTER(FrameDesc), _i32, ctypes.POINTER(StreamFrame),
                                          _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]
    _hg = ctypes.POINTER(HeadGroup)
    L.fxr_head_group_init.argtypes = [_hg, _i32, _i32, _i32, _i32]
    L.fxr_frame_forward_heads.argtypes = [ctypes.POINTER(FrameDesc), _hg] + [_vp] * 11 + \
        [ctypes.c_size_t, _vp]
    L.fxr_head_group_wait.argtypes = [_hg, _vp]
    L.fxr_nccl_unique_id.argtypes = [ctypes.c_char_p]
    L.fxr_nccl_comm_init.argtypes = [_i32, _i32, ctypes.c_char_p, ctypes.POINTER(_vp)]
    L.fxr_nccl_comm_destroy.argtypes = [_vp]
    L.fxr_heads_nccl_workspace_size.argtypes = [ctypes.POINTER(FrameDesc), _hg, _i32]
    L.fxr_heads_nccl_workspace_size.restype = ctypes.c_size_t
    L.fxr_allgather_heads.argtypes = [ctypes.POINTER(FrameDesc), _hg, _vp, _vp, _i32, _vp, _vp, _vp,
                                      _vp, _vp]
    L.fxr_frame_forward_heads_nccl.argtypes = [ctypes.POINTER(FrameDesc), _hg, _vp, _i32] + \
        [_vp] * 12 + [ctypes.c_size_t, _vp]
    L.fxr_ipc_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(_vp), ctypes.POINTER(IpcHandle)]
    L.fxr_ipc_open.argtypes = [ctypes.POINTER(IpcHandle), ctypes.POINTER(_vp)]
    L.fxr_ipc_close.argtypes = [_vp]
    L.fxr_ipc_free.argtypes = [_vp]
    L.fxr_mark_updated.argtypes = [_vp, _vp, _i32, _i32, _vp]
    L.fxr_attention_f32_bhsd.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp]
    _pf = ctypes.POINTER(PluginField)
    _pt = ctypes.POINTER(TensorDesc)
    L.fxr_plugin_create.argtypes = [_pf, _i32]
    L.fxr_plugin_create.restype = _vp
    L.fxr_plugin_clone.argtypes = [_vp]
    L.fxr_plugin_clone.restype = _vp
    L.fxr_plugin_destroy.argtypes = [_vp]
    L.fxr_plugin_destroy.restype = None
    for fn in (L.fxr_plugin_name, L.fxr_plugin_version, L.fxr_plugin_namespace):
        fn.restype = ctypes.c_char_p
    L.fxr_plugin_fields.argtypes = [_vp, _pf, _i32]
    L.fxr_plugin_output_desc.argtypes = [_vp, _pt, _i32, _pt, _i32]
    L.fxr_plugin_supports.argtypes = [_vp, _i32, _pt, _i32, _i32]
    L.fxr_plugin_configure.argtypes = [_vp, _pt, _i32, _pt, _i32]
    L.fxr_plugin_workspace_size.argtypes = [_vp, _pt, _i32]
    L.fxr_plugin_workspace_size.restype = ctypes.c_size_t
    L.fxr_plugin_enqueue.argtypes = [_vp, _pt, _pt, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp,
                                     ctypes.c_size_t, _vp]
    L.fxr_plugin_cache.argtypes = [_vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                   ctypes.POINTER(_vp)]
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


def workspace_min_size(cfg: FrameConfig) -> int:
    d = cfg.desc()
    return int(load().fxr_workspace_min_size(ctypes.byref(d)))


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


def gather_rows(src, idx, dst, count=None, host_count: int = -1, stream=None, n_index_rows=None):
    """dst[m] = src[idx[m]]; indices outside [0, n_index_rows) (default: src's rows) are skipped
    and reported by check_device_error as FXR_ERR_BOUNDS."""
    eb = src.element_size()
    n = src.shape[0] if n_index_rows is None else n_index_rows
    _check(load().fxr_gather_rows(_ptr(src), src.stride(0) * eb, _ptr(idx), _ptr(count), host_count,
                                  _ptr(dst), dst.stride(0) * eb, src[0].numel() * eb if src.dim() > 1 else eb,
                                  n, _stream(stream)))


def scatter_rows(src, idx, dst, count=None, host_count: int = -1, stream=None, n_index_rows=None):
    """dst[idx[m]] = src[m]; indices outside [0, n_index_rows) (default: dst's rows) are skipped
    and reported by check_device_error as FXR_ERR_BOUNDS."""
    eb = src.element_size()
    n = dst.shape[0] if n_index_rows is None else n_index_rows
    _check(load().fxr_scatter_rows(_ptr(src), src.stride(0) * eb, _ptr(idx), _ptr(count), host_count,
                                   _ptr(dst), dst.stride(0) * eb, dst[0].numel() * eb if dst.dim() > 1 else eb,
                                   n, _stream(stream)))


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


def frame_host_workspace_size(cfg: FrameConfig) -> int:
    d = cfg.desc()
    return int(load().fxr_frame_host_workspace_size(ctypes.byref(d)))


def frame_forward_host(cfg: FrameConfig, host_q, host_k, host_v, host_mask, valid, pos, norm_q, norm_k,
                       cache_k, cache_v, host_out, workspace, stream=None):
    """fxr_frame_forward_host: Q, K, V, mask and out are page-locked CPU tensors (pin_memory());
    only the executed rows cross PCIe. Asynchronous on `stream`."""
    d = cfg.desc()
    _check(load().fxr_frame_forward_host(ctypes.byref(d), _ptr(host_q), _ptr(host_k), _ptr(host_v),
                                         _ptr(host_mask), _ptr(valid), _ptr(pos), _ptr(norm_q),
                                         _ptr(norm_k), _ptr(cache_k), _ptr(cache_v), _ptr(host_out),
                                         _ptr(workspace), workspace.numel() * workspace.element_size(),
                                         _stream(stream)))


def frame_forward(cfg: FrameConfig, q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v,
                  out, workspace, stream=None):
    d = cfg.desc()
    _check(load().fxr_frame_forward(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(mask),
                                    _ptr(valid), _ptr(pos), _ptr(norm_q), _ptr(norm_k),
                                    _ptr(cache_k), _ptr(cache_v), _ptr(out), _ptr(workspace),
                                    workspace.numel() * workspace.element_size(), _stream(stream)))


# fxr_frame_step steps
STEP_COMPACT, STEP_GATHER, STEP_GATHER_COMPACT, STEP_ATTENTION, STEP_RESTORE = 0, 1, 2, 3, 4


def frame_step(step: int, cfg: FrameConfig, q, k, v, mask, valid, pos, norm_q, norm_k, cache_k, cache_v,
               out, workspace, stream=None):
    """One step of frame_forward on its workspace layout (fxr_frame_step)."""
    d = cfg.desc()
    _check(load().fxr_frame_step(step, ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(mask),
                                 _ptr(valid), _ptr(pos), _ptr(norm_q), _ptr(norm_k),
                                 _ptr(cache_k), _ptr(cache_v), _ptr(out), _ptr(workspace),
                                 workspace.numel() * workspace.element_size(), _stream(stream)))


def frame_forward_noalloc(cfg: FrameConfig, q, k, v, mask, valid, pos, norm_q, norm_k, cache_k,
                          cache_v, out, stream=None):
    d = cfg.desc()
    _check(load().fxr_frame_forward_noalloc(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(mask),
                                            _ptr(valid), _ptr(pos), _ptr(norm_q), _ptr(norm_k),
                                            _ptr(cache_k), _ptr(cache_v), _ptr(out),
                                            _stream(stream)))


def mark_updated(mask, valid, n_text: int, stream=None):
    _check(load().fxr_mark_updated(_ptr(mask), _ptr(valid), n_text, mask.numel(), _stream(stream)))


def attention_f32_bhsd(q, k, v, out, stream=None):
    """out = softmax(q k^T / sqrt(d)) v for fp32 [B, H, S, D] tensors (SIMT path)."""
    B, H, S, D = q.shape
    _check(load().fxr_attention_f32_bhsd(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, S,
                                         k.shape[2], D, _stream(stream)))


def tensor_desc(shape, dtype_code_: int) -> TensorDesc:
    t = TensorDesc()
    t.nb_dims = len(shape)
    t.dtype = dtype_code_
    for i, n in enumerate(shape):
        t.dims[i] = int(n)
    return t


def _tensor_code(t) -> int:
    import torch
    return FXR_DTYPE_INT32 if t.dtype == torch.int32 else dtype_code(t.dtype)


class SparseAttnPlugin:
    """Python handle on the plugin core of include/fxr_plugin.h (Flux2SparseAttnPlugin).

    Fields are given as keyword arguments: num_heads, head_dim, n_txt, layer_idx (int),
    rope_axes (sequence of 1-4 ints), rope_theta, eps (float).
    """

    _INT = ("num_heads", "head_dim", "n_txt", "layer_idx")
    _FLOAT = ("rope_theta", "eps")

    def __init__(self, _handle=None, **fields):
        L = load()
        if _handle is None:
            keep, arr = [], (PluginField * max(len(fields), 1))()
            for i, (name, val) in enumerate(fields.items()):
                if name == "rope_axes":
                    buf = (ctypes.c_int32 * len(val))(*val)
                    ftype, n = FXR_FIELD_INT32, len(val)
                elif name in self._FLOAT:
                    buf, ftype, n = (ctypes.c_float * 1)(val), FXR_FIELD_FLOAT32, 1
                else:
                    buf, ftype, n = (ctypes.c_int32 * 1)(val), FXR_FIELD_INT32, 1
                keep.append(buf)
                arr[i] = PluginField(name.encode(), ctypes.cast(buf, ctypes.c_void_p), ftype, n)
            _handle = L.fxr_plugin_create(arr, len(fields))
            if not _handle:
                raise FxrError(FXR_ERR_INVALID, L.fxr_last_error_string().decode())
        self._h = _handle
        self._L = L

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            self._L.fxr_plugin_destroy(h)

    def clone(self) -> "SparseAttnPlugin":
        return SparseAttnPlugin(_handle=self._L.fxr_plugin_clone(self._h))

    def fields(self) -> dict:
        n = self._L.fxr_plugin_fields(self._h, None, 0)
        arr = (PluginField * n)()
        self._L.fxr_plugin_fields(self._h, arr, n)
        out = {}
        for f in arr:
            if f.type == FXR_FIELD_FLOAT32:
                vals = list(ctypes.cast(f.data, ctypes.POINTER(ctypes.c_float))[:f.length])
            else:
                vals = list(ctypes.cast(f.data, ctypes.POINTER(ctypes.c_int32))[:f.length])
            out[f.name.decode()] = vals if f.name == b"rope_axes" else vals[0]
        return out

    @staticmethod
    def _descs(tensors):
        arr = (TensorDesc * len(tensors))()
        for i, t in enumerate(tensors):
            arr[i] = tensor_desc(t.shape, _tensor_code(t)) if not isinstance(t, TensorDesc) else t
        return arr

    def output_desc(self, inputs) -> TensorDesc:
        out = TensorDesc()
        _check_plugin(self._L.fxr_plugin_output_desc(self._h, self._descs(inputs), len(inputs),
                                                     ctypes.byref(out), 1))
        return out

    def supports(self, pos: int, io) -> bool:
        return self._L.fxr_plugin_supports(self._h, pos, self._descs(io), len(io) - 1, 1) == 1

    def configure(self, inputs, output=None):
        outs = self._descs([output]) if output is not None else None
        _check_plugin(self._L.fxr_plugin_configure(self._h, self._descs(inputs), len(inputs), outs,
                                                   1 if output is not None else 0))

    def workspace_size(self, inputs) -> int:
        return self._L.fxr_plugin_workspace_size(self._h, self._descs(inputs), len(inputs))

    def enqueue(self, inputs, output, workspace, stream=None):
        ins = self._descs(inputs)
        outd = self._descs([output])
        ptrs = (ctypes.c_void_p * len(inputs))(*[t.data_ptr() for t in inputs])
        optrs = (ctypes.c_void_p * 1)(output.data_ptr())
        _check_plugin(self._L.fxr_plugin_enqueue(self._h, ins, outd, ptrs, optrs, _ptr(workspace),
                                                 workspace.numel() * workspace.element_size(),
                                                 _stream(stream)))

    def cache(self, b: int):
        """Device pointers (cache_k, cache_v, valid) of edit stream b."""
        k, v, valid = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check_plugin(self._L.fxr_plugin_cache(self._h, b, ctypes.byref(k), ctypes.byref(v),
                                               ctypes.byref(valid)))
        return k.value, v.value, valid.value

    def cache_tensors(self, b: int, n_tokens: int, channels: int, dtype):
        """Torch views (no copy) of stream b's K cache [N, C], V cache [N, C] and valid [N]."""
        k, v, valid = self.cache(b)
        return (_device_view(k, (n_tokens, channels), "<u2").view(dtype),
                _device_view(v, (n_tokens, channels), "<u2").view(dtype),
                _device_view(valid, (n_tokens,), "|u1"))


def _device_view(ptr: int, shape, typestr: str):
    import torch

    class _Mem:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                    "data": (ptr, False), "version": 2}
    return torch.as_tensor(_Mem(), device="cuda")


def _check_plugin(status: int):
    if status != 0:
        raise FxrError(status, load().fxr_last_error_string().decode())


# ---- head-sharded frames ------------------------------------------------------------------------
def head_group(world: int, rank: int, n_heads: int, n_tokens: int) -> HeadGroup:
    """fxr_head_group_init: this rank's heads and every rank's attention CTA count."""
    g = HeadGroup()
    _check(load().fxr_head_group_init(ctypes.byref(g), world, rank, n_heads, n_tokens))
    return g


def frame_forward_heads(cfg: FrameConfig, g: HeadGroup, q, k, v, mask, valid, pos, norm_q, norm_k,
                        cache_k, cache_v, workspace, stream=None):
    """One frame of this rank's heads (cfg describes the full frame); see fxr_frame_forward_heads."""
    d = cfg.desc()
    _check(load().fxr_frame_forward_heads(ctypes.byref(d), ctypes.byref(g), _ptr(q), _ptr(k),
                                          _ptr(v), _ptr(mask), _ptr(valid), _ptr(pos),
                                          _ptr(norm_q), _ptr(norm_k), _ptr(cache_k),
                                          _ptr(cache_v), _ptr(workspace),
                                          workspace.numel() * workspace.element_size(),
                                          _stream(stream)))


def head_group_wait(g: HeadGroup, stream=None):
    _check(load().fxr_head_group_wait(ctypes.byref(g), _stream(stream)))


class IpcBuffer:
    """Zero-filled device memory of this process, shareable with the other processes of the node."""

    def __init__(self, nbytes: int):
        self.ptr = ctypes.c_void_p()
        self.handle = IpcHandle()
        _check(load().fxr_ipc_alloc(nbytes, ctypes.byref(self.ptr), ctypes.byref(self.handle)))
        self.nbytes = nbytes

    def handle_bytes(self) -> bytes:
        return bytes(self.handle.bytes)

    def free(self):
        if self.ptr:
            _check(load().fxr_ipc_free(self.ptr))
            self.ptr = ctypes.c_void_p()


def ipc_open(handle: bytes) -> int:
    h = IpcHandle()
    ctypes.memmove(h.bytes, handle, 64)
    p = ctypes.c_void_p()
    _check(load().fxr_ipc_open(ctypes.byref(h), ctypes.byref(p)))
    return p.value


def ipc_close(ptr: int):
    _check(load().fxr_ipc_close(ptr))


def device_view(ptr: int, shape, dtype):
    """Torch tensor over device memory this library allocated or mapped (no copy)."""
    import torch
    code = {torch.bfloat16: "<u2", torch.float16: "<u2", torch.int32: "<i4", torch.uint8: "|u1",
            torch.float32: "<f4"}[dtype]
    t = _device_view(ptr, shape, code)
    return t.view(dtype) if dtype in (torch.bfloat16, torch.float16) else t


# ---- NCCL variant of the head split -----------------------------------------------------------
def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(load().fxr_nccl_unique_id(buf))
    return buf.raw


def nccl_comm_init(world: int, rank: int, uid: bytes) -> int:
    comm = ctypes.c_void_p()
    _check(load().fxr_nccl_comm_init(world, rank, uid, ctypes.byref(comm)))
    return comm.value


def nccl_comm_destroy(comm: int):
    _check(load().fxr_nccl_comm_destroy(comm))


def heads_nccl_workspace_size(cfg: FrameConfig, g: HeadGroup, m_cap: int) -> int:
    d = cfg.desc()
    return load().fxr_heads_nccl_workspace_size(ctypes.byref(d), ctypes.byref(g), m_cap)


def frame_forward_heads_nccl(cfg: FrameConfig, g: HeadGroup, comm: int, m_cap: int, q, k, v, mask,
                             valid, pos, norm_q, norm_k, cache_k, cache_v, out, workspace,
                             stream=None):
    d = cfg.desc()
    _check(load().fxr_frame_forward_heads_nccl(
        ctypes.byref(d), ctypes.byref(g), comm, m_cap, _ptr(q), _ptr(k), _ptr(v), _ptr(mask),
        _ptr(valid), _ptr(pos), _ptr(norm_q), _ptr(norm_k), _ptr(cache_k), _ptr(cache_v),
        _ptr(out), _ptr(workspace), workspace.numel() * workspace.element_size(),
        _stream(stream)))


# ---- independent edit streams in one set of launches --------------------------------------------
def batch_workspace_size(cfg: FrameConfig, n_streams: int) -> int:
    d = cfg.desc()
    return load().fxr_batch_workspace_size(ctypes.byref(d), n_streams)


def frame_forward_batch(cfg: FrameConfig, streams, pos, norm_q, norm_k, workspace, stream=None):
    """streams: list of dicts with q, k, v, mask, valid (or None), cache_k, cache_v, out tensors."""
    d = cfg.desc()
    arr = (StreamFrame * max(len(streams), 1))()
    for b, f in enumerate(streams):
        arr[b] = StreamFrame(*[_ptr(f.get(k)) for k in ("q", "k", "v", "mask", "valid", "cache_k",
                                                         "cache_v", "out")])
    _check(load().fxr_frame_forward_batch(ctypes.byref(d), len(streams), arr, _ptr(pos), _ptr(norm_q),
                                          _ptr(norm_k), _ptr(workspace),
                                          workspace.numel() * workspace.element_size(),
                                          _stream(stream)))


def qkv_project(cfg: FrameConfig, hidden, w_qkv, bias, idx, count, q, k, v, scratch=None,
                stream=None):
    """q/k/v[idx[m]] = hidden[idx[m]] @ w_qkv.T (+ bias) for the executed rows (tcgen05 GEMM).
    scratch: a zeroed uint8 tensor of rows_gemm_scratch_size() bytes (stream-K), or None."""
    d = cfg.desc()
    _check(load().fxr_qkv_project(ctypes.byref(d), _ptr(hidden), hidden.stride(0), hidden.shape[1],
                                  _ptr(w_qkv), _ptr(bias), _ptr(idx), _ptr(count), _ptr(q), _ptr(k),
                                  _ptr(v), _ptr(scratch), scratch.numel() if scratch is not None else 0,
                                  _stream(stream)))


def rows_gemm_scratch_size() -> int:
    return int(load().fxr_rows_gemm_scratch_size())


def rows_gemm_scratch(device="cuda"):
    """A zeroed stream-K scratch area for rows_gemm (one per stream, reused as is)."""
    import torch
    return torch.zeros(rows_gemm_scratch_size(), dtype=torch.uint8, device=device)


def ln_modulate_rows(x, idx, count, y, scale=None, shift=None, eps=1e-6, row0=0, row_end=-1,
                     stream=None):
    """y[m] = (1 + scale) * LayerNorm(x[idx[m]]) + shift for compact rows m in [row0, row_end)."""
    _check(load().fxr_ln_modulate_rows(dtype_code(x.dtype), _ptr(x), x.stride(0), x.shape[1],
                                       _ptr(idx), _ptr(count), row0, row_end, x.shape[0],
                                       _ptr(scale), _ptr(shift), eps, _ptr(y), y.stride(0),
                                       _stream(stream)))


def rows_gemm(operands, outputs, idx, count, n_tokens, bias0=None, bias1=None, residual=None,
              gate=None, row0=0, row_end=-1, scratch=None, stream=None):
    """Executed-row GEMM (fxr_rows_gemm). operands: [(rows, w, gathered)] (1 or 2; rows [*, k],
    w [n_out, k]); outputs: [(rows, cols, scattered, act)] (1 to 4)."""
    d = RowsGemmDesc()
    d.dtype = dtype_code(operands[0][0].dtype)
    d.n_tokens = n_tokens
    d.row0, d.row_end = row0, row_end
    d.n_operands, d.n_outputs = len(operands), len(outputs)
    for i, (rows, w, gathered) in enumerate(operands):   # w may be a column block of a wider W
        d.a[i] = RowsOperand(_ptr(rows), rows.stride(0), w.shape[1], 1 if gathered else 0, _ptr(w),
                             w.stride(0))
    for i, (rows, cols, scattered, act) in enumerate(outputs):
        d.y[i] = RowsOutput(_ptr(rows), rows.stride(0), cols, 1 if scattered else 0, act, 0)
    d.bias0, d.bias1, d.gate = _ptr(bias0), _ptr(bias1), _ptr(gate)
    d.residual = _ptr(residual)
    d.ld_residual = residual.stride(0) if residual is not None else 0
    _check(load().fxr_rows_gemm(ctypes.byref(d), _ptr(idx), _ptr(count), _ptr(scratch),
                                scratch.numel() if scratch is not None else 0, _stream(stream)))


_BLOCK_FIELDS = ("shift", "scale", "gate", "w_qkv", "b_qkv", "norm_q", "norm_k", "w_out", "b_out",
                 "w_mlp0", "b_mlp0", "w_mlp2", "b_mlp2")


def block_stream(**tensors) -> BlockStream:
    """fxr_block_stream from device tensors (missing or None fields are NULL)."""
    bs = BlockStream()
    for n in _BLOCK_FIELDS:
        setattr(bs, n, _ptr(tensors.get(n)))
    return bs


def double_block_workspace_size(cfg: FrameConfig, mlp_hidden: int) -> int:
    d = cfg.desc()
    return int(load().fxr_double_block_workspace_size(ctypes.byref(d), mlp_hidden))


def block_host_workspace_size(cfg: FrameConfig, mlp_hidden: int) -> int:
    d = cfg.desc()
    return int(load().fxr_block_host_workspace_size(ctypes.byref(d), mlp_hidden))


def double_block_forward(cfg: FrameConfig, txt: dict, img: dict, mlp_hidden: int, x_in, x_out, mask,
                         valid, pos, cache_k, cache_v, workspace, ln_eps=1e-6, stream=None, host=False):
    """One double-stream block on the executed rows (fxr_double_block_forward). txt / img: dicts of
    the fxr_block_stream fields (device tensors). host=True: x_in, x_out and mask are page-locked CPU
    tensors (fxr_double_block_forward_host; workspace of block_host_workspace_size bytes)."""
    d = cfg.desc()
    blk = DoubleBlock(block_stream(**txt), block_stream(**img), mlp_hidden, ln_eps)
    fn = load().fxr_double_block_forward_host if host else load().fxr_double_block_forward
    _check(fn(ctypes.byref(d), ctypes.byref(blk), _ptr(x_in), _ptr(x_out), _ptr(mask), _ptr(valid),
              _ptr(pos), _ptr(cache_k), _ptr(cache_v), _ptr(workspace), workspace.numel(), _stream(stream)))


def single_block_workspace_size(cfg: FrameConfig, mlp_hidden: int) -> int:
    d = cfg.desc()
    return int(load().fxr_single_block_workspace_size(ctypes.byref(d), mlp_hidden))


def single_block_forward(cfg: FrameConfig, wts: dict, mlp_hidden: int, x_in, x_out, mask, valid, pos,
                         cache_k, cache_v, workspace, ln_eps=1e-6, stream=None, host=False):
    """One single-stream block on the executed rows (fxr_single_block_forward). wts: dict of the
    fxr_single_block weight fields (device tensors). host=True as for double_block_forward."""
    d = cfg.desc()
    blk = SingleBlock()
    for n in ("shift", "scale", "gate", "w_qkv_mlp", "b_qkv_mlp", "norm_q", "norm_k", "w_out", "b_out"):
        setattr(blk, n, _ptr(wts.get(n)))
    blk.mlp_hidden, blk.ln_eps = mlp_hidden, ln_eps
    fn = load().fxr_single_block_forward_host if host else load().fxr_single_block_forward
    _check(fn(ctypes.byref(d), ctypes.byref(blk), _ptr(x_in), _ptr(x_out), _ptr(mask), _ptr(valid),
              _ptr(pos), _ptr(cache_k), _ptr(cache_v), _ptr(workspace), workspace.numel(), _stream(stream)))
