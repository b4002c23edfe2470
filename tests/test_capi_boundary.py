"""CPU tests of the C-ABI boundary: the library builds and loads, exports every symbol the public
header declares, and rejects bad arguments before touching the GPU."""
import ctypes
import os
import re
import subprocess

import pytest

import fxr

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("fxr.h", "fxr_plugin.h")]


def _declared_symbols():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(fxr_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    import build as B
    B.build()
    return fxr.load()


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_symbols()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", fxr.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (fxr_[a-z0-9_]+)", out))
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    assert sorted(fxr.EXPORTED) == declared
    for s in declared:
        assert hasattr(lib, s)


def test_library_is_sm100a_only_and_self_contained(lib):
    out = subprocess.run(["ldd", fxr.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in out      # static runtime: nothing to resolve against torch's copy
    assert "libtorch" not in out and "libpython" not in out
    assert lib.fxr_abi_version() == 2


def test_frame_desc_layout_matches_header():
    # fxr_frame_desc: 10 int32 + 3 float + int32 reserved = 14*4 = 56 bytes, then 3 int64 -> 80
    assert ctypes.sizeof(fxr.FrameDesc) == 80
    assert fxr.FrameDesc.ld_qkv.offset == 56


def test_workspace_size_and_views(lib):
    cfg = fxr.FrameConfig(n_tokens=4608, n_text=512)
    n = fxr.workspace_size(cfg)
    C = 24 * 128
    assert n >= 4608 * 4 + 4608 * C * 2 * 3
    assert n % 256 == 0
    # the minimum leaves out only the optional split / stream-K slot area
    lo = fxr.workspace_min_size(cfg)
    assert 4608 * 4 + 4608 * C * 2 * 3 <= lo < n and lo % 256 == 0
    assert fxr.workspace_min_size(fxr.FrameConfig(n_tokens=16, n_text=4, dtype="f32", head_dim=0)) == 0


def test_status_codes_match_the_header():
    """Every FXR_ERR_* value of include/fxr.h is the binding's constant of the same name."""
    text = open(HEADERS[0]).read()
    body = text[text.index("typedef enum fxr_status"):text.index("} fxr_status;")]
    codes = dict((k, int(v)) for k, v in re.findall(r"\b(FXR_(?:OK|ERR_[A-Z_]+))\s*=\s*(\d+)", body))
    assert codes["FXR_ERR_BOUNDS"] == 7 and len(codes) == 8
    for name, value in codes.items():
        assert getattr(fxr, name) == value, name


def test_invalid_arguments_rejected_without_gpu(lib):
    d = fxr.FrameConfig(n_tokens=16, n_text=4, head_dim=64).desc()
    st = lib.fxr_attention_active(ctypes.byref(d), None, 0, None, None, None, None, None, None)
    assert st == fxr.FXR_ERR_UNSUPPORTED
    assert b"head_dim" in lib.fxr_last_error_string()
    d = fxr.FrameConfig(n_tokens=16, n_text=4).desc()
    d.rope_axes_dim[0] = 15
    st = lib.fxr_gather_norm_rope(ctypes.byref(d), *([None] * 10), 0, None, None, None, None)
    assert st == fxr.FXR_ERR_INVALID
    assert lib.fxr_mask_compact(None, None, -1, None, None, None) == fxr.FXR_ERR_INVALID
    d = fxr.FrameConfig(n_tokens=16, n_text=4).desc()
    st = lib.fxr_frame_forward(ctypes.byref(d), *([None] * 11), None, 0, None)
    assert st == fxr.FXR_ERR_INVALID
    assert lib.fxr_kv_sync(None, None, None, None, None, 4, 4, 7, None) == fxr.FXR_ERR_INVALID
    d = fxr.FrameConfig(n_tokens=16, n_text=4).desc()
    assert lib.fxr_frame_step(9, ctypes.byref(d), *([None] * 11), None, 0, None) == fxr.FXR_ERR_INVALID
    assert b"step" in lib.fxr_last_error_string()
    assert lib.fxr_frame_step(fxr.STEP_ATTENTION, ctypes.byref(d), *([None] * 11), None, 0, None) == fxr.FXR_ERR_INVALID


def test_frame_steps_match_the_header():
    """The FXR_STEP_* values of include/fxr.h are the binding's STEP_* constants."""
    text = open(HEADERS[0]).read()
    steps = dict((k, int(v)) for k, v in re.findall(r"\bFXR_STEP_([A-Z_]+)\s*=\s*(\d+)", text))
    assert steps == {"COMPACT": 0, "GATHER": 1, "GATHER_COMPACT": 2, "ATTENTION": 3, "RESTORE": 4}
    for name, value in steps.items():
        assert getattr(fxr, "STEP_" + name) == value, name


def test_product_path_has_no_cpu_fallback():
    """The product package never imports or links the oracle."""
    pkg = os.path.join(ROOT, "fluxrt-cpp_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                text = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in text.lower(), f


def test_batch_workspace_and_arguments(lib):
    cfg = fxr.FrameConfig(n_tokens=2816, n_text=512)
    one = fxr.batch_workspace_size(cfg, 1)
    assert one > 0 and fxr.batch_workspace_size(cfg, 8) == 8 * one
    assert fxr.batch_workspace_size(cfg, 20) == 8 * one          # groups of 8 reuse it
    assert fxr.batch_workspace_size(cfg, -1) == 0
    d = cfg.desc()
    assert lib.fxr_frame_forward_batch(ctypes.byref(d), 0, None, None, None, None, None, 0, None) == fxr.FXR_OK
    st = lib.fxr_frame_forward_batch(ctypes.byref(d), 2, None, None, None, None, None, 0, None)
    assert st == fxr.FXR_ERR_INVALID


def test_compaction_row_owner_by_multiply_is_exact():
    """The compacting gather finds the CTA that owns launch row g (g mod grid) and the row's slot
    (g div grid) with q = umulhi(g, ceil(2^32 / grid)) instead of a division (compact_into_list in
    fxr_mem_kernels.cuh, the constant from launch_gather_streams in fxr_capi.cu). Restated here for
    every grid up to 256 CTAs and every row a compacting launch can hold (fewer than 1024 x grid):
    the quotient equals the integer division, as the bound g x grid < 2^32 guarantees."""
    import numpy as np
    for grid in range(2, 257):
        magic = ((1 << 32) + grid - 1) // grid
        g = np.arange(0, 1024 * grid, dtype=np.uint64)
        q = (g * np.uint64(magic)) >> np.uint64(32)
        assert np.array_equal(q, g // np.uint64(grid)), grid
        assert 1024 * grid * grid < (1 << 32)
