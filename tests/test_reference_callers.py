"""The reference's own C++ callers against this library (the drop-in claim of include/fxr_reference_api.h).

oracle/build_ref_callers.sh compiles two of fluxrt-cpp's test programs, unmodified, with their
headers resolved to this library's forwarding headers (include/fluxrt_dropin/) and the caller's own
src/utils/error.h, and links them with lib/libfxr.so alone:
  src/spike/test_spatial_cache.cu    SpatialCache preprocess, output-cache merge and restore
  src/spike/test_gather_scatter.cpp  gather_tokens, scatter_tokens, layer_norm_modulated
CPU: one translation unit holding the reference's error.h and the mirror compiles in either order
(fluxrt::RuntimeError is defined once), and the recipe builds both programs. GPU: the programs
built by build() run and report PASS."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("FXR_REFERENCE_ROOT", "/root/reference")
OUT = os.path.join(ROOT, "oracle", "_ref")
HAVE_REF = os.path.isfile(os.path.join(REF, "src", "utils", "error.h"))


@pytest.mark.skipif(not HAVE_REF, reason="reference sources not on this machine")
@pytest.mark.parametrize("order", ["error_first", "mirror_first"])
def test_mirror_and_reference_error_header_in_one_unit(tmp_path, order):
    inc = ['#include "utils/error.h"', '#include "inference/kernels/spatial_kv_cache.h"',
           '#include "inference/plugins/gather_scatter_kernels.h"',
           '#include "inference/plugins/flux2_kernels.h"', '#include "inference/plugins/attention_kernels.h"']
    if order == "mirror_first":
        inc = inc[1:] + inc[:1]
    src = tmp_path / "tu.cpp"
    src.write_text("\n".join(inc) + """
static void use(float* p, const int32_t* m) {
    fluxrt::kernels::SpatialCache c(4, 2, 4, 2, 2, 1, 1);
    c.preprocess_mask(const_cast<int32_t*>(m));
    fluxrt::plugins::layer_norm_modulated(p, p, nullptr, nullptr, 1e-6f, 2, 4, 0);
    fluxrt::plugins::launch_scale_add(p, p, p, 0.5f, 8, 0);
    fluxrt::plugins::apply_modulation(p, p, p, p, 2, 4, 0);
    fluxrt::plugins::launch_gelu(p, 8, 0);
    fluxrt::plugins::launch_bias_add(p, p, 2, 4, 0);
    fluxrt::plugins::launch_elem_add(p, p, p, 8, 0);
    throw fluxrt::RuntimeError("x");
}
int main() { (void)&use; return 0; }
""")
    # the reference's include root first, as its CMake build sets it (src/CMakeLists.txt:10-13), with
    # the drop-in headers standing in for its inference/ directory
    tree = tmp_path / "src"
    tree.mkdir()
    os.symlink(os.path.join(ROOT, "include", "fluxrt_dropin", "inference"), tree / "inference")
    os.symlink(os.path.join(REF, "src", "utils"), tree / "utils")
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I" + str(tree),
                        "-I" + os.path.join(ROOT, "include"), "-I/usr/local/cuda/include", str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


@pytest.mark.skipif(not HAVE_REF, reason="reference sources not on this machine")
def test_reference_callers_build_against_the_library(tmp_path):
    import build as B
    B.build()
    env = dict(os.environ, FXR_CALLERS_OUT=str(tmp_path))
    r = subprocess.run([os.path.join(ROOT, "oracle", "build_ref_callers.sh")], capture_output=True,
                       text=True, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    for exe in ("ref_test_spatial_cache", "ref_test_gather_scatter"):
        path = tmp_path / exe
        assert path.exists()
        ldd = subprocess.run(["ldd", str(path)], capture_output=True, text=True).stdout
        assert "libfxr.so" in ldd and "not found" not in ldd


@pytest.mark.gpu
@pytest.mark.parametrize("exe,expect", [
    ("ref_test_spatial_cache", ["Preprocess mask OK", "Initial output sync OK",
                                "correctly restored skipped tokens. PASS"]),
    ("ref_test_gather_scatter", ["gather_tokens: PASS", "scatter_tokens: PASS",
                                 "layer_norm_modulated: PASS", "All tests done"]),
])
def test_reference_callers_pass_on_the_gpu(cuda, exe, expect):
    path = os.path.join(OUT, exe)
    if not os.path.exists(path):
        pytest.skip(f"{exe} not built (reference sources absent where build() ran)")
    r = subprocess.run([path], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.stdout, r.stderr)
    for line in expect:
        assert line in r.stdout, r.stdout
    assert "FAIL" not in r.stdout
