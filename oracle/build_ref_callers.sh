#!/usr/bin/env bash
# Compiles two of fluxrt-cpp's own test programs, unmodified and from where they lie, against this
# library's C++ mirror of the reference kernel layer (include/fxr_reference_api.h through the
# forwarding headers of include/fluxrt_dropin/) and links them with fluxrt-cpp_b200/lib/libfxr.so in
# place of the reference's kernels:
#   src/spike/test_spatial_cache.cu    SpatialCache: preprocess + output-cache merge / restore
#   src/spike/test_gather_scatter.cpp  gather_tokens, scatter_tokens, layer_norm_modulated
# The programs include their headers by relative paths ("../inference/...", "../utils/error.h"), so
# they are compiled inside a scratch tree (outside this repository) whose src/spike entries link to
# the reference files, src/inference to include/fluxrt_dropin/inference and src/utils to the
# reference's utils (the caller's own error.h, which the mirror then uses for fluxrt::RuntimeError).
# Binaries go to oracle/_ref/ (git-ignored, copied with the working tree; test_reference_callers.py
# runs them on a GPU). Reference sources: FXR_REFERENCE_ROOT, by default /root/reference.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
repo="$(dirname "$here")"
ref="${FXR_REFERENCE_ROOT:-/root/reference}"
if [[ ! -f "$ref/src/spike/test_spatial_cache.cu" ]]; then
  echo "reference sources not present ($ref): reference callers not built"
  exit 0
fi
lib="$repo/fluxrt-cpp_b200/lib"
[[ -f "$lib/libfxr.so" ]] || { echo "build fluxrt-cpp_b200/lib/libfxr.so first" >&2; exit 1; }
tree="$(mktemp -d /tmp/fxr_callers.XXXXXX)"
trap 'rm -rf "$tree"' EXIT
mkdir -p "$tree/src/spike"
ln -s "$ref/src/spike/test_spatial_cache.cu" "$tree/src/spike/test_spatial_cache.cu"
ln -s "$ref/src/spike/test_gather_scatter.cpp" "$tree/src/spike/test_gather_scatter.cpp"
ln -s "$repo/include/fluxrt_dropin/inference" "$tree/src/inference"
ln -s "$ref/src/utils" "$tree/src/utils"
out="${FXR_CALLERS_OUT:-$here/_ref}"
mkdir -p "$out"
inc=(-I"$tree/src" -I"$repo/include")
link=(-L"$lib" -lfxr -Xlinker -rpath -Xlinker '$ORIGIN/../../fluxrt-cpp_b200/lib' -Xlinker -rpath -Xlinker "$lib")
nvcc -gencode arch=compute_100a,code=sm_100a -O2 -std=c++17 "${inc[@]}" \
  "$tree/src/spike/test_spatial_cache.cu" "${link[@]}" -o "$out/ref_test_spatial_cache"
nvcc -Wno-deprecated-gpu-targets -O2 -std=c++17 "${inc[@]}" -x c++ "$tree/src/spike/test_gather_scatter.cpp" "${link[@]}" \
  -lcudart -o "$out/ref_test_gather_scatter"
echo "$out/ref_test_spatial_cache"
echo "$out/ref_test_gather_scatter"
