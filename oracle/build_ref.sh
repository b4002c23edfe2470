#!/usr/bin/env bash
# Compiles fluxrt-cpp's own CUDA kernels for sm_100a from the reference sources, where they lie
# (FXR_REFERENCE_ROOT, by default the read-only checkout at /root/reference), together with
# oracle/ref_shim.cu, into oracle/_ref/libfxr_refkernels.so. The .so is git-ignored and copied with
# the working tree; machines without the reference sources skip this step and use that copy.
# No reference source is copied into this repository. The reference's TensorRT plugin classes are
# not built: NvInferRuntime.h is absent.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
ref="${FXR_REFERENCE_ROOT:-/root/reference}"
src="$ref/src/inference"
if [[ ! -d "$src" ]]; then
  echo "reference sources not present ($ref): oracle/_ref not built"
  exit 0
fi
out="$here/_ref"
mkdir -p "$out"
nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Xcompiler -fPIC -shared \
  -I"$src/plugins" -I"$src/kernels" -I"$ref/src" \
  "$src/plugins/gather_scatter_kernels.cu" "$src/plugins/flux2_kernels.cu" \
  "$src/plugins/attention_kernels.cu" "$src/kernels/spatial_kv_cache.cu" \
  "$here/ref_shim.cu" -o "$out/libfxr_refkernels.so.tmp"
mv "$out/libfxr_refkernels.so.tmp" "$out/libfxr_refkernels.so"
echo "$out/libfxr_refkernels.so"
