#!/usr/bin/env bash
# Builds the CPU oracle (test infrastructure) into oracle/_build/libfxr_oracle.so.
#   oracle/build_oracle.sh            portable build (x86-64-v3: AVX2 + FMA)
#   oracle/build_oracle.sh native     tuned for the host CPU (used for the timed CPU baseline)
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
out="$here/_build"
mkdir -p "$out"
arch="-march=x86-64-v3"
name="libfxr_oracle.so"
if [[ "${1:-}" == "native" ]]; then arch="-march=native"; name="libfxr_oracle_native.so"; fi
gcc -O3 $arch -fopenmp -fPIC -shared -std=c11 -Wall -Wextra -o "$out/$name.tmp" "$here/fxr_oracle.c" -lm
mv "$out/$name.tmp" "$out/$name"
echo "$out/$name"
