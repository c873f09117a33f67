#!/usr/bin/env bash
# Regenerates the MXFP4 golden vectors in this directory from CUTLASS 4.5.0's host code.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
CUTLASS="${CUTLASS:-$(python3 -c "import os,flashinfer;print(os.path.join(os.path.dirname(flashinfer.__file__),'data','cutlass','include'))")}"
CUDA="${CUDA:-/usr/local/cuda}"
TMP="$(mktemp -d)"
g++ -std=c++17 -O2 -o "$TMP/make_golden_mx" "$HERE/make_golden_mx.cpp" \
    -I"$CUTLASS" -I"$CUDA/include" 2> "$TMP/build.log" || { cat "$TMP/build.log"; exit 1; }
(cd "$HERE" && "$TMP/make_golden_mx")
rm -rf "$TMP"
echo "MX golden vectors written to $HERE"
