#!/usr/bin/env bash
# Regenerates the golden vectors in this directory from the reference's own code:
# the reference header (host part) and the CUTLASS 4.5.0 host converters it calls.
# Needs the reference tree (REF=<dir>, default a directory named "reference" next to this
# repository) and CUTLASS headers; run from any directory.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${REF:-$(cd "$HERE/../../.." && pwd)/reference}"
[ -d "$REF/include/blackhole" ] || { echo "reference tree not found at $REF (set REF=<dir>)" >&2; exit 2; }
CUTLASS="${CUTLASS:-$(python3 -c "import os,flashinfer;print(os.path.join(os.path.dirname(flashinfer.__file__),'data','cutlass','include'))")}"
CUDA="${CUDA:-/usr/local/cuda}"
TMP="$(mktemp -d)"
g++ -std=c++17 -O2 -ffp-contract=off -o "$TMP/make_golden" "$HERE/make_golden.cpp" \
    -I"$REF/include" -I"$CUTLASS" -I"$CUDA/include" 2> "$TMP/build.log" || { cat "$TMP/build.log"; exit 1; }
(cd "$HERE" && "$TMP/make_golden")
rm -rf "$TMP"
echo "golden vectors written to $HERE"
