#!/bin/bash
# Build the reference project's own CUDA kernels, unmodified and compiled from
# where they lie in the reference checkout, into oracle/_ref/libt4ref.so -- a
# GPU-side checker for the tests (never shipped, never measured).
#
# usage: oracle/build_ref.sh [--if-present] [reference checkout]
#   The checkout is the argument, else $T4B_REFERENCE, else /root/reference
#   (where this build container mounts it).  With --if-present a missing
#   checkout is not an error: nothing is built.
#
# Compiles src/kernels/{lop3_dequant,fused_w4a16_gemm,h17_mega_kernel}.cu of the
# reference plus oracle/ref_shim.cu (C-ABI forwarding of the launchers) for
# sm_100a.  Nothing is copied out of the reference tree; the output goes to
# oracle/_ref/ only (git-ignored; it travels with the working tree).
set -euo pipefail
IF_PRESENT=0
if [ "${1:-}" = "--if-present" ]; then IF_PRESENT=1; shift; fi
REF=${1:-${T4B_REFERENCE:-/root/reference}}
if [ ! -d "$REF/src/kernels" ]; then
    if [ "$IF_PRESENT" = 1 ]; then echo "build_ref: no reference checkout at $REF; skipped"; exit 0; fi
    echo "build_ref: no reference checkout at $REF" >&2; exit 1
fi
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="$HERE/_ref"
NVCC=${NVCC:-$(command -v nvcc || echo /usr/local/cuda/bin/nvcc)}
KSRC="$REF/src/kernels"
for f in lop3_dequant.cu fused_w4a16_gemm.cu h17_mega_kernel.cu; do
    [ -f "$KSRC/$f" ] || { echo "build_ref: $KSRC/$f not found" >&2; exit 1; }
done
mkdir -p "$OUT"
TMP="$OUT/libt4ref.so.tmp"
"$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -shared -Xcompiler -fPIC \
    -I"$KSRC" \
    "$KSRC/lop3_dequant.cu" "$KSRC/fused_w4a16_gemm.cu" "$KSRC/h17_mega_kernel.cu" "$HERE/ref_shim.cu" \
    -o "$TMP" -lcudart_static -lrt -ldl -lpthread
mv -f "$TMP" "$OUT/libt4ref.so"
echo "build_ref: wrote $OUT/libt4ref.so"
