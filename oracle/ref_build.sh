#!/bin/bash
# Builds the reference's own CUDA kernels (the second oracle, test infrastructure
# only) from its sources where they lie: the .cu files are concatenated in the
# order compute-cuda/src/runtime.rs:15-29 gives to NVRTC and compiled for
# sm_100a with the options of runtime.rs:160-168 (no FMA contraction, no
# flush-to-zero, IEEE divide and square root).  Output goes to oracle/_ref/ only
# (git-ignored; it travels to GPU machines with the working tree).
# Usage: oracle/ref_build.sh [path of the reference checkout]   (default /root/reference)
# Without the reference sources it builds nothing and exits 0; a cubin newer
# than every source is kept.
set -euo pipefail
REF="${1:-/root/reference}"
SRC="$REF/crates/compute-cuda/src"
OUT="$(cd "$(dirname "$0")" && pwd)/_ref"
NVCC="${NVCC:-/usr/local/cuda/bin/nvcc}"
files=(kernels.cu indexing.cu reductions.cu scatter.cu low_precision.cu statistics.cu attention.cu low_ops.cu
       low_indexing.cu low_scatter.cu low_statistics.cu low_attention.cu convolution.cu float64.cu float64_indexing.cu)
if [ ! -f "$SRC/convolution.cu" ]; then
    echo "reference sources not found under $REF: the second oracle is not built"
    exit 0
fi
mkdir -p "$OUT"
if [ -f "$OUT/reference_kernels.cubin" ]; then
    stale=0
    for f in "${files[@]}"; do [ "$SRC/$f" -nt "$OUT/reference_kernels.cubin" ] && stale=1; done
    if [ "$stale" = 0 ]; then echo "$OUT/reference_kernels.cubin"; exit 0; fi
fi
# the concatenation is a temporary file outside the repository
tmp="$(mktemp --suffix=.cu)"
trap 'rm -f "$tmp"' EXIT
for f in "${files[@]}"; do
    cat "$SRC/$f" >> "$tmp"
    echo >> "$tmp"
done
"$NVCC" -cubin -gencode arch=compute_100a,code=sm_100a -fmad=false -ftz=false -prec-div=true -prec-sqrt=true \
    -o "$OUT/reference_kernels.cubin" "$tmp"
echo "$OUT/reference_kernels.cubin"
