#!/bin/bash
# Builds into oracle/_ref/, compiled directly from the reference tree (no copy):
#  * the reference's GPU kernels (stbl/kernels.cu + kernels.h) for sm_100a, libstbl_ref_kernels.so: the
#    second oracle for the kernels.h compatibility entry points; the GPU tests run both builds on the
#    same inputs and compare them bit for bit, as stbl/cmp_kernels.py does;
#  * the reference's GGUF reader (stbl/gguf.cpp) behind a test-only C shim, libstbl_ref_gguf.so.
# Needs the reference tree (present where the repository is developed, absent on GPU boxes, which use
# the prebuilt files).
set -euo pipefail
HERE=$(cd "$(dirname "$0")" && pwd)
REF=${STBL_REFERENCE:-$HERE/../../reference}   # default: the reference tree next to the repository
if [ ! -f "$REF/stbl/kernels.cu" ]; then
    echo "reference tree not found at $REF; keeping the prebuilt _ref/ (if any)" >&2
    exit 0
fi
mkdir -p "$HERE/_ref"
nvcc -O2 -std=c++17 -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC -shared \
    "$REF/stbl/kernels.cu" -o "$HERE/_ref/libstbl_ref_kernels.so"
echo "built $HERE/_ref/libstbl_ref_kernels.so"
# the reference's GGUF reader (stbl/gguf.cpp) behind a test-only C shim: the second oracle for
# include/stbl_gguf.h (tests/test_gguf.py compares the two readers' tables on the same files)
g++ -O2 -std=c++17 -fPIC -shared -I"$REF/stbl" "$HERE/ref_gguf_shim.cpp" "$REF/stbl/gguf.cpp" \
    -o "$HERE/_ref/libstbl_ref_gguf.so"
echo "built $HERE/_ref/libstbl_ref_gguf.so"
