#!/usr/bin/env bash
# Compile the reference's own CUDA kernel sources, where they lie in the
# read-only reference tree, into oracle/_ref/libwlq_ref_kernels.so.
#
# TEST INFRASTRUCTURE ONLY: the GPU parity tests load this library to run the
# reference kernels (launch_gemv_chunk_csr, launch_gemm_metalog_dora,
# launch_dequant_patch_metalog, launch_fused_dora_epilogue) on the same inputs
# as this package's kernels.  The two .cu files need only the CUDA toolkit;
# the reference's csrc/vllm_binding.cpp needs libtorch and is not built.
# Flags follow the reference's setup.py:20-34, with the arch set to sm_100a.
set -euo pipefail
HERE=$(cd "$(dirname "$0")" && pwd)
# the reference tree: the first argument, else WLQ_REFERENCE_TREE, else a
# directory named "reference" beside this repository
REF=${1:-${WLQ_REFERENCE_TREE:-$(dirname "$(cd "$HERE/.." && pwd -P)")/reference}}
OUT="$HERE/_ref"
mkdir -p "$OUT"
if [ ! -f "$REF/csrc/gemv_kernel.cu" ]; then
  echo "reference tree not found at $REF; skipping" >&2
  exit 0
fi
NVCC=${NVCC:-/usr/local/cuda/bin/nvcc}
"$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++20 --use_fast_math -lineinfo \
  -Xcompiler -fPIC -shared \
  -o "$OUT/libwlq_ref_kernels.so" "$REF/csrc/gemv_kernel.cu" "$REF/csrc/gemm_kernel.cu"
echo "built $OUT/libwlq_ref_kernels.so"
