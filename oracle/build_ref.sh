#!/usr/bin/env bash
# Compiles the reference's own MoE path (src/layer_moe.cpp, src/cuda/matmul_q4.cu,
# src/cuda/moe.cu, and src/cuda/ops.cu for the pre-MoE RMSNorm; unmodified,
# from where they lie in the reference tree) for
# sm_100a into oracle/_ref/libqwenref.so, plus oracle/ref_capi.cpp (C entry
# points).  oracle/ref_shim/qwen_ref_prelude.hpp is force-included to stand in
# for the reference's cuda_utils.hpp, whose macros do not compile as shipped
# (it also supplies the CUDA_CHECK that ops.cu uses without including it).
# Usage: oracle/build_ref.sh <reference_root>
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
if [ $# -lt 1 ]; then
  echo "usage: $0 <reference_root>" >&2
  exit 2
fi
ref="$1"
if [ ! -f "$ref/src/layer_moe.cpp" ]; then
  echo "reference tree not found at $ref; skipping" >&2
  exit 0
fi
out="$here/_ref"
mkdir -p "$out"
NVCC="${NVCC:-/usr/local/cuda/bin/nvcc}"
flags=(-std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC
       -include "$here/ref_shim/qwen_ref_prelude.hpp" -I "$ref/include")
"$NVCC" "${flags[@]}" -c "$ref/src/cuda/matmul_q4.cu" -o "$out/matmul_q4.o"
"$NVCC" "${flags[@]}" -c "$ref/src/cuda/moe.cu" -o "$out/moe.o"
"$NVCC" "${flags[@]}" -c "$ref/src/cuda/ops.cu" -o "$out/ops.o"
"$NVCC" "${flags[@]}" -x cu -c "$ref/src/layer_moe.cpp" -o "$out/layer_moe.o"
"$NVCC" "${flags[@]}" -x cu -c "$here/ref_capi.cpp" -o "$out/ref_capi.o"
"$NVCC" -shared -gencode arch=compute_100a,code=sm_100a -o "$out/libqwenref.so" \
    "$out/matmul_q4.o" "$out/moe.o" "$out/ops.o" "$out/layer_moe.o" "$out/ref_capi.o" -lcudart
rm -f "$out"/*.o
echo "built $out/libqwenref.so"
