#!/usr/bin/env bash
# Builds tests/cpp/shim_test: the C++ drop-in headers and their shim sources
# (qwen-3.5-cuda_b200/cpp) against libqmoe, with the test stand-ins for the
# reference project's config.hpp / cuda_utils.hpp, and the CPU oracle linked
# as the checker.  Output: tests/cpp/_build/shim_test.
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
root="$(cd "$here/../.." && pwd)"
out="$here/_build"
mkdir -p "$out"
cuda="${CUDA_HOME:-/usr/local/cuda}"
g++ -std=c++17 -O2 -Wall -Wextra -Werror \
    -I "$root/include" -I "$here/compat" -I "$cuda/include" \
    "$here/shim_test.cpp" "$root/qwen-3.5-cuda_b200/cpp/matmul_q4_shim.cpp" \
    "$root/qwen-3.5-cuda_b200/cpp/layer_moe_shim.cpp" "$root/qwen-3.5-cuda_b200/cpp/moe_prefill_shim.cpp" \
    -L "$root/qwen-3.5-cuda_b200/qmoe" -lqmoe -L "$root/oracle" -loracle -L "$cuda/lib64" -lcudart \
    -Wl,-rpath,"$root/qwen-3.5-cuda_b200/qmoe" -Wl,-rpath,"$root/oracle" -Wl,-rpath,"$cuda/lib64" \
    -o "$out/shim_test"
echo "built $out/shim_test"
