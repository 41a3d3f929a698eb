#!/usr/bin/env bash
# Builds the CPU oracle (test infrastructure) into oracle/liboracle.so, and
# the host side of the seeded synthetic-tensor generator into
# oracle/libsynth_host.so (the same source the product library compiles, so
# the CPU legs -- tests, the bench's reference arm -- can make the benchmark's
# weight bytes without loading the product library).
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
gcc -O2 -std=c11 -fopenmp -ffp-contract=off -fPIC -shared \
    -o "$here/liboracle.so" "$here/qmoe_oracle.c" -lm
csrc="$here/../qwen-3.5-cuda_b200/csrc"
g++ -O2 -std=c++17 -fopenmp -ffp-contract=off -fPIC -shared -fvisibility=hidden \
    -I "$csrc" -I "$here/../include" -o "$here/libsynth_host.so" "$csrc/synth_host.cpp"
