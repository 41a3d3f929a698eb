#!/usr/bin/env bash
# Builds the CPU oracle (test infrastructure) into oracle/liboracle.so.
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
gcc -O2 -std=c11 -fopenmp -ffp-contract=off -fPIC -shared \
    -o "$here/liboracle.so" "$here/qmoe_oracle.c" -lm
