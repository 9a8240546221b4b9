#!/usr/bin/env bash
# Builds the CPU oracle (test infrastructure) into oracle/_build/librxla_oracle.so.
# x86-64-v3 (AVX2/FMA ISA, no FMA contraction) so the library built here also
# runs on the GPU box's host cores.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
mkdir -p "$here/_build"
gcc -O3 -march=x86-64-v3 -ffp-contract=off -fno-fast-math -fopenmp -fPIC -shared \
    -Wall -Wextra -Wno-unused-parameter \
    -o "$here/_build/librxla_oracle.so" "$here/rxla_oracle.c" -lm
