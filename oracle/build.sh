#!/usr/bin/env bash
# Build recipe for the CPU oracle (test infrastructure only).
# Output: oracle/libpaged_oracle.so next to this script. x86-64-v3 (AVX2/FMA) is
# the baseline ISA so that the library built here also runs on the GPU hosts.
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
gcc -O3 -march=x86-64-v3 -fopenmp -fPIC -shared -std=c11 \
    -o "$here/libpaged_oracle.so" "$here/paged_attention_oracle.c" -lm
