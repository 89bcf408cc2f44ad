#!/usr/bin/env bash
# Builds the oracle (test infrastructure): liboracle.so from sdpa_oracle.c, and
# the reference's own sources via build_ref.sh when the reference is present.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
mkdir -p "$HERE/_build"
gcc -O2 -march=x86-64-v3 -ffp-contract=off -fPIC -shared -std=gnu11 -o "$HERE/_build/liboracle.so" \
  "$HERE/sdpa_oracle.c" -lm -lpthread
"$HERE/build_ref.sh"
