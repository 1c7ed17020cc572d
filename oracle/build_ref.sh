#!/usr/bin/env bash
# Builds the reference's own scalar reference ops from their sources where
# they lie under the reference checkout into oracle/_ref/libsingularity_ref.so.
# Test infrastructure only.  The reference checkout's root comes from the
# first argument or B2_REFERENCE_ROOT; with neither, or when the sources are
# not there, the script skips (exit 0).
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
ref="${1:-${B2_REFERENCE_ROOT:-}}"
out="$here/_ref"
if [ -z "$ref" ] || [ ! -f "$ref/Singularity/tests/test_and_bench_a5.cpp" ]; then
    echo "build_ref: reference sources not present; skipping"
    exit 0
fi
mkdir -p "$out"
# -std=c++23 as the reference Makefile (Singularity/Makefile), ISO mode so fp
# contraction stays off; -fpermissive for the 32-bit pointer casts in the
# (unused, garbage-collected) test main().
g++ -std=c++23 -O2 -fPIC -shared -fpermissive -w -ffp-contract=off \
    -fvisibility=hidden -ffunction-sections -fdata-sections -Wl,--gc-sections \
    -Wl,--no-undefined \
    -I"$ref/Singularity" \
    "$here/singularity_ref_shim.cpp" -o "$out/libsingularity_ref.so"
echo "build_ref: built $out/libsingularity_ref.so"
