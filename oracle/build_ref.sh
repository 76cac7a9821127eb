#!/usr/bin/env bash
# Builds oracle/_ref/ref_dct from the reference's own DCT builder sources.
# TEST INFRASTRUCTURE ONLY.  Reads the reference tree (argument 1, default the
# REF_ROOT environment variable); writes only into oracle/_ref/.
#   lines 124-181: build_dct2 / build_dct2_t / build_idct / build_idct_t /
#                  build_idxst / build_idxst_t
#   lines 252-263: wu/wv eigenvalue weights inside TTNNDCTSolver::init
# The first line of each range is checked so a shifted file fails loudly.
set -euo pipefail
REF="${1:-${REF_ROOT:-}}"
HERE="$(cd "$(dirname "$0")" && pwd)"
SRC="$REF/host/density_scatter_ttnn_server_host.cpp"
OUT="$HERE/_ref"
if [ -z "$REF" ] || [ ! -f "$SRC" ]; then
    echo "build_ref: reference source not found ($SRC); skipping" >&2
    exit 3
fi
mkdir -p "$OUT"
sed -n '124,181p' "$SRC" > "$OUT/ref_builders.inc"
sed -n '252,263p' "$SRC" > "$OUT/ref_weights.inc"
head -1 "$OUT/ref_builders.inc" | grep -q 'DCT-II: C\[k,n\]' || { echo "build_ref: builder range moved" >&2; exit 1; }
head -1 "$OUT/ref_weights.inc" | grep -q 'std::vector<float> wu_v' || { echo "build_ref: weight range moved" >&2; exit 1; }
g++ -std=c++17 -O2 -ffp-contract=off -I"$OUT" "$HERE/ref_dct_driver.cpp" -o "$OUT/ref_dct"
echo "build_ref: built $OUT/ref_dct"
