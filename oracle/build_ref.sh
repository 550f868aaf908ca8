#!/usr/bin/env bash
# Builds the reference's kernels/unfused.cu (from a SparseMoE checkout, never
# copied here) with the harness in oracle/ref_harness.cu into oracle/_ref/, for
# the golden-vector configs listed below.  Test infrastructure only.
#   bash oracle/build_ref.sh [path/to/SparseMoE]     (default: $SPARSEMOE_REF)
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-${SPARSEMOE_REF:-}}"
if [[ -z "$REF" || ! -f "$REF/kernels/unfused.cu" ]]; then
  echo "build_ref.sh: no reference checkout given" >&2; exit 1
fi
mkdir -p "$HERE/_ref"
FLAGS="-O3 -lineinfo --use_fast_math -gencode arch=compute_100a,code=sm_100a"
# name  N   d   B  E  k  up_proj_dim
CONFIGS=(
  "k2 256 512 2 16 2 2"
  "k4 128 256 2 32 4 4"
)
for c in "${CONFIGS[@]}"; do
  read -r name n d b e kk up <<<"$c"
  out="$HERE/_ref/ref_unfused_$name"
  if [[ -x "$out" && "$out" -nt "$HERE/ref_harness.cu" && "$out" -nt "$HERE/ref_shadow/include/config.h" ]]; then
    continue
  fi
  nvcc $FLAGS -DREF_N=$n -DREF_D=$d -DREF_B=$b -DREF_E=$e -DREF_K=$kk -DREF_UP=$up \
       -I "$HERE/ref_shadow" -I "$REF" "$REF/kernels/unfused.cu" "$HERE/ref_harness.cu" -o "$out"
  echo "built $out"
done
