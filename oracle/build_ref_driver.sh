#!/usr/bin/env bash
# Links the reference's unmodified drivers/main.cu (from a SparseMoE checkout,
# never copied here) against libsparsemoe_b200.so instead of the reference's
# inputs/data.cu + kernels/*.cu: the drop-in check.  Output: oracle/_ref/profile_b200.
#   bash oracle/build_ref_driver.sh [path/to/SparseMoE]     (default: $SPARSEMOE_REF)
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REPO="$(cd "$HERE/.." && pwd)"
REF="${1:-${SPARSEMOE_REF:-}}"
if [[ -z "$REF" || ! -f "$REF/drivers/main.cu" ]]; then
  echo "build_ref_driver.sh: no reference checkout given" >&2; exit 1
fi
mkdir -p "$HERE/_ref"
LIBDIR="$REPO/sparsemoe_b200"
nvcc -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -I "$REF" -I "$REF/include" \
     "$REF/drivers/main.cu" -L "$LIBDIR" -lsparsemoe_b200 -Xlinker -rpath,'$ORIGIN/../../sparsemoe_b200' \
     -o "$HERE/_ref/profile_b200"
echo "built $HERE/_ref/profile_b200"
