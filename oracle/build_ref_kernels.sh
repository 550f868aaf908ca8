#!/usr/bin/env bash
# Builds the reference's fused kernels for sm_100a (from a SparseMoE checkout,
# never copied here; test infrastructure, outputs only in oracle/_ref/):
#   * ref_<kernel>: the reference's own program (drivers/main.cu +
#     inputs/data.cu + kernels/<kernel>.cu, its own include/config.h, the
#     flags of its Makefile), to time on a B200 next to this library linked
#     into the same driver (oracle/_ref/profile_b200);
#   * ref_pin_<kernel>: the kernel with oracle/ref_pin.cu at a one-thread-block
#     shape (N=16, d=f=64, E=16, top-1, CAP=16), to check the oracle's
#     restatement of its arithmetic against the kernel itself.
#   bash oracle/build_ref_kernels.sh [path/to/SparseMoE]     (default: $SPARSEMOE_REF)
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-${SPARSEMOE_REF:-}}"
if [[ -z "$REF" || ! -f "$REF/kernels/capacity.cu" ]]; then
  echo "build_ref_kernels.sh: no reference checkout given" >&2; exit 1
fi
mkdir -p "$HERE/_ref"
# the reference Makefile's flags (NVCC_FLAGS, -I. -I./include), for sm_100a
FLAGS="-O3 -lineinfo -Xcompiler -Wall --use_fast_math -gencode arch=compute_100a,code=sm_100a"
for kern in capacity capacity_int8_ptx capacity_int4_ptx capacity_fp8_ptx; do
  out="$HERE/_ref/ref_$kern"
  if [[ ! -x "$out" ]]; then
    nvcc $FLAGS -I "$REF" -I "$REF/include" "$REF/drivers/main.cu" "$REF/inputs/data.cu" \
         "$REF/kernels/$kern.cu" -o "$out" 2> "$HERE/_ref/ref_$kern.build.log"
    echo "built $out"
  fi
  pin="$HERE/_ref/ref_pin_$kern"
  if [[ ! -x "$pin" || "$pin" -ot "$HERE/ref_pin.cu" ]]; then
    nvcc $FLAGS -DREF_N=16 -DREF_D=64 -DREF_B=1 -DREF_E=16 -DREF_K=1 -DREF_UP=1 -DREF_CF=16.0f \
         -I "$HERE/ref_shadow" -I "$REF" "$REF/kernels/$kern.cu" "$HERE/ref_pin.cu" -o "$pin" \
         2> "$HERE/_ref/ref_pin_$kern.build.log"
    echo "built $pin"
  fi
done
