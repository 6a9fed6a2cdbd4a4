#!/usr/bin/env bash
# Compiles the reference's own C++/CUDA path from its sources (read in place,
# never copied) into oracle/_ref/:
#   boa_constrictor  the reference CLI, portability_solved_cpp/README.md:11
#                    build line plus an sm_100a target
#   ref_logits       oracle/ref_harness.cu linked against the reference kernels
#   _gpu_range_cuda_ext*.so  the Python codec's batch range coder: importing
#                    gpu_range_coder.py compiles it (gpu_range_coder.py:14-367);
#                    TMPDIR points its build folder into _ref
# usage: build_ref.sh [reference checkout]
# The checkout is the first argument, else $BOA_REF_DIR, else a folder named
# "reference" beside this repository; without it the script does nothing and
# says so.  Outputs are git-ignored.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${BOA_REF_DIR:-$HERE/../../reference}}/portability_solved_cpp"
OUT="$HERE/_ref"
if [ ! -f "$REF/boa.cpp" ]; then echo "reference sources not found at $REF; skipping"; exit 0; fi
mkdir -p "$OUT"
FLAGS=(-O3 -std=c++17 --fmad=false -DENABLE_GPU -DGPU_DEBUG_LOGITS=0 -DGPU_FAST_EXP=0
       -gencode arch=compute_100a,code=sm_100a)
KERNELS=("$REF/gemm_kernels.cu" "$REF/inference_kernels.cu" "$REF/mamba_kernels.cu"
         "$REF/rnn_kernels.cu" "$REF/range_coder_kernels.cu" "$REF/utility_kernels.cu")
if [ ! -x "$OUT/boa_constrictor" ] || [ "${FORCE:-0}" = 1 ]; then
  nvcc -o "$OUT/boa_constrictor" "$REF/boa.cpp" "${KERNELS[@]}" "${FLAGS[@]}"
fi
if [ ! -x "$OUT/ref_logits" ] || [ "$HERE/ref_harness.cu" -nt "$OUT/ref_logits" ] || [ "${FORCE:-0}" = 1 ]; then
  nvcc -o "$OUT/ref_logits" "$HERE/ref_harness.cu" "${KERNELS[@]}" -I"$REF" "${FLAGS[@]}"
fi
if ! ls "$OUT"/_gpu_range_cuda_ext*.so >/dev/null 2>&1 || [ "${FORCE:-0}" = 1 ]; then
  mkdir -p "$OUT/pyrc_build"
  TMPDIR="$OUT/pyrc_build" python3 -c "import sys; sys.path.insert(0, sys.argv[1]); import gpu_range_coder" \
    "$(dirname "$REF")"
  cp "$OUT"/pyrc_build/gpu_range_build/_gpu_range_cuda_ext*.so "$OUT"/
  rm -rf "$OUT/pyrc_build"
fi
echo "reference build in $OUT"
