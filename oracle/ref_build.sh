#!/bin/bash
# Build the reference's own benchmark (cutlass_gemm_mainloop/cutlass_gemm_bench.cu,
# compiled in place from the read-only reference tree) and the CUTLASS
# comparison library (oracle/cutlass_ref.cu) into oracle/_ref/.
# TEST INFRASTRUCTURE: the outputs are the reference arm of the GPU tests and
# of the per-SM mainloop comparison; no product code links them.
#
# The reference does not vendor CUTLASS (its Makefile points at ../../cutlass);
# the CUTLASS 4.5 headers shipped inside this image's flashinfer package are
# used instead.  nvcc flags are the reference's (cutlass_gemm_mainloop/Makefile:2-3).
# Usage: oracle/ref_build.sh [REF_ROOT]   (skips outputs that already exist)
set -e
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-/root/reference}"
OUT="$HERE/_ref"
SRC="$REF/cutlass_gemm_mainloop/cutlass_gemm_bench.cu"
CUTLASS="${CUTLASS_DIR:-$(python -c 'import flashinfer, os; print(os.path.join(os.path.dirname(flashinfer.__file__), "data", "cutlass"))' 2>/dev/null)}"
if [[ ! -f "$SRC" ]]; then echo "reference source not found at $SRC; nothing to build"; exit 0; fi
if [[ ! -d "$CUTLASS/include/cutlass" ]]; then echo "CUTLASS headers not found ($CUTLASS)"; exit 1; fi
mkdir -p "$OUT"
NVCCFLAGS=(-std=c++17 --expt-relaxed-constexpr "-gencode=arch=compute_100a,code=sm_100a")
INC=(-I"$CUTLASS/include" -I"$CUTLASS/tools/util/include")
MAX_JOBS="${MAX_JOBS:-$(nproc)}"

# Reference single-CTA configurations (TILE_M,TILE_N,TILE_K,STAGES,DTYPE_ID):
# the best BF16 / FP8 points of results.csv (:461, :938) and their stage sweeps.
CONFIGS=(
  "128,256,64,0,0" "128,256,64,2,0" "128,256,64,3,0" "128,256,64,4,0"
  "128,192,64,0,0" "128,128,64,0,0"
  "128,256,128,0,1" "128,256,128,2,1" "128,256,128,3,1" "128,256,128,4,1"
  "128,192,128,0,1" "128,128,128,0,1"
)
jobs=0
for cfg in "${CONFIGS[@]}"; do
  IFS=',' read -r TM TN TK S D <<< "$cfg"
  BIN="$OUT/cutlass_bench_${TM}_${TN}_${TK}_s${S}_d${D}"
  [[ -x "$BIN" ]] && continue
  ( nvcc "${NVCCFLAGS[@]}" "${INC[@]}" -DTILE_M=$TM -DTILE_N=$TN -DTILE_K=$TK -DSTAGES=$S -DDTYPE_ID=$D \
        -o "$BIN" "$SRC" -lcuda > "$BIN.log" 2>&1 && echo "built $(basename "$BIN")" || echo "FAILED $(basename "$BIN")" ) &
  jobs=$((jobs + 1)); if (( jobs >= MAX_JOBS )); then wait -n || true; jobs=$((jobs - 1)); fi
done
LIB="$OUT/libcutlass_ref.so"
if [[ ! -f "$LIB" ]]; then
  ( nvcc "${NVCCFLAGS[@]}" "${INC[@]}" -O3 -Xcompiler -fPIC -shared -o "$LIB" "$HERE/cutlass_ref.cu" -lcuda \
      > "$OUT/libcutlass_ref.log" 2>&1 && echo "built libcutlass_ref.so" || echo "FAILED libcutlass_ref.so" ) &
fi
wait
