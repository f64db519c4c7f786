#!/bin/bash
# Build the CUTLASS comparison library (oracle/cutlass_ref.cu) and, when the
# reference tree is given, the reference's own benchmark binaries
# (cutlass_gemm_mainloop/cutlass_gemm_bench.cu, compiled in place from the
# read-only reference tree) into oracle/_ref/.
# TEST INFRASTRUCTURE: the outputs are the reference arm of the GPU tests and
# of bench.py's same-box comparisons; no product code links them.
#
# The reference does not vendor CUTLASS (its Makefile points at ../../cutlass);
# the CUTLASS 4.5 headers shipped inside this image's flashinfer package are
# used instead (CUTLASS_DIR overrides).  nvcc flags are the reference's
# (cutlass_gemm_mainloop/Makefile:2-3).
#
# Usage: oracle/ref_build.sh [REF_ROOT]
#   REF_ROOT (or $MICROBENCH_REF_ROOT): root of the reference checkout; without
#   it only libcutlass_ref.so is built.  Outputs newer than their sources are kept.
set -e
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-${MICROBENCH_REF_ROOT:-}}"
OUT="$HERE/_ref"
CUTLASS="${CUTLASS_DIR:-$(python -c 'import flashinfer, os; print(os.path.join(os.path.dirname(flashinfer.__file__), "data", "cutlass"))' 2>/dev/null)}"
if [[ ! -d "$CUTLASS/include/cutlass" ]]; then echo "CUTLASS headers not found ($CUTLASS)"; exit 1; fi
mkdir -p "$OUT"
NVCCFLAGS=(-std=c++17 --expt-relaxed-constexpr "-gencode=arch=compute_100a,code=sm_100a")
INC=(-I"$CUTLASS/include" -I"$CUTLASS/tools/util/include")
MAX_JOBS="${MAX_JOBS:-$(nproc)}"
jobs=0
throttle() { jobs=$((jobs + 1)); if (( jobs >= MAX_JOBS )); then wait -n || true; jobs=$((jobs - 1)); fi; }

# The reference's single-CTA configurations (TILE_M,TILE_N,TILE_K,STAGES,DTYPE_ID):
# the best BF16 / FP8 points of results.csv (:461, :938) and their stage sweeps,
# and small TILE_M = 64 tiles, whose time is the per-stage loop cost.
SRC="$REF/cutlass_gemm_mainloop/cutlass_gemm_bench.cu"
if [[ -n "$REF" && -f "$SRC" ]]; then
  CONFIGS=(
    "128,256,64,0,0" "128,256,64,2,0" "128,256,64,3,0" "128,256,64,4,0"
    "128,192,64,0,0" "128,128,64,0,0"
    "128,256,128,0,1" "128,256,128,2,1" "128,256,128,3,1" "128,256,128,4,1"
    "128,192,128,0,1" "128,128,128,0,1"
    "64,16,16,0,0" "64,16,64,0,0" "64,64,64,0,0" "64,16,16,4,0" "64,128,64,0,0"
    "64,16,32,0,1" "64,64,128,0,1"
  )
  for cfg in "${CONFIGS[@]}"; do
    IFS=',' read -r TM TN TK S D <<< "$cfg"
    BIN="$OUT/cutlass_bench_${TM}_${TN}_${TK}_s${S}_d${D}"
    [[ -x "$BIN" ]] && continue
    ( nvcc "${NVCCFLAGS[@]}" "${INC[@]}" -DTILE_M=$TM -DTILE_N=$TN -DTILE_K=$TK -DSTAGES=$S -DDTYPE_ID=$D \
          -o "$BIN" "$SRC" -lcuda > "$BIN.log" 2>&1 && echo "built $(basename "$BIN")" || echo "FAILED $(basename "$BIN")" ) &
    throttle
  done
else
  echo "no reference tree given (argument or MICROBENCH_REF_ROOT): reference binaries skipped"
fi

# The comparison library: two translation units (REF_PART 0 and 2) compiled in parallel.
LIB="$OUT/libcutlass_ref.so"
if [[ ! -f "$LIB" || "$HERE/cutlass_ref.cu" -nt "$LIB" ]]; then
  for part in 0 2; do
    ( nvcc "${NVCCFLAGS[@]}" "${INC[@]}" -O3 -Xcompiler -fPIC -DREF_PART=$part -c \
          -o "$OUT/cutlass_ref_p$part.o" "$HERE/cutlass_ref.cu" > "$OUT/cutlass_ref_p$part.log" 2>&1 \
        && echo "compiled cutlass_ref part $part" || echo "FAILED cutlass_ref part $part (see $OUT/cutlass_ref_p$part.log)" ) &
    throttle
  done
  wait
  if [[ -f "$OUT/cutlass_ref_p0.o" && -f "$OUT/cutlass_ref_p2.o" ]]; then
    nvcc "-gencode=arch=compute_100a,code=sm_100a" -shared -o "$LIB" "$OUT"/cutlass_ref_p{0,2}.o -lcuda \
      && echo "built libcutlass_ref.so"
    rm -f "$OUT"/cutlass_ref_p{0,2}.o
  fi
fi
wait
