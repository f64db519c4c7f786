#!/bin/bash
# Sweep over GEMM mainloop configurations of the sm_100a library; writes
# results.csv in the reference's schema (cutlass_gemm_mainloop/sweep.sh:21):
#   M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS
# so cutlass_gemm_mainloop/plot_results.py reads it unchanged.
#
# Phase 1 builds one harness binary per (TILE_M,TILE_N,TILE_K,STAGES,DTYPE_ID)
# in parallel (MAX_JOBS, skipping binaries already built); phase 2 runs them
# one at a time (exclusive GPU) and appends one line each, or a
# "# FAILED: cfg" / "# BUILD_FAILED: cfg" comment line -- the reference's flow
# (cutlass_gemm_mainloop/sweep.sh:85-149).  The harness is host-only C++ over
# the prebuilt library, so a build takes about a second instead of a minute.
#
# Tile lists: the reference's BF16 and FP8 lists (sweep.sh:28-65: TILE_M 64
# and 128, TILE_K down to one MMA K step -- 32- and 64-byte swizzle rows) plus
# NVFP4 (DTYPE_ID=2) and CTA-pair (TILE_M=256) tiles.
#   SWEEP=focus (default: the 128/256-row tiles at the default TILE_K)
#   SWEEP=full  (every reference tile)
set -e

SCRIPT_DIR="$(cd "$(dirname "$0")" && pwd)"
BUILD_DIR="$SCRIPT_DIR/build"
OUTFILE="${OUTFILE:-$SCRIPT_DIR/results.csv}"
MAX_JOBS="${MAX_JOBS:-$(nproc)}"
SWEEP="${SWEEP:-focus}"

mkdir -p "$BUILD_DIR"
echo "M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS" > "$OUTFILE"

STAGE_LIST=(0 2 3 4 5 6 7 8)

if [[ "$SWEEP" == "full" ]]; then
  BF16_TILES=()
  for TM in 64 128; do for TN in 16 32 64 128 192 256; do for TK in 16 32 64 128 256; do
    BF16_TILES+=("$TM,$TN,$TK"); done; done; done
  FP8_TILES=()
  for TM in 64 128; do for TN in 16 32 64 128 192 256; do for TK in 32 64 128 256 512; do
    FP8_TILES+=("$TM,$TN,$TK"); done; done; done
else
  BF16_TILES=("128,128,64" "128,192,64" "128,256,64" "128,256,128")
  FP8_TILES=("128,128,128" "128,192,128" "128,256,128" "128,256,256")
fi
NVFP4_TILES=("128,128,256" "128,256,256" "256,128,256" "256,256,256")
PAIR_BF16_TILES=("256,256,64" "256,512,64" "256,256,128")
PAIR_FP8_TILES=("256,256,128" "256,512,128" "256,256,256")

ALL_CONFIGS=()
for tile in "${BF16_TILES[@]}" "${PAIR_BF16_TILES[@]}"; do
  IFS=',' read -r TM TN TK <<< "$tile"
  for S in "${STAGE_LIST[@]}"; do ALL_CONFIGS+=("${TM},${TN},${TK},${S},0"); done
done
for tile in "${FP8_TILES[@]}" "${PAIR_FP8_TILES[@]}"; do
  IFS=',' read -r TM TN TK <<< "$tile"
  for S in "${STAGE_LIST[@]}"; do ALL_CONFIGS+=("${TM},${TN},${TK},${S},1"); done
done
for tile in "${NVFP4_TILES[@]}"; do
  IFS=',' read -r TM TN TK <<< "$tile"
  for S in "${STAGE_LIST[@]}"; do ALL_CONFIGS+=("${TM},${TN},${TK},${S},2"); done
done

TOTAL=${#ALL_CONFIGS[@]}
echo "=== Phase 1: Building $TOTAL binaries (max $MAX_JOBS parallel jobs) ==="
make -s -C "$SCRIPT_DIR/.." > /dev/null   # the library itself

job_count=0
for cfg in "${ALL_CONFIGS[@]}"; do
  IFS=',' read -r TM TN TK S D <<< "$cfg"
  BIN_NAME="bench_${TM}_${TN}_${TK}_s${S}_d${D}"
  BIN_PATH="$BUILD_DIR/$BIN_NAME"
  LOG_PATH="$BUILD_DIR/${BIN_NAME}.log"
  if [[ -x "$BIN_PATH" ]]; then continue; fi
  (
    if make -s -C "$SCRIPT_DIR" TILE_M=$TM TILE_N=$TN TILE_K=$TK STAGES=$S DTYPE_ID=$D \
         OUT="$BIN_PATH" > "$LOG_PATH" 2>&1; then
      echo "  [OK] $BIN_NAME"
    else
      echo "  [FAIL] $BIN_NAME (see $LOG_PATH)"
    fi
  ) &
  job_count=$((job_count + 1))
  if (( job_count >= MAX_JOBS )); then
    wait -n 2>/dev/null || true
    job_count=$((job_count - 1))
  fi
done
wait
echo "=== Phase 1 complete ==="

echo "=== Phase 2: Running benchmarks sequentially ==="
done_count=0
for cfg in "${ALL_CONFIGS[@]}"; do
  IFS=',' read -r TM TN TK S D <<< "$cfg"
  BIN_NAME="bench_${TM}_${TN}_${TK}_s${S}_d${D}"
  BIN_PATH="$BUILD_DIR/$BIN_NAME"
  done_count=$((done_count + 1))
  if [[ -x "$BIN_PATH" ]]; then
    echo -ne "  [$done_count/$TOTAL] $BIN_NAME ... "
    if result=$("$BIN_PATH" 2>/dev/null); then
      echo "$result" >> "$OUTFILE"
      echo "$result"
    else
      echo "# FAILED: $cfg" >> "$OUTFILE"
      echo "FAILED"
    fi
  else
    echo "  [$done_count/$TOTAL] $BIN_NAME ... BUILD_FAILED"
    echo "# BUILD_FAILED: $cfg" >> "$OUTFILE"
  fi
done

echo "=== Done. Results in $OUTFILE ==="
wc -l "$OUTFILE"
