#!/bin/bash
# Entry point with the reference's name and environment variables
# (cutlass_gemm_mainloop/sweep.sh: SWEEP, OUTFILE, MAX_JOBS); the sweep itself
# is sweep.py (in process through the library by default, or --binaries for one
# harness binary per configuration).
exec python3 "$(dirname "$0")/sweep.py" "$@"
