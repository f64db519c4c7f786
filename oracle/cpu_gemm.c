/*
 * cpu_gemm.c -- the CPU baseline GEMM.  TEST INFRASTRUCTURE ONLY (see oracle.c):
 * bench.py's cpu_baseline leg and its --impl reference arm time it on the
 * host cores; nothing on the GPU path calls it.
 *
 * The reference has no CPU path (its only GEMM is the CUTLASS SM100 kernel in
 * cutlass_gemm_mainloop/cutlass_gemm_bench.cu:101-156), so this is the
 * "straightforward OpenMP host GEMM" the benchmark plan names: the same
 * D = alpha * A . B^T (A M x K row-major, B N x K, D column-major bf16,
 * cutlass_gemm_bench.cu:103-105) with fp32 accumulation (:69) over
 * dequantised fp32 inputs.  Compiled separately from oracle.c so that it may
 * use FMA contraction and per-ISA clones (the generator must not).
 */
#include <stdint.h>
#include <string.h>
#include <omp.h>

#define EXPORT __attribute__((visibility("default")))

static inline uint16_t f32_to_bf16(float x) {
  uint32_t u; memcpy(&u, &x, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* CPU baseline: a plain OpenMP GEMM with fp32 accumulation over dequantised
 * fp32 inputs (what the reference would run on a host core, had it a CPU
 * path).  Blocked over (M, N) with a 4x4 register tile of dot products along
 * the contiguous K; writes bf16 column-major D rows [0, M). */
__attribute__((target_clones("arch=skylake-avx512", "arch=haswell", "default")))
EXPORT void orc_gemm_omp_f32(const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                             float alpha, uint16_t* D, int64_t ldd) {
  const int64_t MB = 64, NB = 64;
  #pragma omp parallel for schedule(dynamic, 1) collapse(2)
  for (int64_t ib = 0; ib < M; ib += MB) {
    for (int64_t jb = 0; jb < N; jb += NB) {
      for (int64_t i = ib; i < ib + MB && i < M; i += 4) {
        for (int64_t j = jb; j < jb + NB && j < N; j += 4) {
          float acc[4][4][8];
          memset(acc, 0, sizeof(acc));
          int64_t mi = (M - i) < 4 ? (M - i) : 4;
          int64_t nj = (N - j) < 4 ? (N - j) : 4;
          const float* a[4]; const float* b[4];
          for (int x = 0; x < 4; ++x) a[x] = A + (i + (x < mi ? x : 0)) * K;
          for (int y = 0; y < 4; ++y) b[y] = B + (j + (y < nj ? y : 0)) * K;
          int64_t k = 0;
          for (; k + 8 <= K; k += 8)
            for (int x = 0; x < 4; ++x)
              for (int y = 0; y < 4; ++y)
                for (int l = 0; l < 8; ++l) acc[x][y][l] += a[x][k + l] * b[y][k + l];
          for (int x = 0; x < mi; ++x)
            for (int y = 0; y < nj; ++y) {
              float s = 0.0f;
              for (int l = 0; l < 8; ++l) s += acc[x][y][l];
              for (int64_t kk = k; kk < K; ++kk) s += a[x][kk] * b[y][kk];
              D[(i + x) + (j + y) * ldd] = f32_to_bf16(alpha * s);
            }
        }
      }
    }
  }
}

