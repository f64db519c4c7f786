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
#include <stdlib.h>
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
 * path).  Output tiles of 64 x 64 are distributed over threads; for each
 * K-block of 256 the tile's 64 rows of B are packed K-major (64 KiB, stays in
 * L2) and a 4 x 16 outer-product register tile accumulates
 * C[i][j..j+15] += A[i][k] * Bp[k][j..j+15].  Writes bf16 column-major D. */
__attribute__((target_clones("arch=skylake-avx512", "arch=haswell", "default")))
EXPORT void orc_gemm_omp_f32(const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                             float alpha, uint16_t* D, int64_t ldd) {
  enum { MB = 64, NB = 64, KB = 256 };
  const int64_t mt = (M + MB - 1) / MB, nt = (N + NB - 1) / NB;
  #pragma omp parallel
  {
    float* Bp = (float*)aligned_alloc(64, sizeof(float) * KB * NB);
    float* C = (float*)aligned_alloc(64, sizeof(float) * MB * NB);
    #pragma omp for schedule(dynamic, 1)
    for (int64_t t = 0; t < mt * nt; ++t) {
      const int64_t ib = (t / nt) * MB, jb = (t % nt) * NB;
      const int64_t mi_all = (M - ib) < MB ? (M - ib) : MB;
      const int64_t nj_all = (N - jb) < NB ? (N - jb) : NB;
      memset(C, 0, sizeof(float) * MB * NB);
      for (int64_t kb = 0; kb < K; kb += KB) {
        const int64_t kl = (K - kb) < KB ? (K - kb) : KB;
        for (int64_t jj = 0; jj < NB; ++jj)
          for (int64_t kk = 0; kk < kl; ++kk)
            Bp[kk * NB + jj] = jj < nj_all ? B[(jb + jj) * K + kb + kk] : 0.0f;
        for (int64_t i = 0; i < mi_all; i += 4) {
          const float* a[4];
          for (int x = 0; x < 4; ++x) a[x] = A + (ib + i + ((i + x) < mi_all ? x : 0)) * K + kb;
          for (int64_t j = 0; j < NB; j += 16) {
            float c[4][16];
            for (int x = 0; x < 4; ++x)
              for (int l = 0; l < 16; ++l) c[x][l] = C[(i + x) * NB + j + l];
            for (int64_t kk = 0; kk < kl; ++kk) {
              const float* bp = Bp + kk * NB + j;
              for (int x = 0; x < 4; ++x) {
                const float av = a[x][kk];
                for (int l = 0; l < 16; ++l) c[x][l] += av * bp[l];
              }
            }
            for (int x = 0; x < 4; ++x)
              for (int l = 0; l < 16; ++l) C[(i + x) * NB + j + l] = c[x][l];
          }
        }
      }
      for (int64_t i = 0; i < mi_all; ++i)
        for (int64_t j = 0; j < nj_all; ++j) D[(ib + i) + (jb + j) * ldd] = f32_to_bf16(alpha * C[i * NB + j]);
    }
    free(Bp);
    free(C);
  }
}
