/*
 * oracle.c -- CPU oracle for the sm_100a GEMM library.  TEST INFRASTRUCTURE ONLY:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library, and only as the checker or the reported CPU baseline -- never
 * as the thing measured for the GPU path and never as a fallback.
 *
 * What it restates:
 *   - The reference's arithmetic, cutlass_gemm_mainloop/cutlass_gemm_bench.cu:
 *       D = alpha * A . B^T + 0 * C            (:117-118, :196-204)
 *       A row-major M x K, B column-major K x N (= N x K, K contiguous),
 *       D column-major M x N bf16               (:103-105)
 *       fp32 accumulation                        (:69)
 *       FLOPs = 2*M*N*K                          (:249)
 *     restated here as an fp64 GEMM over the dequantised inputs (the
 *     tolerance target: relative Frobenius error 2e-3 for bf16/fp8, 1e-2 for
 *     NVFP4), plus a plain OpenMP fp32-accumulate GEMM that is the CPU
 *     baseline (the reference has no CPU path).
 *   - The seeded synthetic inputs of the benchmark configurations: a
 *     counter-based generator (splitmix64 over (seed, stream, index)), a
 *     Box-Muller normal built only from IEEE +,-,*,/ and sqrt (own series for
 *     ln and cos, so the host and device generators agree bit for bit), and
 *     the quantisers: bf16 and e4m3 (round to nearest even, e4m3 saturating
 *     to +-448), e2m1 (round to nearest even, saturating to +-6) and the
 *     unsigned-e4m3 NVFP4 block scale absmax/6 rounded up.
 *
 * Parity status: the reference pins no numerics for this path (it zero-fills
 * A and B and never reads D, cutlass_gemm_bench.cu:71-75,180-185), so there
 * are no reference golden vectors.  The quantisers are pinned against
 * PyTorch's dtype casts and the GEMM against numpy/torch fp64 matmul through
 * committed fixtures (tests/golden/), and on the GPU against the CUTLASS
 * SM100 kernel family the reference instantiates.
 *
 * Build: oracle/Makefile (gcc, OpenMP, -ffp-contract=off for the generator).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ RNG */

static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
static const uint64_t GOLDEN = 0x9E3779B97F4A7C15ULL;

/* Per-(seed, stream) key; element i draws mix64(key + (i + 1) * GOLDEN). */
static inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64(seed + mix64(stream + GOLDEN));
}
EXPORT uint64_t orc_bits(uint64_t seed, uint64_t stream, uint64_t idx) {
  return mix64(stream_key(seed, stream) + (idx + 1) * GOLDEN);
}

/* uniform[-1, 1) on a 2^-23 grid, exact in fp32. */
static inline float uniform_from_bits(uint64_t r) {
  return (float)(int32_t)(r >> 40) * (1.0f / 8388608.0f) - 1.0f;
}

/* ln(x) for x in (0, 1]: exponent split + atanh series, IEEE ops only. */
static double det_log(double x) {
  uint64_t b; memcpy(&b, &x, 8);
  int e = (int)((b >> 52) & 0x7FF) - 1022;           /* x = f * 2^e, f in [0.5, 1) */
  b = (b & 0x000FFFFFFFFFFFFFULL) | 0x3FE0000000000000ULL;
  double f; memcpy(&f, &b, 8);
  if (f < 0.70710678118654752) { f = f * 2.0; e -= 1; }  /* f in [0.7071, 1.4142) */
  double t = (f - 1.0) / (f + 1.0);
  double t2 = t * t;
  double s = 1.0 / 25.0;
  s = s * t2 + 1.0 / 23.0;
  s = s * t2 + 1.0 / 21.0;
  s = s * t2 + 1.0 / 19.0;
  s = s * t2 + 1.0 / 17.0;
  s = s * t2 + 1.0 / 15.0;
  s = s * t2 + 1.0 / 13.0;
  s = s * t2 + 1.0 / 11.0;
  s = s * t2 + 1.0 / 9.0;
  s = s * t2 + 1.0 / 7.0;
  s = s * t2 + 1.0 / 5.0;
  s = s * t2 + 1.0 / 3.0;
  s = s * t2 + 1.0;
  const double LN2 = 0.69314718055994531;
  return (double)e * LN2 + 2.0 * t * s;
}

/* Taylor series on |x| <= pi/4. */
static double det_cos_small(double x) {
  double x2 = x * x;
  double s = 1.0 / 6402373705728000.0;          /* 1/18! */
  s = -s * x2 + 1.0 / 20922789888000.0;          /* 1/16! */
  s = -s * x2 + 1.0 / 87178291200.0;             /* 1/14! */
  s = -s * x2 + 1.0 / 479001600.0;               /* 1/12! */
  s = -s * x2 + 1.0 / 3628800.0;                 /* 1/10! */
  s = -s * x2 + 1.0 / 40320.0;                   /* 1/8!  */
  s = -s * x2 + 1.0 / 720.0;                     /* 1/6!  */
  s = -s * x2 + 1.0 / 24.0;                      /* 1/4!  */
  s = -s * x2 + 1.0 / 2.0;                       /* 1/2!  */
  s = -s * x2 + 1.0;
  return s;
}
static double det_sin_small(double x) {
  double x2 = x * x;
  double s = 1.0 / 121645100408832000.0;         /* 1/19! */
  s = -s * x2 + 1.0 / 355687428096000.0;         /* 1/17! */
  s = -s * x2 + 1.0 / 1307674368000.0;           /* 1/15! */
  s = -s * x2 + 1.0 / 6227020800.0;              /* 1/13! */
  s = -s * x2 + 1.0 / 39916800.0;                /* 1/11! */
  s = -s * x2 + 1.0 / 362880.0;                  /* 1/9!  */
  s = -s * x2 + 1.0 / 5040.0;                    /* 1/7!  */
  s = -s * x2 + 1.0 / 120.0;                     /* 1/5!  */
  s = -s * x2 + 1.0 / 6.0;                       /* 1/3!  */
  s = -s * x2 + 1.0;
  return s * x;
}
/* cos(2*pi*v) for v in [0, 1), folded with exact subtractions. */
static double det_cos2pi(double v) {
  const double TWO_PI = 6.283185307179586;
  if (v >= 0.5) v = 1.0 - v;                  /* cos symmetric about 1/2 */
  double sign = 1.0;
  if (v > 0.25) { v = 0.5 - v; sign = -1.0; }  /* cos(pi - x) = -cos x */
  if (v > 0.125) return sign * det_sin_small(TWO_PI * (0.25 - v));
  return sign * det_cos_small(TWO_PI * v);
}

static inline float normal_from_bits(uint64_t r) {
  double u1 = ((double)(r >> 32) + 1.0) * (1.0 / 4294967296.0);       /* (0, 1] */
  double u2 = (double)(r & 0xFFFFFFFFULL) * (1.0 / 4294967296.0);     /* [0, 1) */
  double rad = sqrt(-2.0 * det_log(u1));
  return (float)(rad * det_cos2pi(u2));
}

EXPORT float orc_uniform(uint64_t seed, uint64_t stream, uint64_t idx) {
  return uniform_from_bits(orc_bits(seed, stream, idx));
}
EXPORT float orc_normal(uint64_t seed, uint64_t stream, uint64_t idx) {
  return normal_from_bits(orc_bits(seed, stream, idx));
}

/* ----------------------------------------------------------- quantisers */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

EXPORT uint16_t orc_f32_to_bf16(float x) {
  uint32_t u = f2u(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);  /* quiet NaN */
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
EXPORT float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* e4m3 (fn): bias 7, no infinities, max 448, min subnormal 2^-9. */
EXPORT float orc_e4m3_to_f32(uint8_t q) {
  int s = q >> 7, e = (q >> 3) & 0xF, m = q & 7;
  float v;
  if (e == 0xF && m == 7) return NAN;
  if (e == 0) v = (float)m * (1.0f / 512.0f);            /* m * 2^-3 * 2^-6 */
  else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

/* Round to nearest even, saturating to +-448 (cvt.rn.satfinite semantics). */
EXPORT uint8_t orc_f32_to_e4m3(float x) {
  uint32_t u = f2u(x);
  uint8_t sign = (uint8_t)((u >> 24) & 0x80);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7F;     /* NaN */
  float a = fabsf(x);
  if (a >= 448.0f) return sign | 0x7E;                   /* saturate */
  /* Work on the grid of e4m3 values with the exponent of a. */
  int e;
  if (a < 0.015625f) {                                    /* below 2^-6: subnormal grid 2^-9 */
    float q = a * 512.0f;                                 /* exact scaling by 2^9 */
    float r = rintf(q);                                   /* RNE (default rounding mode) */
    return sign | (uint8_t)r;                             /* r = 8 gives exponent 1, mantissa 0 */
  }
  frexpf(a, &e);                                          /* a = f * 2^e, f in [0.5, 1) */
  int E = e - 1;                                          /* a in [2^E, 2^(E+1)) */
  float scaled = ldexpf(a, 3 - E);                        /* in [8, 16), exact */
  float r = rintf(scaled);                                /* 8..16 */
  int m = (int)r - 8;
  if (m == 8) { m = 0; E += 1; }
  int biased = E + 7;
  if (biased > 15 || (biased == 15 && m == 7)) return sign | 0x7E;
  return sign | (uint8_t)((biased << 3) | m);
}

/* e2m1: values 0, 0.5, 1, 1.5, 2, 3, 4, 6. */
EXPORT float orc_e2m1_to_f32(uint8_t q) {
  static const float T[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  float v = T[q & 7];
  return (q & 8) ? -v : v;
}
/* Round to nearest even on the e2m1 grid, saturating to +-6. */
EXPORT uint8_t orc_f32_to_e2m1(float x) {
  uint8_t sign = (f2u(x) >> 31) ? 8 : 0;
  float a = fabsf(x);
  uint8_t c;
  if (a != a) return 0x7;                       /* NaN -> +6 (satfinite) */
  if (a <= 0.25f) c = 0;                        /* tie 0.25 -> 0 (even) */
  else if (a < 0.75f) c = 1;                    /* 0.5 */
  else if (a <= 1.25f) c = 2;                   /* tie 0.75 -> 1.0 (code 2 even), tie 1.25 -> 1.0 */
  else if (a < 1.75f) c = 3;                    /* 1.5 */
  else if (a <= 2.5f) c = 4;                    /* tie 1.75 -> 2 (code 4), tie 2.5 -> 2 */
  else if (a < 3.5f) c = 5;                     /* 3 */
  else if (a <= 5.0f) c = 6;                    /* tie 3.5 -> 4 (code 6), tie 5 -> 4 */
  else c = 7;                                   /* 6 and saturation */
  return sign | c;
}

/* Smallest non-negative e4m3 value >= t (t >= 0), saturating at 448. */
EXPORT uint8_t orc_ue4m3_round_up(float t) {
  if (!(t > 0.0f)) return 0;
  if (t >= 448.0f) return 0x7E;
  uint8_t q = orc_f32_to_e4m3(t);
  if (orc_e4m3_to_f32(q) < t) q = (uint8_t)(q + 1);    /* next representable up */
  return q;
}

/* ----------------------------------------------------- matrix generation */

/* out_dtype: 0 bf16, 1 e4m3; dist: 0 uniform[-1,1), 1 normal(0,1); value = round(dist * scale).
 * Writes rows [row0, row0+rows) (out points at row row0) of a matrix with
 * `cols` columns; element (r, c) uses index r*cols + c. */
EXPORT void orc_generate(void* out, int out_dtype, int dist, float scale,
                         uint64_t seed, uint64_t stream,
                         int64_t row0, int64_t rows, int64_t cols, int64_t ld) {
  uint64_t key = stream_key(seed, stream);
  #pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c) {
      uint64_t idx = (uint64_t)((row0 + r) * cols + c);
      uint64_t bits = mix64(key + (idx + 1) * GOLDEN);
      float v = dist ? normal_from_bits(bits) : uniform_from_bits(bits);
      v = v * scale;
      if (out_dtype == 0) ((uint16_t*)out)[r * ld + c] = orc_f32_to_bf16(v);
      else ((uint8_t*)out)[r * ld + c] = orc_f32_to_e4m3(v);
    }
  }
}

/* Byte offset of scale (row r, scale column c) in the 128x4 interleaved layout. */
EXPORT int64_t orc_sf_offset(int64_t r, int64_t c, int64_t cols) {
  int64_t kblocks = cols / 64;
  return ((r / 128) * kblocks + c / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4);
}

/* NVFP4: normal(0,1)*scale quantised per 16-element block; packed e2m1
 * (low nibble = even column) + ue4m3 scales in the interleaved layout.
 * out_packed / out_scales point at row row0 (a multiple of 128). */
EXPORT void orc_generate_nvfp4(uint8_t* out_packed, uint8_t* out_scales, float scale,
                               uint64_t seed, uint64_t stream,
                               int64_t row0, int64_t rows, int64_t cols) {
  uint64_t key = stream_key(seed, stream);
  #pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t cb = 0; cb < cols / 16; ++cb) {
      float v[16];
      float amax = 0.0f;
      for (int j = 0; j < 16; ++j) {
        uint64_t idx = (uint64_t)((row0 + r) * cols + cb * 16 + j);
        v[j] = normal_from_bits(mix64(key + (idx + 1) * GOLDEN)) * scale;
        float a = fabsf(v[j]);
        if (a > amax) amax = a;
      }
      uint8_t sq = orc_ue4m3_round_up(amax / 6.0f);
      float s = orc_e4m3_to_f32(sq);
      out_scales[orc_sf_offset(r, cb, cols)] = sq;
      for (int j = 0; j < 16; j += 2) {
        uint8_t lo = sq ? orc_f32_to_e2m1(v[j] / s) : 0;
        uint8_t hi = sq ? orc_f32_to_e2m1(v[j + 1] / s) : 0;
        out_packed[r * (cols / 2) + (cb * 16 + j) / 2] = (uint8_t)(lo | (hi << 4));
      }
    }
  }
}

/* ----------------------------------------------------------- dequantise */

/* dtype 0 bf16, 1 e4m3 -> fp32 row-major rows x cols (source row stride ld). */
EXPORT void orc_dequant(const void* in, int dtype, int64_t rows, int64_t cols, int64_t ld, float* out) {
  #pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c)
      out[r * cols + c] = dtype == 0 ? orc_bf16_to_f32(((const uint16_t*)in)[r * ld + c])
                                     : orc_e4m3_to_f32(((const uint8_t*)in)[r * ld + c]);
}

/* NVFP4 -> fp32: value * block scale. Rows r are relative to the buffers. */
EXPORT void orc_dequant_nvfp4(const uint8_t* packed, const uint8_t* scales,
                              int64_t rows, int64_t cols, float* out) {
  #pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      uint8_t byte = packed[r * (cols / 2) + c / 2];
      uint8_t q = (c & 1) ? (byte >> 4) : (byte & 0xF);
      float s = orc_e4m3_to_f32(scales[orc_sf_offset(r, c / 16, cols)]);
      out[r * cols + c] = orc_e2m1_to_f32(q) * s;
    }
}

/* -------------------------------------------------------------- GEMMs */

/* fp64 reference: Dref[i + j*ldd] = alpha * sum_k A[i,k] * B[j,k] over the
 * listed rows/cols (row_idx/col_idx may be NULL = all).  A is Mx K, B N x K,
 * both dequantised fp32 row-major; Dref is column-major over the selection
 * (ldd = number of selected rows). */
EXPORT void orc_gemm_f64(const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                         const int64_t* row_idx, int64_t nrows,
                         const int64_t* col_idx, int64_t ncols,
                         double alpha, double* Dref) {
  if (!row_idx) nrows = M;
  if (!col_idx) ncols = N;
  #pragma omp parallel for schedule(dynamic, 1) collapse(2)
  for (int64_t jb = 0; jb < ncols; jb += 16) {
    for (int64_t ib = 0; ib < nrows; ib += 16) {
      for (int64_t j = jb; j < jb + 16 && j < ncols; ++j) {
        const float* b = B + (col_idx ? col_idx[j] : j) * K;
        for (int64_t i = ib; i < ib + 16 && i < nrows; ++i) {
          const float* a = A + (row_idx ? row_idx[i] : i) * K;
          double acc = 0.0;
          for (int64_t k = 0; k < K; ++k) acc += (double)a[k] * (double)b[k];
          Dref[i + j * nrows] = alpha * acc;
        }
      }
    }
  }
}

/* Relative Frobenius error of a bf16 column-major result (selection) against
 * the fp64 reference: ||D - Dref||_F / ||Dref||_F. */
EXPORT double orc_rel_frobenius(const uint16_t* D, int64_t ldd,
                                const int64_t* row_idx, int64_t nrows,
                                const int64_t* col_idx, int64_t ncols,
                                const double* Dref) {
  double num = 0.0, den = 0.0;
  #pragma omp parallel for reduction(+:num,den) schedule(static)
  for (int64_t j = 0; j < ncols; ++j)
    for (int64_t i = 0; i < nrows; ++i) {
      int64_t r = row_idx ? row_idx[i] : i;
      int64_t c = col_idx ? col_idx[j] : j;
      double d = (double)orc_bf16_to_f32(D[r + c * ldd]);
      double ref = Dref[i + j * nrows];
      num += (d - ref) * (d - ref);
      den += ref * ref;
    }
  return den > 0.0 ? sqrt(num / den) : sqrt(num);
}

EXPORT int orc_num_threads(void) { return omp_get_max_threads(); }
