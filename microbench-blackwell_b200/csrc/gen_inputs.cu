// gen_inputs.cu -- seeded synthetic operands on the device (harness helper).
//
// Every element is a pure function of (seed, stream, index): splitmix64 over
// a per-stream key, then uniform[-1,1) on a 2^-23 grid or a Box-Muller
// normal whose ln and cos are our own series in IEEE double arithmetic with
// every operation explicitly rounded (no FMA contraction), so a host
// implementation of the same steps reproduces the operands bit for bit.
// Rounding to the operand type: bf16 and e4m3 round to nearest even (e4m3
// saturating to +-448); NVFP4 uses one unsigned-e4m3 scale per 16 K elements
// (absmax/6 rounded up, so |x/scale| <= 6) and e2m1 values rounded to nearest
// even.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "gemm_sm100a.h"
#include "device_guard.cuh"

namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

__host__ __device__ inline uint64_t mix64_hd(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
inline uint64_t stream_key(uint64_t seed, uint64_t stream) { return mix64_hd(seed + mix64_hd(stream + kGolden)); }

__device__ __forceinline__ float uniform_from_bits(uint64_t r) {
  return __fsub_rn(__fmul_rn((float)(int32_t)(r >> 40), 1.0f / 8388608.0f), 1.0f);
}

#define DMUL __dmul_rn
#define DADD __dadd_rn
#define DSUB __dsub_rn
#define DDIV __ddiv_rn

// ln(x), x in (0, 1]: x = f * 2^e, f folded into [sqrt(1/2), sqrt(2)), ln f = 2 atanh((f-1)/(f+1)).
__device__ double det_log(double x) {
  uint64_t b = (uint64_t)__double_as_longlong(x);
  int e = (int)((b >> 52) & 0x7FF) - 1022;
  b = (b & 0x000FFFFFFFFFFFFFULL) | 0x3FE0000000000000ULL;
  double f = __longlong_as_double((long long)b);
  if (f < 0.70710678118654752) { f = DMUL(f, 2.0); e -= 1; }
  const double t = DDIV(DSUB(f, 1.0), DADD(f, 1.0));
  const double t2 = DMUL(t, t);
  double s = 1.0 / 25.0;
  s = DADD(DMUL(s, t2), 1.0 / 23.0);
  s = DADD(DMUL(s, t2), 1.0 / 21.0);
  s = DADD(DMUL(s, t2), 1.0 / 19.0);
  s = DADD(DMUL(s, t2), 1.0 / 17.0);
  s = DADD(DMUL(s, t2), 1.0 / 15.0);
  s = DADD(DMUL(s, t2), 1.0 / 13.0);
  s = DADD(DMUL(s, t2), 1.0 / 11.0);
  s = DADD(DMUL(s, t2), 1.0 / 9.0);
  s = DADD(DMUL(s, t2), 1.0 / 7.0);
  s = DADD(DMUL(s, t2), 1.0 / 5.0);
  s = DADD(DMUL(s, t2), 1.0 / 3.0);
  s = DADD(DMUL(s, t2), 1.0);
  const double LN2 = 0.69314718055994531;
  return DADD(DMUL((double)e, LN2), DMUL(DMUL(2.0, t), s));
}

// Taylor series of cos and sin on |x| <= pi/4 (Horner in x^2).
__device__ double det_cos_small(double x) {
  const double x2 = DMUL(x, x);
  double s = 1.0 / 6402373705728000.0;
  s = DADD(DMUL(-s, x2), 1.0 / 20922789888000.0);
  s = DADD(DMUL(-s, x2), 1.0 / 87178291200.0);
  s = DADD(DMUL(-s, x2), 1.0 / 479001600.0);
  s = DADD(DMUL(-s, x2), 1.0 / 3628800.0);
  s = DADD(DMUL(-s, x2), 1.0 / 40320.0);
  s = DADD(DMUL(-s, x2), 1.0 / 720.0);
  s = DADD(DMUL(-s, x2), 1.0 / 24.0);
  s = DADD(DMUL(-s, x2), 1.0 / 2.0);
  s = DADD(DMUL(-s, x2), 1.0);
  return s;
}
__device__ double det_sin_small(double x) {
  const double x2 = DMUL(x, x);
  double s = 1.0 / 121645100408832000.0;
  s = DADD(DMUL(-s, x2), 1.0 / 355687428096000.0);
  s = DADD(DMUL(-s, x2), 1.0 / 1307674368000.0);
  s = DADD(DMUL(-s, x2), 1.0 / 6227020800.0);
  s = DADD(DMUL(-s, x2), 1.0 / 39916800.0);
  s = DADD(DMUL(-s, x2), 1.0 / 362880.0);
  s = DADD(DMUL(-s, x2), 1.0 / 5040.0);
  s = DADD(DMUL(-s, x2), 1.0 / 120.0);
  s = DADD(DMUL(-s, x2), 1.0 / 6.0);
  s = DADD(DMUL(-s, x2), 1.0);
  return DMUL(s, x);
}
// cos(2 pi v), v in [0, 1), folded into [0, 1/8] with exact subtractions.
__device__ double det_cos2pi(double v) {
  const double TWO_PI = 6.283185307179586;
  if (v >= 0.5) v = DSUB(1.0, v);
  double sign = 1.0;
  if (v > 0.25) { v = DSUB(0.5, v); sign = -1.0; }
  if (v > 0.125) return DMUL(sign, det_sin_small(DMUL(TWO_PI, DSUB(0.25, v))));
  return DMUL(sign, det_cos_small(DMUL(TWO_PI, v)));
}

__device__ __forceinline__ float normal_from_bits(uint64_t r) {
  const double u1 = DMUL(DADD((double)(r >> 32), 1.0), 1.0 / 4294967296.0);
  const double u2 = DMUL((double)(r & 0xFFFFFFFFULL), 1.0 / 4294967296.0);
  const double rad = __dsqrt_rn(DMUL(-2.0, det_log(u1)));
  return __double2float_rn(DMUL(rad, det_cos2pi(u2)));
}

__device__ __forceinline__ uint8_t to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t q) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)q, __NV_E4M3);
  return __half2float(__half(h));
}
// e2m1 round to nearest even, saturating to +-6 (same decision table as a
// comparison ladder on |x| with ties going to the even code).
__device__ __forceinline__ uint8_t to_e2m1(float x) {
  const uint8_t sign = (__float_as_uint(x) >> 31) ? 8 : 0;
  const float a = fabsf(x);
  uint8_t c;
  if (a <= 0.25f) c = 0;
  else if (a < 0.75f) c = 1;
  else if (a <= 1.25f) c = 2;
  else if (a < 1.75f) c = 3;
  else if (a <= 2.5f) c = 4;
  else if (a < 3.5f) c = 5;
  else if (a <= 5.0f) c = 6;
  else c = 7;
  return sign | c;
}
__device__ __forceinline__ uint8_t ue4m3_round_up(float t) {
  if (!(t > 0.0f)) return 0;
  if (t >= 448.0f) return 0x7E;
  uint8_t q = to_e4m3(t);
  if (e4m3_to_f32(q) < t) q = (uint8_t)(q + 1);
  return q;
}

__global__ void generate_kernel(void* out, int out_dtype, int dist, float scale, uint64_t key,
                                int64_t row0, int64_t rows, int64_t cols, int64_t ld) {
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const uint64_t idx = (uint64_t)((row0 + r) * cols + c);
    const uint64_t bits = mix64(key + (idx + 1) * kGolden);
    float v = dist ? normal_from_bits(bits) : uniform_from_bits(bits);
    v = __fmul_rn(v, scale);
    if (out_dtype == GEMM_DTYPE_BF16)
      reinterpret_cast<__nv_bfloat16*>(out)[r * ld + c] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<uint8_t*>(out)[r * ld + c] = to_e4m3(v);
  }
}

// One thread per 16-element block.
__global__ void generate_nvfp4_kernel(uint8_t* packed, uint8_t* scales, float scale, uint64_t key,
                                      int64_t row0, int64_t rows, int64_t cols) {
  const int64_t nblk = cols / 16;
  const int64_t kblocks = cols / 64;
  const int64_t total = rows * nblk;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nblk, cb = i - r * nblk;
    float v[16];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint64_t idx = (uint64_t)((row0 + r) * cols + cb * 16 + j);
      v[j] = __fmul_rn(normal_from_bits(mix64(key + (idx + 1) * kGolden)), scale);
      amax = fmaxf(amax, fabsf(v[j]));
    }
    const uint8_t sq = ue4m3_round_up(__fdiv_rn(amax, 6.0f));
    const float s = e4m3_to_f32(sq);
    scales[((r / 128) * kblocks + cb / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (cb % 4)] = sq;
    uint8_t* dst = packed + r * (cols / 2) + cb * 8;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const uint8_t lo = sq ? to_e2m1(__fdiv_rn(v[j], s)) : 0;
      const uint8_t hi = sq ? to_e2m1(__fdiv_rn(v[j + 1], s)) : 0;
      dst[j / 2] = (uint8_t)(lo | (hi << 4));
    }
  }
}

int grid_for(int64_t work) {
  int64_t g = (work + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  return (int)g;
}

}  // namespace

extern "C" int gemm_sm100a_generate(void* out, int32_t out_dtype, int32_t dist, float scale,
                                    uint64_t seed, uint64_t stream_id,
                                    int64_t row0, int64_t rows, int64_t cols, int64_t ld,
                                    void* cuda_stream) {
  if (!out || rows < 0 || cols < 0 || ld < cols) return GEMM_ERR_BAD_ARGS;
  if (out_dtype != GEMM_DTYPE_BF16 && out_dtype != GEMM_DTYPE_FP8_E4M3) return GEMM_ERR_BAD_ARGS;
  if (rows == 0 || cols == 0) return GEMM_OK;
  StreamDeviceGuard guard(reinterpret_cast<cudaStream_t>(cuda_stream));
  if (!guard.ok) return GEMM_ERR_LAUNCH;
  generate_kernel<<<grid_for(rows * cols), 256, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(
      out, out_dtype, dist, scale, stream_key(seed, stream_id), row0, rows, cols, ld);
  if (cudaGetLastError() != cudaSuccess) return GEMM_ERR_LAUNCH;
  return GEMM_OK;
}

extern "C" int gemm_sm100a_generate_nvfp4(void* out_packed, void* out_scales, float scale,
                                          uint64_t seed, uint64_t stream_id,
                                          int64_t row0, int64_t rows, int64_t cols,
                                          void* cuda_stream) {
  if (!out_packed || !out_scales || rows < 0 || cols % 64 != 0 || rows % 128 != 0 || row0 % 128 != 0)
    return GEMM_ERR_BAD_ARGS;
  if (rows == 0 || cols == 0) return GEMM_OK;
  StreamDeviceGuard guard(reinterpret_cast<cudaStream_t>(cuda_stream));
  if (!guard.ok) return GEMM_ERR_LAUNCH;
  generate_nvfp4_kernel<<<grid_for(rows * (cols / 16)), 256, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(
      reinterpret_cast<uint8_t*>(out_packed), reinterpret_cast<uint8_t*>(out_scales), scale,
      stream_key(seed, stream_id), row0, rows, cols);
  if (cudaGetLastError() != cudaSuccess) return GEMM_ERR_LAUNCH;
  return GEMM_OK;
}
