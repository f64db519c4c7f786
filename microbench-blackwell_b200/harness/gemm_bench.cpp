// gemm_bench.cpp -- drop-in host harness for the sm_100a GEMM library.
//
// Keeps the surface of the reference benchmark
// cutlass_gemm_mainloop/cutlass_gemm_bench.cu:
//   * compile-time knobs TILE_M, TILE_N, TILE_K, STAGES (0 = auto), DTYPE_ID
//     with the same defaults (cutlass_gemm_bench.cu:34-49), plus CTA_GROUP
//     (1 or 2; TILE_M = 256 implies 2), CLUSTER_M, CLUSTER_N and DTYPE_ID = 2
//     for NVFP4;
//   * with no arguments it runs the reference experiment: one CTA (one CTA
//     pair for CTA_GROUP 2), M = TILE_M, N = TILE_N, K = 131072, zero-filled
//     inputs, 1 warm-up and 20 timed launches (cutlass_gemm_bench.cu:52-55,
//     158-246), and prints exactly the reference's CSV line
//         M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS
//     (cutlass_gemm_bench.cu:253-257); exit status 1 when the configuration
//     cannot be implemented (cutlass_gemm_bench.cu:211-224);
//   * with arguments it runs full problems:
//         --m M --n N --k K [--init zero|seeded] [--seed S] [--iters I]
//         [--warmup W] [--check] [--ngpus G] [--allgather] [--fused-gather] [--raster R]
//         [--max-ctas C]
//     and appends cta_group,ngpus,allgather_ms,relerr (and fused_ms with
//     --fused-gather) to the line.  With
//     --ngpus G > 1 the GEMM is split along N (A replicated, B and D
//     column-sliced; GPU g owns columns [g*N/G, (g+1)*N/G)), timed as the
//     maximum over GPUs; --fused-gather times GEMM + gather in one launch per
//     GPU (gemm_sm100a_launch_gather: each GPU's epilogue also stores its slice
//     into every other GPU's full D over NVLink) and checks the gathered D
//     bitwise against the slices; --allgather gathers the bf16 D slices into a full
//     D on every GPU with one ncclAllGather (timed separately).
//
// All GEMM work goes through the C ABI (gemm_sm100a_launch); the harness
// owns every buffer.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <random>
#include <string>
#include <vector>

#include "gemm_sm100a.h"

#ifndef TILE_M
#define TILE_M 128
#endif
#ifndef TILE_N
#define TILE_N 128
#endif
#ifndef TILE_K
#define TILE_K 64
#endif
#ifndef STAGES
#define STAGES 0
#endif
#ifndef DTYPE_ID
#define DTYPE_ID 0
#endif
#ifndef CTA_GROUP
#define CTA_GROUP (TILE_M > 128 ? 2 : 1)
#endif
#ifndef CLUSTER_M
#define CLUSTER_M CTA_GROUP
#endif
#ifndef CLUSTER_N
#define CLUSTER_N 1
#endif

#if DTYPE_ID == 0
static const char* kDtype = "BF16";
#elif DTYPE_ID == 1
static const char* kDtype = "FP8_E4M3";
#elif DTYPE_ID == 2
static const char* kDtype = "NVFP4";
#else
#error "Unknown DTYPE_ID (0=BF16, 1=FP8_E4M3, 2=NVFP4)"
#endif

static constexpr int64_t kRefK = 131072;  // the reference's K (cutlass_gemm_bench.cu:53)

#define CK(x)                                                                           \
  do {                                                                                  \
    cudaError_t e_ = (x);                                                               \
    if (e_ != cudaSuccess) {                                                            \
      fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
      exit(1);                                                                          \
    }                                                                                   \
  } while (0)
#define NK(x)                                                                           \
  do {                                                                                  \
    ncclResult_t r_ = (x);                                                              \
    if (r_ != ncclSuccess) {                                                            \
      fprintf(stderr, "NCCL error %s at %s:%d\n", ncclGetErrorString(r_), __FILE__, __LINE__); \
      exit(1);                                                                          \
    }                                                                                   \
  } while (0)

struct Options {
  bool full = false;           // any size argument given
  int64_t m = TILE_M, n = TILE_N, k = kRefK;
  bool seeded = false;
  uint64_t seed = 0;
  int iters = 20, warmup = 1;
  bool check = false;
  int ngpus = 1;
  bool allgather = false;
  bool fused_gather = false;
  int raster = 0;
  int max_ctas = -1;           // -1: single CTA (pair) in reference mode, all SMs otherwise
};

static Options parse(int argc, char** argv) {
  Options o;
  bool init_given = false;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() -> const char* {
      if (i + 1 >= argc) { fprintf(stderr, "missing value for %s\n", a.c_str()); exit(2); }
      return argv[++i];
    };
    if (a == "--m") { o.m = atoll(next()); o.full = true; }
    else if (a == "--n") { o.n = atoll(next()); o.full = true; }
    else if (a == "--k") { o.k = atoll(next()); o.full = true; }
    else if (a == "--init") { o.seeded = std::string(next()) == "seeded"; init_given = true; }
    else if (a == "--seed") { o.seed = strtoull(next(), nullptr, 10); }
    else if (a == "--iters") { o.iters = atoi(next()); }
    else if (a == "--warmup") { o.warmup = atoi(next()); }
    else if (a == "--check") { o.check = true; }
    else if (a == "--ngpus") { o.ngpus = atoi(next()); o.full = true; }
    else if (a == "--allgather") { o.allgather = true; }
    else if (a == "--fused-gather") { o.fused_gather = true; }
    else if (a == "--raster") { o.raster = atoi(next()); }
    else if (a == "--max-ctas") { o.max_ctas = atoi(next()); }
    else { fprintf(stderr, "unknown argument %s\n", a.c_str()); exit(2); }
  }
  if (o.full && !init_given) o.seeded = true;     // full problems use the seeded inputs
  if (o.check) o.seeded = true;
  if (o.max_ctas < 0) o.max_ctas = o.full ? 0 : CTA_GROUP;
  return o;
}

// ------------------------------------------------------------------ host decoders for --check
static float bf16_to_f32(uint16_t h) { uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f; }
static float e4m3_to_f32(uint8_t q) {
  int s = q >> 7, e = (q >> 3) & 0xF, m = q & 7;
  if (e == 0xF && m == 7) return NAN;
  float v = e == 0 ? (float)m / 512.0f : ldexpf(1.0f + m / 8.0f, e - 7);
  return s ? -v : v;
}
static float e2m1_to_f32(uint8_t q) {
  static const float T[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  return (q & 8) ? -T[q & 7] : T[q & 7];
}
static int64_t sf_offset(int64_t r, int64_t c, int64_t k) {
  return ((r / 128) * (k / 64) + c / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4);
}
static int64_t sf_bytes(int64_t rows, int64_t k) { return ((rows + 127) / 128) * (k / 64) * 512; }

struct DeviceGemm {
  int dev = 0;
  cudaStream_t stream = nullptr;
  int64_t n_local = 0, n0 = 0;
  void *a = nullptr, *b = nullptr, *d = nullptr, *sfa = nullptr, *sfb = nullptr, *dfull = nullptr;
  void* dfused = nullptr;   // full M x N D written by every GPU's fused-gather launch
  int32_t* status = nullptr;
  GemmArgs args{};
  cudaEvent_t e0{}, e1{}, g0{}, g1{};
};

static size_t row_bytes(int64_t k) { return DTYPE_ID == 0 ? (size_t)k * 2 : (DTYPE_ID == 1 ? (size_t)k : (size_t)k / 2); }

int main(int argc, char** argv) {
  Options o = parse(argc, argv);
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (o.ngpus < 1 || o.ngpus > ndev) { fprintf(stderr, "need %d GPUs, found %d\n", o.ngpus, ndev); return 1; }
  if (o.n % o.ngpus != 0) { fprintf(stderr, "N (%lld) must divide evenly over %d GPUs\n", (long long)o.n, o.ngpus); return 1; }

  std::vector<DeviceGemm> g(o.ngpus);
  const int64_t n_local = o.n / o.ngpus;
  for (int i = 0; i < o.ngpus; ++i) {
    DeviceGemm& x = g[i];
    x.dev = i;
    x.n_local = n_local;
    x.n0 = (int64_t)i * n_local;
    CK(cudaSetDevice(i));
    CK(cudaStreamCreateWithFlags(&x.stream, cudaStreamNonBlocking));
    CK(cudaMalloc(&x.a, row_bytes(o.k) * o.m));
    CK(cudaMalloc(&x.b, row_bytes(o.k) * n_local));
    CK(cudaMalloc(&x.d, (size_t)o.m * n_local * 2));
    CK(cudaMalloc(&x.status, sizeof(int32_t)));
    CK(cudaMemsetAsync(x.status, 0, sizeof(int32_t), x.stream));
    if (DTYPE_ID == 2) {
      CK(cudaMalloc(&x.sfa, sf_bytes(o.m, o.k)));
      CK(cudaMalloc(&x.sfb, sf_bytes(n_local, o.k)));
    }
    if (!o.seeded) {  // the reference zero-fills A and B (cutlass_gemm_bench.cu:72-75,183-184)
      CK(cudaMemsetAsync(x.a, 0, row_bytes(o.k) * o.m, x.stream));
      CK(cudaMemsetAsync(x.b, 0, row_bytes(o.k) * n_local, x.stream));
      if (DTYPE_ID == 2) {
        CK(cudaMemsetAsync(x.sfa, 0, sf_bytes(o.m, o.k), x.stream));
        CK(cudaMemsetAsync(x.sfb, 0, sf_bytes(n_local, o.k), x.stream));
      }
    } else if (DTYPE_ID == 2) {
      if (gemm_sm100a_generate_nvfp4(x.a, x.sfa, 1.0f, o.seed, 0, 0, o.m, o.k, x.stream) ||
          gemm_sm100a_generate_nvfp4(x.b, x.sfb, 1.0f, o.seed, 1, x.n0, n_local, o.k, x.stream)) {
        fprintf(stderr, "NVFP4 generation needs M, N/ngpus multiples of 128 and K of 64\n");
        return 1;
      }
    } else {
      // bf16: uniform[-1,1); e4m3: N(0,1)/4 (config 3)
      const int dist = DTYPE_ID == 0 ? 0 : 1;
      const float scale = DTYPE_ID == 0 ? 1.0f : 0.25f;
      if (gemm_sm100a_generate(x.a, DTYPE_ID, dist, scale, o.seed, 0, 0, o.m, o.k, o.k, x.stream) ||
          gemm_sm100a_generate(x.b, DTYPE_ID, dist, scale, o.seed, 1, x.n0, n_local, o.k, o.k, x.stream)) {
        fprintf(stderr, "generation failed\n");
        return 1;
      }
    }
    GemmArgs& a = x.args;
    memset(&a, 0, sizeof(a));
    a.struct_size = sizeof(GemmArgs);
    a.dtype = DTYPE_ID;
    a.m = o.m; a.n = n_local; a.k = o.k;
    a.a = x.a; a.lda = o.k;
    a.b = x.b; a.ldb = o.k;
    a.d = x.d; a.ldd = o.m;
    a.sfa = x.sfa; a.sfb = x.sfb;
    a.alpha = 1.0f;
    a.tile_m = TILE_M; a.tile_n = TILE_N; a.tile_k = TILE_K; a.stages = STAGES;
    a.cta_group = CTA_GROUP; a.cluster_m = CLUSTER_M;
    a.max_ctas = o.max_ctas;
    a.raster_group = o.raster;
    a.status = x.status;
    if (CLUSTER_N != 1) { fprintf(stderr, "Cannot implement: CLUSTER_N=%d (only 1)\n", CLUSTER_N); return 1; }
    GemmInfo info;
    memset(&info, 0, sizeof(info));
    if (gemm_sm100a_query(&a, &info) != GEMM_OK) {
      fprintf(stderr, "Cannot implement: TILE_M=%d TILE_N=%d TILE_K=%d STAGES=%d dtype=%s error=%s\n",
              TILE_M, TILE_N, TILE_K, STAGES, kDtype, info.reason);
      return 1;
    }
    CK(cudaEventCreate(&x.e0)); CK(cudaEventCreate(&x.e1));
    CK(cudaEventCreate(&x.g0)); CK(cudaEventCreate(&x.g1));
  }

  auto launch_all = [&]() {
    for (auto& x : g) {
      CK(cudaSetDevice(x.dev));
      int rc = gemm_sm100a_launch(&x.args, x.stream);
      if (rc != GEMM_OK) { fprintf(stderr, "launch failed: %s\n", gemm_sm100a_strerror(rc)); exit(1); }
    }
  };
  for (int w = 0; w < o.warmup; ++w) launch_all();
  for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaStreamSynchronize(x.stream)); }

  for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaEventRecord(x.e0, x.stream)); }
  for (int it = 0; it < o.iters; ++it) launch_all();
  for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaEventRecord(x.e1, x.stream)); }
  float ms_max = 0.0f;
  for (auto& x : g) {
    CK(cudaSetDevice(x.dev));
    CK(cudaEventSynchronize(x.e1));
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, x.e0, x.e1));
    ms_max = std::max(ms_max, ms);
    int32_t detail = 0;
    if (gemm_sm100a_read_status(x.status, x.stream, &detail) != GEMM_OK) {
      fprintf(stderr, "device wait timed out on GPU %d (status 0x%08x)\n", x.dev, (unsigned)detail);
      return 1;
    }
  }
  const float avg_ms = ms_max / o.iters;

  // ---------------------------------------------------------------- optional all-gather of D
  float ag_ms = 0.0f;
  if (o.allgather && o.ngpus > 1) {
    std::vector<ncclComm_t> comms(o.ngpus);
    std::vector<int> devs(o.ngpus);
    for (int i = 0; i < o.ngpus; ++i) devs[i] = i;
    NK(ncclCommInitAll(comms.data(), o.ngpus, devs.data()));
    for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaMalloc(&x.dfull, (size_t)o.m * o.n * 2)); }
    auto gather = [&]() {
      NK(ncclGroupStart());
      for (int i = 0; i < o.ngpus; ++i)
        NK(ncclAllGather(g[i].d, g[i].dfull, (size_t)o.m * n_local, ncclBfloat16, comms[i], g[i].stream));
      NK(ncclGroupEnd());
    };
    gather();  // warm-up
    for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaStreamSynchronize(x.stream)); CK(cudaEventRecord(x.g0, x.stream)); }
    gather();
    for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaEventRecord(x.g1, x.stream)); }
    for (auto& x : g) {
      CK(cudaSetDevice(x.dev));
      CK(cudaEventSynchronize(x.g1));
      float ms = 0.0f;
      CK(cudaEventElapsedTime(&ms, x.g0, x.g1));
      ag_ms = std::max(ag_ms, ms);
    }
    for (auto& c : comms) ncclCommDestroy(c);
  }

  // ---------------------------------------------------------------- optional fused GEMM + gather
  float fused_ms = 0.0f;
  if (o.fused_gather && o.ngpus > 1) {
    if (o.ngpus - 1 > 7) { fprintf(stderr, "--fused-gather supports up to 8 GPUs\n"); return 1; }
    for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaMalloc(&x.dfused, (size_t)o.m * o.n * 2)); }
    std::vector<std::vector<void*>> peers(o.ngpus);
    std::vector<GemmArgs> fargs(o.ngpus);
    for (auto& x : g) {
      fargs[x.dev] = x.args;
      fargs[x.dev].d = (uint16_t*)x.dfused + x.n0 * o.m;             // this GPU's slice of its full D
      for (auto& y : g)
        if (y.dev != x.dev) peers[x.dev].push_back((uint16_t*)y.dfused + x.n0 * o.m);   // same slice, peers' D
    }
    auto launch_fused = [&]() {
      for (auto& x : g) {
        CK(cudaSetDevice(x.dev));
        int rc = gemm_sm100a_launch_gather(&fargs[x.dev], peers[x.dev].data(), (int32_t)peers[x.dev].size(), x.stream);
        if (rc != GEMM_OK) { fprintf(stderr, "fused launch failed: %s\n", gemm_sm100a_strerror(rc)); exit(1); }
      }
    };
    auto sync_all = [&]() { for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaStreamSynchronize(x.stream)); } };
    for (int w = 0; w < std::max(1, o.warmup); ++w) launch_fused();
    sync_all();
    // Every GPU finished its warm-up stores into every D before timing starts.
    for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaEventRecord(x.g0, x.stream)); }
    // GPU x only ever writes slice x (of every D), so back-to-back launches
    // need no cross-GPU ordering; each GPU's time includes its remote stores.
    for (int it = 0; it < o.iters; ++it) launch_fused();
    for (auto& x : g) { CK(cudaSetDevice(x.dev)); CK(cudaEventRecord(x.g1, x.stream)); }
    for (auto& x : g) {
      CK(cudaSetDevice(x.dev));
      CK(cudaEventSynchronize(x.g1));
      float ms = 0.0f;
      CK(cudaEventElapsedTime(&ms, x.g0, x.g1));
      fused_ms = std::max(fused_ms, ms / o.iters);
      int32_t detail = 0;
      if (gemm_sm100a_read_status(x.status, x.stream, &detail) != GEMM_OK) {
        fprintf(stderr, "device wait timed out on GPU %d (status 0x%08x)\n", x.dev, (unsigned)detail);
        return 1;
      }
    }
    // Bitwise check: sampled columns of every slice, on every GPU, against the
    // owner's own result from the plain launches above.
    std::mt19937_64 rng(o.seed + 777);
    std::vector<uint16_t> got(o.m), want(o.m);
    for (auto& x : g)
      for (auto& y : g)
        for (int sidx = 0; sidx < 10; ++sidx) {
          const int64_t cl = sidx == 0 ? 0 : (sidx == 1 ? n_local - 1 : (int64_t)(rng() % (uint64_t)n_local));
          CK(cudaSetDevice(x.dev));
          CK(cudaMemcpy(got.data(), (uint16_t*)x.dfused + (y.n0 + cl) * o.m, (size_t)o.m * 2, cudaMemcpyDeviceToHost));
          CK(cudaSetDevice(y.dev));
          CK(cudaMemcpy(want.data(), (uint16_t*)y.d + cl * o.m, (size_t)o.m * 2, cudaMemcpyDeviceToHost));
          if (memcmp(got.data(), want.data(), (size_t)o.m * 2) != 0) {
            fprintf(stderr, "fused gather mismatch: GPU %d, slice of GPU %d, column %lld\n", x.dev, y.dev, (long long)cl);
            return 1;
          }
        }
  }

  // ---------------------------------------------------------------- optional sampled fp64 check
  double relerr = -1.0;
  if (o.check) {
    std::mt19937_64 rng(o.seed + 12345);
    const int S = 48;
    std::vector<int64_t> rows(S), cols(S);
    for (auto& r : rows) r = (int64_t)(rng() % (uint64_t)o.m);
    for (auto& c : cols) c = (int64_t)(rng() % (uint64_t)o.n);
    const size_t rb = row_bytes(o.k);
    std::vector<uint8_t> arow(rb), brow(rb);
    std::vector<uint8_t> sfa_h, sfb_h;
    std::vector<std::vector<float>> A(S, std::vector<float>(o.k)), B(S, std::vector<float>(o.k));
    auto decode = [&](const uint8_t* raw, const std::vector<uint8_t>& sf, int64_t r, std::vector<float>& out) {
      for (int64_t c = 0; c < o.k; ++c) {
        if (DTYPE_ID == 0) { uint16_t h; memcpy(&h, raw + 2 * c, 2); out[c] = bf16_to_f32(h); }
        else if (DTYPE_ID == 1) out[c] = e4m3_to_f32(raw[c]);
        else {
          const uint8_t byte = raw[c / 2];
          out[c] = e2m1_to_f32((c & 1) ? (byte >> 4) : (byte & 0xF)) * e4m3_to_f32(sf[sf_offset(r, c / 16, o.k)]);
        }
      }
    };
    double num = 0.0, den = 0.0;
    std::vector<std::vector<uint8_t>> sfb_dev(o.ngpus);
    if (DTYPE_ID == 2) {
      sfa_h.resize(sf_bytes(o.m, o.k));
      CK(cudaSetDevice(g[0].dev));
      CK(cudaMemcpy(sfa_h.data(), g[0].sfa, sfa_h.size(), cudaMemcpyDeviceToHost));
      for (auto& x : g) {
        sfb_dev[x.dev].resize(sf_bytes(n_local, o.k));
        CK(cudaSetDevice(x.dev));
        CK(cudaMemcpy(sfb_dev[x.dev].data(), x.sfb, sfb_dev[x.dev].size(), cudaMemcpyDeviceToHost));
      }
    }
    for (int i = 0; i < S; ++i) {
      const DeviceGemm& x = g[cols[i] / n_local];
      const int64_t cl = cols[i] - x.n0;
      CK(cudaSetDevice(g[0].dev));
      CK(cudaMemcpy(arow.data(), (const uint8_t*)g[0].a + rb * rows[i], rb, cudaMemcpyDeviceToHost));
      CK(cudaSetDevice(x.dev));
      CK(cudaMemcpy(brow.data(), (const uint8_t*)x.b + rb * cl, rb, cudaMemcpyDeviceToHost));
      decode(arow.data(), sfa_h, rows[i], A[i]);
      decode(brow.data(), DTYPE_ID == 2 ? sfb_dev[x.dev] : sfb_h, cl, B[i]);
    }
    for (int i = 0; i < S; ++i)
      for (int j = 0; j < S; ++j) {
        double ref = 0.0;
        for (int64_t c = 0; c < o.k; ++c) ref += (double)A[i][c] * (double)B[j][c];
        const DeviceGemm& x = g[cols[j] / n_local];
        uint16_t h;
        CK(cudaSetDevice(x.dev));
        CK(cudaMemcpy(&h, (const uint16_t*)x.d + rows[i] + (cols[j] - x.n0) * o.m, 2, cudaMemcpyDeviceToHost));
        const double v = bf16_to_f32(h);
        num += (v - ref) * (v - ref);
        den += ref * ref;
      }
    relerr = den > 0 ? std::sqrt(num / den) : std::sqrt(num);
  }

  const double flops = 2.0 * (double)o.m * (double)o.n * (double)o.k;   // cutlass_gemm_bench.cu:249
  const double tflops = (flops / (avg_ms * 1e-3)) / 1e12;
  std::cout << o.m << "," << o.n << "," << o.k << "," << TILE_M << "," << TILE_N << "," << TILE_K << ","
            << STAGES << "," << kDtype << "," << avg_ms << "," << tflops;
  if (o.full) std::cout << "," << CTA_GROUP << "," << o.ngpus << "," << ag_ms << "," << relerr;
  if (o.full && o.fused_gather) std::cout << "," << fused_ms;
  std::cout << std::endl;

  for (auto& x : g) {
    cudaSetDevice(x.dev);
    cudaFree(x.a); cudaFree(x.b); cudaFree(x.d); cudaFree(x.status);
    if (x.sfa) cudaFree(x.sfa);
    if (x.sfb) cudaFree(x.sfb);
    if (x.dfull) cudaFree(x.dfull);
    if (x.dfused) cudaFree(x.dfused);
  }
  if (o.check && relerr > (DTYPE_ID == 2 ? 1e-2 : 2e-3)) {
    fprintf(stderr, "check failed: relative Frobenius error %.3e\n", relerr);
    return 1;
  }
  return 0;
}
