/*
 * gemm_sm100a.h -- C ABI of the B200 (sm_100a) dense GEMM mainloop library.
 *
 * The library replaces the CUTLASS SM100 GEMM that the reference benchmark
 * cutlass_gemm_mainloop/cutlass_gemm_bench.cu instantiates (GEMM types at
 * cutlass_gemm_bench.cu:101-156) and drives through
 * Gemm::can_implement / initialize / run (cutlass_gemm_bench.cu:206-239).
 * The math is the reference's:
 *
 *     D = alpha * (A . B^T) + beta * C      (the reference runs beta = 0 with no C source,
 *                                            cutlass_gemm_bench.cu:117-118,196-204; its
 *                                            LinearCombination epilogue also takes beta and C)
 *
 *   A  M x K, row-major   (K contiguous)      cutlass_gemm_bench.cu:103 LayoutA = RowMajor
 *   B  N x K, "K-major"   (K contiguous)      cutlass_gemm_bench.cu:104 LayoutB = ColumnMajor (K x N)
 *   D  M x N, column-major (M contiguous), bf16  cutlass_gemm_bench.cu:105 LayoutD = ColumnMajor
 *   accumulate in fp32                         cutlass_gemm_bench.cu:69 ElementAccumulator = float
 *
 * Element types: bf16 and fp8 e4m3 as in the reference (DTYPE_ID 0 and 1,
 * cutlass_gemm_bench.cu:57-66), plus NVFP4 (DTYPE_ID 2): packed e2m1 values
 * with one unsigned e4m3 scale per 16 consecutive K elements of each row.
 *
 * Ownership: the caller owns every buffer (A, B, scale factors, D and the
 * optional status word). The launcher allocates nothing and throws nothing;
 * its only global state is a once-initialised driver entry point and a
 * mutex-guarded record of the kernels whose shared-memory limit it has raised
 * on each device, so concurrent calls on different streams or devices are safe.
 */
#ifndef GEMM_SM100A_H
#define GEMM_SM100A_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element type selector; the numeric values equal the reference's DTYPE_ID
 * (cutlass_gemm_bench.cu:57-66) with NVFP4 appended. */
enum {
  GEMM_DTYPE_BF16     = 0,
  GEMM_DTYPE_FP8_E4M3 = 1,
  GEMM_DTYPE_NVFP4    = 2
};

/* Return codes. */
enum {
  GEMM_OK               = 0,
  GEMM_ERR_CANNOT_IMPLEMENT = -1,  /* shape, alignment, knob or smem limit (Gemm::can_implement, cutlass_gemm_bench.cu:211-218) */
  GEMM_ERR_LAUNCH       = -2,      /* CUDA launch / driver error (Gemm::initialize / run failure, cutlass_gemm_bench.cu:220-224) */
  GEMM_ERR_TIMEOUT      = -3,      /* a device-side bounded wait ran out; read back from the status word */
  GEMM_ERR_BAD_ARGS     = -4       /* null pointer, struct-size mismatch */
};

/* Layout of D (and C): the reference's LayoutD is column-major
 * (cutlass_gemm_bench.cu:105); row-major is the other LinearCombination layout. */
enum {
  GEMM_LAYOUT_COL_MAJOR = 0,   /* M contiguous, element (i, j) at i + j * ld */
  GEMM_LAYOUT_ROW_MAJOR = 1    /* N contiguous, element (i, j) at i * ld + j */
};

/* Flags. */
enum {
  /* Fault injection for tests of the timeout path: the producer warp issues
   * no loads, so every consumer wait runs out after timeout_ms and the kernel
   * records GEMM_ERR_TIMEOUT in *status and returns.  Never used for timing. */
  GEMM_FLAG_INJECT_STALL = 1u << 0,
  /* Store D straight from registers instead of staging each chunk in shared
   * memory for a TMA store (the fallback when the staging buffers do not fit
   * next to the ring); for comparisons of the two epilogues. */
  GEMM_FLAG_DIRECT_EPILOGUE = 1u << 1
};

/*
 * GemmArgs: one GEMM problem plus the kernel knobs.
 *
 * Knob names and defaults follow the reference's compile-time macros
 * (cutlass_gemm_bench.cu:34-49: TILE_M=128, TILE_N=128, TILE_K=64,
 * STAGES=0 meaning "auto", DTYPE_ID=0); here they are runtime fields.
 * cta_group (1 or 2) selects 1-SM or 2-SM (CTA pair) MMAs; cluster_m is the
 * number of CTAs per cluster along M and must equal cta_group (no load uses
 * cluster multicast).
 *
 * Leading dimensions are in ELEMENTS (for NVFP4, elements are 4-bit; lda and
 * ldb must then be even).  All base pointers must be 16-byte aligned and
 * lda*elem_bytes, ldb*elem_bytes, ldd*2 multiples of 16 (the reference's
 * 128-bit AlignmentA/B/D, cutlass_gemm_bench.cu:110-112).
 *
 * NVFP4 scale factors (sfa for A, sfb for B) are unsigned e4m3 bytes in the
 * 128-row x 4-scale interleaved atom layout: for row r and scale column c
 * (c = k / 16) the byte offset is
 *     ((r / 128) * (K / 64) + c / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4)
 * NVFP4 needs m a multiple of the MMA M (128, or 256 for cta_group 2), n a
 * multiple of tile_n and k a multiple of tile_k; the scale buffers then hold
 * (m / 128) * (k / 64) and (n / 128) * (k / 64) atoms of 512 bytes.
 */
typedef struct GemmArgs {
  uint32_t struct_size;   /* sizeof(GemmArgs), guards ABI drift */
  int32_t  dtype;         /* GEMM_DTYPE_* */
  int64_t  m, n, k;
  const void* a;  int64_t lda;
  const void* b;  int64_t ldb;
  void*       d;  int64_t ldd;
  const void* sfa;        /* NVFP4 only */
  const void* sfb;        /* NVFP4 only */
  float    alpha;         /* D = alpha * acc; 1.0 in the reference */
  int32_t  tile_m;        /* per-MMA M: 64 or 128 (cta_group 1), 256 (cta_group 2); 0 = default */
  int32_t  tile_n;        /* cta_group 1: 16, 32, 64, 128, 192, 256; cta_group 2: 64, 128, 192, 256, 512;
                             NVFP4: 128 or 256; 0 = default (256) */
  int32_t  tile_k;        /* K per pipeline stage: one or two 32-byte MMA K steps (bf16 16/32, fp8 32/64),
                             or 1, 2 or 4 128-byte swizzle atoms (bf16 64/128/256, fp8 128/256/512,
                             NVFP4 256/512/1024); 0 = one atom */
  int32_t  stages;        /* shared-memory ring depth; 0 = auto (as many as fit) */
  int32_t  cta_group;     /* 1 or 2; 0 = default (1) */
  int32_t  cluster_m;     /* CTAs per cluster along M; 0 = cta_group */
  int32_t  max_ctas;      /* grid cap; 0 = one CTA per SM (persistent); 1 = single-CTA mainloop mode */
  int32_t  raster_group;  /* tile order for L2 reuse: G > 0 groups of G M-tiles (M fastest), G < 0 groups of -G N-tiles (N fastest); 0 = default */
  int32_t* status;        /* optional device int32: 0 on success, GEMM_ERR_TIMEOUT (and where) on a device wait timeout */
  uint32_t timeout_ms;    /* device wait budget; 0 = default (4000 ms) */
  uint32_t flags;         /* GEMM_FLAG_* */
  int32_t  l2_prefetch;   /* warm L2 this many k-blocks ahead of the shared-memory ring; 0 = default, < 0 = off */
  unsigned long long* clock_out; /* optional device [2]: every CTA adds the SM cycles and nanoseconds it
                                    spent in the launch (zero it first; cycles / ns = the launch's mean
                                    effective SM clock under power capping) */
  /* Epilogue (CUTLASS LinearCombination, cutlass_gemm_bench.cu:117-118,196-204):
   * D = alpha * scale_a * scale_b * (A . B^T) + beta * C, computed in fp32 and
   * rounded once to bf16.  C is bf16 with D's layout and leading dimension ldc
   * (16-byte aligned, ldc a multiple of 8), read only when beta != 0; C may be D. */
  float    beta;          /* 0 in the reference */
  const void* c;          /* bf16 C, or NULL when beta == 0 */
  int64_t  ldc;
  int32_t  d_layout;      /* GEMM_LAYOUT_*; 0 = column-major as in the reference */
  float    scale_a;       /* per-tensor dequantisation scale of A (fp8: "per-tensor fp32 scale"); 0 means 1.0 */
  float    scale_b;       /* per-tensor scale of B; 0 means 1.0 */
} GemmArgs;

/* What a launch would do; filled by gemm_sm100a_query. */
typedef struct GemmInfo {
  uint32_t struct_size;
  int32_t  tile_m, tile_n, tile_k, stages, cta_group, cluster_m;
  int32_t  max_stages;           /* stages that fit in 227 KiB of shared memory */
  int64_t  smem_bytes_per_stage; /* per CTA */
  int64_t  smem_bytes;           /* dynamic shared memory per CTA */
  int32_t  tmem_columns;         /* tensor-memory columns allocated per CTA */
  int32_t  grid_ctas;            /* CTAs launched */
  int64_t  num_tiles;            /* output tiles (per CTA pair for cta_group 2) */
  int32_t  num_sms;
  int32_t  can_implement;        /* 1 if gemm_sm100a_launch would accept the arguments */
  char     reason[128];          /* why not, when can_implement == 0 */
  int32_t  epilogue_staging_buffers; /* shared-memory staging buffers per epilogue group (TMA-store
                                        epilogue); 0 = D stored directly from registers */
} GemmInfo;

/*
 * Validate the arguments and resolve defaults / auto stages without
 * launching.  Replaces Gemm::can_implement + Gemm::get_workspace_size
 * (cutlass_gemm_bench.cu:208-218); the workspace is always zero bytes.
 * Returns GEMM_OK or GEMM_ERR_CANNOT_IMPLEMENT / GEMM_ERR_BAD_ARGS.
 */
int gemm_sm100a_query(const GemmArgs* args, GemmInfo* info);

/*
 * Enqueue D = alpha * A . B^T on `stream` (a cudaStream_t; 0 = legacy default
 * stream).  Replaces Gemm::initialize + Gemm::run (cutlass_gemm_bench.cu:220-239):
 * each call encodes the TMA descriptors on the host and issues exactly one
 * kernel launch.  Asynchronous: a device wait timeout is reported through
 * args->status, read it with gemm_sm100a_read_status after synchronising.
 * Returns GEMM_OK, GEMM_ERR_CANNOT_IMPLEMENT, GEMM_ERR_BAD_ARGS or GEMM_ERR_LAUNCH.
 */
int gemm_sm100a_launch(const GemmArgs* args, void* stream);

/*
 * gemm_sm100a_launch, fused with an all-gather of D across the GPUs of one
 * box: the epilogue also stores every element of this launch's D block into
 * each of `n_peers` (at most 7) further buffers, typically the same block of
 * the full D on the other GPUs of an N-split, so the gather overlaps the GEMM
 * instead of following it (replaces the GEMM + ncclAllGather pair the N-split
 * harness otherwise issues; the reference is single-GPU and has none).
 * Each peer buffer uses args->ldd and must hold the same m x n block as
 * args->d (checked against its allocation before the launch); D must be
 * column-major (GEMM_ERR_CANNOT_IMPLEMENT otherwise).  Peer pointers must be device memory this GPU can reach: the call
 * enables peer access to other GPUs' memory and returns GEMM_ERR_BAD_ARGS for
 * host memory, unreachable devices or misaligned pointers.  Only D is
 * gathered; completion on every GPU means the full D is complete there.
 * It pays off while the D bytes each GPU sends are small next to its GEMM
 * time: on B200, config 5 split over 2 GPUs ran 33 % faster than GEMM +
 * ncclAllGather, over 8 GPUs 23 % slower (the epilogue's 64-byte stores move
 * ~370 GB/s per GPU over NVLink, NCCL ~580 GB/s).
 */
int gemm_sm100a_launch_gather(const GemmArgs* args, void* const* peer_d, int32_t n_peers, void* stream);

/*
 * Synchronise `stream`, copy the device status word back and map it to a
 * return code (GEMM_OK or GEMM_ERR_TIMEOUT); *detail (optional) receives the
 * raw word, which encodes the waiting role and pipeline stage.
 */
int gemm_sm100a_read_status(const int32_t* status, void* stream, int32_t* detail);

/* Static description of a return code. */
const char* gemm_sm100a_strerror(int code);

/* Library version, major*10000 + minor*100 + patch. */
int gemm_sm100a_version(void);

/*
 * Seeded input generation on the device (harness helper, not part of the
 * GEMM).  Every element is a pure function of (seed, stream_id, index), so
 * any GPU can regenerate any slice of a matrix and a host checker can
 * regenerate any element.
 *   dist: 0 = uniform[-1,1), 1 = normal(0,1)
 *   out_dtype: GEMM_DTYPE_BF16 or GEMM_DTYPE_FP8_E4M3 (round to nearest even,
 *   fp8 saturating); values are multiplied by `scale` before rounding.
 * Generates rows [row0, row0+rows) of a rows_total x cols row-major matrix
 * (row stride ld elements); element (r, c) uses index r*cols + c.
 */
int gemm_sm100a_generate(void* out, int32_t out_dtype, int32_t dist, float scale,
                         uint64_t seed, uint64_t stream_id,
                         int64_t row0, int64_t rows, int64_t cols, int64_t ld,
                         void* cuda_stream);

/*
 * NVFP4 quantisation of a seeded normal(0,1)*scale matrix on the device:
 * writes packed e2m1 values (two per byte, low nibble = even column) and the
 * unsigned-e4m3 block scales (absmax/6 rounded up) in the interleaved layout
 * described above.  Rows [row0, row0+rows) of a matrix with `cols` columns
 * (cols a multiple of 64, row0 and rows multiples of 128).
 */
int gemm_sm100a_generate_nvfp4(void* out_packed, void* out_scales, float scale,
                               uint64_t seed, uint64_t stream_id,
                               int64_t row0, int64_t rows, int64_t cols,
                               void* cuda_stream);

/*
 * Measured tcgen05 dense peak (replaces the reference's umma_throughput/umma_tput.cu
 * probe, kernel :286-544, with an NVFP4 kind and a whole-GPU mode added).
 * Launches `num_ctas` CTAs (a multiple of cta_group; one per SM at most), each
 * issuing `iters` groups of `depth` back-to-back M=128*cta_group, N=256 MMAs of
 * `dtype` from shared memory, one commit per group.  results (device, caller-owned,
 * 3*num_ctas uint64) receives per CTA {clock64 cycles, %globaltimer ns, status}
 * (zeros for the non-issuing CTA of a pair).  Returns GEMM_OK, GEMM_ERR_BAD_ARGS
 * or GEMM_ERR_LAUNCH; asynchronous on `stream`.
 */
int gemm_sm100a_umma_peak(int32_t dtype, int32_t cta_group, int32_t num_ctas, int32_t depth,
                          int32_t iters, unsigned long long* results, void* stream);

/*
 * TMA-2D HBM read-throughput probe (replaces the reference's
 * tma2d_throughput/tma2d_tput.cu: kernel :42-126, launch :131-219).  Launches
 * ctas_per_sm one-warp CTAs per SM (227 KiB of shared memory each, as the
 * reference pins it), which stream the 32-bit words of `buf` (read as a
 * (bytes / (4 * box_width)) x box_width row-major tensor, whole box_rows-row
 * tiles only) through a `stages`-deep ring of (box_rows x box_width) TMA
 * tiles.  results (device, caller-owned, 5 * num_SMs * ctas_per_sm uint64)
 * receives per CTA {clock64 cycles, %globaltimer ns, tiles loaded, XOR of the
 * first 32 words of every tile it loaded, status (0, or 3 if a load wait ran
 * out after 2 s)}.  box_width: 4..256 words, a multiple of 4; box_rows 1..256;
 * tiles of at least 128 bytes.  Time it with events on `stream` after
 * flushing L2: bytes / time is the TMA read roof.  Returns GEMM_OK,
 * GEMM_ERR_BAD_ARGS, GEMM_ERR_CANNOT_IMPLEMENT (ring over shared memory) or
 * GEMM_ERR_LAUNCH; asynchronous.
 */
int gemm_sm100a_tma_read_probe(const void* buf, int64_t bytes, int32_t box_width, int32_t box_rows,
                               int32_t stages, int32_t ctas_per_sm, unsigned long long* results, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GEMM_SM100A_H */
