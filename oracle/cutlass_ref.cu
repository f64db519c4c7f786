// cutlass_ref.cu -- CUTLASS comparison library.  TEST INFRASTRUCTURE ONLY:
// built by oracle/ref_build.sh into oracle/_ref/libcutlass_ref.so and loaded
// only by GPU tests and bench.py's reference-context numbers.
//
// The reference benchmark (cutlass_gemm_mainloop/cutlass_gemm_bench.cu)
// zero-fills its inputs and never reads D (:71-75, :180-185), so it cannot
// check results.  This file instantiates the CUTLASS SM100 kernel family the
// reference builds (:101-156: CollectiveBuilder, A row-major, B column-major,
// D column-major bf16, LinearCombination<bf16, float, void, float>, fp32
// accumulate) and runs it on caller-provided device buffers over the whole
// GPU, so the sm_100a library can be compared with it on identical seeded
// inputs:
//
//   id 0  bf16 1SM 128x256x64, 4 stages  (the reference's best bf16 point,
//         results.csv:461; KernelTmaWarpSpecialized1SmSm100 +
//         NoSmemWarpSpecialized1Sm, cluster 1x1x1, exactly :107-136)
//   id 1  e4m3 1SM 128x256x128, auto stages (results.csv:938)
//   id 4  NVFP4 1SM 128x256x256 (KernelTmaWarpSpecialized1SmNvf4Sm100), the
//         reference family extended to the block-scaled type (the reference
//         has no NVFP4, :58-66)
//
// Every kernel here runs on a cluster of one CTA.  CUTLASS's 2SM schedules need
// a 2x1 cluster, a form this pool treats as a cluster-multicast TMA load (which
// would bar every multi-GPU run), so they are not instantiated.  The NVFP4
// scale buffers use CUTLASS's K-major 128x4 scale atom (Sm1xxBlockScaledConfig,
// tiled K-blocks fastest), the byte layout the sm_100a library takes, so both
// kernels read the same buffers.
//
// REF_PART selects which instantiations this translation unit compiles
// (0: ids 0-1, 2: id 4, -1: all) so the build can run the slow CUTLASS
// compilations in parallel; every part defines its own entry.
#include <cuda_runtime.h>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/numeric_types.h"
#include "cutlass/float_subbyte.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"
#include "cutlass/detail/sm100_blockscaled_layout.hpp"

#ifndef REF_PART
#define REF_PART -1
#endif

using namespace cute;

namespace {

template <class Gemm>
int run_adapter(typename Gemm::Arguments const& args, cudaStream_t stream) {
  Gemm op;
  if (Gemm::get_workspace_size(args) != 0) return -5;   // these configurations need none
  if (op.can_implement(args) != cutlass::Status::kSuccess) return -1;
  if (op.initialize(args, nullptr, stream) != cutlass::Status::kSuccess) return -2;
  if (op.run(stream) != cutlass::Status::kSuccess) return -2;
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

cutlass::KernelHardwareInfo hw_info(int sm_count) {
  cutlass::KernelHardwareInfo hw;
  hw.device_id = 0;
  cudaGetDevice(&hw.device_id);
  hw.sm_count = sm_count;
  return hw;
}

// Dense bf16 / e4m3 GEMM of the reference family.
template <class ElementAB, int TM, int TN, int TK, int Stages, class MainSched, class EpiSched>
struct RefGemm {
  using LayoutA = cutlass::layout::RowMajor;
  using LayoutB = cutlass::layout::ColumnMajor;
  using LayoutD = cutlass::layout::ColumnMajor;
  using ElementD = cutlass::bfloat16_t;
  using Cluster = Shape<_1, _1, _1>;
  using Tile = Shape<Int<TM>, Int<TN>, Int<TK>>;
  static constexpr int AlignAB = 128 / cutlass::sizeof_bits<ElementAB>::value;
  static constexpr int AlignD = 128 / cutlass::sizeof_bits<ElementD>::value;

  using Epi = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, Tile, Cluster,
      cutlass::epilogue::collective::EpilogueTileAuto, float, float,
      void, LayoutD, AlignD, ElementD, LayoutD, AlignD, EpiSched,
      cutlass::epilogue::fusion::LinearCombination<ElementD, float, void, float>>::CollectiveOp;
  using StageType = std::conditional_t<Stages == 0,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epi::SharedStorage))>,
      cutlass::gemm::collective::StageCount<Stages>>;
  using Main = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp,
      ElementAB, LayoutA, AlignAB, ElementAB, LayoutB, AlignAB, float,
      Tile, Cluster, StageType, MainSched>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Main, Epi>;
  using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;

  static int run(const void* A, const void* B, void* D, int M, int N, int K, int sm_count,
                 cudaStream_t stream) {
    using SA = typename Gemm::GemmKernel::StrideA;
    using SB = typename Gemm::GemmKernel::StrideB;
    using SD = typename Gemm::GemmKernel::StrideD;
    auto sa = cutlass::make_cute_packed_stride(SA{}, cute::make_shape(M, K, 1));
    auto sb = cutlass::make_cute_packed_stride(SB{}, cute::make_shape(N, K, 1));
    auto sd = cutlass::make_cute_packed_stride(SD{}, cute::make_shape(M, N, 1));
    typename Gemm::Arguments args{
        cutlass::gemm::GemmUniversalMode::kGemm, {M, N, K, 1},
        {static_cast<const ElementAB*>(A), sa, static_cast<const ElementAB*>(B), sb},
        {{1.0f, 0.0f}, nullptr, sd, static_cast<ElementD*>(D), sd}, hw_info(sm_count)};
    return run_adapter<Gemm>(args, stream);
  }
};

// NVFP4 block-scaled GEMM (e2m1 values, ue4m3 scale per 16 K elements).
template <int TM, int TN, int TK, class MainSched>
struct RefNvf4 {
  using ElementAB = cutlass::nv_float4_t<cutlass::float_e2m1_t>;
  using LayoutA = cutlass::layout::RowMajor;
  using LayoutB = cutlass::layout::ColumnMajor;
  using LayoutD = cutlass::layout::ColumnMajor;
  using ElementD = cutlass::bfloat16_t;
  using Cluster = Shape<_1, _1, _1>;
  using Tile = Shape<Int<TM>, Int<TN>, Int<TK>>;
  static constexpr int AlignAB = 32;
  static constexpr int AlignD = 128 / cutlass::sizeof_bits<ElementD>::value;

  using Epi = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassBlockScaledTensorOp, Tile, Cluster,
      cutlass::epilogue::collective::EpilogueTileAuto, float, float,
      void, LayoutD, AlignD, ElementD, LayoutD, AlignD,
      cutlass::epilogue::collective::EpilogueScheduleAuto>::CollectiveOp;
  using Main = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassBlockScaledTensorOp,
      ElementAB, LayoutA, AlignAB, ElementAB, LayoutB, AlignAB, float, Tile, Cluster,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epi::SharedStorage))>,
      MainSched>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Main, Epi>;
  using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
  using Cfg = typename Kernel::CollectiveMainloop::Sm1xxBlkScaledConfig;

  static int run(const void* A, const void* B, const void* SFA, const void* SFB, void* D, int M, int N, int K,
                 int sm_count, cudaStream_t stream) {
    using SA = typename Gemm::GemmKernel::StrideA;
    using SB = typename Gemm::GemmKernel::StrideB;
    using SD = typename Gemm::GemmKernel::StrideD;
    using DataT = typename ElementAB::DataType;
    using SfT = typename ElementAB::ScaleFactorType;
    auto sa = cutlass::make_cute_packed_stride(SA{}, cute::make_shape(M, K, 1));
    auto sb = cutlass::make_cute_packed_stride(SB{}, cute::make_shape(N, K, 1));
    auto sd = cutlass::make_cute_packed_stride(SD{}, cute::make_shape(M, N, 1));
    auto lsfa = Cfg::tile_atom_to_shape_SFA(cute::make_shape(M, N, K, 1));
    auto lsfb = Cfg::tile_atom_to_shape_SFB(cute::make_shape(M, N, K, 1));
    typename Gemm::Arguments args{
        cutlass::gemm::GemmUniversalMode::kGemm, {M, N, K, 1},
        {static_cast<const DataT*>(A), sa, static_cast<const DataT*>(B), sb,
         static_cast<const SfT*>(SFA), lsfa, static_cast<const SfT*>(SFB), lsfb},
        {{1.0f, 0.0f}, nullptr, sd, static_cast<ElementD*>(D), sd}, hw_info(sm_count)};
    return run_adapter<Gemm>(args, stream);
  }
};

using namespace cutlass::gemm;
using namespace cutlass::epilogue;

}  // namespace

// Per-part entry: returns -6 for an id another part implements.
#define PART_ENTRY(P) cutlass_ref_part##P

#if REF_PART == 0 || REF_PART == -1
extern "C" int PART_ENTRY(0)(int id, const void* A, const void* B, const void*, const void*, void* D, int M, int N,
                             int K, int sms, cudaStream_t s) {
  if (id == 0)
    return RefGemm<cutlass::bfloat16_t, 128, 256, 64, 4, KernelTmaWarpSpecialized1SmSm100,
                   NoSmemWarpSpecialized1Sm>::run(A, B, D, M, N, K, sms, s);
  if (id == 1)
    return RefGemm<cutlass::float_e4m3_t, 128, 256, 128, 0, KernelTmaWarpSpecialized1SmSm100,
                   NoSmemWarpSpecialized1Sm>::run(A, B, D, M, N, K, sms, s);
  return -6;
}
#endif
#if REF_PART == 2 || REF_PART == -1
extern "C" int PART_ENTRY(2)(int id, const void* A, const void* B, const void* SFA, const void* SFB, void* D, int M,
                             int N, int K, int sms, cudaStream_t s) {
  if (id == 4)
    return RefNvf4<128, 256, 256, KernelTmaWarpSpecialized1SmNvf4Sm100>::run(A, B, SFA, SFB, D, M, N, K, sms, s);
  return -6;
}
#endif

#if REF_PART == 0 || REF_PART == -1
extern "C" int cutlass_ref_part2(int, const void*, const void*, const void*, const void*, void*, int, int, int, int,
                                 cudaStream_t);

// Run kernel `id` (table above) on device buffers: D (column-major M x N bf16)
// = A . B^T.  sfa / sfb are the NVFP4 scale buffers (id 4, else unused).
// sm_count <= 0 uses every SM of the current device.  Returns 0 on success,
// -1 can't implement, -2 launch error, -4 unknown id.
extern "C" int cutlass_ref_run(int id, const void* A, const void* B, const void* sfa, const void* sfb, void* D,
                               int M, int N, int K, int sm_count, void* stream) {
  if (sm_count <= 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (id) {
    case 0: case 1: return cutlass_ref_part0(id, A, B, sfa, sfb, D, M, N, K, sm_count, s);
    case 4: return cutlass_ref_part2(id, A, B, sfa, sfb, D, M, N, K, sm_count, s);
  }
  return -4;
}

// Earlier entry kept for callers of the 1SM reference points: dtype 0 = id 0, 1 = id 1.
extern "C" int cutlass_ref_gemm(int dtype, const void* A, const void* B, void* D, int M, int N, int K, int sm_count,
                                void* stream) {
  if (dtype != 0 && dtype != 1) return -4;
  return cutlass_ref_run(dtype, A, B, nullptr, nullptr, D, M, N, K, sm_count, stream);
}
#endif
