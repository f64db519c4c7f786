// cutlass_ref.cu -- CUTLASS comparison library.  TEST INFRASTRUCTURE ONLY:
// built by oracle/ref_build.sh into oracle/_ref/libcutlass_ref.so and loaded
// only by GPU tests and bench.py's reference-context numbers.
//
// The reference benchmark (cutlass_gemm_mainloop/cutlass_gemm_bench.cu)
// zero-fills its inputs and never reads D (:71-75, :180-185), so it cannot
// check results.  This file instantiates the same CUTLASS SM100 kernel family
// the reference builds (:101-156: CollectiveBuilder, Sm100 +
// KernelTmaWarpSpecialized1SmSm100 mainloop, NoSmemWarpSpecialized1Sm
// epilogue, LinearCombination<bf16, float, void, float>, A row-major,
// B column-major, D column-major, cluster 1x1x1) at the reference's best
// tiles (BF16 128x256x64 S=4, results.csv:461; FP8 128x256x128 auto stages,
// results.csv:938) and runs it on caller-provided device buffers over the
// whole GPU, so the sm_100a library can be compared with it on identical
// seeded inputs.
#include <cuda_runtime.h>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/numeric_types.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

using namespace cute;

namespace {

template <class ElementAB, int TM, int TN, int TK, int Stages>
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
      void, LayoutD, AlignD, ElementD, LayoutD, AlignD,
      cutlass::epilogue::NoSmemWarpSpecialized1Sm,
      cutlass::epilogue::fusion::LinearCombination<ElementD, float, void, float>>::CollectiveOp;
  using StageType = std::conditional_t<Stages == 0,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epi::SharedStorage))>,
      cutlass::gemm::collective::StageCount<Stages>>;
  using Main = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp,
      ElementAB, LayoutA, AlignAB, ElementAB, LayoutB, AlignAB, float,
      Tile, Cluster, StageType, cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;
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
    cutlass::KernelHardwareInfo hw;
    hw.device_id = 0;
    cudaGetDevice(&hw.device_id);
    hw.sm_count = sm_count;
    typename Gemm::Arguments args{
        cutlass::gemm::GemmUniversalMode::kGemm, {M, N, K, 1},
        {static_cast<const ElementAB*>(A), sa, static_cast<const ElementAB*>(B), sb},
        {{1.0f, 0.0f}, nullptr, sd, static_cast<ElementD*>(D), sd}, hw};
    Gemm op;
    if (Gemm::get_workspace_size(args) != 0) return -5;   // these configurations need none
    if (op.can_implement(args) != cutlass::Status::kSuccess) return -1;
    if (op.initialize(args, nullptr, stream) != cutlass::Status::kSuccess) return -2;
    if (op.run(stream) != cutlass::Status::kSuccess) return -2;
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
};

using RefBf16 = RefGemm<cutlass::bfloat16_t, 128, 256, 64, 4>;
using RefE4m3 = RefGemm<cutlass::float_e4m3_t, 128, 256, 128, 0>;

}  // namespace

// dtype: 0 bf16 (128x256x64, 4 stages), 1 e4m3 (128x256x128, auto stages).
// sm_count <= 0 uses every SM of the current device.  Returns 0 on success.
extern "C" int cutlass_ref_gemm(int dtype, const void* A, const void* B, void* D,
                                int M, int N, int K, int sm_count, void* stream) {
  if (sm_count <= 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == 0) return RefBf16::run(A, B, D, M, N, K, sm_count, s);
  if (dtype == 1) return RefE4m3::run(A, B, D, M, N, K, sm_count, s);
  return -4;
}
