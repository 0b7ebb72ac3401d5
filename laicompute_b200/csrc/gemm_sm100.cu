// Dense fp16 GEMM on the 5th-generation tensor cores (tcgen05.mma, TMEM
// accumulators, TMA loads) for the batched prompt prefill:
//   C[M][N] (fp32) = A[M][K] (fp16, row-major) x W[N][K]^T (fp16, row-major weights [out][in])
// Built from CUTLASS's sm100 collective mainloop / epilogue builders with a
// 1x1x1 cluster (no multicast loads: every operand is this GPU's own memory).
#include <cuda_runtime.h>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

namespace laic {
namespace {

using namespace cute;

using ElementA = cutlass::half_t;
using LayoutA = cutlass::layout::RowMajor;
constexpr int kAlignA = 8;
using ElementB = cutlass::half_t;
using LayoutB = cutlass::layout::ColumnMajor;  // W[N][K] row-major = K x N column-major
constexpr int kAlignB = 8;
using ElementC = float;
using LayoutC = cutlass::layout::RowMajor;
constexpr int kAlignC = 4;
using ElementAcc = float;

using MmaTile = Shape<_128, _128, _64>;
using Cluster = Shape<_1, _1, _1>;

using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTile, Cluster,
    cutlass::epilogue::collective::EpilogueTileAuto, ElementAcc, ElementAcc, ElementC, LayoutC, kAlignC, ElementC,
    LayoutC, kAlignC, cutlass::epilogue::collective::EpilogueScheduleAuto>::CollectiveOp;

using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElementA, LayoutA, kAlignA, ElementB, LayoutB, kAlignB,
    ElementAcc, MmaTile, Cluster,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
    cutlass::gemm::collective::KernelScheduleAuto>::CollectiveOp;

using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue, void>;
using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;

typename Gemm::Arguments make_args(int M, int N, int K, const void* A, const void* W, float* C) {
    using StrideA = typename Gemm::GemmKernel::StrideA;
    using StrideB = typename Gemm::GemmKernel::StrideB;
    using StrideC = typename Gemm::GemmKernel::StrideC;
    using StrideD = typename Gemm::GemmKernel::StrideD;
    const StrideA sa = cutlass::make_cute_packed_stride(StrideA{}, cute::make_shape(M, K, 1));
    const StrideB sb = cutlass::make_cute_packed_stride(StrideB{}, cute::make_shape(N, K, 1));
    const StrideC sc = cutlass::make_cute_packed_stride(StrideC{}, cute::make_shape(M, N, 1));
    const StrideD sd = cutlass::make_cute_packed_stride(StrideD{}, cute::make_shape(M, N, 1));
    typename Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                  {M, N, K, 1},
                                  {reinterpret_cast<const ElementA*>(A), sa, reinterpret_cast<const ElementB*>(W), sb},
                                  {{1.f, 0.f}, C, sc, C, sd}};
    return args;
}

}  // namespace

// Workspace bytes the GEMM of this shape needs (0 when it needs none).
size_t gemm_f16_workspace(int M, int N, int K) {
    return Gemm::get_workspace_size(make_args(M, N, K, nullptr, nullptr, nullptr));
}

// C = A x W^T. Shapes: K a multiple of 8, N a multiple of 4. Returns a CUDA error code
// (cudaErrorInvalidValue when CUTLASS rejects the shape).
cudaError_t gemm_f16(int M, int N, int K, const void* A, const void* W, float* C, void* workspace, size_t ws_bytes,
                     cudaStream_t st) {
    Gemm gemm;
    auto args = make_args(M, N, K, A, W, C);
    if (gemm.can_implement(args) != cutlass::Status::kSuccess) return cudaErrorInvalidValue;
    if (Gemm::get_workspace_size(args) > ws_bytes) return cudaErrorInvalidValue;
    if (gemm.initialize(args, workspace, st) != cutlass::Status::kSuccess) return cudaErrorInvalidValue;
    if (gemm.run(st) != cutlass::Status::kSuccess) return cudaErrorLaunchFailure;
    return cudaGetLastError();
}

}  // namespace laic
