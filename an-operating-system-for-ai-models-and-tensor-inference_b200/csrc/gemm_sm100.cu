// Dense projections for prefill: D[M,N] (f32) = A[M,K] (bf16, row-major) x
// W[N,K]^T (bf16, row-major weights) + beta * C, on the 5th-generation
// tensor cores (tcgen05.mma, operands staged in shared memory by TMA,
// accumulator in TMEM), instantiated from the CUTLASS/CuTe SM100 templates.
//
// The reference's gemm_bf16 (crates/tensor_core/src/gemm_bf16.rs:297-383)
// multiplies bf16 weights by f32 activations with f32 sums. The tensor cores
// take bf16 on both sides, so callers pass each activation as the exact sum
// of three bf16 values (hi, mid, lo; prefill.h kSplitParts), stacked as row
// blocks [hi; mid; lo] of A: one GEMM then yields the three partial outputs
// and the consumer adds them. Every activation bit and every product is
// exact; only the f32 accumulation order differs from the reference's.
// (CUTLASS's stream-K tile scheduler measured slower here than one output
// tile per CTA: 5.27 vs 4.86 ms for a 128-token prefill.)
#include <cutlass/cutlass.h>
#include <cutlass/epilogue/collective/collective_builder.hpp>
#include <cutlass/gemm/collective/collective_builder.hpp>
#include <cutlass/gemm/device/gemm_universal_adapter.h>
#include <cutlass/gemm/kernel/gemm_universal.hpp>
#include <cutlass/util/packed_stride.hpp>
#include <cute/tensor.hpp>

#include "gemm_sm100.h"
#include "kernels.h"

namespace myos {
namespace {

using namespace cute;

using ElementA = cutlass::bfloat16_t;
using ElementB = cutlass::bfloat16_t;
using LayoutA = cutlass::layout::RowMajor;     // activations: K contiguous
using LayoutB = cutlass::layout::ColumnMajor;  // W[N,K] row-major is K x N column-major
using LayoutC = cutlass::layout::RowMajor;
using MmaTile = Shape<_128, _128, _64>;
using ClusterShape = Shape<_1, _1, _1>;

using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTile, ClusterShape,
    cutlass::epilogue::collective::EpilogueTileAuto, float, float, float, LayoutC, 4, float,
    LayoutC, 4, cutlass::epilogue::collective::EpilogueScheduleAuto>::CollectiveOp;

using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElementA, LayoutA, 8, ElementB, LayoutB,
    8, float, MmaTile, ClusterShape,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(
        sizeof(typename Epilogue::SharedStorage))>,
    cutlass::gemm::collective::KernelScheduleAuto>::CollectiveOp;

using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue>;
using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;

typename Gemm::Arguments make_args(int M, int N, int K, const uint16_t* A, const uint16_t* W,
                                   const float* C, float* D, float beta, int ldw = 0) {
  using StrideA = typename Gemm::GemmKernel::StrideA;
  using StrideB = typename Gemm::GemmKernel::StrideB;
  using StrideC = typename Gemm::GemmKernel::StrideC;
  using StrideD = typename Gemm::GemmKernel::StrideD;
  const StrideA sa = cutlass::make_cute_packed_stride(StrideA{}, {M, K, 1});
  StrideB sb = cutlass::make_cute_packed_stride(StrideB{}, {N, K, 1});
  if (ldw > K) cute::get<0>(sb) = ldw;  // W row n starts n * ldw elements in
  const StrideC sc = cutlass::make_cute_packed_stride(StrideC{}, {M, N, 1});
  const StrideD sd = cutlass::make_cute_packed_stride(StrideD{}, {M, N, 1});
  typename Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                {M, N, K, 1},
                                {reinterpret_cast<const ElementA*>(A), sa,
                                 reinterpret_cast<const ElementB*>(W), sb},
                                {{1.0f, beta}, C ? C : D, sc, D, sd}};
  return args;
}

}  // namespace

bool gemm_supported(int M, int N, int K) {
  // 16-byte aligned rows for the TMA copies (8 bf16 / 4 f32 elements)
  return M > 0 && N > 0 && K > 0 && K % 8 == 0 && N % 4 == 0;
}

size_t gemm_workspace_bytes(int M, int N, int K) {
  return Gemm::get_workspace_size(make_args(M, N, K, nullptr, nullptr, nullptr, nullptr, 0.0f));
}

cudaError_t gemm_bf16_f32(int M, int N, int K, const uint16_t* A, const uint16_t* W,
                          const float* C, float* D, float beta, void* workspace,
                          size_t workspace_bytes, cudaStream_t st, int ldw) {
  if (!gemm_supported(M, N, K) || (ldw && (ldw < K || ldw % 8))) return cudaErrorInvalidValue;
  const typename Gemm::Arguments args = make_args(M, N, K, A, W, C, D, beta, ldw);
  Gemm g;
  if (g.can_implement(args) != cutlass::Status::kSuccess) return cudaErrorInvalidValue;
  if (Gemm::get_workspace_size(args) > workspace_bytes) return cudaErrorInvalidValue;
  if (g.initialize(args, workspace, st) != cutlass::Status::kSuccess) return cudaErrorInvalidValue;
  if (g.run(st) != cutlass::Status::kSuccess) return cudaErrorLaunchFailure;
  return counted(cudaGetLastError());
}

}  // namespace myos
