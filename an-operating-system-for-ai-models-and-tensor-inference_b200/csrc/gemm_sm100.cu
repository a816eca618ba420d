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
#ifndef CUTLASS_ENABLE_GDC_FOR_SM100
#error "gemm_sm100.cu needs CUTLASS_ENABLE_GDC_FOR_SM100 (programmatic dependent launch waits)"
#endif
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
// One SM per 128 x 128 output tile, no clusters. (Measured against it and
// dropped: 128 x 256 tiles for the wide projections, slower.)
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

// 64 x 128 tiles (MMA M = 64) for row counts that are a multiple of 64 but
// not of 128 (three bf16 terms of 64 sequences: 192 rows), where 128-row
// tiles would compute a third of their second tile for nothing.
using MmaTile64 = Shape<_64, _128, _64>;

using Epilogue64 = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTile64, ClusterShape,
    cutlass::epilogue::collective::EpilogueTileAuto, float, float, float, LayoutC, 4, float,
    LayoutC, 4, cutlass::epilogue::collective::EpilogueScheduleAuto>::CollectiveOp;

using Mainloop64 = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElementA, LayoutA, 8, ElementB, LayoutB,
    8, float, MmaTile64, ClusterShape,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(
        sizeof(typename Epilogue64::SharedStorage))>,
    cutlass::gemm::collective::KernelScheduleAuto>::CollectiveOp;

using Kernel64 =
    cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop64, Epilogue64>;
using Gemm64 = cutlass::gemm::device::GemmUniversalAdapter<Kernel64>;

template <class G>
typename G::Arguments make_args(int M, int N, int K, const uint16_t* A, const uint16_t* W,
                                const float* C, float* D, float beta, int ldw = 0,
                                int splits = 1) {
  using StrideA = typename G::GemmKernel::StrideA;
  using StrideB = typename G::GemmKernel::StrideB;
  using StrideC = typename G::GemmKernel::StrideC;
  using StrideD = typename G::GemmKernel::StrideD;
  // Split-K as the batch mode: batch l multiplies the K slice
  // [l * Kc, (l + 1) * Kc) of A and W (the same rows, Kc elements further on)
  // and writes its own [M, N] block of D, so D holds `splits` partial
  // products that the consumer adds in a fixed order.
  const int Kc = K / splits;
  StrideA sa = cutlass::make_cute_packed_stride(StrideA{}, {M, Kc, splits});
  cute::get<0>(sa) = K;
  cute::get<2>(sa) = Kc;
  StrideB sb = cutlass::make_cute_packed_stride(StrideB{}, {N, Kc, splits});
  cute::get<0>(sb) = ldw > K ? ldw : K;  // W row n starts n * ldw elements in
  cute::get<2>(sb) = Kc;
  const StrideC sc = cutlass::make_cute_packed_stride(StrideC{}, {M, N, splits});
  const StrideD sd = cutlass::make_cute_packed_stride(StrideD{}, {M, N, splits});
  typename G::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                {M, N, Kc, splits},
                                {reinterpret_cast<const ElementA*>(A), sa,
                                 reinterpret_cast<const ElementB*>(W), sb},
                                {{1.0f, beta}, C ? C : D, sc, D, sd}};
  return args;
}

template <class G>
cudaError_t run(int M, int N, int K, const uint16_t* A, const uint16_t* W, const float* C, float* D,
                float beta, void* workspace, size_t workspace_bytes, cudaStream_t st, int ldw,
                int splits, bool pdl) {
  const typename G::Arguments args = make_args<G>(M, N, K, A, W, C, D, beta, ldw, splits);
  G g;
  if (g.can_implement(args) != cutlass::Status::kSuccess) return cudaErrorInvalidValue;
  if (G::get_workspace_size(args) > workspace_bytes) return cudaErrorInvalidValue;
  if (g.initialize(args, workspace, st) != cutlass::Status::kSuccess) return cudaErrorInvalidValue;
  // pdl: launched with a programmatic edge to the previous kernel; the
  // kernel's loading warps wait for it (griddepcontrol.wait, compiled in by
  // CUTLASS_ENABLE_GDC_FOR_SM100) before their first global read
  if (g.run(st, nullptr, pdl) != cutlass::Status::kSuccess) return cudaErrorLaunchFailure;
  return counted(cudaGetLastError());
}

}  // namespace

bool gemm_supported(int M, int N, int K) {
  // 16-byte aligned rows for the TMA copies (8 bf16 / 4 f32 elements)
  return M > 0 && N > 0 && K > 0 && K % 8 == 0 && N % 4 == 0;
}

size_t gemm_workspace_bytes(int M, int N, int K) {
  const size_t a =
      Gemm::get_workspace_size(make_args<Gemm>(M, N, K, nullptr, nullptr, nullptr, nullptr, 0.0f));
  const size_t b = Gemm64::get_workspace_size(
      make_args<Gemm64>(M, N, K, nullptr, nullptr, nullptr, nullptr, 0.0f));
  return a > b ? a : b;
}

bool gemm_use64(int M, bool allow) { return allow && M % 128 != 0 && M % 64 == 0; }

int gemm_pick_splits(int M, int N, int K, int sms, bool m64) {
  // One 128 x 128 output tile per CTA: a projection with fewer tiles than
  // SMs streams its weights through a fraction of the chip (each SM pulls
  // its tile's K extent alone), so the K extent is cut into slices of whole
  // 64-wide k-blocks until the tiles x slices fill the SMs once, keeping at
  // least four k-blocks per slice.
  const int tm = gemm_use64(M, m64) ? 64 : 128;
  const long tiles = (long)((M + tm - 1) / tm) * ((N + 127) / 128);
  if (K % 64 != 0 || tiles * 2 > sms) return 1;
  const int kb = K / 64;
  int best = 1;
  for (int s = 2; s <= kMaxSplits; ++s)
    if (kb % s == 0 && kb / s >= 4 && tiles * s <= sms) best = s;
  return best;
}

cudaError_t gemm_bf16_f32(int M, int N, int K, const uint16_t* A, const uint16_t* W,
                          const float* C, float* D, float beta, void* workspace,
                          size_t workspace_bytes, cudaStream_t st, int ldw, int splits, bool pdl,
                          bool m64) {
  if (!gemm_supported(M, N, K) || (ldw && (ldw < K || ldw % 8))) return cudaErrorInvalidValue;
  if (splits < 1 || splits > kMaxSplits || K % splits || (K / splits) % 8 ||
      (splits > 1 && (C || beta != 0.0f)))
    return cudaErrorInvalidValue;
  if (gemm_use64(M, m64))
    return run<Gemm64>(M, N, K, A, W, C, D, beta, workspace, workspace_bytes, st, ldw, splits, pdl);
  return run<Gemm>(M, N, K, A, W, C, D, beta, workspace, workspace_bytes, st, ldw, splits, pdl);
}

}  // namespace myos
