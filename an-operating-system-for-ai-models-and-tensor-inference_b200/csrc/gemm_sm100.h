// Prefill projections on the sm_100 tensor cores (gemm_sm100.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace myos {

// D[M,N] = A[M,K] x W[N,K]^T + beta * C (C may be null when beta == 0); A and
// W bf16 row-major (W's rows ldw >= K elements apart; 0: K), C and D f32
// row-major; stream-ordered, no allocation.
//
// splits > 1 (split-K; C null, beta 0): K is cut into `splits` equal slices
// (K / splits a multiple of 8) and D receives `splits` consecutive [M, N]
// blocks, block l = A[:, l*Kc:(l+1)*Kc] x W[:, l*Kc:(l+1)*Kc]^T; the caller
// adds them.
constexpr int kMaxSplits = 8;
bool gemm_supported(int M, int N, int K);
size_t gemm_workspace_bytes(int M, int N, int K);
// Slices that let an [M, N] output's 128 x 128 tiles fill `sms` SMs once
// (1 when the tiles already cover half of them or K is not 64-aligned).
// m64: 64-row tiles allowed (as gemm_use64).
int gemm_pick_splits(int M, int N, int K, int sms, bool m64 = true);
// Whether an M-row projection runs on 64 x 128 tiles (allowed, and M a
// multiple of 64 but not of 128) instead of 128 x 128.
bool gemm_use64(int M, bool allow);
// pdl: launch with a programmatic edge to the previous kernel in the stream
// (the GEMM reads nothing before that kernel has finished).
cudaError_t gemm_bf16_f32(int M, int N, int K, const uint16_t* A, const uint16_t* W,
                          const float* C, float* D, float beta, void* workspace,
                          size_t workspace_bytes, cudaStream_t st, int ldw = 0, int splits = 1,
                          bool pdl = false, bool m64 = true);

}  // namespace myos
