// Element-wise and attention kernels of the GEMM prefill (prefill.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace myos {

// Each f32 activation enters the tensor cores as the exact sum of three
// bf16 terms (hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid):
// 8 + 8 + 8 significand bits, every subtraction exact in f32), stacked as
// row blocks [hi; mid; lo] of A, so one GEMM pass over the weights gives
// three partial outputs whose sum (hi + mid) + lo the consumers form.
constexpr int kSplitParts = 3;

cudaError_t pf_embed(float* X, const uint16_t* embed, const uint32_t* ids, int n, int K,
                     cudaStream_t st);
cudaError_t pf_norm_split(uint16_t* A, const float* X, const float* gamma, int n, int K, float eps,
                          cudaStream_t st);
cudaError_t pf_bias(float* Q, const float* D, const float* bias, int n, int N, cudaStream_t st);
// Rows are tokens p0.. of one sequence, or (rowpos non-null) the next token
// of sequence t at position rowpos[t] with its cache rowstride elements on.
cudaError_t pf_rope_store(float* Q, void* kc, void* vc, int kv_bf16, const float* cos_t,
                          const float* sin_t, int p0, int n, int Hq, int Hkv, int d, int S,
                          cudaStream_t st, const int* rowpos = nullptr, size_t rowstride = 0);
bool pf_attn_supported(int d, int G);
cudaError_t pf_attn(float* out, const float* Q, const void* kc, const void* vc, int kv_bf16, int p0,
                    int n, int Hq, int Hkv, int d, int S, float scale, cudaStream_t st,
                    const int* rowpos = nullptr, size_t rowstride = 0);
// Greedy token per row of stacked logit parts D[3B, V]; tok[b], and
// out[b * out_stride + step] when out is non-null.
cudaError_t pf_row_argmax(uint32_t* tok, uint32_t* out, int out_stride, int step, const float* D,
                          int B, int V, cudaStream_t st);
cudaError_t pf_rows_copy(float* dst, const float* src, const int* src_row, int B, int K,
                         cudaStream_t st);
cudaError_t pf_pos_advance(int* rowpos, int B, cudaStream_t st);
cudaError_t pf_resid(float* X, const float* D, int n, int N, cudaStream_t st);
// D[t] = (X ? X[t] : 0) + D[t] + D[n + t] over rows t < n (in place; the
// tensor-parallel part before the sum over ranks).
cudaError_t pf_resid_part(float* D, const float* X, int n, int N, cudaStream_t st);
cudaError_t pf_swiglu_split(uint16_t* A, const float* D, int n, int I, cudaStream_t st);

}  // namespace myos
