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
// Projection outputs D hold `sp` K slices of 3n partial rows each
// (gemm_sm100.h split-K); the consumers below add them in a fixed order.
//
// Q[t] = QKV projection + bias, then RoPE of the q and k heads and the K/V
// store. Rows are tokens p0.. of one sequence, or (rowpos non-null) the next
// token of sequence t at position rowpos[t] with its cache rowstride
// elements on.
cudaError_t pf_qkv_post(float* Q, const float* D, int sp, const float* bias, void* kc, void* vc,
                        int kv_bf16, const float* cos_t, const float* sin_t, int p0, int n, int Hq,
                        int Hkv, int d, int S, cudaStream_t st, const int* rowpos = nullptr,
                        size_t rowstride = 0);
bool pf_attn_supported(int d, int G);
// Raises the shared-memory limit of the split attention (once per device,
// with that device current, before the first pf_attn there) and reads
// MYOS_GEMM_PDL (0: launch the GEMM path without programmatic dependent
// launch).
cudaError_t pf_init();
// Whether the GEMM path's kernels (and its GEMMs) launch with PDL.
bool pf_pdl();
// Causal GQA per row, split over the keys, then merged into A as the o_proj
// input's three terms. Splits of 64 keys (longer past kAttnMaxSplits); the
// partials o_part (rows * Hq * splits * d floats) and ml (rows * Hq * splits)
// come from the caller, sized by pf_attn_splits(max_keys) for the largest
// position + 1 of any row. arrive (n * Hkv zeroed counters, left zeroed):
// where the key-split kernel runs, the last split of each (row, KV head) to
// finish merges that row's heads itself instead of a merge launch. work (2
// zeroed counters, left zeroed): the key-split kernel's blocks take items
// past their first from a shared queue instead of a fixed stride.
constexpr int kAttnMaxSplits = 64;
int pf_attn_splits(int max_keys, int* ch);
cudaError_t pf_attn(uint16_t* A, float* o_part, float2* ml, const float* Q, const void* kc,
                    const void* vc, int kv_bf16, int p0, int n, int Hq, int Hkv, int d, int S,
                    float scale, int max_keys, int sms, cudaStream_t st,
                    const int* rowpos = nullptr, size_t rowstride = 0,
                    unsigned* arrive = nullptr, unsigned* work = nullptr);
// Greedy token per row of stacked logit parts D[3B, V]; tok[b], and
// out[b * out_stride + step] when out is non-null. part: B * pf_argmax_chunks(V)
// float2 of scratch. d_step non-null: step = *d_step, read on the device, and
// out written only while step < out_stride.
int pf_argmax_chunks(int V);
cudaError_t pf_row_argmax(uint32_t* tok, uint32_t* out, int out_stride, int step, const float* D,
                          float2* part, int B, int V, cudaStream_t st,
                          const int* d_step = nullptr);
// tok[b] = feed_t[*d_step * B + b] (teacher-forced batched steps).
cudaError_t pf_feed(uint32_t* tok, const uint32_t* feed_t, const int* d_step, int B,
                    cudaStream_t st);
cudaError_t pf_rows_copy(float* dst, const float* src, const int* src_row, int B, int K,
                         cudaStream_t st);
// rowpos[b] += 1 for b < B, and *d_step += 1 when d_step is non-null.
cudaError_t pf_pos_advance(int* rowpos, int B, cudaStream_t st, int* d_step = nullptr);
// X[t] += projection; with gamma also A = the three bf16 terms of
// RMSNorm(X[t]) * gamma (the next projection's input).
cudaError_t pf_resid_norm(float* X, const float* D, int sp, const float* gamma, uint16_t* A, int n,
                          int N, float eps, cudaStream_t st);
// D[t] = (X ? X[t] : 0) + projection over rows t < n (in place over the first
// hi rows; the tensor-parallel part before the sum over ranks).
cudaError_t pf_resid_part(float* D, const float* X, int n, int N, int sp, cudaStream_t st);
cudaError_t pf_swiglu_split(uint16_t* A, const float* D, int n, int I, int sp, cudaStream_t st);

}  // namespace myos
