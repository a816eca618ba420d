// Prefill of a chunk of n prompt tokens as dense projections (gemm_sm100.cu)
// with these kernels around them; the structure of the reference's prefill
// (crates/model_core/src/qwen25_block.rs:323-543): GEMM QKV, per-token bias,
// RoPE and KV store, per-position causal GQA, GEMM o_proj + residual,
// RMSNorm, GEMM gate|up, SwiGLU, GEMM down + residual.
//
// Activations reach the tensor cores as three stacked bf16 terms (prefill.h
// kSplitParts): rows t, n + t and 2n + t of A hold hi, mid and lo of x_t,
// whose sum is x_t exactly, so (D[t] + D[n + t]) + D[2n + t] is the
// projection of the full f32 activation with exact products. The
// element-wise steps keep the reference's operation order (no contraction).
#include <math.h>

#include "common.cuh"
#include "prefill.h"
#include "kernels.h"

namespace myos {
namespace {

constexpr int kT = 256;

MYOS_DEV uint16_t bf16_rn(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Row t of A's three blocks: hi, mid, lo with hi + mid + lo == y exactly.
MYOS_DEV void put_split(uint16_t* A, int n, int t, int K, int j, float y) {
  const uint16_t hi = bf16_rn(y);
  const float r1 = __fsub_rn(y, __uint_as_float((uint32_t)hi << 16));
  const uint16_t mid = bf16_rn(r1);
  const float r2 = __fsub_rn(r1, __uint_as_float((uint32_t)mid << 16));
  A[(size_t)t * K + j] = hi;
  A[(size_t)(n + t) * K + j] = mid;
  A[(size_t)(2 * n + t) * K + j] = bf16_rn(r2);
}

// The projection of row t: its three partial outputs, (hi + mid) + lo.
MYOS_DEV float part_sum(const float* D, int n, int t, int N, int j) {
  return __fadd_rn(__fadd_rn(D[(size_t)t * N + j], D[(size_t)(n + t) * N + j]),
                   D[(size_t)(2 * n + t) * N + j]);
}

MYOS_DEV float bsum(float v, float* red) { return block_sum(v, red); }

// X[t] = embedding row of ids[t] (exact promotion).
__global__ void k_pf_embed(float* X, const uint16_t* embed, const uint32_t* ids, int K) {
  const int t = blockIdx.x;
  const uint16_t* row = embed + (size_t)ids[t] * K;
  for (int j = threadIdx.x; j < K; j += blockDim.x) X[(size_t)t * K + j] = bf16_at(row + j);
}

// A[t], A[n + t], A[2n + t] = the three bf16 terms of gamma * (x * inv),
// inv = 1 / sqrtf(mean(x^2) + eps) (bf16.rs:231-270); gamma null: of x.
__global__ void __launch_bounds__(kT) k_pf_norm_split(uint16_t* A, const float* X, const float* gamma,
                                                      int n, int K, float eps) {
  __shared__ float red[33];
  const int t = blockIdx.x;
  const float* x = X + (size_t)t * K;
  float inv = 1.0f;
  if (gamma) {
    float ss = 0.0f;
    for (int j = threadIdx.x; j < K; j += blockDim.x) ss = fmaf(x[j], x[j], ss);
    ss = bsum(ss, red);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
  }
  for (int j = threadIdx.x; j < K; j += blockDim.x)
    put_split(A, n, t, K, j, gamma ? __fmul_rn(gamma[j], __fmul_rn(x[j], inv)) : x[j]);
}

// Q[t] = projection + bias (bf16.rs:147-158).
__global__ void k_pf_bias(float* Q, const float* D, const float* bias, int n, int N) {
  const int t = blockIdx.x;
  for (int j = threadIdx.x; j < N; j += blockDim.x)
    Q[(size_t)t * N + j] = __fadd_rn(part_sum(D, n, t, N, j), bias[j]);
}

// NeoX rotation of token t's q heads and KV heads at position p0 + t
// (rope.rs:145-184), then K and V stored at that slot (KvCache::store_at).
template <typename KT>
__global__ void k_pf_rope_store(float* Q, KT* kc, KT* vc, const float* cos_t, const float* sin_t,
                                int p0, int Hq, int Hkv, int d, int S, const int* rowpos,
                                size_t rowstride) {
  // row t is token t of one sequence (position p0 + t), or with rowpos the
  // next token of sequence t (position rowpos[t], cache rowstride elements on)
  const int t = blockIdx.x, pos = rowpos ? rowpos[t] : p0 + t, half = d >> 1;
  const int N = (Hq + 2 * Hkv) * d;
  if (rowpos) {
    kc += (size_t)t * rowstride;
    vc += (size_t)t * rowstride;
  }
  float* q = Q + (size_t)t * N;
  const float* cs = cos_t + (size_t)pos * half;
  const float* sn = sin_t + (size_t)pos * half;
  for (int i = threadIdx.x; i < (Hq + Hkv) * half; i += blockDim.x) {
    const int h = i / half, p = i - h * half;
    float* x = q + h * d;  // heads 0..Hq-1 are q, Hq.. are k
    const float x0 = x[p], x1 = x[p + half];
    x[p] = __fsub_rn(__fmul_rn(x0, cs[p]), __fmul_rn(x1, sn[p]));
    x[p + half] = __fadd_rn(__fmul_rn(x1, cs[p]), __fmul_rn(x0, sn[p]));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < Hkv * d; i += blockDim.x) {
    const int g = i / d, e = i - g * d;
    const size_t slot = ((size_t)g * S + pos) * d + e;
    if constexpr (sizeof(KT) == 4) {
      kc[slot] = q[(Hq + g) * d + e];
      vc[slot] = q[(Hq + Hkv + g) * d + e];
    } else {
      kc[slot] = __float2bfloat16_rn(q[(Hq + g) * d + e]);
      vc[slot] = __float2bfloat16_rn(q[(Hq + Hkv + g) * d + e]);
    }
  }
}

template <typename KT>
MYOS_DEV float4 kv4(const KT* p);
template <>
MYOS_DEV float4 kv4<float>(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}
template <>
MYOS_DEV float4 kv4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p));
  return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
}

// Causal GQA for token t (position p0 + t) and KV head g: keys 0..pos from
// the cache, online softmax over tiles of 32 (one warp per query head, lane
// per key), p * v accumulated per lane over dims [4 lane, 4 lane + 4)
// (+128 for d > 128); out = sum / L (gqa.rs:174-218, reassociated).
template <typename KT, int D>
__global__ void __launch_bounds__(kT) k_pf_attn(float* out, const float* Q, const KT* kcache,
                                                const KT* vcache, int p0, int Hq, int Hkv, int S,
                                                float scale, const int* rowpos, size_t rowstride) {
  constexpr int kTile = 32, ds = D + 4;
  __shared__ __align__(16) float qs[8 * D];
  __shared__ __align__(16) float ks[kTile * ds];
  __shared__ __align__(16) float vs[kTile * ds];
  const int t = blockIdx.x, g = blockIdx.y, G = Hq / Hkv, pos = rowpos ? rowpos[t] : p0 + t;
  if (rowpos) {
    kcache += (size_t)t * rowstride;
    vcache += (size_t)t * rowstride;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = (Hq + 2 * Hkv) * D;
  const float* q = Q + (size_t)t * N + (size_t)g * G * D;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) qs[i] = q[i];
  const KT* kc = kcache + (size_t)g * S * D;
  const KT* vc = vcache + (size_t)g * S * D;
  float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  float m_run = -INFINITY, l_run = 0.0f;
  for (int t0 = 0; t0 <= pos; t0 += kTile) {
    const int nk = min(kTile, pos + 1 - t0);
    __syncthreads();  // qs staged / previous tile consumed
    for (int i = threadIdx.x; i < nk * (D / 4); i += blockDim.x) {
      const int tt = i / (D / 4), e = (i - tt * (D / 4)) * 4;
      *reinterpret_cast<float4*>(ks + tt * ds + e) = kv4<KT>(kc + (size_t)(t0 + tt) * D + e);
      *reinterpret_cast<float4*>(vs + tt * ds + e) = kv4<KT>(vc + (size_t)(t0 + tt) * D + e);
    }
    __syncthreads();
    if (warp < G) {
      const float* qh = qs + warp * D;
      float sc = -INFINITY;
      if (lane < nk) {
        const float* kr = ks + lane * ds;
        float p0s = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
        for (int e = 0; e < D; e += 4) {
          const float4 a = *reinterpret_cast<const float4*>(qh + e);
          const float4 b = *reinterpret_cast<const float4*>(kr + e);
          p0s = fmaf(a.x, b.x, p0s);
          p1 = fmaf(a.y, b.y, p1);
          p2 = fmaf(a.z, b.z, p2);
          p3 = fmaf(a.w, b.w, p3);
        }
        sc = __fmul_rn((p0s + p1) + (p2 + p3), scale);
      }
      const float mn = fmaxf(m_run, warp_max(sc));
      const float cf = expf(m_run - mn);
      const float p = lane < nk ? expf(sc - mn) : 0.0f;
      l_run = fmaf(l_run, cf, warp_sum(p));
      m_run = mn;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        acc[j].x *= cf;
        acc[j].y *= cf;
        acc[j].z *= cf;
        acc[j].w *= cf;
      }
#pragma unroll 8
      for (int k = 0; k < nk; ++k) {
        const float pk = __shfl_sync(0xffffffffu, p, k);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int e = 4 * lane + 128 * j;
          if (e < D) {
            const float4 v = *reinterpret_cast<const float4*>(vs + k * ds + e);
            acc[j].x = fmaf(pk, v.x, acc[j].x);
            acc[j].y = fmaf(pk, v.y, acc[j].y);
            acc[j].z = fmaf(pk, v.z, acc[j].z);
            acc[j].w = fmaf(pk, v.w, acc[j].w);
          }
        }
      }
    }
  }
  if (warp < G) {
    float* o = out + (size_t)t * Hq * D + (size_t)(g * G + warp) * D;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int e = 4 * lane + 128 * j;
      if (e < D)
        *reinterpret_cast<float4*>(o + e) =
            make_float4(__fdiv_rn(acc[j].x, l_run), __fdiv_rn(acc[j].y, l_run),
                        __fdiv_rn(acc[j].z, l_run), __fdiv_rn(acc[j].w, l_run));
    }
  }
}

// X[t] += projection (residual after o_proj / down_proj).
__global__ void k_pf_resid(float* X, const float* D, int n, int N) {
  const int t = blockIdx.x;
  for (int j = threadIdx.x; j < N; j += blockDim.x)
    X[(size_t)t * N + j] = __fadd_rn(X[(size_t)t * N + j], part_sum(D, n, t, N, j));
}

// Tensor-parallel form: this rank's part of the residual update, written in
// place over the hi rows of D: X + projection on the rank that carries the
// residual (X non-null), the projection elsewhere; the ranks' parts are then summed.
__global__ void k_pf_resid_part(float* D, const float* X, int n, int N) {
  const int t = blockIdx.x;
  for (int j = threadIdx.x; j < N; j += blockDim.x) {
    const float dl = part_sum(D, n, t, N, j);
    D[(size_t)t * N + j] = X ? __fadd_rn(X[(size_t)t * N + j], dl) : dl;
  }
}

// h = (g / (1 + expf(-g))) * u (swiglu.rs:113-131) from the stacked gate|up
// projection, written as three bf16 terms for the down projection.
__global__ void k_pf_swiglu_split(uint16_t* A, const float* D, int n, int I) {
  const int t = blockIdx.x, N = 2 * I;
  for (int j = threadIdx.x; j < I; j += blockDim.x) {
    const float g = part_sum(D, n, t, N, j);
    const float u = part_sum(D, n, t, N, I + j);
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    put_split(A, n, t, I, j, __fmul_rn(s, u));
  }
}

// Greedy token of each row from the stacked logit parts: logits_b[j] =
// (D[b][j] + D[B + b][j]) + D[2B + b][j]; the first maximum with strict >, NaN and -inf never
// win, none -> 0 (model_core/src/lib.rs:157-167). Records the token.
__global__ void __launch_bounds__(kT) k_row_argmax(uint32_t* tok, uint32_t* out, int out_stride,
                                                   int step, const float* D, int B, int V) {
  __shared__ float bvs[kT / 32];
  __shared__ uint32_t bis[kT / 32];
  const int b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float v = part_sum(D, B, b, V, j);
    if (v > bv) {  // j grows per thread: strict > keeps the first
      bv = v;
      bi = (uint32_t)j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    bvs[warp] = bv;
    bis[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    for (int w = 0; w < kT / 32; ++w)
      if (bvs[w] > v || (bvs[w] == v && bis[w] < i)) {
        v = bvs[w];
        i = bis[w];
      }
    const uint32_t t = i == 0xffffffffu ? 0u : i;
    tok[b] = t;
    if (out) out[(size_t)b * out_stride + step] = t;
  }
}

__global__ void k_rows_copy(float* dst, const float* src, const int* src_row, int K) {
  const int b = blockIdx.x;
  for (int j = threadIdx.x; j < K; j += blockDim.x)
    dst[(size_t)b * K + j] = src[(size_t)src_row[b] * K + j];
}

__global__ void k_pos_advance(int* rowpos, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) rowpos[b] += 1;
}

}  // namespace

cudaError_t pf_row_argmax(uint32_t* tok, uint32_t* out, int out_stride, int step, const float* D,
                          int B, int V, cudaStream_t st) {
  k_row_argmax<<<B, kT, 0, st>>>(tok, out, out_stride, step, D, B, V);
  return counted(cudaGetLastError());
}

cudaError_t pf_rows_copy(float* dst, const float* src, const int* src_row, int B, int K,
                         cudaStream_t st) {
  k_rows_copy<<<B, kT, 0, st>>>(dst, src, src_row, K);
  return counted(cudaGetLastError());
}

cudaError_t pf_pos_advance(int* rowpos, int B, cudaStream_t st) {
  k_pos_advance<<<(B + 127) / 128, 128, 0, st>>>(rowpos, B);
  return counted(cudaGetLastError());
}

cudaError_t pf_embed(float* X, const uint16_t* embed, const uint32_t* ids, int n, int K,
                     cudaStream_t st) {
  k_pf_embed<<<n, kT, 0, st>>>(X, embed, ids, K);
  return counted(cudaGetLastError());
}

cudaError_t pf_norm_split(uint16_t* A, const float* X, const float* gamma, int n, int K, float eps,
                          cudaStream_t st) {
  k_pf_norm_split<<<n, kT, 0, st>>>(A, X, gamma, n, K, eps);
  return counted(cudaGetLastError());
}

cudaError_t pf_bias(float* Q, const float* D, const float* bias, int n, int N, cudaStream_t st) {
  k_pf_bias<<<n, kT, 0, st>>>(Q, D, bias, n, N);
  return counted(cudaGetLastError());
}

cudaError_t pf_rope_store(float* Q, void* kc, void* vc, int kv_bf16, const float* cos_t,
                          const float* sin_t, int p0, int n, int Hq, int Hkv, int d, int S,
                          cudaStream_t st, const int* rowpos, size_t rowstride) {
  if (kv_bf16)
    k_pf_rope_store<__nv_bfloat16><<<n, kT, 0, st>>>(Q, (__nv_bfloat16*)kc, (__nv_bfloat16*)vc,
                                                      cos_t, sin_t, p0, Hq, Hkv, d, S, rowpos,
                                                      rowstride);
  else
    k_pf_rope_store<float><<<n, kT, 0, st>>>(Q, (float*)kc, (float*)vc, cos_t, sin_t, p0, Hq, Hkv,
                                             d, S, rowpos, rowstride);
  return counted(cudaGetLastError());
}

bool pf_attn_supported(int d, int G) { return (d == 64 || d == 128) && G <= 8; }

cudaError_t pf_attn(float* out, const float* Q, const void* kc, const void* vc, int kv_bf16, int p0,
                    int n, int Hq, int Hkv, int d, int S, float scale, cudaStream_t st,
                    const int* rowpos, size_t rowstride) {
  const dim3 grid(n, Hkv);
#define MYOS_PF_ATTN(D)                                                                     \
  if (d == D) {                                                                             \
    if (kv_bf16)                                                                            \
      k_pf_attn<__nv_bfloat16, D><<<grid, kT, 0, st>>>(out, Q, (const __nv_bfloat16*)kc,    \
                                                       (const __nv_bfloat16*)vc, p0, Hq,    \
                                                       Hkv, S, scale, rowpos, rowstride);   \
    else                                                                                    \
      k_pf_attn<float, D><<<grid, kT, 0, st>>>(out, Q, (const float*)kc, (const float*)vc, \
                                               p0, Hq, Hkv, S, scale, rowpos, rowstride);   \
    return counted(cudaGetLastError());                                                              \
  }
  MYOS_PF_ATTN(64)
  MYOS_PF_ATTN(128)
#undef MYOS_PF_ATTN
  return cudaErrorInvalidValue;
}

cudaError_t pf_resid(float* X, const float* D, int n, int N, cudaStream_t st) {
  k_pf_resid<<<n, kT, 0, st>>>(X, D, n, N);
  return counted(cudaGetLastError());
}

cudaError_t pf_resid_part(float* D, const float* X, int n, int N, cudaStream_t st) {
  k_pf_resid_part<<<n, kT, 0, st>>>(D, X, n, N);
  return counted(cudaGetLastError());
}

cudaError_t pf_swiglu_split(uint16_t* A, const float* D, int n, int I, cudaStream_t st) {
  k_pf_swiglu_split<<<n, kT, 0, st>>>(A, D, n, I);
  return counted(cudaGetLastError());
}

}  // namespace myos
