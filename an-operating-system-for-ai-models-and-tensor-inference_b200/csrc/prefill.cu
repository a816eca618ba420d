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

#include <algorithm>
#include <cstdlib>

#include <cooperative_groups.h>

#include "common.cuh"
#include "prefill.h"
#include "gemm_sm100.h"
#include "kernels.h"

namespace myos {
namespace {

namespace cg = cooperative_groups;

// Programmatic dependent launch between the kernels of the GEMM path: each
// kernel waits for the previous kernel of the stream to finish (and its
// memory to be visible) before its first global access, then lets the next
// one be scheduled, so launches overlap their predecessors' tails.
bool g_pdl = true;  // MYOS_GEMM_PDL=0 at pf_init: plain stream order
// prompt chunks whose rows reach at least this many keys use the row-tiled
// attention (MYOS_PF_ATTN_ROWS_MIN at pf_init; the per-row split kernel below)
int g_rows_min = 1024;
// the per-row split attention with keys split over the warps
// (k_pf_attn_warps; D = 128, 5..8 query heads per KV head); MYOS_PF_ATTN_WARPS
// at pf_init, 0: the dims-split k_pf_attn_split
bool g_attn_warps = true;
// with it, the last split of a (row, KV head) merges the splits
// (MYOS_PF_MERGE_FUSED at pf_init, 0: a separate merge launch)
bool g_merge_fused = true;
// items per block up to which the merge is fused (measured: a 128-id prompt
// chunk, 1.7 items a block, 2.52 -> 2.46 ms; 32 batched rows at 512 keys,
// 1.95 items, 2.24-2.34 -> 2.075 ms per step; 64 batched rows, 3.9 items,
// 2.775 -> 2.783 ms per step; 256-row chunks of 512-id prompts, 14 items,
// 645 -> 726 ms)
constexpr int kMergeFusedItems = 2;
// with it, blocks past their first item take items from a shared queue
// (MYOS_PF_ATTN_DYN at pf_init, 0: a fixed stride over the items) when a
// block has more than kAttnDynItems items on average (measured: 256-row
// chunks of 512-id prompts, 14 items a block, 64 prompts 658 -> 607 ms; 64
// batched rows, 3.9 items, 2.821 -> 2.848 ms per step; a 128-id chunk, 1.7
// items, 2.49 -> 2.57 ms: the first pending item's atomic delays every block)
bool g_attn_dyn = true;
constexpr int kAttnDynItems = 4;

MYOS_DEV void pdl_begin() {
  pdl_wait();
  pdl_launch();
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = g_pdl ? 1 : 0;
  return counted(cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...));
}

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

// The projection of row t from D's partial outputs: `sp` K slices (blocks of
// 3n rows, gemm_sm100.h split-K), each with its hi, mid and lo rows; summed
// (hi + mid) + lo within a slice, then slice by slice in order.
MYOS_DEV float part_sum(const float* D, int n, int t, int N, int j, int sp) {
  const size_t blk = (size_t)kSplitParts * n * N;
  float acc = 0.0f;
  for (int l = 0; l < sp; ++l) {
    const float* Dl = D + (size_t)l * blk;
    const float v = __fadd_rn(__fadd_rn(Dl[(size_t)t * N + j], Dl[(size_t)(n + t) * N + j]),
                              Dl[(size_t)(2 * n + t) * N + j]);
    acc = l ? __fadd_rn(acc, v) : v;
  }
  return acc;
}

// part_sum of columns j..j+3 (N % 4 == 0, j % 4 == 0): every slice's three
// partial rows are loaded before any is added, so the loads overlap.
MYOS_DEV float4 part_sum4(const float* D, int n, int t, int N, int j, int sp) {
  const size_t blk = (size_t)kSplitParts * n * N;
  float4 a[kMaxSplits], b[kMaxSplits], c[kMaxSplits];
#pragma unroll
  for (int l = 0; l < kMaxSplits; ++l)
    if (l < sp) {
      const float* Dl = D + (size_t)l * blk;
      a[l] = __ldcs(reinterpret_cast<const float4*>(Dl + (size_t)t * N + j));
      b[l] = __ldcs(reinterpret_cast<const float4*>(Dl + (size_t)(n + t) * N + j));
      c[l] = __ldcs(reinterpret_cast<const float4*>(Dl + (size_t)(2 * n + t) * N + j));
    }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int l = 0; l < kMaxSplits; ++l)
    if (l < sp) {
      const float4 v = make_float4(__fadd_rn(__fadd_rn(a[l].x, b[l].x), c[l].x),
                                   __fadd_rn(__fadd_rn(a[l].y, b[l].y), c[l].y),
                                   __fadd_rn(__fadd_rn(a[l].z, b[l].z), c[l].z),
                                   __fadd_rn(__fadd_rn(a[l].w, b[l].w), c[l].w));
      acc = l ? make_float4(__fadd_rn(acc.x, v.x), __fadd_rn(acc.y, v.y), __fadd_rn(acc.z, v.z),
                            __fadd_rn(acc.w, v.w))
              : v;
    }
  return acc;
}

MYOS_DEV float bsum(float v, float* red) { return block_sum(v, red); }

// X[t] = embedding row of ids[t] (exact promotion).
__global__ void k_pf_embed(float* X, const uint16_t* embed, const uint32_t* ids, int K) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int t = blockIdx.x;
  const uint16_t* row = embed + (size_t)ids[t] * K;
  for (int j = threadIdx.x; j < K; j += blockDim.x) X[(size_t)t * K + j] = bf16_at(row + j);
}

// A[t], A[n + t], A[2n + t] = the three bf16 terms of gamma * (x * inv),
// inv = 1 / sqrtf(mean(x^2) + eps) (bf16.rs:231-270); gamma null: of x.
__global__ void __launch_bounds__(kT) k_pf_norm_split(uint16_t* A, const float* X, const float* gamma,
                                                      int n, int K, float eps) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
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

// Token t's q|k|v row from the QKV projection: projection + bias
// (bf16.rs:147-158); the NeoX rotation of the q heads and KV heads at the
// row's position (rope.rs:145-184); q into Q, K and V stored at that slot of
// the cache (KvCache::store_at). Row t is token t of one sequence (position
// p0 + t), or (rowpos non-null) the next token of sequence t at position
// rowpos[t] with its cache rowstride elements on. Block (t, y) takes
// 256 / d heads, one thread per rotation pair (p, p + d/2).
template <typename KT>
__global__ void __launch_bounds__(128) k_pf_qkv_post(float* Q, const float* D, int sp,
                                                     const float* bias, KT* kc, KT* vc,
                                                     const float* cos_t, const float* sin_t, int p0,
                                                     int Hq, int Hkv, int d, int S,
                                                     const int* rowpos, size_t rowstride) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int t = blockIdx.x, n = gridDim.x, half = d >> 1;
  const int h = blockIdx.y * (256 / d) + threadIdx.x / half, p = threadIdx.x % half;
  if (h >= Hq + 2 * Hkv) return;
  const int pos = rowpos ? rowpos[t] : p0 + t;
  const int N = (Hq + 2 * Hkv) * d, j = h * d + p;
  float x0 = __fadd_rn(part_sum(D, n, t, N, j, sp), bias[j]);
  float x1 = __fadd_rn(part_sum(D, n, t, N, j + half, sp), bias[j + half]);
  if (h < Hq + Hkv) {  // q and k heads rotate
    const float cs = cos_t[(size_t)pos * half + p], sn = sin_t[(size_t)pos * half + p];
    const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    const float y1 = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x0, sn));
    x0 = y0;
    x1 = y1;
  }
  float* q = Q + (size_t)t * N;
  q[j] = x0;
  q[j + half] = x1;
  if (h < Hq) return;
  const bool is_k = h < Hq + Hkv;
  const int g = is_k ? h - Hq : h - Hq - Hkv;
  KT* cache = is_k ? kc : vc;
  if (rowpos) cache += (size_t)t * rowstride;
  const size_t slot = ((size_t)g * S + pos) * d + p;
  if constexpr (sizeof(KT) == 4) {
    cache[slot] = x0;
    cache[slot + half] = x1;
  } else {
    cache[slot] = __float2bfloat16_rn(x0);
    cache[slot + half] = __float2bfloat16_rn(x1);
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

// Causal GQA per row, split over the keys. Row t (token t at position
// p0 + t of one sequence, or with rowpos the next token of sequence t at
// rowpos[t], its cache rowstride elements on) and KV head g: block
// (s, g, t) takes keys [s * ch, min((s + 1) * ch, pos + 1)) in tiles of 32
// (one warp per query head, lane per key for the scores, online softmax
// over the tiles, lane per D/32 dims for p * v) and leaves the unnormalised
// partial: o_part[row][head][s][D], ml[row][head][s] = (running max, sum of
// exponentials). k_pf_attn_merge combines the splits (gqa.rs:174-218,
// reassociated: the softmax is taken split by split, then rescaled).
constexpr int kAttnTile = 32;

MYOS_DEV void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
MYOS_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MYOS_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Shared memory of k_pf_attn_split: two slots of (q heads of the group, K
// tile, V tile) with K/V rows padded to D + 4 floats, the per-warp partial
// scores, the tile's probabilities [key][head] and the heads' rescale factors.
constexpr int kAttnWarps = kT / 32;
template <int D>
constexpr int attn_slot_floats() {
  return 8 * D + 2 * kAttnTile * (D + 4);
}
template <int D>
constexpr size_t attn_smem_bytes() {
  return (size_t)(2 * attn_slot_floats<D>() + kAttnWarps * 8 * kAttnTile + kAttnTile * 8 + 8) *
         sizeof(float);
}

// One (row, KV head, split) item of the split attention and its tiles.
struct AttnItem {
  int item, tile, nt;  // item index (>= n_items: none), tile within it, its tiles
  int t, g, s, k0, k1;
};

// Causal GQA per row, split over the keys (see pf_attn), on a persistent
// grid: block b takes items b, b + gridDim.x, ... (item = (row t, KV head g,
// split s), s fastest) and walks their 32-key tiles as one stream, the next
// tile's copies (q, K, V; asynchronous for f32) in flight while this one is
// computed, across item boundaries. Per tile: scores: warp w takes dims
// [w D/8, (w+1) D/8) of every head, lane = key (each K element is read from
// shared memory once, the q values are broadcasts), the 8 partial sums meet
// in shared memory in warp order; softmax: warp h owns head h's running max
// and sum; p * v: lane = (key group, head pair, 4 dims) of warp w's dims, so
// each V element read serves two heads, the key groups summed by shuffles
// when the item ends.
template <typename KT, int D>
__global__ void __launch_bounds__(kT, 2) k_pf_attn_split(float* o_part, float2* ml, const float* Q,
                                                         const KT* kcache, const KT* vcache, int p0,
                                                         int n, int Hq, int Hkv, int S, float scale,
                                                         int ch, int ns, const int* rowpos,
                                                         size_t rowstride) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  constexpr int ds = D + 4, V4 = D / 4;
  constexpr int DW = D / kAttnWarps;    // dims per warp (16 or 8)
  constexpr int CW = DW / 4;            // float4 chunks per warp
  constexpr int LK = CW * 4;            // lanes per key group in p * v (chunk x head pair)
  constexpr int KG = 32 / LK;           // key groups (2 or 4)
  constexpr int SLOT = attn_slot_floats<D>();
  constexpr int kPer = (kAttnTile * V4 + kT - 1) / kT;  // float4s of K (and of V) per thread
  extern __shared__ __align__(16) float sm[];
  float* red = sm + 2 * SLOT;                    // [warps][8][32]
  float* pr = red + kAttnWarps * 8 * kAttnTile;  // [32][8]
  float* cfs = pr + kAttnTile * 8;               // [8]
  const int G = Hq / Hkv, n_items = n * Hkv * ns;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = (Hq + 2 * Hkv) * D;

  auto open_item = [&](AttnItem& it, int item) {  // first non-empty item from `item` on
    for (; item < n_items; item += gridDim.x) {
      const int s = item % ns, g = (item / ns) % Hkv, t = item / (ns * Hkv);
      const int pos = rowpos ? rowpos[t] : p0 + t, k0 = s * ch;
      if (k0 > pos) continue;  // this row has fewer splits
      it.item = item;
      it.tile = 0;
      it.t = t;
      it.g = g;
      it.s = s;
      it.k0 = k0;
      it.k1 = min(k0 + ch, pos + 1);
      it.nt = (it.k1 - k0 + kAttnTile - 1) / kAttnTile;
      return;
    }
    it.item = n_items;
  };
  auto advance = [&](AttnItem it) {
    if (++it.tile < it.nt) return it;
    open_item(it, it.item + gridDim.x);
    return it;
  };
  auto stage = [&](const AttnItem& it, int slot) {
    float* qs = sm + slot * SLOT;
    float* ks = qs + 8 * D;
    float* vs = ks + kAttnTile * ds;
    const size_t cofs = (rowpos ? (size_t)it.t * rowstride : 0) + (size_t)it.g * S * D;
    const KT* kc = kcache + cofs;
    const KT* vc = vcache + cofs;
    const int t0 = it.k0 + it.tile * kAttnTile, nk = min(kAttnTile, it.k1 - t0);
    const float* q = Q + (size_t)it.t * N + (size_t)it.g * G * D;
    for (int i = threadIdx.x; i < G * V4; i += kT) cp_async16(qs + 4 * i, q + 4 * i);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = threadIdx.x + i * kT, tt = idx / V4, e = (idx - tt * V4) * 4;
      if (tt < nk) {
        if constexpr (sizeof(KT) == 4) {
          cp_async16(ks + tt * ds + e, kc + (size_t)(t0 + tt) * D + e);
          cp_async16(vs + tt * ds + e, vc + (size_t)(t0 + tt) * D + e);
        } else {
          *reinterpret_cast<float4*>(ks + tt * ds + e) = kv4<KT>(kc + (size_t)(t0 + tt) * D + e);
          *reinterpret_cast<float4*>(vs + tt * ds + e) = kv4<KT>(vc + (size_t)(t0 + tt) * D + e);
        }
      }
    }
    cp_async_commit();
  };

  // p * v lane roles
  const int kg = lane / LK, hp = (lane % LK) / CW, cq = lane % CW;
  const int dv = warp * DW + cq * 4;  // this lane's 4 dims
  float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  float m_run = -INFINITY, l_run = 0.0f;  // warp h < G: head h

  AttnItem cur;
  open_item(cur, blockIdx.x);
  if (cur.item >= n_items) return;
  stage(cur, 0);
  AttnItem nxt = advance(cur);
  int slot = 0;
  while (cur.item < n_items) {
    if (nxt.item < n_items) {
      stage(nxt, slot ^ 1);
      cp_async_wait<1>();  // this tile's group has landed
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // every thread's copies of this tile are visible
    const float* qs = sm + slot * SLOT;
    const float* ks = qs + 8 * D;
    const float* vs = ks + kAttnTile * ds;
    const int nk = min(kAttnTile, cur.k1 - (cur.k0 + cur.tile * kAttnTile));
    {  // partial scores of key `lane` over this warp's dims, heads < G: even
       // and odd dims summed apart (packed f32x2 FMAs), then added
      float2 sc[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) sc[h] = make_float2(0.0f, 0.0f);
      if (lane < nk) {
#pragma unroll
        for (int c = 0; c < CW; ++c) {
          const int e = warp * DW + 4 * c;
          const float4 kv = *reinterpret_cast<const float4*>(ks + lane * ds + e);
          const float2 k01 = make_float2(kv.x, kv.y), k23 = make_float2(kv.z, kv.w);
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            if (h < G) {
              const float4 qv = *reinterpret_cast<const float4*>(qs + h * D + e);
              sc[h] = __ffma2_rn(make_float2(qv.x, qv.y), k01, sc[h]);
              sc[h] = __ffma2_rn(make_float2(qv.z, qv.w), k23, sc[h]);
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 8; ++h)
        red[(warp * 8 + h) * kAttnTile + lane] = __fadd_rn(sc[h].x, sc[h].y);
    }
    __syncthreads();
    if (warp < G) {  // online softmax of head `warp` over this tile
      float sc = -INFINITY;
      if (lane < nk) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) v = __fadd_rn(v, red[(w * 8 + warp) * kAttnTile + lane]);
        sc = __fmul_rn(v, scale);
      }
      const float mn = fmaxf(m_run, warp_max(sc));
      const float cf = expf(m_run - mn);
      const float pk = lane < nk ? expf(sc - mn) : 0.0f;
      l_run = fmaf(l_run, cf, warp_sum(pk));
      m_run = mn;
      pr[lane * 8 + warp] = pk;
      if (lane == 0) cfs[warp] = cf;
    } else {
      pr[lane * 8 + warp] = 0.0f;
      if (lane == 0) cfs[warp] = 1.0f;
    }
    __syncthreads();
    {  // p * v for heads 2hp, 2hp + 1 on dims dv..dv+3, keys kg, kg + KG, ...
      const float c0 = cfs[2 * hp], c1 = cfs[2 * hp + 1];
      acc[0].x *= c0; acc[0].y *= c0; acc[0].z *= c0; acc[0].w *= c0;
      acc[1].x *= c1; acc[1].y *= c1; acc[1].z *= c1; acc[1].w *= c1;
      float2 a0 = make_float2(acc[0].x, acc[0].y), a1 = make_float2(acc[0].z, acc[0].w);
      float2 b0 = make_float2(acc[1].x, acc[1].y), b1 = make_float2(acc[1].z, acc[1].w);
#pragma unroll 4
      for (int k = kg; k < nk; k += KG) {  // packed f32x2 FMAs, per element as fmaf
        const float4 v = *reinterpret_cast<const float4*>(vs + k * ds + dv);
        const float2 pp = *reinterpret_cast<const float2*>(pr + k * 8 + 2 * hp);
        const float2 v01 = make_float2(v.x, v.y), v23 = make_float2(v.z, v.w);
        const float2 px = make_float2(pp.x, pp.x), py = make_float2(pp.y, pp.y);
        a0 = __ffma2_rn(px, v01, a0);
        a1 = __ffma2_rn(px, v23, a1);
        b0 = __ffma2_rn(py, v01, b0);
        b1 = __ffma2_rn(py, v23, b1);
      }
      acc[0] = make_float4(a0.x, a0.y, a1.x, a1.y);
      acc[1] = make_float4(b0.x, b0.y, b1.x, b1.y);
    }
    if (cur.tile + 1 == cur.nt) {  // the item is done: its partial out, then a fresh state
      // key groups summed in a fixed order (xor tree over the group bits)
#pragma unroll
      for (int o = LK; o < 32; o <<= 1)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          acc[j].x += __shfl_xor_sync(0xffffffffu, acc[j].x, o);
          acc[j].y += __shfl_xor_sync(0xffffffffu, acc[j].y, o);
          acc[j].z += __shfl_xor_sync(0xffffffffu, acc[j].z, o);
          acc[j].w += __shfl_xor_sync(0xffffffffu, acc[j].w, o);
        }
      const size_t base = ((size_t)cur.t * Hq + (size_t)cur.g * G) * ns + cur.s;
      if (kg == 0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int h = 2 * hp + j;
          if (h < G) *reinterpret_cast<float4*>(o_part + (base + (size_t)h * ns) * D + dv) = acc[j];
        }
      }
      if (warp < G && lane == 0) ml[base + (size_t)warp * ns] = make_float2(m_run, l_run);
      acc[0] = acc[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      m_run = -INFINITY;
      l_run = 0.0f;
    }
    __syncthreads();  // this slot, the scores and the probabilities are consumed
    cur = nxt;
    nxt = advance(nxt);
    slot ^= 1;
  }
}

// out = (sum over splits of o_s * e^(m_s - M)) / (sum of l_s * e^(m_s - M)),
// M the largest split maximum, for query head h of row t over its nsr
// splits; written into A as the three bf16 terms of the o_proj input (n
// rows, row length Hq * D). One warp: lanes hold the split weights (s =
// lane, lane + 32), then D/32 dims each, splits in order. The partials are
// read through L2 (other blocks may have written them in this launch).
template <int D>
MYOS_DEV void merge_head(uint16_t* A, const float* o_part, const float2* ml, int n, int t, int h,
                         int Hq, int ns, int nsr, int lane) {
  constexpr int E = D / 32;
  const size_t base = ((size_t)t * Hq + h) * ns;
  const float2 a0 = lane < nsr ? __ldcg(ml + base + lane) : make_float2(-INFINITY, 0.0f);
  const float2 a1 = lane + 32 < nsr ? __ldcg(ml + base + lane + 32) : make_float2(-INFINITY, 0.0f);
  const float M = warp_max(fmaxf(a0.x, a1.x));
  const float w0 = lane < nsr ? expf(a0.x - M) : 0.0f;
  const float w1 = lane + 32 < nsr ? expf(a1.x - M) : 0.0f;
  const float L = warp_sum(fmaf(a1.y, w1, __fmul_rn(a0.y, w0)));
  float o[E];
#pragma unroll
  for (int e = 0; e < E; ++e) o[e] = 0.0f;
  const float* op = o_part + base * D + lane * E;
#pragma unroll 4
  for (int s = 0; s < nsr; ++s) {
    const float w = __shfl_sync(0xffffffffu, s < 32 ? w0 : w1, s & 31);
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = fmaf(__ldcg(op + (size_t)s * D + e), w, o[e]);
  }
#pragma unroll
  for (int e = 0; e < E; ++e) put_split(A, n, t, Hq * D, h * D + lane * E + e, __fdiv_rn(o[e], L));
}

// One step of the halving exchange that sums a warp's partial dot products:
// of the first N values a lane keeps the half its `bit` selects (the upper
// half when set), adds its partner's (lane ^ off) copy of that half and
// stores the sums in s[0, N/2). After N = 32, 16, 8, 4, 2 with off = N / 2,
// lane L holds the warp-wide sum of value L.
template <int N>
MYOS_DEV void halve_sum(float (&s)[32], bool bit, int off) {
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const float lo = s[i], hi = s[i + N / 2];
    const float keep = bit ? hi : lo, send = bit ? lo : hi;
    s[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
  }
}

// The split attention of k_pf_attn_split (same items, persistent grid,
// double-buffered 32-key tiles, same partial outputs for k_pf_attn_merge)
// with a tile's work split by keys instead of dims (D = 128, G query heads
// per KV head): warp w owns keys 4w..4w+3 of every tile and keeps its own
// running max, sum and p * v accumulator per head; lane = 4 dims of every
// head, q held in registers for the item. The 4 keys x 8 heads partial dot
// products over a lane's dims are summed across the warp by the halving
// exchange, leaving (head h, key j) in lane 4h + j, where the online
// softmax runs over the warp's 4 keys with two shuffles. A tile needs no
// block barrier besides the staging one; when an item ends the 8 warps'
// states meet in shared memory and are combined in warp order.
// Shared memory of k_pf_attn_warps: three slots of (q heads of the group,
// K tile, V tile), rows unpadded.
constexpr int kWarpsSlot = 8 * 128 + 2 * kAttnTile * 128;
constexpr size_t kWarpsSmem = 3 * kWarpsSlot * sizeof(float);

template <typename KT, int G>
__global__ void __launch_bounds__(kT, 2) k_pf_attn_warps(float* o_part, float2* ml, const float* Q,
                                                         const KT* kcache, const KT* vcache, int p0,
                                                         int n, int Hq, int Hkv, int S, float scale,
                                                         int ch, int ns, const int* rowpos,
                                                         size_t rowstride, uint16_t* A,
                                                         unsigned* arrive, unsigned* work) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  constexpr int D = 128, ds = D, V4 = D / 4;  // rows unpadded: a warp reads whole rows
  constexpr int SLOT = kWarpsSlot;
  constexpr int kPer = (kAttnTile * V4 + kT - 1) / kT;  // float4s of K (and of V) per thread
  constexpr int KW = kAttnTile / kAttnWarps;            // keys of a warp per tile
  static_assert(KW == 4 && G >= 1 && G <= 8, "4 keys x 8 heads fill the 32 lanes");
  static_assert(kAttnWarps * G * D + 2 * kAttnWarps * 8 <= SLOT, "warp states fit a slot");
  extern __shared__ __align__(16) float sm[];
  const int n_items = n * Hkv * ns;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = (Hq + 2 * Hkv) * D;

  // Static items (work null): block b takes the non-empty items among b,
  // b + grid, ... Dynamic items: block b starts on item b (or the queue's
  // first non-empty one), then takes the queue's next: work[0] counts the
  // items handed out past the grid, work[1] the blocks done, and the last
  // block done resets both. Thread 0 takes an item a tile ahead of its use
  // (`pending`, passed through shared memory at the tile's end barrier).
  __shared__ int s_q[2];
  int pending = n_items;
  auto item_empty = [&](int item) {  // a split past its row's last key
    const int t = item / (ns * Hkv);
    return (item % ns) * ch > (rowpos ? rowpos[t] : p0 + t);
  };
  auto take = [&](unsigned ticket) {  // thread 0: the first non-empty item from a ticket on
    int i = (int)gridDim.x + (int)ticket;
    while (i < n_items && item_empty(i)) i = (int)gridDim.x + (int)atomicAdd(work, 1u);
    return min(i, n_items);
  };
  auto open_item = [&](AttnItem& it, int item) {  // first non-empty item from `item` on
    for (; item < n_items; item += gridDim.x) {
      const int s = item % ns, g = (item / ns) % Hkv, t = item / (ns * Hkv);
      const int pos = rowpos ? rowpos[t] : p0 + t, k0 = s * ch;
      if (k0 > pos) {  // this row has fewer splits
        if (work) break;  // (never: the queue hands out non-empty items)
        continue;
      }
      it.item = item;
      it.tile = 0;
      it.t = t;
      it.g = g;
      it.s = s;
      it.k0 = k0;
      it.k1 = min(k0 + ch, pos + 1);
      it.nt = (it.k1 - k0 + kAttnTile - 1) / kAttnTile;
      return;
    }
    it.item = n_items;
  };
  auto advance = [&](AttnItem it, bool& used) {
    if (++it.tile < it.nt) return it;
    if (work) {
      used = true;
      open_item(it, pending);
    } else {
      open_item(it, it.item + gridDim.x);
    }
    return it;
  };
  auto stage = [&](const AttnItem& it, int slot) {
    float* qs = sm + slot * SLOT;
    float* ks = qs + 8 * D;
    float* vs = ks + kAttnTile * ds;
    const size_t cofs = (rowpos ? (size_t)it.t * rowstride : 0) + (size_t)it.g * S * D;
    const KT* kc = kcache + cofs;
    const KT* vc = vcache + cofs;
    const int t0 = it.k0 + it.tile * kAttnTile, nk = min(kAttnTile, it.k1 - t0);
    const float* q = Q + (size_t)it.t * N + (size_t)it.g * G * D;
    for (int i = threadIdx.x; i < G * V4; i += kT) cp_async16(qs + 4 * i, q + 4 * i);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = threadIdx.x + i * kT, tt = idx / V4, e = (idx - tt * V4) * 4;
      if (tt < nk) {
        if constexpr (sizeof(KT) == 4) {
          cp_async16(ks + tt * ds + e, kc + (size_t)(t0 + tt) * D + e);
          cp_async16(vs + tt * ds + e, vc + (size_t)(t0 + tt) * D + e);
        } else {
          *reinterpret_cast<float4*>(ks + tt * ds + e) = kv4<KT>(kc + (size_t)(t0 + tt) * D + e);
          *reinterpret_cast<float4*>(vs + tt * ds + e) = kv4<KT>(vc + (size_t)(t0 + tt) * D + e);
        }
      }
    }
    cp_async_commit();
  };

  const int hl = lane >> 2, jl = lane & 3;  // the (head, key) of this lane's summed score
  const int kb = warp * KW;                 // this warp's first key of a tile
  float4 q[G], acc[G];
  float m_h = -INFINITY, l_h = 0.0f;  // head hl over this warp's keys of the item

  AttnItem cur;
  if (work) {
    if (threadIdx.x == 0) {
      const int first = item_empty(blockIdx.x) ? take(atomicAdd(work, 1u)) : (int)blockIdx.x;
      s_q[0] = first;
      s_q[1] = first < n_items ? take(atomicAdd(work, 1u)) : n_items;
    }
    __syncthreads();
    open_item(cur, s_q[0]);
    pending = s_q[1];
  } else {
    open_item(cur, blockIdx.x);
  }
  AttnItem nxt = cur;
  if (cur.item < n_items) {
    stage(cur, 0);
    bool used = false;
    nxt = advance(cur, used);
    if (nxt.item < n_items) stage(nxt, 1);
    else cp_async_commit();  // an empty group keeps one group per tile
    if (used) {              // block-uniform: refill the pending item
      __syncthreads();
      if (threadIdx.x == 0) s_q[1] = pending < n_items ? take(atomicAdd(work, 1u)) : n_items;
      __syncthreads();
      pending = s_q[1];
    }
  }
  int slot = 0;
  while (cur.item < n_items) {
    bool used = false;
    const AttnItem nxt2 = advance(nxt, used);
    if (nxt2.item < n_items) stage(nxt2, slot == 0 ? 2 : slot - 1);
    else cp_async_commit();
    cp_async_wait<2>();  // this tile's group has landed; two more in flight
    __syncthreads();     // every thread's copies of this tile are visible
    // the refill's ticket now, its use at the tile's end (latency hidden)
    const bool refill = used && threadIdx.x == 0 && pending < n_items;
    const unsigned ticket = refill ? atomicAdd(work, 1u) : 0u;
    const float* qs = sm + slot * SLOT;
    const float* ks = qs + 8 * D;
    const float* vs = ks + kAttnTile * ds;
    const int nk = min(kAttnTile, cur.k1 - (cur.k0 + cur.tile * kAttnTile));
    if (cur.tile == 0) {  // a new item: its q, a fresh state
#pragma unroll
      for (int h = 0; h < G; ++h) {
        q[h] = *reinterpret_cast<const float4*>(qs + h * D + 4 * lane);
        acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      m_h = -INFINITY;
      l_h = 0.0f;
    }
    if (kb < nk) {  // warp-uniform: this warp has keys in the tile
      float s[32];  // value 4h + j: head h, key kb + j, over this lane's dims
#pragma unroll
      for (int j = 0; j < KW; ++j) {
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (kb + j < nk) kv = *reinterpret_cast<const float4*>(ks + (kb + j) * ds + 4 * lane);
        const float2 k01 = make_float2(kv.x, kv.y), k23 = make_float2(kv.z, kv.w);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          if (h < G) {
            float2 t = __ffma2_rn(make_float2(q[h].x, q[h].y), k01, make_float2(0.f, 0.f));
            t = __ffma2_rn(make_float2(q[h].z, q[h].w), k23, t);
            s[4 * h + j] = __fadd_rn(t.x, t.y);
          } else {
            s[4 * h + j] = 0.0f;
          }
        }
      }
      halve_sum<32>(s, lane & 16, 16);
      halve_sum<16>(s, lane & 8, 8);
      halve_sum<8>(s, lane & 4, 4);
      halve_sum<4>(s, lane & 2, 2);
      halve_sum<2>(s, lane & 1, 1);
      // online softmax of head hl over the warp's keys of this tile
      const bool valid = hl < G && kb + jl < nk;
      const float sc = valid ? __fmul_rn(s[0], scale) : -INFINITY;
      float mx = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m_h, mx);
      const float cf = mn == -INFINITY ? 1.0f : expf(m_h - mn);
      const float p = valid ? expf(sc - mn) : 0.0f;
      float ps = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 1));
      ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 2));
      l_h = fmaf(l_h, cf, ps);
      m_h = mn;
      // p * v on this lane's 4 dims of every head
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float c = __shfl_sync(0xffffffffu, cf, 4 * h);
        acc[h].x *= c;
        acc[h].y *= c;
        acc[h].z *= c;
        acc[h].w *= c;
      }
#pragma unroll
      for (int j = 0; j < KW; ++j) {
        if (kb + j < nk) {  // warp-uniform
          const float4 v = *reinterpret_cast<const float4*>(vs + (kb + j) * ds + 4 * lane);
          const float2 v01 = make_float2(v.x, v.y), v23 = make_float2(v.z, v.w);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float pj = __shfl_sync(0xffffffffu, p, 4 * h + j);
            const float2 pp = make_float2(pj, pj);
            const float2 a01 = __ffma2_rn(pp, v01, make_float2(acc[h].x, acc[h].y));
            const float2 a23 = __ffma2_rn(pp, v23, make_float2(acc[h].z, acc[h].w));
            acc[h] = make_float4(a01.x, a01.y, a23.x, a23.y);
          }
        }
      }
    }
    if (cur.tile + 1 == cur.nt) {  // the item is done: combine the warps' states
      __syncthreads();             // every warp is done with this slot's tile
      float* wacc = sm + slot * SLOT;             // [warp][head][D]
      float* wml = wacc + kAttnWarps * G * D;     // [warp][head] (max, sum)
#pragma unroll
      for (int h = 0; h < G; ++h)
        *reinterpret_cast<float4*>(wacc + (warp * G + h) * D + 4 * lane) = acc[h];
      if (jl == 0 && hl < G) {
        wml[2 * (warp * G + hl)] = m_h;
        wml[2 * (warp * G + hl) + 1] = l_h;
      }
      __syncthreads();
      const size_t base = ((size_t)cur.t * Hq + (size_t)cur.g * G) * ns + cur.s;
      for (int o = threadIdx.x; o < G * V4; o += kT) {  // (head, 4 dims)
        const int h = o / V4, e = (o - h * V4) * 4;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wml[2 * (w * G + h)]);
        float L = 0.0f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
          const float mw = wml[2 * (w * G + h)];
          const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
          const float4 a = *reinterpret_cast<const float4*>(wacc + (w * G + h) * D + e);
          L = fmaf(wml[2 * (w * G + h) + 1], f, L);
          O.x = fmaf(a.x, f, O.x);
          O.y = fmaf(a.y, f, O.y);
          O.z = fmaf(a.z, f, O.z);
          O.w = fmaf(a.w, f, O.w);
        }
        *reinterpret_cast<float4*>(o_part + (base + (size_t)h * ns) * D + e) = O;
        if (e == 0) ml[base + (size_t)h * ns] = make_float2(M, L);
      }
      if (arrive) {  // the last split of (row, KV head) to finish merges them
        __shared__ int merge_n;
        __syncthreads();  // the block's partials are written ...
        if (threadIdx.x == 0) {
          __threadfence();  // ... and visible device-wide before it counts
          const int pos = rowpos ? rowpos[cur.t] : p0 + cur.t;
          const int nsr = min(ns, pos / ch + 1);  // splits holding keys of this row
          unsigned* cnt = arrive + (size_t)cur.t * Hkv + cur.g;
          const bool last = atomicAdd(cnt, 1u) == (unsigned)(nsr - 1);
          if (last) *cnt = 0u;  // ready for the next launch
          merge_n = last ? nsr : 0;
        }
        __syncthreads();
        if (merge_n && warp < G) {
          __threadfence();
          merge_head<D>(A, o_part, ml, n, cur.t, cur.g * G + warp, Hq, ns, merge_n, lane);
        }
      }
    }
    if (used && threadIdx.x == 0) s_q[1] = refill ? take(ticket) : n_items;
    __syncthreads();  // this slot is consumed
    if (used) pending = s_q[1];
    cur = nxt;
    nxt = nxt2;
    slot = slot == 2 ? 0 : slot + 1;
  }
  if (work && threadIdx.x == 0 && atomicAdd(work + 1, 1u) == gridDim.x - 1) {
    work[0] = 0u;  // every block has taken its last item: the queue is
    work[1] = 0u;  // ready for the next launch
  }
}

// Causal GQA for a chunk of prompt rows, tiled over rows as well as keys
// (D = 128, long contexts): block (ti, g, s) takes rows [16 ti, 16 ti + 16),
// every query head of KV head g (warp h = head h) and the keys [s ch,
// (s + 1) ch) at or before each row's position. Each 32-key tile of K and V
// is staged once for all 16 x G query vectors. Scores: lane (rr, kk) holds
// rows 4 rr..4 rr+3 x keys kk, kk+8, kk+16, kk+24 (conflict-free reads of the
// padded rows); online softmax per row across the 8 lanes of its group;
// p * v: lane = 4 dims x all 16 rows. Writes the same split partials as
// k_pf_attn_split (merged by k_pf_attn_merge).
constexpr int kRowTile = 16;
template <int D>
constexpr size_t attn_rows_smem_bytes(int G) {
  return ((size_t)G * kRowTile * (D + 4) + 2 * kAttnTile * (D + 4) +
          (size_t)G * kAttnTile * kRowTile + (size_t)G * kRowTile) *
         sizeof(float);
}

template <typename KT>
__global__ void __launch_bounds__(256) k_pf_attn_rows(float* o_part, float2* ml, const float* Q,
                                                      const KT* kcache, const KT* vcache, int p0,
                                                      int n, int Hq, int Hkv, int S, float scale,
                                                      int ch, int ns) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  constexpr int D = 128, ds = D + 4, V4 = D / 4;
  const int ti = blockIdx.x, g = blockIdx.y, sidx = blockIdx.z, G = Hq / Hkv;
  const int r0 = ti * kRowTile, r1 = min(n, r0 + kRowTile);
  const int k0 = sidx * ch;
  if (k0 > p0 + r1 - 1) return;  // every row of the tile ends before this split
  const int k1 = min(k0 + ch, p0 + r1);  // keys of the tile's last row end at p0 + r1 - 1
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                                 // [G][16][ds]
  float* ks = qs + (size_t)G * kRowTile * ds;     // [32][ds]
  float* vs = ks + kAttnTile * ds;                // [32][ds]
  float* ps = vs + kAttnTile * ds;                // [G][32 keys][16 rows]
  float* rsc = ps + (size_t)G * kAttnTile * kRowTile;  // [G][16] rescale factors
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nt = blockDim.x;
  const int N = (Hq + 2 * Hkv) * D;
  // q rows of the G heads (rows past n read as zeros)
  for (int i = threadIdx.x; i < G * kRowTile * V4; i += nt) {
    const int h = i / (kRowTile * V4), rem = i - h * kRowTile * V4, r = rem / V4,
              e = (rem - r * V4) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < n) v = *reinterpret_cast<const float4*>(Q + (size_t)(r0 + r) * N + (size_t)(g * G + h) * D + e);
    *reinterpret_cast<float4*>(qs + ((size_t)h * kRowTile + r) * ds + e) = v;
  }
  const KT* kc = kcache + (size_t)g * S * D;
  const KT* vc = vcache + (size_t)g * S * D;
  const int h = warp;                  // this warp's query head (warps >= G only load)
  const int rr = lane >> 3, kk = lane & 7;
  float m_run[4], l_run[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.0f;
  }
  float4 o[kRowTile];  // p * v: rows 0..15 x dims 4 lane..4 lane+3
#pragma unroll
  for (int r = 0; r < kRowTile; ++r) o[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t0 = k0; t0 < k1; t0 += kAttnTile) {
    const int nk = min(kAttnTile, k1 - t0);
    __syncthreads();  // the previous tile is consumed (and q staged)
    for (int i = threadIdx.x; i < kAttnTile * V4; i += nt) {
      const int tt = i / V4, e = (i - tt * V4) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (tt < nk) {
        kv = kv4<KT>(kc + (size_t)(t0 + tt) * D + e);
        vv = kv4<KT>(vc + (size_t)(t0 + tt) * D + e);
      }
      *reinterpret_cast<float4*>(ks + tt * ds + e) = kv;
      *reinterpret_cast<float4*>(vs + tt * ds + e) = vv;
    }
    __syncthreads();
    if (h < G) {
      // scores of rows 4rr+i and keys kk+8j
      float2 sc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[i][j] = make_float2(0.f, 0.f);
      const float* qh = qs + ((size_t)h * kRowTile + 4 * rr) * ds;
#pragma unroll 4
      for (int e = 0; e < D; e += 4) {
        float4 qv[4], kv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(qh + i * ds + e);
#pragma unroll
        for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(ks + (kk + 8 * j) * ds + e);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sc[i][j] = __ffma2_rn(make_float2(qv[i].x, qv[i].y), make_float2(kv[j].x, kv[j].y), sc[i][j]);
            sc[i][j] = __ffma2_rn(make_float2(qv[i].z, qv[i].w), make_float2(kv[j].z, kv[j].w), sc[i][j]);
          }
      }
      // mask, online softmax per row (its 32 keys live in the 8 lanes kk)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 4 * rr + i, pos = p0 + r0 + r;
        float s[4], mt = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int key = kk + 8 * j, kp = t0 + key;
          s[j] = (key < nk && kp <= pos && r0 + r < n)
                     ? __fmul_rn(__fadd_rn(sc[i][j].x, sc[i][j].y), scale)
                     : -INFINITY;
          mt = fmaxf(mt, s[j]);
        }
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
        const float mn = fmaxf(m_run[i], mt);
        const float cf = mn == -INFINITY ? 1.0f : expf(m_run[i] - mn);
        float ls = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p = s[j] == -INFINITY ? 0.0f : expf(s[j] - mn);
          ps[((size_t)h * kAttnTile + kk + 8 * j) * kRowTile + r] = p;
          ls += p;
        }
        ls += __shfl_xor_sync(0xffffffffu, ls, 1);
        ls += __shfl_xor_sync(0xffffffffu, ls, 2);
        ls += __shfl_xor_sync(0xffffffffu, ls, 4);
        l_run[i] = fmaf(l_run[i], cf, ls);
        m_run[i] = mn;
        if (kk == 0) rsc[h * kRowTile + r] = cf;
      }
      __syncwarp();
      // p * v: this lane's 4 dims for all 16 rows
      const float* rs = rsc + h * kRowTile;
#pragma unroll
      for (int r = 0; r < kRowTile; ++r) {
        const float c = rs[r];
        o[r].x *= c;
        o[r].y *= c;
        o[r].z *= c;
        o[r].w *= c;
      }
      const float* ph = ps + (size_t)h * kAttnTile * kRowTile;
      for (int k = 0; k < nk; ++k) {
        const float4 v = *reinterpret_cast<const float4*>(vs + k * ds + 4 * lane);
        const float2 v01 = make_float2(v.x, v.y), v23 = make_float2(v.z, v.w);
#pragma unroll
        for (int r4 = 0; r4 < kRowTile; r4 += 4) {
          const float4 p = *reinterpret_cast<const float4*>(ph + k * kRowTile + r4);
          const float pr[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float2 a = make_float2(o[r4 + u].x, o[r4 + u].y), b = make_float2(o[r4 + u].z, o[r4 + u].w);
            a = __ffma2_rn(make_float2(pr[u], pr[u]), v01, a);
            b = __ffma2_rn(make_float2(pr[u], pr[u]), v23, b);
            o[r4 + u] = make_float4(a.x, a.y, b.x, b.y);
          }
        }
      }
      __syncwarp();  // ps and rsc are rewritten by the next tile
    }
  }
  if (h < G) {
#pragma unroll
    for (int r = 0; r < kRowTile; ++r) {
      if (r0 + r >= n || p0 + r0 + r < k0) continue;  // no keys of this split for the row
      const size_t slot = ((size_t)(r0 + r) * Hq + (size_t)g * G + h) * ns + sidx;
      *reinterpret_cast<float4*>(o_part + slot * D + 4 * lane) = o[r];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 4 * rr + i;
      if (kk == 0 && r0 + r < n && p0 + r0 + r >= k0) {
        const size_t slot = ((size_t)(r0 + r) * Hq + (size_t)g * G + h) * ns + sidx;
        ml[slot] = make_float2(m_run[i], l_run[i]);
      }
    }
  }
}

// One warp per (row, head) over merge_head (the kernel form of the merge).
template <int D>
__global__ void __launch_bounds__(128) k_pf_attn_merge(uint16_t* A, const float* o_part,
                                                       const float2* ml, int p0, int Hq, int ch,
                                                       int ns, const int* rowpos) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int t = blockIdx.x, n = gridDim.x, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (h >= Hq) return;
  const int pos = rowpos ? rowpos[t] : p0 + t;
  merge_head<D>(A, o_part, ml, n, t, h, Hq, ns, min(ns, pos / ch + 1), lane);
}

// X[t] += projection (the residual after o_proj / down_proj); then, with
// gamma, A[t], A[n + t], A[2n + t] = the three bf16 terms of
// gamma * (x * inv), inv = 1 / sqrtf(mean(x^2) + eps) of the updated row (the
// next RMSNorm, bf16.rs:231-270). A row is one cluster of kResidParts
// blocks, block r owning the r-th quarter of the columns (four adjacent
// columns per thread and step, held in registers); the quarters' sums of
// squares meet in distributed shared memory and are added in rank order.
constexpr int kResidParts = 4, kResidThreads = 128, kResidVec = 4;
__global__ void __cluster_dims__(kResidParts, 1, 1) __launch_bounds__(kResidThreads)
    k_pf_resid_norm(float* X, const float* D, int sp, const float* gamma, uint16_t* A, int N,
                    float eps) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  __shared__ float red[33];
  __shared__ float part_ss;
  const int r = blockIdx.x, t = blockIdx.y, n = gridDim.y;
  const int w = N / kResidParts, c0 = r * w;  // N % (4 * kResidParts) == 0
  float* x = X + (size_t)t * N;
  float4 v[kResidVec];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kResidVec; ++i) {
    const int j = c0 + 4 * (threadIdx.x + i * kResidThreads);
    if (j < c0 + w) {
      const float4 p = part_sum4(D, n, t, N, j, sp);
      const float4 o = *reinterpret_cast<const float4*>(x + j);
      v[i] = make_float4(__fadd_rn(o.x, p.x), __fadd_rn(o.y, p.y), __fadd_rn(o.z, p.z),
                         __fadd_rn(o.w, p.w));
      *reinterpret_cast<float4*>(x + j) = v[i];
      ss = fmaf(v[i].x, v[i].x, ss);
      ss = fmaf(v[i].y, v[i].y, ss);
      ss = fmaf(v[i].z, v[i].z, ss);
      ss = fmaf(v[i].w, v[i].w, ss);
    }
  }
  if (!gamma) return;  // the whole cluster (gamma is uniform)
  ss = bsum(ss, red);
  if (threadIdx.x == 0) part_ss = ss;
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  float tot = 0.0f;
#pragma unroll
  for (int q = 0; q < kResidParts; ++q) tot = __fadd_rn(tot, *cl.map_shared_rank(&part_ss, q));
  cl.sync();  // every peer has read this block's part_ss
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)N), eps)));
#pragma unroll
  for (int i = 0; i < kResidVec; ++i) {
    const int j = c0 + 4 * (threadIdx.x + i * kResidThreads);
    if (j < c0 + w) {
      put_split(A, n, t, N, j, __fmul_rn(gamma[j], __fmul_rn(v[i].x, inv)));
      put_split(A, n, t, N, j + 1, __fmul_rn(gamma[j + 1], __fmul_rn(v[i].y, inv)));
      put_split(A, n, t, N, j + 2, __fmul_rn(gamma[j + 2], __fmul_rn(v[i].z, inv)));
      put_split(A, n, t, N, j + 3, __fmul_rn(gamma[j + 3], __fmul_rn(v[i].w, inv)));
    }
  }
}

// Tensor-parallel form: this rank's part of the residual update, written in
// place over the first hi rows of D: X + projection on the rank that carries
// the residual (X non-null), the projection elsewhere; the ranks' parts are
// then summed.
__global__ void k_pf_resid_part(float* D, const float* X, int n, int N, int sp) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int t = blockIdx.x;
  for (int j = threadIdx.x; j < N; j += blockDim.x) {
    const float dl = part_sum(D, n, t, N, j, sp);  // reads D[t][j] before it is replaced
    D[(size_t)t * N + j] = X ? __fadd_rn(X[(size_t)t * N + j], dl) : dl;
  }
}

// h = (g / (1 + expf(-g))) * u (swiglu.rs:113-131) from the stacked gate|up
// projection, written as three bf16 terms for the down projection; four
// adjacent columns per thread (I % 4 == 0), partials summed as part_sum does.
__global__ void __launch_bounds__(kT) k_pf_swiglu_split(uint16_t* A, const float* D, int I, int sp) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int t = blockIdx.x, n = gridDim.x, N = 2 * I;
  const int j = 4 * (blockIdx.y * blockDim.x + threadIdx.x);
  if (j >= I) return;
  float g[4], u[4];
  for (int l = 0; l < sp; ++l) {
    const float* Dl = D + (size_t)l * kSplitParts * n * N;
    const float* r0 = Dl + (size_t)t * N;
    const float* r1 = Dl + (size_t)(n + t) * N;
    const float* r2 = Dl + (size_t)(2 * n + t) * N;
    const float4 g0 = __ldcs(reinterpret_cast<const float4*>(r0 + j));
    const float4 g1 = __ldcs(reinterpret_cast<const float4*>(r1 + j));
    const float4 g2 = __ldcs(reinterpret_cast<const float4*>(r2 + j));
    const float4 u0 = __ldcs(reinterpret_cast<const float4*>(r0 + I + j));
    const float4 u1 = __ldcs(reinterpret_cast<const float4*>(r1 + I + j));
    const float4 u2 = __ldcs(reinterpret_cast<const float4*>(r2 + I + j));
    const float ga[4] = {g0.x, g0.y, g0.z, g0.w}, gb[4] = {g1.x, g1.y, g1.z, g1.w},
                gc[4] = {g2.x, g2.y, g2.z, g2.w};
    const float ua[4] = {u0.x, u0.y, u0.z, u0.w}, ub[4] = {u1.x, u1.y, u1.z, u1.w},
                uc[4] = {u2.x, u2.y, u2.z, u2.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float gv = __fadd_rn(__fadd_rn(ga[i], gb[i]), gc[i]);
      const float uv = __fadd_rn(__fadd_rn(ua[i], ub[i]), uc[i]);
      g[i] = l ? __fadd_rn(g[i], gv) : gv;
      u[i] = l ? __fadd_rn(u[i], uv) : uv;
    }
  }
  uint16_t hi[4], mid[4], lo[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float s = __fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i])));
    const float y = __fmul_rn(s, u[i]);
    hi[i] = bf16_rn(y);
    const float e1 = __fsub_rn(y, __uint_as_float((uint32_t)hi[i] << 16));
    mid[i] = bf16_rn(e1);
    lo[i] = bf16_rn(__fsub_rn(e1, __uint_as_float((uint32_t)mid[i] << 16)));
  }
  auto pack = [](const uint16_t* v) {
    return make_uint2((uint32_t)v[0] | ((uint32_t)v[1] << 16), (uint32_t)v[2] | ((uint32_t)v[3] << 16));
  };
  *reinterpret_cast<uint2*>(A + (size_t)t * I + j) = pack(hi);
  *reinterpret_cast<uint2*>(A + (size_t)(n + t) * I + j) = pack(mid);
  *reinterpret_cast<uint2*>(A + (size_t)(2 * n + t) * I + j) = pack(lo);
}

// Greedy token of each row from the stacked logit parts: logits_b[j] =
// (D[b][j] + D[B + b][j]) + D[2B + b][j]; the first maximum with strict >,
// NaN and -inf never win, none -> 0 (model_core/src/lib.rs:157-167).
// Stage 1: block (b, c) takes columns [c * kArgChunk, (c + 1) * kArgChunk)
// and leaves its best (value, index) in part[b][c]; stage 2 picks among a
// row's chunks (larger value, or equal value and smaller index) and records
// the token.
constexpr int kArgChunk = 4096;
MYOS_DEV void amax_take(float& bv, uint32_t& bi, float v, uint32_t i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

__global__ void __launch_bounds__(kT) k_row_argmax_part(float2* part, const float* D, int B, int V,
                                                        int vec) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  __shared__ float bvs[kT / 32];
  __shared__ uint32_t bis[kT / 32];
  const int b = blockIdx.x, c = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j0 = c * kArgChunk, j1 = min(V, j0 + kArgChunk);
  const float* r0 = D + (size_t)b * V;
  const float* r1 = D + (size_t)(B + b) * V;
  const float* r2 = D + (size_t)(2 * B + b) * V;
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  if (vec) {  // V % 4 == 0: four adjacent columns per thread, all loads issued first
    constexpr int kPer = kArgChunk / 4 / kT;
    float4 a[kPer], bb[kPer], cc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int j = j0 + 4 * (threadIdx.x + i * kT);
      if (j < j1) {
        a[i] = __ldcs(reinterpret_cast<const float4*>(r0 + j));
        bb[i] = __ldcs(reinterpret_cast<const float4*>(r1 + j));
        cc[i] = __ldcs(reinterpret_cast<const float4*>(r2 + j));
      }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {  // j grows per thread: strict > keeps the first
      const int j = j0 + 4 * (threadIdx.x + i * kT);
      if (j < j1) {
        const float v0 = __fadd_rn(__fadd_rn(a[i].x, bb[i].x), cc[i].x);
        const float v1 = __fadd_rn(__fadd_rn(a[i].y, bb[i].y), cc[i].y);
        const float v2 = __fadd_rn(__fadd_rn(a[i].z, bb[i].z), cc[i].z);
        const float v3 = __fadd_rn(__fadd_rn(a[i].w, bb[i].w), cc[i].w);
        if (v0 > bv) { bv = v0; bi = (uint32_t)j; }
        if (v1 > bv) { bv = v1; bi = (uint32_t)j + 1; }
        if (v2 > bv) { bv = v2; bi = (uint32_t)j + 2; }
        if (v3 > bv) { bv = v3; bi = (uint32_t)j + 3; }
      }
    }
  } else {
    for (int j = j0 + threadIdx.x; j < j1; j += kT) {
      const float v = __fadd_rn(__fadd_rn(r0[j], r1[j]), r2[j]);
      if (v > bv) {
        bv = v;
        bi = (uint32_t)j;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    amax_take(bv, bi, ov, oi);
  }
  if (lane == 0) {
    bvs[warp] = bv;
    bis[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    for (int w = 0; w < kT / 32; ++w) amax_take(v, i, bvs[w], bis[w]);
    part[(size_t)b * gridDim.y + c] = make_float2(v, __uint_as_float(i));
  }
}

__global__ void k_row_argmax_fin(uint32_t* tok, uint32_t* out, int out_stride, int step,
                                 const int* d_step, const float2* part, int nc) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int b = blockIdx.x, lane = threadIdx.x;
  if (d_step) {  // the step index lives on the device (graph replays)
    step = *d_step;
    if (step >= out_stride) out = nullptr;
  }
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  for (int c = lane; c < nc; c += 32) {
    const float2 p = part[(size_t)b * nc + c];
    amax_take(bv, bi, p.x, __float_as_uint(p.y));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    amax_take(bv, bi, ov, oi);
  }
  if (lane == 0) {
    const uint32_t t = bi == 0xffffffffu ? 0u : bi;
    tok[b] = t;
    if (out) out[(size_t)b * out_stride + step] = t;
  }
}

__global__ void k_rows_copy(float* dst, const float* src, const int* src_row, int K) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int b = blockIdx.x;
  for (int j = threadIdx.x; j < K; j += blockDim.x)
    dst[(size_t)b * K + j] = src[(size_t)src_row[b] * K + j];
}

__global__ void k_pos_advance(int* rowpos, int B, int* d_step) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) rowpos[b] += 1;
  if (d_step && b == 0) *d_step += 1;
}

// Teacher-forced token of each row at the device-held step: tok[b] =
// feed_t[step * B + b].
__global__ void k_feed(uint32_t* tok, const uint32_t* feed_t, const int* d_step, int B) {
  pdl_begin();  // the previous kernel of the stream has finished (PDL)
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) tok[b] = feed_t[(size_t)(*d_step) * B + b];
}

}  // namespace

int pf_argmax_chunks(int V) { return (V + kArgChunk - 1) / kArgChunk; }

cudaError_t pf_row_argmax(uint32_t* tok, uint32_t* out, int out_stride, int step, const float* D,
                          float2* part, int B, int V, cudaStream_t st, const int* d_step) {
  const int nc = pf_argmax_chunks(V);
  if (cudaError_t e = launch(k_row_argmax_part, dim3(B, nc), kT, 0, st, part, D, B, V,
                             (int)(V % 4 == 0)))
    return e;
  return launch(k_row_argmax_fin, B, 32, 0, st, tok, out, out_stride, step, d_step, part, nc);
}

cudaError_t pf_rows_copy(float* dst, const float* src, const int* src_row, int B, int K,
                         cudaStream_t st) {
  return launch(k_rows_copy, B, kT, 0, st,
                dst, src, src_row, K);
}

cudaError_t pf_pos_advance(int* rowpos, int B, cudaStream_t st, int* d_step) {
  return launch(k_pos_advance, (B + 127) / 128, 128, 0, st,
                rowpos, B, d_step);
}

cudaError_t pf_feed(uint32_t* tok, const uint32_t* feed_t, const int* d_step, int B,
                    cudaStream_t st) {
  return launch(k_feed, (B + 127) / 128, 128, 0, st,
                tok, feed_t, d_step, B);
}

cudaError_t pf_embed(float* X, const uint16_t* embed, const uint32_t* ids, int n, int K,
                     cudaStream_t st) {
  return launch(k_pf_embed, n, kT, 0, st,
                X, embed, ids, K);
}

cudaError_t pf_norm_split(uint16_t* A, const float* X, const float* gamma, int n, int K, float eps,
                          cudaStream_t st) {
  return launch(k_pf_norm_split, n, kT, 0, st,
                A, X, gamma, n, K, eps);
}

cudaError_t pf_qkv_post(float* Q, const float* D, int sp, const float* bias, void* kc, void* vc,
                        int kv_bf16, const float* cos_t, const float* sin_t, int p0, int n, int Hq,
                        int Hkv, int d, int S, cudaStream_t st, const int* rowpos,
                        size_t rowstride) {
  if ((d != 64 && d != 128) || sp < 1 || sp > kMaxSplits) return cudaErrorInvalidValue;
  const dim3 grid(n, (Hq + 2 * Hkv + 256 / d - 1) / (256 / d));
  if (kv_bf16)
    return launch(k_pf_qkv_post<__nv_bfloat16>, grid, 128, 0, st, Q, D, sp, bias,
                  (__nv_bfloat16*)kc, (__nv_bfloat16*)vc, cos_t, sin_t, p0, Hq, Hkv, d, S, rowpos,
                  rowstride);
  return launch(k_pf_qkv_post<float>, grid, 128, 0, st, Q, D, sp, bias, (float*)kc, (float*)vc,
                cos_t, sin_t, p0, Hq, Hkv, d, S, rowpos, rowstride);
}

bool pf_attn_supported(int d, int G) { return (d == 64 || d == 128) && G <= 8; }

bool pf_pdl() { return g_pdl; }

cudaError_t pf_init() {
  const char* pe = getenv("MYOS_GEMM_PDL");
  g_pdl = !(pe && pe[0] == '0');
#define MYOS_PF_SMEM(KT, D)                                                                \
  if (cudaError_t e = cudaFuncSetAttribute(k_pf_attn_split<KT, D>,                         \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                           (int)attn_smem_bytes<D>()))                     \
    return e;
  MYOS_PF_SMEM(float, 64)
  MYOS_PF_SMEM(float, 128)
  MYOS_PF_SMEM(__nv_bfloat16, 64)
  MYOS_PF_SMEM(__nv_bfloat16, 128)
#define MYOS_PF_SMEM_W(KT, G)                                                              \
  if (cudaError_t e = cudaFuncSetAttribute(k_pf_attn_warps<KT, G>,                         \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                           (int)kWarpsSmem))                               \
    return e;                                                                              \
  if (cudaError_t e = cudaFuncSetAttribute(k_pf_attn_warps<KT, G>,                         \
                                           cudaFuncAttributePreferredSharedMemoryCarveout, \
                                           100))                                           \
    return e;
  MYOS_PF_SMEM_W(float, 5)
  MYOS_PF_SMEM_W(float, 6)
  MYOS_PF_SMEM_W(float, 7)
  MYOS_PF_SMEM_W(float, 8)
  MYOS_PF_SMEM_W(__nv_bfloat16, 5)
  MYOS_PF_SMEM_W(__nv_bfloat16, 6)
  MYOS_PF_SMEM_W(__nv_bfloat16, 7)
  MYOS_PF_SMEM_W(__nv_bfloat16, 8)
#undef MYOS_PF_SMEM_W
#undef MYOS_PF_SMEM
  const char* aw = getenv("MYOS_PF_ATTN_WARPS");
  g_attn_warps = !(aw && aw[0] == '0');
  const char* mf = getenv("MYOS_PF_MERGE_FUSED");
  g_merge_fused = !(mf && mf[0] == '0');
  const char* ad = getenv("MYOS_PF_ATTN_DYN");
  g_attn_dyn = !(ad && ad[0] == '0');
  const int rows_smem = (int)attn_rows_smem_bytes<128>(8);
  if (cudaError_t e = cudaFuncSetAttribute(
          k_pf_attn_rows<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, rows_smem))
    return e;
  if (cudaError_t e = cudaFuncSetAttribute(k_pf_attn_rows<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, rows_smem))
    return e;
  const char* rm = getenv("MYOS_PF_ATTN_ROWS_MIN");
  g_rows_min = rm ? atoi(rm) : 1024;
  return cudaSuccess;
}

int pf_attn_splits(int max_keys, int* ch) {
  // two 32-key tiles per split (the second's copies overlap the first's
  // math), or more so that a row has at most kAttnMaxSplits of them
  int c = 2 * kAttnTile;
  while ((max_keys + c - 1) / c > kAttnMaxSplits) c += kAttnTile;
  *ch = c;
  return (max_keys + c - 1) / c;
}

cudaError_t pf_attn(uint16_t* A, float* o_part, float2* ml, const float* Q, const void* kc,
                    const void* vc, int kv_bf16, int p0, int n, int Hq, int Hkv, int d, int S,
                    float scale, int max_keys, int sms, cudaStream_t st, const int* rowpos,
                    size_t rowstride, unsigned* arrive, unsigned* work) {
  if (!pf_attn_supported(d, Hq / Hkv) || max_keys < 1 || sms < 1) return cudaErrorInvalidValue;
  if (!rowpos && d == 128 && max_keys >= g_rows_min) {  // a long prompt chunk: row tiles
    int ch = 256;
    while ((max_keys + ch - 1) / ch > kAttnMaxSplits) ch += 256;
    const int ns = (max_keys + ch - 1) / ch, G = Hq / Hkv;
    const dim3 grid((n + kRowTile - 1) / kRowTile, Hkv, ns);
    const size_t smem = attn_rows_smem_bytes<128>(G);
    cudaError_t e = kv_bf16
                        ? launch(k_pf_attn_rows<__nv_bfloat16>, grid, 32 * G, smem, st, o_part, ml,
                                 Q, (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc, p0, n, Hq,
                                 Hkv, S, scale, ch, ns)
                        : launch(k_pf_attn_rows<float>, grid, 32 * G, smem, st, o_part, ml, Q,
                                 (const float*)kc, (const float*)vc, p0, n, Hq, Hkv, S, scale, ch,
                                 ns);
    if (e != cudaSuccess) return e;
    return launch(k_pf_attn_merge<128>, dim3(n, (Hq + 3) / 4), 128, 0, st, A, o_part, ml, p0, Hq,
                  ch, ns, rowpos);
  }
  int ch = 0;
  const int ns = pf_attn_splits(max_keys, &ch);
  const long items = (long)n * Hkv * ns;
  const dim3 grid((unsigned)std::min<long>(items, 2L * sms));  // two resident blocks per SM
  cudaError_t e = cudaSuccess;
  const int G = Hq / Hkv;
  if (g_attn_warps && d == 128 && G >= 5 && G <= 8) {
    const size_t smem = kWarpsSmem;
    // the merge sits on a block's path at an item's end: fused only while a
    // block has few items (many items: one merge launch is cheaper)
    if (!g_merge_fused || items > kMergeFusedItems * (long)grid.x) arrive = nullptr;
    if (!g_attn_dyn || items <= kAttnDynItems * (long)grid.x) work = nullptr;
#define MYOS_PF_ATTN_W(GG)                                                                     \
  if (G == GG)                                                                                 \
    e = kv_bf16 ? launch(k_pf_attn_warps<__nv_bfloat16, GG>, grid, kT, smem, st, o_part, ml, Q, \
                         (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc, p0, n, Hq, Hkv, S, \
                         scale, ch, ns, rowpos, rowstride, A, arrive, work)                     \
                : launch(k_pf_attn_warps<float, GG>, grid, kT, smem, st, o_part, ml, Q,         \
                         (const float*)kc, (const float*)vc, p0, n, Hq, Hkv, S, scale, ch, ns,  \
                         rowpos, rowstride, A, arrive, work);
    MYOS_PF_ATTN_W(5)
    MYOS_PF_ATTN_W(6)
    MYOS_PF_ATTN_W(7)
    MYOS_PF_ATTN_W(8)
#undef MYOS_PF_ATTN_W
    if (e != cudaSuccess || arrive) return e;
    return launch(k_pf_attn_merge<128>, dim3(n, (Hq + 3) / 4), 128, 0, st, A, o_part, ml, p0, Hq,
                  ch, ns, rowpos);
  }
#define MYOS_PF_ATTN(D)                                                                         \
  if (d == D) {                                                                                 \
    const size_t smem = attn_smem_bytes<D>();                                                   \
    e = kv_bf16 ? launch(k_pf_attn_split<__nv_bfloat16, D>, grid, kT, smem, st, o_part, ml, Q,  \
                         (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc, p0, n, Hq, Hkv, S, \
                         scale, ch, ns, rowpos, rowstride)                                      \
                : launch(k_pf_attn_split<float, D>, grid, kT, smem, st, o_part, ml, Q,          \
                         (const float*)kc, (const float*)vc, p0, n, Hq, Hkv, S, scale, ch, ns,  \
                         rowpos, rowstride);                                                    \
  }
  MYOS_PF_ATTN(64)
  MYOS_PF_ATTN(128)
#undef MYOS_PF_ATTN
  if (e != cudaSuccess) return e;
  const dim3 mgrid(n, (Hq + 3) / 4);
  if (d == 64)
    return launch(k_pf_attn_merge<64>, mgrid, 128, 0, st, A, o_part, ml, p0, Hq, ch, ns, rowpos);
  return launch(k_pf_attn_merge<128>, mgrid, 128, 0, st, A, o_part, ml, p0, Hq, ch, ns, rowpos);
}

cudaError_t pf_resid_norm(float* X, const float* D, int sp, const float* gamma, uint16_t* A, int n,
                          int N, float eps, cudaStream_t st) {
  if (N % (4 * kResidParts) || N > 4 * kResidVec * kResidThreads * kResidParts || sp < 1 ||
      sp > kMaxSplits)
    return cudaErrorInvalidValue;
  return launch(k_pf_resid_norm, dim3(kResidParts, n), kResidThreads, 0, st,
                X, D, sp, gamma, A, N, eps);
}

cudaError_t pf_resid_part(float* D, const float* X, int n, int N, int sp, cudaStream_t st) {
  return launch(k_pf_resid_part, n, kT, 0, st,
                D, X, n, N, sp);
}

cudaError_t pf_swiglu_split(uint16_t* A, const float* D, int n, int I, int sp, cudaStream_t st) {
  if (I % 4) return cudaErrorInvalidValue;
  const dim3 grid(n, (I / 4 + kT - 1) / kT);
  return launch(k_pf_swiglu_split, grid, kT, 0, st,
                A, D, I, sp);
}

}  // namespace myos
