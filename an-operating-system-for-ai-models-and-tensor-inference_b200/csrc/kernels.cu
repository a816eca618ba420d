// sm_100a kernels of the Qwen2.5 decode step.
//
// Every GEMV here is HBM-bound (one flop per weight byte), so the design
// goal is to keep DRAM streaming across kernel boundaries:
//   * each block owns a contiguous row range and issues a bulk L2 prefetch
//     of (the head of) that range BEFORE its programmatic-dependency wait,
//     so a kernel's weights stream in while its predecessor still runs;
//   * weights are read with 16-byte streaming loads (L1 no-allocate), several
//     rows and chunks in flight per lane, promoted to f32 by shift/mask;
//   * the input vector is staged once per block in shared memory, with the
//     RMSNorm of the reference (bf16.rs:231-270) fused into that staging;
//   * epilogues fuse the QKV bias (bf16.rs:147-158), the residual add
//     (qwen25_block.rs:172-178), SiLU(gate)*up (swiglu.rs:113-131,254-261)
//     and the first-maximum argmax (model_core/src/lib.rs:157-167).
// Reductions use a fixed shuffle tree per row, so results are identical run
// to run (the reference's DET gate), though not the serial chain's bits.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace myos {

constexpr int kThreads = 256;
constexpr int kMaxG = 8;

// ------------------------------------------------------------------ staging
// Vector layout (K % 8 == 0): chunk c's first four values at xs[4c..], its
// last four at xs[K/2 + 4c..], so a lane's two float4 reads hit distinct banks.
MYOS_DEV void stage_input(float* xs, int K, bool vec, const GemvInput& in, float* red) {
  const int nt = blockDim.x;
  const uint16_t* erow = nullptr;
  if (in.embed) {
    const uint32_t tok = in.feed ? in.feed[in.ctl->step] : in.ctl->argmax;
    erow = in.embed + (size_t)tok * (size_t)K;
    if (blockIdx.x == 0 && threadIdx.x == 0) in.ctl->fed = tok;
  }
  float inv = 1.0f;
  if (in.gamma) {
    float ss = 0.0f;
    for (int j = threadIdx.x; j < K; j += nt) {
      const float v = erow ? bf16_at(erow + j) : in.x[j];
      ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    // 1 / sqrtf(mean + eps): IEEE sqrt and division, as bf16.rs:263-270.
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), in.eps)));
  }
  const int half = K >> 1;
  for (int j = threadIdx.x; j < K; j += nt) {
    const float v = erow ? bf16_at(erow + j) : in.x[j];
    if (erow && in.x_store && blockIdx.x == 0) in.x_store[j] = v;
    // gamma * (x * inv): two rounded products, reference order.
    const float s = in.gamma ? __fmul_rn(in.gamma[j], __fmul_rn(v, inv)) : v;
    int dst = j;
    if (vec) {
      const int c = j >> 3, e = j & 7;
      dst = e < 4 ? (c * 4 + e) : (half + c * 4 + (e - 4));
    }
    xs[dst] = s;
  }
  __syncthreads();
}

// NR rows at once, U chunks of 16 bytes in flight per row per lane.
template <int NR, int U>
MYOS_DEV void dot_rows_vec(const uint4* const* w, const float4* xlo, const float4* xhi,
                           int nchunk, int lane, float* out) {
  float acc[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
  int c = lane;
  for (; c + 32 * (U - 1) < nchunk; c += 32 * U) {
    uint4 u[NR][U];
#pragma unroll
    for (int i = 0; i < U; ++i)
#pragma unroll
      for (int r = 0; r < NR; ++r) u[r][i] = ld_stream(w[r] + c + 32 * i);
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const float4 lo = xlo[c + 32 * i], hi = xhi[c + 32 * i];
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[r] = dot8(u[r][i], lo, hi, acc[r]);
    }
  }
  for (; c < nchunk; c += 32) {
    const float4 lo = xlo[c], hi = xhi[c];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = dot8(ld_stream(w[r] + c), lo, hi, acc[r]);
  }
#pragma unroll
  for (int r = 0; r < NR; ++r) out[r] = warp_sum(acc[r]);
}

// Any K (fixtures use K = 2): one element per lane step.
MYOS_DEV float dot_row_scalar(const uint16_t* w, const float* xs, int K, int lane) {
  float acc = 0.0f;
  for (int j = lane; j < K; j += 32) acc = fmaf(bf16_at(w + j), xs[j], acc);
  return warp_sum(acc);
}

MYOS_DEV float silu_mul(float g, float u) {
  // z / (1 + expf(-z)), then one multiply (swiglu.rs:113-115, 254-261).
  const float a = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(a, u);
}

// The reference keeps index i only if logits[i] > best, best starting at
// -inf: NaN and -inf never win, ties keep the lower index, and with no
// candidate the answer is 0.
MYOS_DEV bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > -INFINITY && (v > bv || (v == bv && i < bi));
}

template <int EPI>
MYOS_DEV void epilogue(const GemvArgs& a, int row, float v, float v2, float& bv, uint32_t& bi,
                       int lane) {
  if (EPI == EPI_ARGMAX) {
    if (better(v, (uint32_t)row, bv, bi)) {
      bv = v;
      bi = (uint32_t)row;
    }
  }
  if (lane != 0) return;
  if (EPI == EPI_STORE || EPI == EPI_ARGMAX) a.y[row] = v;
  if (EPI == EPI_BIAS) a.y[row] = __fadd_rn(v, a.bias[row]);
  if (EPI == EPI_RESID) a.y[row] = __fadd_rn(a.y[row], v);
  if (EPI == EPI_SWIGLU) a.y[row] = silu_mul(v, v2);
}

template <int EPI>
__global__ void __launch_bounds__(kThreads) k_gemv(GemvArgs a) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  __shared__ float red[33];
  __shared__ float wbv[kThreads / 32];
  __shared__ uint32_t wbi[kThreads / 32];
  __shared__ int last_block;

  const int G = gridDim.x, b = blockIdx.x;
  const int r0 = (int)((long long)b * a.M / G);
  const int r1 = (int)((long long)(b + 1) * a.M / G);
  const size_t row_bytes = (size_t)a.K * 2;
  if (a.prefetch_cap) {
    size_t bytes = (size_t)(r1 - r0) * row_bytes;
    if (EPI == EPI_SWIGLU) bytes = bytes < a.prefetch_cap / 2 ? bytes : a.prefetch_cap / 2;
    else if (bytes > a.prefetch_cap) bytes = a.prefetch_cap;
    prefetch_range(a.w + (size_t)r0 * a.K, bytes);
    if (EPI == EPI_SWIGLU) prefetch_range(a.w2 + (size_t)r0 * a.K, bytes);
  }
  pdl_wait();
  pdl_launch();

  const bool vec = (a.K & 7) == 0 && ((uintptr_t)a.w & 15) == 0 &&
                   (EPI != EPI_SWIGLU || ((uintptr_t)a.w2 & 15) == 0);
  stage_input(xs, a.K, vec, a.in, red);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  if (vec) {
    const float4* xlo = reinterpret_cast<const float4*>(xs);
    const float4* xhi = reinterpret_cast<const float4*>(xs + (a.K >> 1));
    const int nchunk = a.K >> 3;
    int row = r0 + warp;
    if (EPI == EPI_SWIGLU) {
      for (; row < r1; row += nw) {
        const uint4* w[2] = {reinterpret_cast<const uint4*>(a.w + (size_t)row * a.K),
                             reinterpret_cast<const uint4*>(a.w2 + (size_t)row * a.K)};
        float o[2];
        dot_rows_vec<2, 4>(w, xlo, xhi, nchunk, lane, o);
        epilogue<EPI>(a, row, o[0], o[1], bv, bi, lane);
      }
    } else {
      for (; row + nw < r1; row += 2 * nw) {
        const uint4* w[2] = {reinterpret_cast<const uint4*>(a.w + (size_t)row * a.K),
                             reinterpret_cast<const uint4*>(a.w + (size_t)(row + nw) * a.K)};
        float o[2];
        dot_rows_vec<2, 4>(w, xlo, xhi, nchunk, lane, o);
        epilogue<EPI>(a, row, o[0], 0.0f, bv, bi, lane);
        epilogue<EPI>(a, row + nw, o[1], 0.0f, bv, bi, lane);
      }
      if (row < r1) {
        const uint4* w[1] = {reinterpret_cast<const uint4*>(a.w + (size_t)row * a.K)};
        float o[1];
        dot_rows_vec<1, 8>(w, xlo, xhi, nchunk, lane, o);
        epilogue<EPI>(a, row, o[0], 0.0f, bv, bi, lane);
      }
    }
  } else {
    for (int row = r0 + warp; row < r1; row += nw) {
      const float g = dot_row_scalar(a.w + (size_t)row * a.K, xs, a.K, lane);
      const float u = EPI == EPI_SWIGLU ? dot_row_scalar(a.w2 + (size_t)row * a.K, xs, a.K, lane)
                                        : 0.0f;
      epilogue<EPI>(a, row, g, u, bv, bi, lane);
    }
  }

  if (EPI == EPI_ARGMAX) {
    if (lane == 0) {
      wbv[warp] = bv;
      wbi[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = -INFINITY;
      uint32_t i = 0xffffffffu;
      for (int w = 0; w < nw; ++w)
        if (better(wbv[w], wbi[w], v, i)) {
          v = wbv[w];
          i = wbi[w];
        }
      a.part_val[b] = v;
      a.part_idx[b] = i;
      __threadfence();
      const unsigned prev = atomicAdd(a.counter, 1u);
      last_block = prev == (unsigned)(G - 1);
    }
    __syncthreads();
    if (last_block && threadIdx.x == 0) {
      __threadfence();
      float v = -INFINITY;
      uint32_t i = 0xffffffffu;
      for (int q = 0; q < G; ++q) {
        const float pv = __ldcg(a.part_val + q);
        const uint32_t pi = __ldcg(a.part_idx + q);
        if (better(pv, pi, v, i)) {
          v = pv;
          i = pi;
        }
      }
      const uint32_t tok = i == 0xffffffffu ? 0u : i;
      StepCtl* ctl = a.in.ctl;
      const uint32_t s = ctl->step;
      if (a.rec_fed) a.rec_fed[s] = ctl->fed;
      if (a.rec_argmax) a.rec_argmax[s] = ctl->argmax;
      ctl->argmax = tok;
      ctl->pos = ctl->pos + 1;
      ctl->step = s + 1;
      *a.counter = 0u;
    }
  }
}

// ------------------------------------------------------------------ attention
template <typename KT>
MYOS_DEV float kv_load(const KT* p);
template <>
MYOS_DEV float kv_load<float>(const float* p) {
  return *p;
}
template <>
MYOS_DEV float kv_load<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename KT>
MYOS_DEV KT kv_from(float v);
template <>
MYOS_DEV float kv_from<float>(float v) {
  return v;
}
template <>
MYOS_DEV __nv_bfloat16 kv_from<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// NeoX half-rotate (rope.rs:145-184): y0 = x0*c - x1*s, y1 = x1*c + x0*s,
// each product rounded before the add; c, s from the host libm table.
MYOS_DEV float rope_lane(const float* x, int e, int d, const float* cs, const float* sn) {
  const int half = d >> 1;
  const int p = e < half ? e : e - half;
  const float x0 = x[p], x1 = x[p + half];
  const float c = cs[p], s = sn[p];
  return e < half ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s))
                  : __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

// Split-KV decode attention (flash-decoding). Block (s, g): keys of split s
// for KV head g, serving its G query heads (gqa.rs:96-105: heads
// [g*G, (g+1)*G) read KV head g). Each warp runs an online softmax over
// its keys; warps merge in shared memory; splits merge in the last block
// to arrive, in split order.
template <int DPL, typename KT>
__global__ void __launch_bounds__(kThreads) k_attn(AttnArgs a) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int d = a.d, G = a.G;
  float* qs = sm;                    // [G][d]
  float* knew = qs + G * d;          // [d]
  float* vnew = knew + d;            // [d]
  float* wm = vnew + d;              // [8][G]
  float* wl = wm + 8 * G;            // [8][G]
  float* wo = wl + 8 * G;            // [8][G][d]
  __shared__ int last_block;

  const int s = blockIdx.x, g = blockIdx.y;
  const int nt = blockDim.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const KT* kc = reinterpret_cast<const KT*>(a.kc) + (size_t)g * a.S * d;
  const KT* vc = reinterpret_cast<const KT*>(a.vc) + (size_t)g * a.S * d;

  pdl_wait();
  pdl_launch();

  int nkeys, pos = -1;
  if (a.decode) {
    pos = (int)a.ctl->pos;
    nkeys = pos + 1;
  } else {
    nkeys = a.nkeys_fixed;
  }
  const int kb = s * a.chunk;
  const int ke = min(kb + a.chunk, nkeys);
  const int half = d >> 1;
  const float* cs = a.decode ? a.cos_t + (size_t)pos * half : nullptr;
  const float* sn = a.decode ? a.sin_t + (size_t)pos * half : nullptr;

  for (int i = threadIdx.x; i < G * d; i += nt) {
    const int hh = i / d, e = i - hh * d;
    const float* qh = a.q + (size_t)(g * G + hh) * d;
    qs[i] = a.decode ? rope_lane(qh, e, d, cs, sn) : qh[e];
  }
  const bool has_new = a.decode && pos >= kb && pos < ke;
  if (has_new) {
    const float* kh = a.q + (size_t)a.Hq * d + (size_t)g * d;
    const float* vh = a.q + (size_t)(a.Hq + a.Hkv) * d + (size_t)g * d;
    KT* kdst = const_cast<KT*>(kc) + (size_t)pos * d;
    KT* vdst = const_cast<KT*>(vc) + (size_t)pos * d;
    for (int e = threadIdx.x; e < d; e += nt) {
      const KT kq = kv_from<KT>(rope_lane(kh, e, d, cs, sn));
      const KT vq = kv_from<KT>(vh[e]);
      knew[e] = kv_load<KT>(&kq);
      vnew[e] = kv_load<KT>(&vq);
      kdst[e] = kq;  // the cache slot for this position (KvCache::store)
      vdst[e] = vq;
    }
  }
  __syncthreads();

  float qr[kMaxG][DPL];
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh)
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int e = lane + 32 * j;
      qr[hh][j] = (hh < G && e < d) ? qs[hh * d + e] : 0.0f;
    }
  float m[kMaxG], l[kMaxG], acc[kMaxG][DPL];
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[hh][j] = 0.0f;
  }

  for (int t = kb + warp; t < ke; t += (nt >> 5)) {
    float kv[DPL], vv[DPL];
    const bool is_new = has_new && t == pos;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int e = lane + 32 * j;
      if (e < d) {
        kv[j] = is_new ? knew[e] : kv_load<KT>(kc + (size_t)t * d + e);
        vv[j] = is_new ? vnew[e] : kv_load<KT>(vc + (size_t)t * d + e);
      } else {
        kv[j] = 0.0f;
        vv[j] = 0.0f;
      }
    }
#pragma unroll
    for (int hh = 0; hh < kMaxG; ++hh) {
      if (hh < G) {
        float part = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) part = fmaf(qr[hh][j], kv[j], part);
        // score = dot * scale (gqa.rs:189-191), scale = 1/sqrtf(d)
        const float sc = __fmul_rn(warp_sum(part), a.scale);
        const float mn = fmaxf(m[hh], sc);
        const float corr = expf(m[hh] - mn);
        const float p = expf(sc - mn);
        l[hh] = fmaf(l[hh], corr, p);
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[hh][j] = fmaf(acc[hh][j], corr, p * vv[j]);
        m[hh] = mn;
      }
    }
  }

  // Merge warps.
#pragma unroll
  for (int hh = 0; hh < kMaxG; ++hh) {
    if (hh < G) {
      if (lane == 0) {
        wm[warp * G + hh] = m[hh];
        wl[warp * G + hh] = l[hh];
      }
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        const int e = lane + 32 * j;
        if (e < d) wo[(warp * G + hh) * d + e] = acc[hh][j];
      }
    }
  }
  __syncthreads();
  const int nwarps = nt >> 5;
  for (int i = threadIdx.x; i < G * d; i += nt) {
    const int hh = i / d, e = i - hh * d;
    float M = -INFINITY;
    for (int w = 0; w < nwarps; ++w) M = fmaxf(M, wm[w * G + hh]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int w = 0; w < nwarps; ++w) {
        const float f = expf(wm[w * G + hh] - M);
        L = fmaf(wl[w * G + hh], f, L);
        O = fmaf(wo[(w * G + hh) * d + e], f, O);
      }
    }
    const size_t pidx = ((size_t)g * a.nsplit + s) * G + hh;
    a.part_o[pidx * d + e] = O;
    if (e == 0) {
      a.part_m[pidx] = M;
      a.part_l[pidx] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.counters + g, 1u);
    last_block = prev == (unsigned)(a.nsplit - 1);
  }
  __syncthreads();
  if (!last_block) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * d; i += nt) {
    const int hh = i / d, e = i - hh * d;
    float M = -INFINITY;
    for (int q = 0; q < a.nsplit; ++q)
      M = fmaxf(M, __ldcg(a.part_m + ((size_t)g * a.nsplit + q) * G + hh));
    float L = 0.0f, O = 0.0f;
    for (int q = 0; q < a.nsplit; ++q) {
      const size_t pidx = ((size_t)g * a.nsplit + q) * G + hh;
      const float mq = __ldcg(a.part_m + pidx);
      if (mq == -INFINITY) continue;
      const float f = expf(mq - M);
      L = fmaf(__ldcg(a.part_l + pidx), f, L);
      O = fmaf(__ldcg(a.part_o + pidx * d + e), f, O);
    }
    a.out[(size_t)(g * G + hh) * d + e] = __fdiv_rn(O, L);
  }
  if (threadIdx.x == 0) a.counters[g] = 0u;
}

// ------------------------------------------------------------------ small kernels
__global__ void k_step_end(StepCtl* ctl) {
  pdl_wait();
  pdl_launch();
  if (threadIdx.x == 0) {
    ctl->pos = ctl->pos + 1;
    ctl->step = ctl->step + 1;
  }
}

// Two-stage argmax over an f32 vector: per-block first maximum, then the
// last block to arrive reduces the block results in block order.
__global__ void __launch_bounds__(kThreads) k_argmax(const float* v, int n, float* part_val,
                                                     uint32_t* part_idx, unsigned* counter,
                                                     uint32_t* out) {
  __shared__ float wbv[kThreads / 32];
  __shared__ uint32_t wbi[kThreads / 32];
  __shared__ int last_block;
  const int G = gridDim.x, b = blockIdx.x;
  const int r0 = (int)((long long)b * n / G), r1 = (int)((long long)(b + 1) * n / G);
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x)
    if (better(v[i], (uint32_t)i, bv, bi)) {
      bv = v[i];
      bi = (uint32_t)i;
    }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    wbv[warp] = bv;
    wbi[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float rv = -INFINITY;
    uint32_t ri = 0xffffffffu;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
      if (better(wbv[w], wbi[w], rv, ri)) {
        rv = wbv[w];
        ri = wbi[w];
      }
    part_val[b] = rv;
    part_idx[b] = ri;
    __threadfence();
    last_block = atomicAdd(counter, 1u) == (unsigned)(G - 1);
  }
  __syncthreads();
  if (last_block && threadIdx.x == 0) {
    __threadfence();
    float rv = -INFINITY;
    uint32_t ri = 0xffffffffu;
    for (int q = 0; q < G; ++q) {
      const float pv = __ldcg(part_val + q);
      const uint32_t pi = __ldcg(part_idx + q);
      if (better(pv, pi, rv, ri)) {
        rv = pv;
        ri = pi;
      }
    }
    *out = ri == 0xffffffffu ? 0u : ri;
    *counter = 0u;
  }
}

// One vector: y = gamma * (x * inv_rms), the staging math of the GEMVs.
__global__ void __launch_bounds__(kThreads) k_rmsnorm(float* y, const float* x, const float* gamma,
                                                      int n, float eps) {
  __shared__ float red[33];
  float ss = 0.0f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) ss = fmaf(x[j], x[j], ss);
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
  for (int j = threadIdx.x; j < n; j += blockDim.x) y[j] = __fmul_rn(gamma[j], __fmul_rn(x[j], inv));
}

__global__ void k_swiglu_mul(float* h, const float* gate, const float* up, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    h[i] = silu_mul(gate[i], up[i]);
}

__global__ void k_rope(float* y, const float* x, int len, int d, const float* cs, const float* sn) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < len; i += gridDim.x * blockDim.x) {
    const int h = i / d, e = i - h * d;
    y[i] = rope_lane(x + (size_t)h * d, e, d, cs, sn);
  }
}

// ------------------------------------------------------------------ launchers
static cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                   bool pdl, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

size_t gemv_smem_bytes(int K) { return (size_t)((K + 7) & ~7) * sizeof(float); }

cudaError_t launch_gemv(int epi, const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(grid), dim3(kThreads), gemv_smem_bytes(a.K), st, pdl, attr);
  switch (epi) {
    case EPI_STORE: return cudaLaunchKernelEx(&cfg, k_gemv<EPI_STORE>, a);
    case EPI_BIAS: return cudaLaunchKernelEx(&cfg, k_gemv<EPI_BIAS>, a);
    case EPI_RESID: return cudaLaunchKernelEx(&cfg, k_gemv<EPI_RESID>, a);
    case EPI_SWIGLU: return cudaLaunchKernelEx(&cfg, k_gemv<EPI_SWIGLU>, a);
    case EPI_ARGMAX: return cudaLaunchKernelEx(&cfg, k_gemv<EPI_ARGMAX>, a);
  }
  return cudaErrorInvalidValue;
}

int attn_dpl(int d) { return d <= 32 ? 1 : d <= 64 ? 2 : d <= 128 ? 4 : 8; }

size_t attn_smem_bytes(int G, int d) {
  return (size_t)(G * d + 2 * d + 16 * G + 8 * G * d) * sizeof(float);
}

template <int DPL>
static cudaError_t launch_attn_dpl(const AttnArgs& a, int kv_bf16, cudaLaunchConfig_t& cfg) {
  if (kv_bf16) return cudaLaunchKernelEx(&cfg, k_attn<DPL, __nv_bfloat16>, a);
  return cudaLaunchKernelEx(&cfg, k_attn<DPL, float>, a);
}

cudaError_t launch_attention(const AttnArgs& a, int kv_bf16, cudaStream_t st, bool pdl) {
  if (a.G > kMaxG || a.d > 256 || a.d <= 0) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(a.nsplit, a.Hkv), dim3(kThreads),
                                    attn_smem_bytes(a.G, a.d), st, pdl, attr);
  switch (attn_dpl(a.d)) {
    case 1: return launch_attn_dpl<1>(a, kv_bf16, cfg);
    case 2: return launch_attn_dpl<2>(a, kv_bf16, cfg);
    case 4: return launch_attn_dpl<4>(a, kv_bf16, cfg);
    default: return launch_attn_dpl<8>(a, kv_bf16, cfg);
  }
}

cudaError_t launch_step_end(StepCtl* ctl, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(32), 0, st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, k_step_end, ctl);
}

cudaError_t launch_argmax(const float* v, int n, float* part_val, uint32_t* part_idx,
                          unsigned* counter, uint32_t* out, int grid, cudaStream_t st) {
  k_argmax<<<grid, kThreads, 0, st>>>(v, n, part_val, part_idx, counter, out);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_mul(float* h, const float* gate, const float* up, int n,
                              cudaStream_t st) {
  int grid = (n + kThreads - 1) / kThreads;
  if (grid > 1184) grid = 1184;
  if (grid < 1) grid = 1;
  k_swiglu_mul<<<grid, kThreads, 0, st>>>(h, gate, up, n);
  return cudaGetLastError();
}

cudaError_t launch_rope(float* y, const float* x, int len, int head_dim, const float* cos_row,
                        const float* sin_row, cudaStream_t st) {
  int grid = (len + kThreads - 1) / kThreads;
  if (grid < 1) grid = 1;
  k_rope<<<grid, kThreads, 0, st>>>(y, x, len, head_dim, cos_row, sin_row);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(float* y, const float* x, const float* gamma, int n, float eps,
                           cudaStream_t st) {
  k_rmsnorm<<<1, kThreads, 0, st>>>(y, x, gamma, n, eps);
  return cudaGetLastError();
}

cudaError_t kernels_init() {
  // Dynamic shared-memory limits are per device: raise them once for each.
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t status = cudaGetDevice(&dev);
  if (status != cudaSuccess) return status;
  if (dev < 64 && (done_mask >> dev) & 1ull) return cudaSuccess;
  if (dev < 64) done_mask |= 1ull << dev;
  const int gemv_max = 200 * 1024;  // staged K up to 51200 floats
  const int attn_max = 200 * 1024;
  cudaError_t e;
#define MYOS_SET(kern, bytes)                                                               \
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)) != \
      cudaSuccess)                                                                          \
    return e;
  MYOS_SET(k_gemv<EPI_STORE>, gemv_max)
  MYOS_SET(k_gemv<EPI_BIAS>, gemv_max)
  MYOS_SET(k_gemv<EPI_RESID>, gemv_max)
  MYOS_SET(k_gemv<EPI_SWIGLU>, gemv_max)
  MYOS_SET(k_gemv<EPI_ARGMAX>, gemv_max)
  MYOS_SET((k_attn<1, float>), attn_max)
  MYOS_SET((k_attn<2, float>), attn_max)
  MYOS_SET((k_attn<4, float>), attn_max)
  MYOS_SET((k_attn<8, float>), attn_max)
  MYOS_SET((k_attn<1, __nv_bfloat16>), attn_max)
  MYOS_SET((k_attn<2, __nv_bfloat16>), attn_max)
  MYOS_SET((k_attn<4, __nv_bfloat16>), attn_max)
  MYOS_SET((k_attn<8, __nv_bfloat16>), attn_max)
#undef MYOS_SET
  return cudaSuccess;
}

}  // namespace myos
