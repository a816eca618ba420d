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
#include <stdlib.h>

#include <cooperative_groups.h>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace myos {

constexpr int kThreads = 256;
constexpr int kMaxG = 8;

// ------------------------------------------------------------------ staging
// Vector layout (K % 8 == 0): chunk c's first four values at xs[4c..], its
// last four at xs[K/2 + 4c..], so a lane's two float4 reads hit distinct banks.
//
// The input is read with 16-byte loads issued in batches of kStageBatch per
// thread before any shared-memory store, so staging costs about one L2 round
// trip instead of one per element.
constexpr int kStageBatch = 4;

// Weights (never written): read-only path. Activations written by the
// previous kernel: L2 only (__ldcg), read once per block then kept in smem.
MYOS_DEV float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
MYOS_DEV float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

MYOS_DEV void unpack8(const uint4& u, float4& lo, float4& hi) {
  lo = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
  hi = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
}

// Timeline stamps (KTrace): called by thread 0 of each block after the
// dependency wait (the step counter is only stable then).
MYOS_DEV uint64_t* trace_begin(const KTrace& t, const StepCtl* ctl, uint64_t t_start) {
  if (!t.buf || threadIdx.x != 0) return nullptr;
  uint64_t* row = t.buf + ((size_t)(ctl->step % kTraceSteps) * t.nslot + t.slot) * kTraceWidth;
  atomicMin(reinterpret_cast<unsigned long long*>(row), (unsigned long long)t_start);
  atomicMin(reinterpret_cast<unsigned long long*>(row + 1), (unsigned long long)global_ns());
  return row;
}
MYOS_DEV void trace_end(uint64_t* row) {
  if (row) atomicMax(reinterpret_cast<unsigned long long*>(row + 2), (unsigned long long)global_ns());
}
MYOS_DEV void trace_mark(uint64_t* row, int k) {
  if (row) atomicMax(reinterpret_cast<unsigned long long*>(row + k), (unsigned long long)global_ns());
}

MYOS_DEV void cpa16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
MYOS_DEV void cpa_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Attention-merge staging: x = merge of the split partials of the splits
// holding keys 0..pos. Per head h (KV head g = h / G): M = max_q m_q,
// f_q = expf(m_q - M), L = sum_q l_q f_q, x = (sum_q o_q f_q) / L, sums in
// split order (the reference's e / sum, gqa.rs:283-307, reassociated).
// All partials are copied into shared memory at once (scratch after xs).
MYOS_DEV void stage_merge(float* xs, int K, bool vec, const GemvInput& in, float* mb) {
  const int nt = blockDim.x;
  const int G = in.m_G, d = in.m_d, ns = in.m_nsplit, Hq = K / d, Hkv = Hq / G;
  const int nkeys = (int)in.ctl->pos + 1;
  int ne = (nkeys + in.m_chunk - 1) / in.m_chunk;
  if (ne > ns) ne = ns;
  float* po = mb;                       // [Hkv][ns][G][d] (valid splits filled)
  float* fs = po + (size_t)Hkv * ns * G * d;  // [Hkv][ns][G]
  float* ls = fs + Hkv * ns * G;
  float* Ls = ls + Hkv * ns * G;        // [Hq]
  const int per_g = ne * G * d;         // contiguous floats of one KV head's valid splits
  if ((d & 3) == 0) {
    const int q4 = per_g >> 2;
    for (int i = threadIdx.x; i < Hkv * q4; i += nt) {
      const int g = i / q4, r = i - g * q4;
      const size_t off = (size_t)g * ns * G * d + 4 * (size_t)r;
      cpa16(po + off, in.part_o + off);
    }
  } else {
    for (int i = threadIdx.x; i < Hkv * per_g; i += nt) {
      const int g = i / per_g, r = i - g * per_g;
      const size_t off = (size_t)g * ns * G * d + r;
      po[off] = __ldcg(in.part_o + off);
    }
  }
  const int per_m = ne * G;
  for (int i = threadIdx.x; i < Hkv * per_m; i += nt) {
    const int g = i / per_m, r = i - g * per_m;
    const int off = g * ns * G + r;
    fs[off] = __ldcg(in.part_m + off);
    ls[off] = __ldcg(in.part_l + off);
  }
  cpa_wait_all();
  __syncthreads();
  if (threadIdx.x < Hq) {
    const int h = threadIdx.x, g = h / G, hh = h - g * G;
    float M = -INFINITY;
    for (int q = 0; q < ne; ++q) M = fmaxf(M, fs[(g * ns + q) * G + hh]);
    float L = 0.0f;
    for (int q = 0; q < ne; ++q) {
      const int i = (g * ns + q) * G + hh;
      const float f = fs[i] == -INFINITY ? 0.0f : expf(fs[i] - M);
      fs[i] = f;
      L = fmaf(ls[i], f, L);
    }
    Ls[h] = L;
  }
  __syncthreads();
  for (int o = threadIdx.x; o < K; o += nt) {
    const int h = o / d, e = o - h * d, g = h / G, hh = h - g * G;
    float O = 0.0f;
    for (int q = 0; q < ne; ++q) {
      const int i = (g * ns + q) * G + hh;
      O = fmaf(po[(size_t)i * d + e], fs[i], O);
    }
    const float v = __fdiv_rn(O, Ls[h]);
    if (vec) {
      const int c = o >> 3, r = o & 7;
      xs[r < 4 ? (c * 4 + r) : ((K >> 1) + c * 4 + (r - 4))] = v;
    } else {
      xs[o] = v;
    }
  }
  __syncthreads();
}

// Staging for K % 256 == 0 in one round trip. Thread t owns chunks
// c = t + i*blockDim.x (8 values: 4 at xs[4c], 4 at xs[K/2 + 4c]); all its
// x (or bf16 embedding) loads are issued at once (K <= kStageOne * 8 *
// blockDim.x). The RMSNorm weight of the thread's chunks arrives in
// registers, loaded before the dependency wait (it depends on no kernel);
// the norm y = gamma * (x * inv), inv = 1 / sqrtf(mean(x^2) + eps)
// (bf16.rs:231-270) then needs one block reduction and no further load.
constexpr int kStageOne = 5;
constexpr int kGammaRegs = 3;

template <int NG>
MYOS_DEV void gamma_preload(const GemvInput& in, int K, float4 (&g0)[NG], float4 (&g1)[NG]) {
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < (K >> 3)) {
      g0[i] = ldg4(in.gamma + 8 * c);
      g1[i] = ldg4(in.gamma + 8 * c + 4);
    }
  }
}

template <int NG, int NS = kStageOne>
MYOS_DEV void stage_one_trip(float* xs, int K, const GemvInput& in, float* red, bool has_g,
                             const float4 (&g0)[NG], const float4 (&g1)[NG]) {
  const int nt = blockDim.x, nchunk = K >> 3, half = K >> 1;
  float4* xlo = reinterpret_cast<float4*>(xs);
  float4* xhi = reinterpret_cast<float4*>(xs + half);
  const uint16_t* erow = nullptr;
  if (in.embed) {
    const uint32_t tok = in.feed ? in.feed[in.ctl->step] : in.ctl->argmax;
    erow = in.embed + (size_t)tok * (size_t)K;
    if (blockIdx.x == 0 && threadIdx.x == 0) in.ctl->fed = tok;
  }
  float4 lo[NS], hi[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    const int c = threadIdx.x + i * nt;
    if (c < nchunk) {
      if (erow) {
        unpack8(__ldg(reinterpret_cast<const uint4*>(erow) + c), lo[i], hi[i]);
      } else {
        lo[i] = ldcg4(in.x + 8 * c);
        hi[i] = ldcg4(in.x + 8 * c + 4);
      }
    }
  }
  if (erow && in.x_store && blockIdx.x == 0) {  // block 0 also stores the embedding row
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      const int c = threadIdx.x + i * nt;
      if (c < nchunk) {
        reinterpret_cast<float4*>(in.x_store)[2 * c] = lo[i];
        reinterpret_cast<float4*>(in.x_store)[2 * c + 1] = hi[i];
      }
    }
  }
  if (has_g) {
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      if (threadIdx.x + i * nt < nchunk) {
        ss = fmaf(lo[i].x, lo[i].x, ss);
        ss = fmaf(lo[i].y, lo[i].y, ss);
        ss = fmaf(lo[i].z, lo[i].z, ss);
        ss = fmaf(lo[i].w, lo[i].w, ss);
        ss = fmaf(hi[i].x, hi[i].x, ss);
        ss = fmaf(hi[i].y, hi[i].y, ss);
        ss = fmaf(hi[i].z, hi[i].z, ss);
        ss = fmaf(hi[i].w, hi[i].w, ss);
      }
    }
    ss = block_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), in.eps)));
#pragma unroll
    for (int i = 0; i < NG; ++i) {
      const float4 a = lo[i], b = hi[i], ga = g0[i], gb = g1[i];
      lo[i] = make_float4(__fmul_rn(ga.x, __fmul_rn(a.x, inv)), __fmul_rn(ga.y, __fmul_rn(a.y, inv)),
                          __fmul_rn(ga.z, __fmul_rn(a.z, inv)), __fmul_rn(ga.w, __fmul_rn(a.w, inv)));
      hi[i] = make_float4(__fmul_rn(gb.x, __fmul_rn(b.x, inv)), __fmul_rn(gb.y, __fmul_rn(b.y, inv)),
                          __fmul_rn(gb.z, __fmul_rn(b.z, inv)), __fmul_rn(gb.w, __fmul_rn(b.w, inv)));
    }
  }
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    const int c = threadIdx.x + i * nt;
    if (c < nchunk) {
      xlo[c] = lo[i];
      xhi[c] = hi[i];
    }
  }
  __syncthreads();
}

MYOS_DEV void stage_input(float* xs, int K, bool vec, const GemvInput& in, float* red) {
  const int nt = blockDim.x;
  if (in.part_o) {
    stage_merge(xs, K, vec, in, xs + ((K + 7) & ~7));
    return;
  }
  const uint16_t* erow = nullptr;
  if (in.embed) {
    const uint32_t tok = in.feed ? in.feed[in.ctl->step] : in.ctl->argmax;
    erow = in.embed + (size_t)tok * (size_t)K;
    if (blockIdx.x == 0 && threadIdx.x == 0) in.ctl->fed = tok;
  }
  const int half = K >> 1;
  if (vec) {
    // 1. raw copy into the split layout (block 0 also stores the embedding row)
    const int nchunk = K >> 3;
    float4* xlo = reinterpret_cast<float4*>(xs);
    float4* xhi = reinterpret_cast<float4*>(xs + half);
    for (int c0 = threadIdx.x; c0 < nchunk; c0 += nt * kStageBatch) {
      float4 lo[kStageBatch], hi[kStageBatch];
#pragma unroll
      for (int i = 0; i < kStageBatch; ++i) {
        const int c = c0 + i * nt;
        if (c < nchunk) {
          if (erow) {
            unpack8(__ldg(reinterpret_cast<const uint4*>(erow) + c), lo[i], hi[i]);
          } else {
            lo[i] = ldcg4(in.x + 8 * c);
            hi[i] = ldcg4(in.x + 8 * c + 4);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kStageBatch; ++i) {
        const int c = c0 + i * nt;
        if (c < nchunk) {
          xlo[c] = lo[i];
          xhi[c] = hi[i];
          if (erow && in.x_store && blockIdx.x == 0) {
            reinterpret_cast<float4*>(in.x_store)[2 * c] = lo[i];
            reinterpret_cast<float4*>(in.x_store)[2 * c + 1] = hi[i];
          }
        }
      }
    }
    __syncthreads();
    if (!in.gamma) return;
    // 2. RMSNorm in place: gamma * (x * inv), inv = 1 / sqrtf(mean + eps)
    float ss = 0.0f;
    for (int j = threadIdx.x; j < K; j += nt) ss = fmaf(xs[j], xs[j], ss);
    ss = block_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), in.eps)));
    for (int c = threadIdx.x; c < nchunk; c += nt) {
      const float4 g0 = ldg4(in.gamma + 8 * c), g1 = ldg4(in.gamma + 8 * c + 4);
      float4 a = xlo[c], b = xhi[c];
      a = make_float4(__fmul_rn(g0.x, __fmul_rn(a.x, inv)), __fmul_rn(g0.y, __fmul_rn(a.y, inv)),
                      __fmul_rn(g0.z, __fmul_rn(a.z, inv)), __fmul_rn(g0.w, __fmul_rn(a.w, inv)));
      b = make_float4(__fmul_rn(g1.x, __fmul_rn(b.x, inv)), __fmul_rn(g1.y, __fmul_rn(b.y, inv)),
                      __fmul_rn(g1.z, __fmul_rn(b.z, inv)), __fmul_rn(g1.w, __fmul_rn(b.w, inv)));
      xlo[c] = a;
      xhi[c] = b;
    }
    __syncthreads();
    return;
  }
  // Generic widths (test fixtures): element-wise.
  float inv = 1.0f;
  if (in.gamma) {
    float ss = 0.0f;
    for (int j = threadIdx.x; j < K; j += nt) {
      const float v = erow ? bf16_at(erow + j) : in.x[j];
      ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), in.eps)));
  }
  for (int j = threadIdx.x; j < K; j += nt) {
    const float v = erow ? bf16_at(erow + j) : in.x[j];
    if (erow && in.x_store && blockIdx.x == 0) in.x_store[j] = v;
    xs[j] = in.gamma ? __fmul_rn(in.gamma[j], __fmul_rn(v, inv)) : v;
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
                       int lane, unsigned tp_epoch = 0) {
  if (EPI == EPI_ARGMAX) {
    if (better(v, (uint32_t)row, bv, bi)) {
      bv = v;
      bi = (uint32_t)row;
    }
  }
  if (lane != 0) return;
  if (EPI == EPI_STORE || EPI == EPI_ARGMAX) a.y[row] = v;
  if (EPI == EPI_BIAS) a.y[row] = __fadd_rn(v, a.bias[row]);
  if (EPI == EPI_RESID) {
    const float r = __fadd_rn(a.res_zero ? 0.0f : (a.res ? a.res[row] : a.y[row]), v);
    if (a.push.n) {
#pragma unroll
      for (int p = 0; p < kMaxTp; ++p)
        if (p < a.push.n) tp_store(a.push.out[p] + 2 * row, r, tp_epoch);
    } else {
      a.y[row] = r;
    }
  }
  if (EPI == EPI_SWIGLU) a.y[row] = silu_mul(v, v2);
}

// Block-level first maximum, then the last block to arrive picks among the
// per-block results (all its threads, the same total order) and advances
// the step control
// (greedy_token then KvCache::advance, qwen25_block.rs:765-780).
MYOS_DEV void argmax_finish(const GemvArgs& a, float bv, uint32_t bi, float* wbv, uint32_t* wbi,
                            int* last_block) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int G = gridDim.x, b = blockIdx.x;
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
    *last_block = prev == (unsigned)(G - 1);
  }
  __syncthreads();
  if (!*last_block) return;  // block-uniform
  // The last block picks among the G block candidates with every thread:
  // "better" is a total order (larger value, then smaller index; NaN never
  // wins), so the pick does not depend on the reduction order.
  __threadfence();
  float v = -INFINITY;
  uint32_t i = 0xffffffffu;
  for (int q = threadIdx.x; q < G; q += blockDim.x) {
    const float pv = __ldcg(a.part_val + q);
    const uint32_t pi = __ldcg(a.part_idx + q);
    if (better(pv, pi, v, i)) {
      v = pv;
      i = pi;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
  if (lane == 0) {
    wbv[warp] = v;
    wbi[warp] = i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 0; w < nw; ++w)
      if (better(wbv[w], wbi[w], v, i)) {
        v = wbv[w];
        i = wbi[w];
      }
    if (a.tp_cand || a.push.n) {  // this rank's vocab slice: hand over for the global pick
      const float iv = __uint_as_float(i == 0xffffffffu ? i : i + a.row0);
      if (a.push.n) {
        const unsigned e = __ldcg(a.push.seq) + 1u;
#pragma unroll
        for (int p = 0; p < kMaxTp; ++p)
          if (p < a.push.n) {
            tp_store(a.push.out[p], v, e);
            tp_store(a.push.out[p] + 2, iv, e);
          }
      } else {
        a.tp_cand[0] = v;
        a.tp_cand[1] = iv;
      }
      *a.counter = 0u;
      return;
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

  if (EPI == EPI_ARGMAX) argmax_finish(a, bv, bi, wbv, wbi, &last_block);
}

// ------------------------------------------------------------------ streaming GEMV
// K % 256 == 0 (every Qwen2.5 width): each lane owns P = K/256 chunks of
// 16 bytes per row (chunk lane + 32j, so a warp reads 512 contiguous bytes
// per j). A warp walks its rows as a flat sequence of batches of U chunks
// (NR weight rows per output row), double-buffered in registers: batch b+1
// is in flight while batch b is consumed, across row boundaries. Batch 0 is
// issued before the programmatic-dependency wait, so its DRAM latency
// overlaps the predecessor kernel and the input staging.
// This block's share of the strided ranges in a.pf_ptr, requested into L2.
MYOS_DEV void l2_prefetch_slices(const GemvArgs& a) {
  const int nr = 2 * a.pf_n;
  for (int r = blockIdx.x + gridDim.x * threadIdx.x; r < nr; r += gridDim.x * blockDim.x)
    prefetch_range_1(static_cast<const char*>(a.pf_ptr[r / a.pf_n]) + (size_t)(r % a.pf_n) * a.pf_stride,
                     a.pf_bytes[0]);
}

template <int NR, int U>
MYOS_DEV void load_batch(uint4 (&buf)[NR][U], const uint16_t* const* wbase, int K, int row,
                         int j0, int P, int lane) {
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const uint4* w = reinterpret_cast<const uint4*>(wbase[r] + (size_t)row * K);
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const int j = j0 + i;
      if (j < P) buf[r][i] = ld_stream(w + lane + 32 * j);
      else buf[r][i] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

template <int EPI, int NR, int U>
__global__ void __launch_bounds__(kThreads, 2) k_gemv_stream(GemvArgs a) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  __shared__ float red[33];
  __shared__ float wbv[kThreads / 32];
  __shared__ uint32_t wbi[kThreads / 32];
  __shared__ int last_block;

  const int G = gridDim.x, b = blockIdx.x;
  const int r0 = (int)((long long)b * a.M / G);
  const int r1 = (int)((long long)(b + 1) * a.M / G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int P = a.K >> 8;                   // chunks per lane per row
  const int nbr = (P + U - 1) / U;          // batches per row
  const int nrw = r1 - r0 > warp ? (r1 - r0 - warp + nw - 1) / nw : 0;  // rows of this warp
  const int nb = nrw * nbr;
  const uint16_t* wbase[NR];
  wbase[0] = a.w;
  if (NR > 1) wbase[NR - 1] = a.w2;

  if (a.prefetch_cap) {
    size_t bytes = (size_t)(r1 - r0) * (size_t)a.K * 2;
    const size_t cap = NR > 1 ? a.prefetch_cap / 2 : a.prefetch_cap;
    if (bytes > cap) bytes = cap;
#pragma unroll
    for (int r = 0; r < NR; ++r) prefetch_range(wbase[r] + (size_t)r0 * a.K, bytes);
  }
  const uint64_t t_start = a.tr.buf ? global_ns() : 0;
  // one-trip staging when the thread's chunks fit the register budget
  const int nchunk = a.K >> 3, nt = blockDim.x;
  const bool has_g = a.in.gamma != nullptr;
  const bool one = !a.in.part_o && nchunk <= kStageOne * nt && (!has_g || nchunk <= kGammaRegs * nt);
  float4 g0[kGammaRegs], g1[kGammaRegs];
  if (one && has_g) gamma_preload<kGammaRegs>(a.in, a.K, g0, g1);
  uint4 cur[NR][U], nxt[NR][U];
  if (nb > 0) load_batch<NR, U>(cur, wbase, a.K, r0 + warp, 0, P, lane);
  if (a.pf_mode) l2_prefetch_slices(a);
  pdl_wait();
  pdl_launch();
  const unsigned tp_epoch = (EPI == EPI_RESID && a.push.n) ? __ldcg(a.push.seq) + 1u : 0u;
  uint64_t* trow = trace_begin(a.tr, a.in.ctl, t_start);
  if (one) stage_one_trip<kGammaRegs>(xs, a.K, a.in, red, has_g, g0, g1);
  else stage_input(xs, a.K, true, a.in, red);
  trace_mark(trow, 3);  // input staged

  const float4* xlo = reinterpret_cast<const float4*>(xs);
  const float4* xhi = reinterpret_cast<const float4*>(xs + (a.K >> 1));
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  float acc[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
  for (int bt = 0; bt < nb; ++bt) {
    const int rb = bt / nbr, jb = bt - rb * nbr;
    if (bt + 1 < nb) {
      const int rn = (bt + 1) / nbr;
      load_batch<NR, U>(nxt, wbase, a.K, r0 + warp + nw * rn, ((bt + 1) - rn * nbr) * U, P, lane);
    }
    const int j0 = jb * U;
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const int j = j0 + i;
      if (j < P) {
        const float4 lo = xlo[lane + 32 * j], hi = xhi[lane + 32 * j];
#pragma unroll
        for (int r = 0; r < NR; ++r) acc[r] = dot8(cur[r][i], lo, hi, acc[r]);
      }
    }
    if (jb == nbr - 1) {
      const int row = r0 + warp + nw * rb;
      float o[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        o[r] = warp_sum(acc[r]);
        acc[r] = 0.0f;
      }
      epilogue<EPI>(a, row, o[0], NR > 1 ? o[NR - 1] : 0.0f, bv, bi, lane, tp_epoch);
    }
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int i = 0; i < U; ++i) cur[r][i] = nxt[r][i];
  }

  if (EPI == EPI_ARGMAX) argmax_finish(a, bv, bi, wbv, wbi, &last_block);
  if (a.tr.buf) {  // block-uniform
    __syncthreads();
    trace_end(trow);
  }
}

// ------------------------------------------------------------------ fused MLP
// One block per SM, 16 warps. A warp's work is a sequence of weight batches,
// each 2P 16-byte chunks per lane, double-buffered in registers exactly as
// in k_gemv_stream (the first batch is issued before the dependency wait):
//   batches 0..3: one (gate, up) row pair each (row c0 + warp + 16 i); the
//     lane-strided dot products and SiLU(gate)*up are those of the gate|up
//     GEMV, so the activations are the same bits;
//   then: down_proj rows in groups of four, eight lanes per row, each lane
//     one 16-byte chunk of the block's 64 columns against the activations of
//     those 8 columns (held in registers); the 8 lanes' products are summed
//     by a fixed xor tree into part[row][b].
// Reduction: after the grid-wide arrival, warp w of block b sums part[row][.]
// for the rows [b H / grid, (b+1) H / grid) assigned to it, lane-strided in
// block order then a fixed shuffle tree, and adds the sum to resid[row]
// (the reference's x + mlp, qwen25_block.rs:287).
constexpr int kMlpThreads = 512;
constexpr int kMlpWarps = kMlpThreads / 32;
constexpr int kMlpRowsPerWarp = kMlpSlice / kMlpWarps;  // gate|up rows per warp

MYOS_DEV unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <int P>
MYOS_DEV void mlp_load(uint4 (&buf)[2 * P], const MlpArgs& a, int slice, int bt, int warp, int lane,
                       int gpw) {
  const int c0 = slice * kMlpSlice;
  constexpr int UB = 2 * P;
  if (bt < kMlpRowsPerWarp) {
    const size_t r = (size_t)(c0 + warp + kMlpWarps * bt);
    const uint4* g = reinterpret_cast<const uint4*>(a.wg + r * a.H) + lane;
    const uint4* u = reinterpret_cast<const uint4*>(a.wu + r * a.H) + lane;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      buf[i] = ld_stream(g + 32 * i);
      buf[P + i] = ld_stream(u + 32 * i);
    }
  } else {
    const int j = bt - kMlpRowsPerWarp;
    // row r of the block's slice at base + r * ld (64 columns, 128 bytes)
    const uint16_t* base = a.wd_slices ? a.wd_slices + (size_t)slice * a.H * kMlpSlice : a.wd + c0;
    const size_t ld = a.wd_slices ? (size_t)kMlpSlice : (size_t)a.I;
#pragma unroll
    for (int i = 0; i < UB; ++i) {
      const int gi = j * UB + i;
      const int row = 4 * (warp + kMlpWarps * gi) + (lane >> 3);
      if (gi < gpw && row < a.H)
        buf[i] = ld_stream(reinterpret_cast<const uint4*>(base + (size_t)row * ld) + (lane & 7));
      else
        buf[i] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

__global__ void k_mlp_relayout(const uint4* wd, uint4* dst, int H, int I) {
  const size_t per_blk = (size_t)H * (kMlpSlice / 8);  // 16-byte chunks of one slice
  const size_t n = per_blk * (size_t)(I / kMlpSlice);
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < n;
       t += (size_t)gridDim.x * blockDim.x) {
    const size_t blk = t / per_blk, rem = t - blk * per_blk;
    const size_t row = rem / (kMlpSlice / 8), ch = rem - row * (kMlpSlice / 8);
    dst[t] = wd[(row * (size_t)I + blk * kMlpSlice) / 8 + ch];
  }
}

template <int P>
__global__ void __launch_bounds__(kMlpThreads, 1) k_mlp(MlpArgs a) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);  // [H] normed input, split layout
  __shared__ float red[33];
  __shared__ __align__(16) float acts[kMlpSlice];
  __shared__ int wait_failed;
  constexpr int UB = 2 * P;
  const int b = blockIdx.x, nblk = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H, c0 = b * kMlpSlice;
  const int gpw = (H / 4 + kMlpWarps - 1) / kMlpWarps;  // down row groups per warp
  const int nbt = kMlpRowsPerWarp + (gpw + UB - 1) / UB;

  const uint64_t t_start = a.tr.buf ? global_ns() : 0;
  GemvInput in = {};
  in.x = a.resid;
  in.ctl = a.ctl;
  in.gamma = a.gamma;
  in.eps = a.eps;
  float4 g0[1], g1[1];  // H <= 8 * kMlpThreads: one chunk per thread
  gamma_preload<1>(in, H, g0, g1);
  uint4 cur[UB], nxt[UB];
  mlp_load<P>(cur, a, b, 0, warp, lane, gpw);
  if (threadIdx.x == 0) wait_failed = 0;
  pdl_wait();
  pdl_launch();
  uint64_t* trow = trace_begin(a.tr, a.ctl, t_start);
  stage_one_trip<1, 1>(xs, H, in, red, true, g0, g1);
  trace_mark(trow, 3);  // input staged

  const float4* xlo = reinterpret_cast<const float4*>(xs);
  const float4* xhi = reinterpret_cast<const float4*>(xs + (H >> 1));
  float4 alo = make_float4(0.f, 0.f, 0.f, 0.f), ahi = alo;
  for (int bt = 0; bt < nbt; ++bt) {
    if (bt + 1 < nbt) mlp_load<P>(nxt, a, b, bt + 1, warp, lane, gpw);
    if (bt < kMlpRowsPerWarp) {
      float g = 0.0f, u = 0.0f;
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const float4 lo = xlo[lane + 32 * i], hi = xhi[lane + 32 * i];
        g = dot8(cur[i], lo, hi, g);
        u = dot8(cur[P + i], lo, hi, u);
      }
      g = warp_sum(g);
      u = warp_sum(u);
      if (lane == 0) acts[warp + kMlpWarps * bt] = silu_mul(g, u);
      if (bt == kMlpRowsPerWarp - 1) {  // every warp: all activations of the block
        __syncthreads();
        alo = reinterpret_cast<const float4*>(acts)[2 * (lane & 7)];
        ahi = reinterpret_cast<const float4*>(acts)[2 * (lane & 7) + 1];
        trace_mark(trow, 4);  // activations done
      }
    } else {
      const int j = bt - kMlpRowsPerWarp;
#pragma unroll
      for (int i = 0; i < UB; ++i) {
        float v = dot8(cur[i], alo, ahi, 0.0f);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        const int gi = j * UB + i;
        const int row = 4 * (warp + kMlpWarps * gi) + (lane >> 3);
        if ((lane & 7) == 0 && gi < gpw && row < H) a.part[(size_t)row * nblk + b] = v;
      }
    }
#pragma unroll
    for (int i = 0; i < UB; ++i) cur[i] = nxt[i];
  }

  // this warp's first output row: its residual does not change until the
  // sums below, so read it while the other blocks finish
  const int q0 = (int)((long long)b * H / nblk), q1 = (int)((long long)(b + 1) * H / nblk);
  const float res0 = (lane == 0 && q0 + warp < q1) ? __ldcg(a.resid + q0 + warp) : 0.0f;
  // grid-wide arrival: every block's shares written before any block sums
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long old = atomicAdd(a.arrive, 1ull);
    const unsigned long long target = (old / (unsigned long long)nblk + 1ull) * (unsigned long long)nblk;
    if (ld_acquire_u64(a.arrive) < target) {
      const uint64_t t0 = global_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_u64(a.arrive) >= target) break;
        if ((i & 63u) == 0 && global_ns() - t0 > a.wait_ns) {
          atomicOr(a.err, kErrMlpWait);
          wait_failed = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  trace_mark(trow, 5);  // all shares written
  if (!wait_failed) {
    for (int row = q0 + warp; row < q1; row += kMlpWarps) {
      const float* pr = a.part + (size_t)row * nblk;
      constexpr int kP = 8;  // nblk <= 256: every load of the lane in flight at once
      float v[kP];
#pragma unroll
      for (int i = 0; i < kP; ++i) v[i] = lane + 32 * i < nblk ? __ldcg(pr + lane + 32 * i) : 0.0f;
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < kP; ++i) s += v[i];
      s = warp_sum(s);
      if (lane == 0) a.resid[row] = __fadd_rn(row == q0 + warp ? res0 : __ldcg(a.resid + row), s);
    }
  }
  if (a.tr.buf) {  // block-uniform
    __syncthreads();
    trace_end(trow);
  }
}

int mlp_grid(int H, int I, int num_sms) {
  if (H != 1024 && H != 1280 && H != 1536) return 0;
  if (I % kMlpSlice != 0) return 0;
  const int g = I / kMlpSlice;
  if (g > num_sms || g > 256 || 4 * g < 3 * num_sms) return 0;
  return g;
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

// Four consecutive cache elements (16 B of f32 or 8 B of bf16), via L2:
// the cache is written by earlier launches.
template <typename KT>
MYOS_DEV float4 kv_load4(const KT* p);
template <>
MYOS_DEV float4 kv_load4<float>(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}
template <>
MYOS_DEV float4 kv_load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p));
  return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
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

// Split-KV decode attention (flash-decoding). Block (s, g) covers keys
// [s*chunk, (s+1)*chunk) for KV head g and its G query heads (gqa.rs:96-105:
// heads [g*G, (g+1)*G) read KV head g). Keys are processed in tiles of 32:
//   1. the tile's K and V rows are copied to shared memory (coalesced); the
//      first tile, and the rotation row, are loaded before the dependency
//      wait: cached keys below pos do not depend on the preceding kernel;
//   2. (head, key) scores = (q . k) * scale (gqa.rs:189-191,
//      scale = 1/sqrtf(d)), four threads per dot product when d % 16 == 0;
//   3. one warp per head runs the online softmax over the tile's 32 scores
//      (running max, expf(s - max), running sum);
//   4. threads accumulate p * v for their (head, lane) outputs.
// The block writes (unnormalised output, max, sum) per head. With
// defer_merge the o_proj staging merges the splits; otherwise the last block
// of KV head g to finish merges them in split order and divides by the sum
// (the reference's e / sum, gqa.rs:283-307, up to reassociation).
constexpr int kTile = 32;

template <typename KT>
MYOS_DEV void attn_tile_load(const KT* kc, const KT* vc, int d, int t0, int nk, int skip,
                             float* ks, float* vs) {
  const int nt = blockDim.x, ds = d + 4;
  if ((d & 3) == 0) {
    // quads of 4 elements; all of this thread's loads in flight together
    const int qpr = d >> 2, nqd = nk * qpr;
    constexpr int kQ = kTile * 64 / kThreads;  // d <= 256: at most 8 quads per thread
    float4 kq[kQ], vq[kQ];
#pragma unroll
    for (int j = 0; j < kQ; ++j) {
      const int i = threadIdx.x + nt * j;
      if (i < nqd) {
        const int tt = i / qpr, e = (i - tt * qpr) * 4;
        if (t0 + tt != skip) {
          kq[j] = kv_load4<KT>(kc + (size_t)(t0 + tt) * d + e);
          vq[j] = kv_load4<KT>(vc + (size_t)(t0 + tt) * d + e);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kQ; ++j) {
      const int i = threadIdx.x + nt * j;
      if (i < nqd) {
        const int tt = i / qpr, e = (i - tt * qpr) * 4;
        if (t0 + tt != skip) {
          *reinterpret_cast<float4*>(ks + tt * ds + e) = kq[j];
          *reinterpret_cast<float4*>(vs + tt * ds + e) = vq[j];
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < nk * d; i += nt) {
      const int tt = i / d, e = i - tt * d;
      if (t0 + tt == skip) continue;
      ks[tt * ds + e] = kv_load<KT>(kc + (size_t)(t0 + tt) * d + e);
      vs[tt * ds + e] = kv_load<KT>(vc + (size_t)(t0 + tt) * d + e);
    }
  }
}

template <int DPL, typename KT>
__global__ void __launch_bounds__(kThreads) k_attn(AttnArgs a) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int d = a.d, G = a.G, half = d >> 1;
  const int ds = d + 4;                   // padded row stride (float4 reads conflict-free)
  float* qs = sm;                         // [G][d] rotated q
  float* ks = qs + G * d;                 // [kTile][ds]
  float* vs = ks + kTile * ds;            // [kTile][ds]
  float* ps = vs + kTile * ds;            // [G][kTile]
  float* corr = ps + G * kTile;           // [G]
  float* knew = corr + kMaxG;             // [d] rotated new k (as cached)
  float* vnew = knew + d;                 // [d]
  float* qraw = vnew + d;                 // [G][d] q before rotation
  float* cst = qraw + G * d;              // [d/2] rotation row
  float* snt = cst + half;                // [d/2]
  float* kraw = snt + half;               // [d]
  float* vraw = kraw + d;                 // [d]
  __shared__ int last_block;

  const int s = blockIdx.x, g = blockIdx.y;
  const int nt = blockDim.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  KT* kc = reinterpret_cast<KT*>(a.kc) + (size_t)g * a.S * d;
  KT* vc = reinterpret_cast<KT*>(a.vc) + (size_t)g * a.S * d;

  // The position is set before the step's first kernel started, and the
  // cached keys below it by earlier steps, so both are read before the wait.
  int nkeys, pos = -1;
  if (a.decode) {
    pos = (int)a.ctl->pos;
    nkeys = pos + 1;
  } else {
    nkeys = a.nkeys_fixed;
  }
  const int kb = s * a.chunk;
  const int ke = min(kb + a.chunk, nkeys);
  const bool has_new = a.decode && pos >= kb && pos < ke;
  if (a.defer_merge && kb >= ke) return;  // no keys: the merge skips this split
  const uint64_t t_start = a.tr.buf ? global_ns() : 0;
  if (kb < ke) attn_tile_load<KT>(kc, vc, d, kb, min(kTile, ke - kb), has_new ? pos : -1, ks, vs);
  if (a.decode)
    for (int i = threadIdx.x; i < half; i += nt) {
      cst[i] = __ldg(a.cos_t + (size_t)pos * half + i);
      snt[i] = __ldg(a.sin_t + (size_t)pos * half + i);
    }

  pdl_wait();
  pdl_launch();
  uint64_t* trow = a.decode ? trace_begin(a.tr, a.ctl, t_start) : nullptr;

  {
    // q of the G heads and, when this split holds the new key, its k and v:
    // every load issued before the first store.
    float* qdst = a.decode ? qraw : qs;
    const int nq = G * d;
    const int ntot = nq + (has_new ? 2 * d : 0);
    const float* qsrc = a.q + (size_t)g * G * d;
    const float* ksrc = a.q + (size_t)a.Hq * d + (size_t)g * d;
    const float* vsrc = a.q + (size_t)(a.Hq + a.Hkv) * d + (size_t)g * d;
    constexpr int kJ = (kMaxG * 256 + 2 * 256) / kThreads;
    float val[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int v = threadIdx.x + nt * j;
      if (v < ntot)
        val[j] = v < nq ? __ldcg(qsrc + v)
                        : (v < nq + d ? __ldcg(ksrc + (v - nq)) : __ldcg(vsrc + (v - nq - d)));
    }
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int v = threadIdx.x + nt * j;
      if (v < ntot) {
        if (v < nq) qdst[v] = val[j];
        else if (v < nq + d) kraw[v - nq] = val[j];
        else vraw[v - nq - d] = val[j];
      }
    }
    if (a.decode) {
      __syncthreads();
      for (int i = threadIdx.x; i < nq; i += nt) {
        const int hh = i / d, e = i - hh * d;
        qs[i] = rope_lane(qraw + hh * d, e, d, cst, snt);
      }
      if (has_new) {
        const int tt = pos - kb;  // the new key sits in the first tile when tt < kTile
        for (int e = threadIdx.x; e < d; e += nt) {
          const KT kq = kv_from<KT>(rope_lane(kraw, e, d, cst, snt));
          const KT vq = kv_from<KT>(vraw[e]);
          knew[e] = kv_load<KT>(&kq);
          vnew[e] = kv_load<KT>(&vq);
          kc[(size_t)pos * d + e] = kq;  // the cache slot for this position (KvCache::store)
          vc[(size_t)pos * d + e] = vq;
          if (tt < kTile) {
            ks[tt * ds + e] = knew[e];
            vs[tt * ds + e] = vnew[e];
          }
        }
      }
    }
  }

  trace_mark(trow, 3);  // q staged and rotated (this thread's part)
  // Output slots: thread owns outputs o = threadIdx.x + nt*i of G*d.
  constexpr int kMaxOut = kMaxG * 256 / kThreads;
  float acc[kMaxOut];
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) acc[i] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;  // valid in lane 0.. of warp h < G (head h)

  for (int t0 = kb; t0 < ke; t0 += kTile) {
    const int nk = min(kTile, ke - t0);
    if (t0 != kb) {
      __syncthreads();  // previous tile fully consumed
      attn_tile_load<KT>(kc, vc, d, t0, nk, has_new ? pos : -1, ks, vs);
      if (has_new && pos >= t0 && pos < t0 + nk)
        for (int e = threadIdx.x; e < d; e += nt) {
          ks[(pos - t0) * ds + e] = knew[e];
          vs[(pos - t0) * ds + e] = vnew[e];
        }
    }
    __syncthreads();
    if ((d & 15) == 0) {
      // four threads per (head, key): quarter dot products, then two shuffles
      const int qd4 = d >> 2;
      for (int i = threadIdx.x; i < G * kTile * 4; i += nt) {
        const int hk = i >> 2, part = i & 3;
        const int hh = hk / kTile, tt = hk - hh * kTile;
        float dot = 0.0f;
        if (tt < nk) {
          const float* qh = qs + hh * d + part * qd4;
          const float* kr = ks + tt * ds + part * qd4;
          for (int e = 0; e < qd4; e += 4) {
            const float4 qv = *reinterpret_cast<const float4*>(qh + e);
            const float4 kv = *reinterpret_cast<const float4*>(kr + e);
            dot = fmaf(qv.x, kv.x, dot);
            dot = fmaf(qv.y, kv.y, dot);
            dot = fmaf(qv.z, kv.z, dot);
            dot = fmaf(qv.w, kv.w, dot);
          }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        if (part == 0) ps[hh * kTile + tt] = tt < nk ? __fmul_rn(dot, a.scale) : -INFINITY;
      }
    } else {
      for (int i = threadIdx.x; i < G * kTile; i += nt) {
        const int hh = i / kTile, tt = i - hh * kTile;
        float sc = -INFINITY;
        if (tt < nk) {
          const float* qh = qs + hh * d;
          const float* kr = ks + tt * ds;
          float dot = 0.0f;
          for (int e = 0; e < d; ++e) dot = fmaf(qh[e], kr[e], dot);
          sc = __fmul_rn(dot, a.scale);
        }
        ps[hh * kTile + tt] = sc;
      }
    }
    __syncthreads();
    if (warp < G) {
      const float sc = ps[warp * kTile + lane];
      const float mt = warp_max(sc);
      const float mn = fmaxf(m_run, mt);
      const float cf = expf(m_run - mn);  // 0 on the first tile (m_run = -inf)
      const float p = lane < nk ? expf(sc - mn) : 0.0f;
      l_run = fmaf(l_run, cf, warp_sum(p));
      m_run = mn;
      ps[warp * kTile + lane] = p;
      if (lane == 0) corr[warp] = cf;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxOut; ++i) {
      const int o = threadIdx.x + nt * i;
      if (o < G * d) {
        const int hh = o / d, e = o - hh * d;
        const float* ph = ps + hh * kTile;
        float v = acc[i] * corr[hh];
        for (int tt = 0; tt < nk; ++tt) v = fmaf(ph[tt], vs[tt * ds + e], v);
        acc[i] = v;
      }
    }
  }

  trace_mark(trow, 4);  // tiles done (thread 0's view)
  // This split's partial: (sum_t e_t v_t, max, sum) per head.
  const size_t pbase = ((size_t)g * a.nsplit + s) * G;
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) {
    const int o = threadIdx.x + nt * i;
    if (o < G * d) a.part_o[pbase * d + o] = acc[i];
  }
  if (warp < G && lane == 0) {
    a.part_m[pbase + warp] = m_run;
    a.part_l[pbase + warp] = l_run;
  }
  if (a.defer_merge) {
    if (a.tr.buf) {  // block-uniform
      __syncthreads();
      trace_end(trow);
    }
    return;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.counters + g, 1u);
    last_block = prev == (unsigned)(a.nsplit - 1);
  }
  __syncthreads();
  trace_mark(trow, 5);  // counted in
  if (!last_block) return;
  __threadfence();
  // Merge: factor f_q = expf(m_q - M) per (split, head), staged in shared memory.
  float* fs = sm;                    // [nsplit][G]
  float* ls = sm + a.nsplit * G;     // [nsplit][G]
  float* Ls = ls + a.nsplit * G;     // [G]
  const size_t gbase = (size_t)g * a.nsplit * G;
  for (int i = threadIdx.x; i < a.nsplit * G; i += nt) {
    const float mq = __ldcg(a.part_m + gbase + i);
    const float lq = __ldcg(a.part_l + gbase + i);
    fs[i] = mq;
    ls[i] = lq;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int hh = threadIdx.x;
    float M = -INFINITY;
    for (int q = 0; q < a.nsplit; ++q) M = fmaxf(M, fs[q * G + hh]);
    float L = 0.0f;
    for (int q = 0; q < a.nsplit; ++q) {
      const float mq = fs[q * G + hh];
      const float f = mq == -INFINITY ? 0.0f : expf(mq - M);
      fs[q * G + hh] = f;
      L = fmaf(ls[q * G + hh], f, L);
    }
    Ls[hh] = L;
  }
  __syncthreads();
  for (int o = threadIdx.x; o < G * d; o += nt) {
    const int hh = o / d;
    float O = 0.0f;
    int q = 0;
    for (; q + 8 <= a.nsplit; q += 8) {
      float po[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) po[u] = __ldcg(a.part_o + (gbase + (size_t)(q + u) * G) * d + o);
#pragma unroll
      for (int u = 0; u < 8; ++u) O = fmaf(po[u], fs[(q + u) * G + hh], O);
    }
    for (; q < a.nsplit; ++q) O = fmaf(__ldcg(a.part_o + (gbase + (size_t)q * G) * d + o), fs[q * G + hh], O);
    a.out[(size_t)g * G * d + o] = __fdiv_rn(O, Ls[hh]);
  }
  if (threadIdx.x == 0) a.counters[g] = 0u;
  if (a.tr.buf) {  // block-uniform
    __syncthreads();
    trace_end(trow);
  }
}

// Compact decode attention. The per-kernel step launches this kernel on a
// handful of SMs once per layer, so its instructions are fetched cold on
// every launch: the code is kept short (copies through cp.async, rolled
// loops) and the work per thread simple. Block (s, g) covers keys
// [s*chunk, (s+1)*chunk) of KV head g; warp h < G serves query head g*G + h:
//   lane t scores key t of the tile: (q . k_t) * scale (gqa.rs:189-191);
//   the warp runs the online softmax over the tile (max, expf(s - max), sum);
//   lane l accumulates p_t * v_t for dims [4l, 4l+4) (+128 for d > 128).
// The first tile and the rotation row are copied before the dependency wait.
// The split partials are merged by the o_proj staging (defer_merge) or by
// the last block of the KV head to finish, one warp per head, splits in order.
template <typename KT>
MYOS_DEV void dec_tile_issue(const KT* kc, const KT* vc, int d, int t0, int nk, int skip,
                             float* ks, float* vs, uint4* raw, int tid, int nt) {
  constexpr int per = 16 / sizeof(KT);  // elements per 16-byte piece
  const int ppr = d / per, ds = d + 4;
  for (int i = tid; i < nk * ppr; i += nt) {
    const int tt = i / ppr, e = (i - tt * ppr) * per;
    if (t0 + tt == skip) continue;
    const KT* ksrc = kc + (size_t)(t0 + tt) * d + e;
    const KT* vsrc = vc + (size_t)(t0 + tt) * d + e;
    if (sizeof(KT) == 4) {
      cpa16(ks + tt * ds + e, ksrc);
      cpa16(vs + tt * ds + e, vsrc);
    } else {
      cpa16(raw + i, ksrc);
      cpa16(raw + kTile * ppr + i, vsrc);
    }
  }
}

// Completes this thread's copies; bf16 rows are widened by the thread that
// copied them.
template <typename KT>
MYOS_DEV void dec_tile_finish(int d, int t0, int nk, int skip, float* ks, float* vs,
                              const uint4* raw, int tid, int nt) {
  cpa_wait_all();
  if (sizeof(KT) == 4) return;
  const int ppr = d / 8, ds = d + 4;
  for (int i = tid; i < nk * ppr; i += nt) {
    const int tt = i / ppr, e = (i - tt * ppr) * 8;
    if (t0 + tt == skip) continue;
    float4 lo, hi;
    unpack8(raw[i], lo, hi);
    *reinterpret_cast<float4*>(ks + tt * ds + e) = lo;
    *reinterpret_cast<float4*>(ks + tt * ds + e + 4) = hi;
    unpack8(raw[kTile * ppr + i], lo, hi);
    *reinterpret_cast<float4*>(vs + tt * ds + e) = lo;
    *reinterpret_cast<float4*>(vs + tt * ds + e + 4) = hi;
  }
}

// Per-tile work areas of k_attn_dec after the partials: the warps' partial
// scores [8 warps][8 heads][kTile], the probabilities [kTile][8] and the
// heads' rescale factors [8].
constexpr int kDecWarps = kThreads / 32;
constexpr size_t kDecWork = (size_t)kDecWarps * 8 * kTile + (size_t)kTile * 8 + 8;

// Cluster merge inbox of k_attn_dec: the partials (output, max, sum) the
// cluster's blocks push for the heads this block merges, slot w * ns + q for
// its w-th head and split q (at most 2 * kMaxG slots: ceil(G / ns) * ns).
constexpr int kDecInbox = 2 * kMaxG;

size_t attn_dec_smem_bytes(int G, int d) {
  // q, two padded tiles, new k/v, rotation row, raw bf16 tile rows, the
  // block's partial (output, max, sum), the tile work, the merge inbox
  return ((size_t)G * d + 2 * kTile * (d + 4) + 3 * (size_t)d + (size_t)kTile * d +
          (size_t)G * d + 2 * kMaxG + kDecWork + (size_t)kDecInbox * (d + 2)) *
         sizeof(float);
}

// One warp merges one head over the splits q < ne that hold keys:
// M = max m_q, f_q = expf(m_q - M), L = sum l_q f_q, out = (sum o_q f_q) / L
// (the reference's e / sum, gqa.rs:283-307, reassociated). Lane q holds split
// q's max and sum (32 splits per round); the outputs accumulate in split
// order, 8 splits' loads in flight at a time. src.m(q), src.l(q) and
// src.o(q, e) read split q's partial (float4 at dim e).
template <class Src>
MYOS_DEV void merge_head(const Src& src, int ne, int d, int lane, float* out) {
  if (ne <= 8) {
    // one round of loads: the outputs, maxima and sums of every split at once
    float4 po[2][8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int e = 4 * lane + 128 * j;
        po[j][u] = (u < ne && e < d) ? src.o(u, e) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    const float mq = lane < ne ? src.m(lane) : -INFINITY;
    const float lq = lane < ne ? src.l(lane) : 0.0f;
    const float M = warp_max(mq);
    const float f = mq == -INFINITY ? 0.0f : expf(mq - M);
    const float L = warp_sum(lq * f);
    float4 O[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float fu = __shfl_sync(0xffffffffu, f, u);
      if (u < ne)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          O[j].x = fmaf(po[j][u].x, fu, O[j].x);
          O[j].y = fmaf(po[j][u].y, fu, O[j].y);
          O[j].z = fmaf(po[j][u].z, fu, O[j].z);
          O[j].w = fmaf(po[j][u].w, fu, O[j].w);
        }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int e = 4 * lane + 128 * j;
      if (e < d)
        *reinterpret_cast<float4*>(out + e) = make_float4(
            __fdiv_rn(O[j].x, L), __fdiv_rn(O[j].y, L), __fdiv_rn(O[j].z, L), __fdiv_rn(O[j].w, L));
    }
    return;
  }
  float M = -INFINITY;
  for (int q0 = 0; q0 < ne; q0 += 32)
    M = fmaxf(M, warp_max(q0 + lane < ne ? src.m(q0 + lane) : -INFINITY));
  float Lp = 0.0f;
  float4 O[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  // kMergeBatch splits' outputs in flight per round of loads (the merge
  // of many splits is a chain of L2 round trips)
  constexpr int kMergeBatch = 16;
  for (int q0 = 0; q0 < ne; q0 += 32) {
    const int q = q0 + lane;
    const float mq = q < ne ? src.m(q) : -INFINITY;
    const float f = mq == -INFINITY ? 0.0f : expf(mq - M);
    if (q < ne) Lp = fmaf(src.l(q), f, Lp);
    const int nr = min(32, ne - q0);
    for (int u0 = 0; u0 < nr; u0 += kMergeBatch) {
      float4 po[2][kMergeBatch];
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int e = 4 * lane + 128 * j;
          po[j][u] = (u0 + u < nr && e < d) ? src.o(q0 + u0 + u, e) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        const float fu = __shfl_sync(0xffffffffu, f, (u0 + u) & 31);
        if (u0 + u < nr)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            O[j].x = fmaf(po[j][u].x, fu, O[j].x);
            O[j].y = fmaf(po[j][u].y, fu, O[j].y);
            O[j].z = fmaf(po[j][u].z, fu, O[j].z);
            O[j].w = fmaf(po[j][u].w, fu, O[j].w);
          }
      }
    }
  }
  const float L = warp_sum(Lp);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int e = 4 * lane + 128 * j;
    if (e < d)
      *reinterpret_cast<float4*>(out + e) = make_float4(
          __fdiv_rn(O[j].x, L), __fdiv_rn(O[j].y, L), __fdiv_rn(O[j].z, L), __fdiv_rn(O[j].w, L));
  }
}

// Split partials in global memory (head row r(q) = (g*ns + q)*G + h).
struct GlobalPartials {
  const float *pm, *pl, *po;
  size_t base;  // (g*ns)*G + h
  int G, d;
  MYOS_DEV size_t row(int q) const { return base + (size_t)q * G; }
  MYOS_DEV float m(int q) const { return __ldcg(pm + row(q)); }
  MYOS_DEV float l(int q) const { return __ldcg(pl + row(q)); }
  MYOS_DEV float4 o(int q, int e) const {
    return __ldcg(reinterpret_cast<const float4*>(po + row(q) * d + e));
  }
};

// Split partials pushed into this block's shared memory (split q at q).
struct LocalPartials {
  const float *po, *pm, *pl;
  int d;
  MYOS_DEV float m(int q) const { return pm[q]; }
  MYOS_DEV float l(int q) const { return pl[q]; }
  MYOS_DEV float4 o(int q, int e) const {
    return *reinterpret_cast<const float4*>(po + (size_t)q * d + e);
  }
};

template <typename KT, int D>
__global__ void __launch_bounds__(kThreads, 1) k_attn_dec(AttnArgs a) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  constexpr int d = D, half = D / 2, ds = D + 4;  // head dim fixed at compile time
  const int G = a.G;
  float* qs = sm;                   // [G][d]
  float* ks = qs + G * d;           // [kTile][ds]
  float* vs = ks + kTile * ds;      // [kTile][ds]
  float* kn = vs + kTile * ds;      // [d] new k
  float* vn = kn + d;               // [d] new v
  float* cs = vn + d;               // [d/2]
  float* sn = cs + half;            // [d/2]
  uint4* raw = reinterpret_cast<uint4*>(sn + half);
  __shared__ int last_block;
  const int s = blockIdx.x, g = blockIdx.y, ns = a.nsplit;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  KT* kc = reinterpret_cast<KT*>(a.kc) + (size_t)g * a.S * d;
  KT* vc = reinterpret_cast<KT*>(a.vc) + (size_t)g * a.S * d;
  // The position is set before the step's first kernel started, and the
  // cached keys below it by earlier steps: both are read before the wait.
  const int pos = (int)a.ctl->pos;
  const int kb = s * a.chunk, ke = min(kb + a.chunk, pos + 1);
  const bool has_new = pos >= kb && pos < ke;
  if (a.defer_merge && kb >= ke) return;  // no keys: the merge skips this split
  const uint64_t t_start = a.tr.buf ? global_ns() : 0;
  if (kb < ke) dec_tile_issue<KT>(kc, vc, d, kb, min(kTile, ke - kb), pos, ks, vs, raw, threadIdx.x, blockDim.x);
  const float4* c4 = reinterpret_cast<const float4*>(a.cos_t + (size_t)pos * half);
  const float4* s4 = reinterpret_cast<const float4*>(a.sin_t + (size_t)pos * half);
  for (int i = threadIdx.x; i < (half >> 2); i += blockDim.x) {
    cpa16(reinterpret_cast<float4*>(cs) + i, c4 + i);
    cpa16(reinterpret_cast<float4*>(sn) + i, s4 + i);
  }

  pdl_wait();
  pdl_launch();
  uint64_t* trow = trace_begin(a.tr, a.ctl, t_start);

  // q of the G heads; the new k and v when this split holds position pos
  const int nq4 = G * d / 4, d4 = d / 4;
  const float4* q4 = reinterpret_cast<const float4*>(a.q + (size_t)g * G * d);
  const float4* k4 = reinterpret_cast<const float4*>(a.q + (size_t)(a.Hq + g) * d);
  const float4* v4 = reinterpret_cast<const float4*>(a.q + (size_t)(a.Hq + a.Hkv + g) * d);
  for (int i = threadIdx.x; i < nq4 + (has_new ? 2 * d4 : 0); i += blockDim.x) {
    if (i < nq4) cpa16(reinterpret_cast<float4*>(qs) + i, q4 + i);
    else if (i < nq4 + d4) cpa16(reinterpret_cast<float4*>(kn) + (i - nq4), k4 + (i - nq4));
    else cpa16(reinterpret_cast<float4*>(vn) + (i - nq4 - d4), v4 + (i - nq4 - d4));
  }
  if (kb < ke) dec_tile_finish<KT>(d, kb, min(kTile, ke - kb), pos, ks, vs, raw, threadIdx.x, blockDim.x);
  cpa_wait_all();
  __syncthreads();
  trace_mark(trow, 3);  // q, new k/v and the first tile in shared memory
  // NeoX rotation in place (rope.rs:145-184): y0 = x0*c - x1*s, y1 = x1*c + x0*s
  for (int i = threadIdx.x; i < (G + (has_new ? 1 : 0)) * half; i += blockDim.x) {
    const int h = i / half, p = i - h * half;
    float* x = h < G ? qs + h * d : kn;
    const float x0 = x[p], x1 = x[p + half];
    x[p] = __fsub_rn(__fmul_rn(x0, cs[p]), __fmul_rn(x1, sn[p]));
    x[p + half] = __fadd_rn(__fmul_rn(x1, cs[p]), __fmul_rn(x0, sn[p]));
  }
  __syncthreads();
  if (has_new) {
    for (int e = threadIdx.x; e < d; e += blockDim.x) {
      const KT kq = kv_from<KT>(kn[e]), vq = kv_from<KT>(vn[e]);
      kc[(size_t)pos * d + e] = kq;  // KvCache::store for this position
      vc[(size_t)pos * d + e] = vq;
      kn[e] = kv_load<KT>(&kq);
      vn[e] = kv_load<KT>(&vq);
      if (pos - kb < kTile) {
        ks[(pos - kb) * ds + e] = kn[e];
        vs[(pos - kb) * ds + e] = vn[e];
      }
    }
    __syncthreads();
  }

  trace_mark(trow, 4);  // rotated, new key stored
  // Tile work layout (8 warps): scores: warp w takes dims [w D/8, (w+1) D/8)
  // of every head, lane = key, each K element read from shared memory once
  // (q values are broadcasts); the 8 partial sums meet in shared memory and
  // are added in warp order; softmax: warp h < G owns head h's running max
  // and sum; p * v: lane = (key group kg, head pair hp, 4 dims) of warp w's
  // dims, so each V element read serves two heads; the key groups are summed
  // by shuffles after the last tile.
  constexpr int DW = D / kDecWarps, CW = DW / 4, LK = CW * 4, KG = 32 / LK;
  float* red = reinterpret_cast<float*>(raw) + kTile * d + G * d + 2 * kMaxG;  // [8][8][kTile]
  float* pr = red + kDecWarps * 8 * kTile;                                    // [kTile][8]
  float* cfs = pr + kTile * 8;                                                // [8]
  const int kg = lane / LK, hp = (lane % LK) / CW, cq = lane % CW;
  const int dv = warp * DW + cq * 4;  // this lane's 4 dims in p * v
  float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  float m_run = -INFINITY, l_run = 0.0f;  // warp h < G: head h
  for (int t0 = kb; t0 < ke; t0 += kTile) {
    const int nk = min(kTile, ke - t0);
    if (t0 != kb) {  // later tiles
      __syncthreads();
      // f32 rows are copied straight into ks/vs now; bf16 rows were copied
      // into `raw` while the previous tile was computed
      if (sizeof(KT) == 4) dec_tile_issue<KT>(kc, vc, d, t0, nk, pos, ks, vs, raw, threadIdx.x, blockDim.x);
      dec_tile_finish<KT>(d, t0, nk, pos, ks, vs, raw, threadIdx.x, blockDim.x);
      if (has_new && pos >= t0 && pos < t0 + nk)
        for (int e = threadIdx.x; e < d; e += blockDim.x) {
          ks[(pos - t0) * ds + e] = kn[e];
          vs[(pos - t0) * ds + e] = vn[e];
        }
      __syncthreads();
    }
    // bf16: the next tile's rows into `raw` (widened by every thread after
    // this tile, so `raw` is free), in flight during this tile's math
    if (sizeof(KT) == 2 && t0 + kTile < ke)
      dec_tile_issue<KT>(kc, vc, d, t0 + kTile, min(kTile, ke - t0 - kTile), pos, ks, vs, raw,
                         threadIdx.x, blockDim.x);
    {  // partial scores of key `lane` over this warp's dims, heads < G
      float sc[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) sc[h] = 0.0f;
      if (lane < nk) {
#pragma unroll
        for (int c = 0; c < CW; ++c) {
          const int e = warp * DW + 4 * c;
          const float4 kv = *reinterpret_cast<const float4*>(ks + lane * ds + e);
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            if (h < G) {
              const float4 qv = *reinterpret_cast<const float4*>(qs + h * d + e);
              sc[h] = fmaf(qv.x, kv.x, sc[h]);
              sc[h] = fmaf(qv.y, kv.y, sc[h]);
              sc[h] = fmaf(qv.z, kv.z, sc[h]);
              sc[h] = fmaf(qv.w, kv.w, sc[h]);
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 8; ++h) red[(warp * 8 + h) * kTile + lane] = sc[h];
    }
    __syncthreads();
    if (warp < G) {  // online softmax of head `warp` over this tile
      float sc = -INFINITY;
      if (lane < nk) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) v = __fadd_rn(v, red[(w * 8 + warp) * kTile + lane]);
        sc = __fmul_rn(v, a.scale);
      }
      const float mn = fmaxf(m_run, warp_max(sc));
      const float cf = expf(m_run - mn);  // 0 on the first tile (m_run = -inf)
      const float p = lane < nk ? expf(sc - mn) : 0.0f;
      l_run = fmaf(l_run, cf, warp_sum(p));
      m_run = mn;
      pr[lane * 8 + warp] = p;
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
      for (int t = kg; t < nk; t += KG) {  // packed f32x2 FMAs, per element as fmaf
        const float4 v = *reinterpret_cast<const float4*>(vs + t * ds + dv);
        const float2 pp = *reinterpret_cast<const float2*>(pr + t * 8 + 2 * hp);
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
  }
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
  trace_mark(trow, 5);  // tiles done
  const int ne = min(ns, (pos + a.chunk) / a.chunk);  // splits that hold keys
  if (a.cluster) {
    // The blocks of KV head g form one cluster (rank = split). Each block
    // pushes its partial of head h into the shared memory of block h % ns
    // (which merges head h, as its (h / ns)-th head) with remote stores;
    // after one cluster barrier the merge reads only local shared memory,
    // and no block touches a peer's memory again.
    float* in_o = red + kDecWork;                // [kDecInbox][d]
    float* in_m = in_o + (size_t)kDecInbox * d;  // [kDecInbox]
    float* in_l = in_m + kDecInbox;              // [kDecInbox]
    cg::cluster_group cl = cg::this_cluster();
    if (kg == 0)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int h = 2 * hp + j;
        if (h < G) {
          float* dst = cl.map_shared_rank(in_o, h % ns) + (size_t)((h / ns) * ns + s) * d + dv;
          *reinterpret_cast<float4*>(dst) = acc[j];
        }
      }
    if (warp < G && lane == 0) {
      const int slot = (warp / ns) * ns + s, r = warp % ns;
      *cl.map_shared_rank(in_m + slot, r) = m_run;
      *cl.map_shared_rank(in_l + slot, r) = l_run;
    }
    cl.sync();
    trace_mark(trow, 6);  // partials pushed and visible
    // block s merges heads s, s + ns, ... (its w-th head on warp w)
    const int h = s + ns * warp;
    if (h < G) {
      LocalPartials src = {in_o + (size_t)warp * ns * d, in_m + warp * ns, in_l + warp * ns, d};
      merge_head(src, ne, d, lane, a.out + ((size_t)g * G + h) * d);
    }
    trace_mark(trow, 7);  // merged
  } else {
    const size_t pb = ((size_t)g * ns + s) * G;  // partial row of (g, s, head 0)
    if (kg == 0)
#pragma unroll
      for (int j = 0; j < 2; ++j)
        if (2 * hp + j < G)
          *reinterpret_cast<float4*>(a.part_o + (pb + 2 * hp + j) * d + dv) = acc[j];
    if (warp < G && lane == 0) {
      a.part_m[pb + warp] = m_run;
      a.part_l[pb + warp] = l_run;
    }
    if (!a.defer_merge) {
      // The last G blocks of KV head g to arrive merge one query head each
      // (h = 0 for the last), once every split's partial is written: warp w
      // folds splits [w per, (w + 1) per) (one round of loads), then warp 0
      // combines the 8 warp results in warp order. Each wait is bounded.
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        last_block = -1;
        const unsigned long long old = atomicAdd(a.arrive + g, 1ull);
        const int k = ns - 1 - (int)(old % (unsigned long long)ns);
        if (k < G) {
          const unsigned long long target = (old / (unsigned long long)ns + 1ull) * ns;
          bool ok = true;
          if (ld_acquire_u64(a.arrive + g) < target) {
            const uint64_t t0 = global_ns();
            for (uint32_t i = 1;; ++i) {
              if (ld_acquire_u64(a.arrive + g) >= target) break;
              if ((i & 63u) == 0 && global_ns() - t0 > 1000000000ull) {
                atomicOr(&a.ctl->err, kErrAttnWait);
                ok = false;
                break;
              }
            }
          }
          if (ok) last_block = k;
        }
      }
      __syncthreads();
      if (last_block >= 0) {
        __threadfence();
        const int h = last_block;
        const size_t hb = (size_t)g * ns * G + h;  // partial row of split q: hb + q * G
        constexpr int JD = D > 128 ? 2 : 1;
        const int per = (ne + kDecWarps - 1) / kDecWarps;  // <= 20 (ne <= 160)
        const int q0 = warp * per, q1 = min(ne, q0 + per);
        float* wo = red;                          // [8][D] warp outputs
        float* wm = red + kDecWarps * D;          // [8] warp maxima
        float* wl = wm + kDecWarps;               // [8] warp sums
        const int q = q0 + lane;
        const float mq = q < q1 ? __ldcg(a.part_m + hb + (size_t)q * G) : -INFINITY;
        const float lq = q < q1 ? __ldcg(a.part_l + hb + (size_t)q * G) : 0.0f;
        constexpr int kW = 20;
        float4 po[JD][kW];
#pragma unroll
        for (int u = 0; u < kW; ++u)
#pragma unroll
          for (int j = 0; j < JD; ++j) {
            const int e = 4 * lane + 128 * j;
            po[j][u] = (q0 + u < q1 && e < D)
                           ? __ldcg(reinterpret_cast<const float4*>(a.part_o + (hb + (size_t)(q0 + u) * G) * D + e))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        const float Mw = warp_max(mq);
        const float fq = mq == -INFINITY ? 0.0f : expf(mq - Mw);
        const float Lw = warp_sum(lq * fq);
        float4 Ow[JD];
#pragma unroll
        for (int j = 0; j < JD; ++j) Ow[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < kW; ++u) {
          const float fu = __shfl_sync(0xffffffffu, fq, u);
          if (q0 + u < q1)
#pragma unroll
            for (int j = 0; j < JD; ++j) {
              Ow[j].x = fmaf(po[j][u].x, fu, Ow[j].x);
              Ow[j].y = fmaf(po[j][u].y, fu, Ow[j].y);
              Ow[j].z = fmaf(po[j][u].z, fu, Ow[j].z);
              Ow[j].w = fmaf(po[j][u].w, fu, Ow[j].w);
            }
        }
#pragma unroll
        for (int j = 0; j < JD; ++j) {
          const int e = 4 * lane + 128 * j;
          if (e < D) *reinterpret_cast<float4*>(wo + warp * D + e) = Ow[j];
        }
        if (lane == 0) {
          wm[warp] = Mw;
          wl[warp] = Lw;
        }
        __syncthreads();
        if (warp == 0) {
          float M = -INFINITY;
#pragma unroll
          for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, wm[w]);
          float L = 0.0f;
          float4 O[JD];
#pragma unroll
          for (int j = 0; j < JD; ++j) O[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int w = 0; w < kDecWarps; ++w) {
            const float f = wm[w] == -INFINITY ? 0.0f : expf(wm[w] - M);
            L = fmaf(wl[w], f, L);
#pragma unroll
            for (int j = 0; j < JD; ++j) {
              const int e = 4 * lane + 128 * j;
              if (e < D) {
                const float4 o = *reinterpret_cast<const float4*>(wo + w * D + e);
                O[j].x = fmaf(o.x, f, O[j].x);
                O[j].y = fmaf(o.y, f, O[j].y);
                O[j].z = fmaf(o.z, f, O[j].z);
                O[j].w = fmaf(o.w, f, O[j].w);
              }
            }
          }
          float* outp = a.out + ((size_t)g * G + h) * D;
#pragma unroll
          for (int j = 0; j < JD; ++j) {
            const int e = 4 * lane + 128 * j;
            if (e < D)
              *reinterpret_cast<float4*>(outp + e) =
                  make_float4(__fdiv_rn(O[j].x, L), __fdiv_rn(O[j].y, L), __fdiv_rn(O[j].z, L),
                              __fdiv_rn(O[j].w, L));
          }
        }
      }
    }
  }
  if (a.tr.buf) {  // block-uniform
    __syncthreads();
    trace_end(trow);
  }
}

// ------------------------------------------------------------------ small kernels
// Ranks hold contiguous vocab slices in rank order, so the first maximum over
// their candidates (strict >, then the lower index) is the global one.
__global__ void k_tp_pick(const float* cands, int n, unsigned* seq, StepCtl* ctl,
                          uint32_t* rec_fed, uint32_t* rec_argmax) {
  pdl_wait();
  pdl_launch();
  if (threadIdx.x != 0) return;
  const unsigned e = seq ? __ldcg(seq) + 1u : 0u;
  float v = -INFINITY;
  uint32_t i = 0xffffffffu;
  for (int r = 0; r < n; ++r) {
    float cv, ciw;
    if (seq) {  // pushed words (value, epoch), (index bits, epoch)
      if (!tp_wait_word(cands + 4 * r, e, &ctl->err, &cv) ||
          !tp_wait_word(cands + 4 * r + 2, e, &ctl->err, &ciw))
        return;  // error bit set; the step is not advanced
    } else {
      cv = cands[2 * r];
      ciw = cands[2 * r + 1];
    }
    const uint32_t ci = __float_as_uint(ciw);
    if (better(cv, ci, v, i)) {
      v = cv;
      i = ci;
    }
  }
  if (seq) *seq = e;
  const uint32_t s = ctl->step;
  if (rec_fed) rec_fed[s] = ctl->fed;
  if (rec_argmax) rec_argmax[s] = ctl->argmax;
  ctl->argmax = i == 0xffffffffu ? 0u : i;
  ctl->pos = ctl->pos + 1;
  ctl->step = s + 1;
}

cudaError_t launch_tp_pick(const float* cands, int n, unsigned* seq, StepCtl* ctl,
                           uint32_t* rec_fed, uint32_t* rec_argmax, cudaStream_t st) {
  k_tp_pick<<<1, 32, 0, st>>>(cands, n, seq, ctl, rec_fed, rec_argmax);
  return counted(cudaGetLastError());
}

constexpr int kReduceThreads = 256;

// One element per thread over ceil(H / 256) blocks: every rank's word for it
// is loaded at once (one round trip), then only words not yet current are
// polled. The last block to finish advances the epoch.
__global__ void __launch_bounds__(kReduceThreads) k_tp_reduce(TpReduceArgs r) {
  pdl_launch();  // the next projection may start streaming its weights
  pdl_wait();
  const unsigned e = __ldcg(r.seq) + 1u;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < r.H) {
    unsigned long long w[kMaxTp];
#pragma unroll
    for (int p = 0; p < kMaxTp; ++p)
      if (p < r.n) w[p] = tp_load(r.inbox + 2 * ((size_t)p * r.H + i));
    bool ok = true;
    float s = 0.0f;
#pragma unroll
    for (int p = 0; p < kMaxTp; ++p) {
      if (p >= r.n || !ok) continue;
      float t = __uint_as_float((unsigned)w[p]);
      if ((unsigned)(w[p] >> 32) != e)
        ok = tp_wait_word(r.inbox + 2 * ((size_t)p * r.H + i), e, r.err, &t, r.wait_ns);
      s = p == 0 ? t : __fadd_rn(s, t);
    }
    if (ok) r.out[i] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(r.done, 1u) == gridDim.x - 1) {
      *r.done = 0u;
      if (!(*(volatile uint32_t*)r.err & kErrTpWait)) *r.seq = e;
    }
  }
}

cudaError_t launch_tp_reduce(const TpReduceArgs& r, cudaStream_t st, bool pdl) {
  if (r.n < 1 || r.n > kMaxTp) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((r.H + kReduceThreads - 1) / kReduceThreads);
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return counted(cudaLaunchKernelEx(&cfg, k_tp_reduce, r));
}

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
// MYOS_GEMV_KIND=legacy selects the row-at-a-time GEMV (every width) instead
// of the streaming one for A/B timing.
static int gemv_kind() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("MYOS_GEMV_KIND");
    v = (e && e[0] == 'l') ? 2 : 1;
  }
  return v;
}
static bool getenv_legacy() { return gemv_kind() == 2; }

// MYOS_ATTN=tiled selects the general attention kernel for decode too.
static bool attn_compact() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("MYOS_ATTN");
    v = !(e && e[0] == 't');
  }
  return v != 0;
}

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

// Batch width U for the streaming GEMV: the largest U <= 8 that divides the
// per-lane chunk count P (so no batch is partly empty), else 8. Two weight
// matrices (SwiGLU) halve the budget so both buffers fit in registers.
// Chunks per batch: as deep as the register budget allows (each warp keeps
// two batches in flight, so depth sets its share of DRAM bandwidth), then
// the smallest size giving that many batches a row (fewest idle slots in a
// row's last batch).
static int env_int(const char* name, int def);
static int pick_batch(int P, int NR) {
  // NR = 2 keeps both matrices' batches in registers: up to 6 chunks fit
  // without spilling (-Xptxas -v); 6 measured 10.8 us for the 1.5B gate/up
  // against 11.95 us at 4 (MYOS_GEMV_UMAX2 overrides)
  int umax = NR > 1 ? env_int("MYOS_GEMV_UMAX2", 6) : 8;
  if (umax < 3) umax = 3;
  if (umax > (NR > 1 ? 6 : 8)) umax = NR > 1 ? 6 : 8;
  if (P <= umax) return P < 3 ? 3 : P;
  const int nbr = (P + umax - 1) / umax;
  int u = (P + nbr - 1) / nbr;
  return u < 3 ? 3 : u;
}

template <int EPI, int NR>
static cudaError_t launch_stream(const GemvArgs& a, int U, cudaLaunchConfig_t& cfg) {
  switch (U) {
    case 3: return counted(cudaLaunchKernelEx(&cfg, k_gemv_stream<EPI, NR, 3>, a));
    case 4: return counted(cudaLaunchKernelEx(&cfg, k_gemv_stream<EPI, NR, 4>, a));
    case 5: return counted(cudaLaunchKernelEx(&cfg, k_gemv_stream<EPI, NR, 5>, a));
    case 6: return counted(cudaLaunchKernelEx(&cfg, k_gemv_stream<EPI, NR, 6>, a));
    case 7: return counted(cudaLaunchKernelEx(&cfg, k_gemv_stream<EPI, NR, 7>, a));
    default: return counted(cudaLaunchKernelEx(&cfg, k_gemv_stream<EPI, NR, 8>, a));
  }
}

static int env_int(const char* name, int def) {
  const char* e = getenv(name);
  return e && *e ? atoi(e) : def;
}

int gemv_grid(int M, int K, int NR, int num_sms) {
  // Up to two blocks per SM, at least MYOS_GEMV_MIN_ROWS (8) rows a block.
  // MYOS_GEMV_BALANCE=1: past one block per SM, exactly two per SM with the
  // rows spread over fewer warps (gemv_warps). Measured slower for the 1.5B
  // step (every extra block stages the whole input vector again: down_proj
  // 8.7 -> 9.0 us), so off by default.
  const int min_rows = env_int("MYOS_GEMV_MIN_ROWS", 8);
  int g = (M + min_rows - 1) / min_rows;
  if (g > num_sms && env_int("MYOS_GEMV_BALANCE", 0)) g = 2 * num_sms;
  if (g > 2 * num_sms) g = 2 * num_sms;
  return g < 1 ? 1 : g;
}

int gemv_warps(int M, int K, int NR, bool has_gamma, int grid) {
  const int full = kThreads / 32;
  if (!env_int("MYOS_GEMV_BALANCE", 0) || grid < 1) return full;
  const int rows = (M + grid - 1) / grid;           // most rows a block holds
  const int per_warp = (rows + full - 1) / full;    // rows a warp takes at full width
  int nw = (rows + per_warp - 1) / per_warp;        // fewest warps with that many each
  const int nchunk = K >> 3, per = has_gamma ? kGammaRegs : kStageOne;
  const int nw_min = (nchunk + per * 32 - 1) / (per * 32);  // one-trip staging
  if (nw_min > full) return full;  // staged in several trips: all threads help
  if (nw < nw_min) nw = nw_min;
  (void)NR;
  return nw < 1 ? 1 : (nw > full ? full : nw);
}

cudaError_t launch_gemv(int epi, const GemvArgs& a0, int grid, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  if (a0.push.n &&  // the peer push lives in the streaming kernel only
      ((a0.K % 256) != 0 || ((uintptr_t)a0.w & 15) != 0 || getenv_legacy() || a0.in.part_o ||
       a0.push.n > kMaxTp))
    return cudaErrorNotSupported;
  const GemvArgs& a = a0;
  size_t smem = gemv_smem_bytes(a.K);
  if (a.in.part_o) smem += merge_smem_bytes(a.K / a.in.m_d, a.in.m_nsplit, a.in.m_d);
  cudaLaunchConfig_t cfg = make_cfg(dim3(grid), dim3(kThreads), smem, st, pdl, attr);
  const bool stream = (a.K % 256) == 0 && ((uintptr_t)a.w & 15) == 0 &&
                      (epi != EPI_SWIGLU || ((uintptr_t)a.w2 & 15) == 0) && !getenv_legacy();
  if (stream) {
    if (a.warps > 0 && a.warps < kThreads / 32) cfg.blockDim = dim3(32 * a.warps);
    const int P = a.K / 256;
    switch (epi) {
      case EPI_STORE: return launch_stream<EPI_STORE, 1>(a, pick_batch(P, 1), cfg);
      case EPI_BIAS: return launch_stream<EPI_BIAS, 1>(a, pick_batch(P, 1), cfg);
      case EPI_RESID: return launch_stream<EPI_RESID, 1>(a, pick_batch(P, 1), cfg);
      case EPI_SWIGLU: return launch_stream<EPI_SWIGLU, 2>(a, pick_batch(P, 2), cfg);
      case EPI_ARGMAX: return launch_stream<EPI_ARGMAX, 1>(a, pick_batch(P, 1), cfg);
    }
    return cudaErrorInvalidValue;
  }
  switch (epi) {
    case EPI_STORE: return counted(cudaLaunchKernelEx(&cfg, k_gemv<EPI_STORE>, a));
    case EPI_BIAS: return counted(cudaLaunchKernelEx(&cfg, k_gemv<EPI_BIAS>, a));
    case EPI_RESID: return counted(cudaLaunchKernelEx(&cfg, k_gemv<EPI_RESID>, a));
    case EPI_SWIGLU: return counted(cudaLaunchKernelEx(&cfg, k_gemv<EPI_SWIGLU>, a));
    case EPI_ARGMAX: return counted(cudaLaunchKernelEx(&cfg, k_gemv<EPI_ARGMAX>, a));
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_mlp(const MlpArgs& a, int grid, cudaStream_t st, bool pdl) {
  if (grid <= 0 || grid * kMlpSlice != a.I || a.H % 256 != 0 || !a.arrive || !a.err)
    return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg =
      make_cfg(dim3(grid), dim3(kMlpThreads), gemv_smem_bytes(a.H), st, pdl, attr);
  switch (a.H / 256) {
    case 4: return counted(cudaLaunchKernelEx(&cfg, k_mlp<4>, a));
    case 5: return counted(cudaLaunchKernelEx(&cfg, k_mlp<5>, a));
    case 6: return counted(cudaLaunchKernelEx(&cfg, k_mlp<6>, a));
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_mlp_relayout(const uint16_t* wd, uint16_t* dst, int H, int I, cudaStream_t st) {
  if (I % kMlpSlice != 0 || ((uintptr_t)wd & 15) || ((uintptr_t)dst & 15)) return cudaErrorInvalidValue;
  k_mlp_relayout<<<1184, 256, 0, st>>>(reinterpret_cast<const uint4*>(wd), reinterpret_cast<uint4*>(dst), H, I);
  return counted(cudaGetLastError());
}

int attn_dpl(int d) { return d <= 32 ? 1 : d <= 64 ? 2 : d <= 128 ? 4 : 8; }

size_t attn_smem_bytes(int G, int d) {
  // qs, two padded tiles, probabilities, corrections, new K/V row, raw q,
  // rotation row, raw new K/V
  return (size_t)(2 * G * d + 2 * kTile * (d + 4) + G * kTile + kMaxG + 5 * d) * sizeof(float);
}

size_t merge_smem_bytes(int Hq, int nsplit, int d) {
  // partials [Hq*nsplit*d], factors and sums [2*Hq*nsplit], per-head totals [Hq]
  return ((size_t)Hq * nsplit * d + 2 * (size_t)Hq * nsplit + Hq) * sizeof(float);
}

template <int DPL>
static cudaError_t launch_attn_dpl(const AttnArgs& a, int kv_bf16, cudaLaunchConfig_t& cfg) {
  if (kv_bf16) return counted(cudaLaunchKernelEx(&cfg, k_attn<DPL, __nv_bfloat16>, a));
  return counted(cudaLaunchKernelEx(&cfg, k_attn<DPL, float>, a));
}

cudaError_t launch_attention(const AttnArgs& a, int kv_bf16, cudaStream_t st, bool pdl) {
  if (a.G > kMaxG || a.d > 256 || a.d <= 0) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  if (a.decode && (a.d == 64 || a.d == 128 || a.d == 256) && attn_compact()) {
    if (a.cluster && (a.nsplit > 8 || a.defer_merge)) return cudaErrorInvalidValue;
    cudaLaunchAttribute attrs[2];
    cudaLaunchConfig_t cfg = make_cfg(dim3(a.nsplit, a.Hkv), dim3(kThreads),
                                      attn_dec_smem_bytes(a.G, a.d), st, pdl, attrs);
    if (a.cluster) {
      attrs[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
      attrs[cfg.numAttrs].val.clusterDim.x = a.nsplit;
      attrs[cfg.numAttrs].val.clusterDim.y = 1;
      attrs[cfg.numAttrs].val.clusterDim.z = 1;
      ++cfg.numAttrs;
    }
#define MYOS_ATTN_LAUNCH(KT, D) return counted(cudaLaunchKernelEx(&cfg, k_attn_dec<KT, D>, a))
    switch (a.d) {
      case 64:
        if (kv_bf16) MYOS_ATTN_LAUNCH(__nv_bfloat16, 64);
        MYOS_ATTN_LAUNCH(float, 64);
      case 128:
        if (kv_bf16) MYOS_ATTN_LAUNCH(__nv_bfloat16, 128);
        MYOS_ATTN_LAUNCH(float, 128);
      case 256:
        if (kv_bf16) MYOS_ATTN_LAUNCH(__nv_bfloat16, 256);
        MYOS_ATTN_LAUNCH(float, 256);
    }
#undef MYOS_ATTN_LAUNCH
    return cudaErrorInvalidValue;
  }
  // The split merge reuses the tile buffers for (2 nsplit + 1) * G floats.
  size_t smem = attn_smem_bytes(a.G, a.d);
  const size_t merge = (size_t)(2 * a.nsplit + 1) * a.G * sizeof(float);
  if (merge > smem) smem = merge;
  cudaLaunchConfig_t cfg = make_cfg(dim3(a.nsplit, a.Hkv), dim3(kThreads), smem, st, pdl, attr);
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
  return counted(cudaLaunchKernelEx(&cfg, k_step_end, ctl));
}

cudaError_t launch_argmax(const float* v, int n, float* part_val, uint32_t* part_idx,
                          unsigned* counter, uint32_t* out, int grid, cudaStream_t st) {
  k_argmax<<<grid, kThreads, 0, st>>>(v, n, part_val, part_idx, counter, out);
  return counted(cudaGetLastError());
}

cudaError_t launch_swiglu_mul(float* h, const float* gate, const float* up, int n,
                              cudaStream_t st) {
  int grid = (n + kThreads - 1) / kThreads;
  if (grid > 1184) grid = 1184;
  if (grid < 1) grid = 1;
  k_swiglu_mul<<<grid, kThreads, 0, st>>>(h, gate, up, n);
  return counted(cudaGetLastError());
}

cudaError_t launch_rope(float* y, const float* x, int len, int head_dim, const float* cos_row,
                        const float* sin_row, cudaStream_t st) {
  int grid = (len + kThreads - 1) / kThreads;
  if (grid < 1) grid = 1;
  k_rope<<<grid, kThreads, 0, st>>>(y, x, len, head_dim, cos_row, sin_row);
  return counted(cudaGetLastError());
}

cudaError_t launch_rmsnorm(float* y, const float* x, const float* gamma, int n, float eps,
                           cudaStream_t st) {
  k_rmsnorm<<<1, kThreads, 0, st>>>(y, x, gamma, n, eps);
  return counted(cudaGetLastError());
}

static std::atomic<uint64_t> g_launches{0};

cudaError_t counted(cudaError_t e, uint64_t n) {
  if (e == cudaSuccess) g_launches.fetch_add(n, std::memory_order_relaxed);
  return e;
}
void launches_uncount(uint64_t n) { g_launches.fetch_sub(n, std::memory_order_relaxed); }
uint64_t launches_total() { return g_launches.load(std::memory_order_relaxed); }

static std::mutex g_init_mu;
static unsigned long long g_init_mask = 0;  // devices whose limits are raised (under g_init_mu)

static cudaError_t raise_limits();

cudaError_t kernels_init() {
  // Dynamic shared-memory limits are per device: raise them once for each,
  // and count a device done only after every attribute call succeeded. The
  // lock keeps a second host thread from launching a large-smem kernel
  // before the first has raised the limit.
  int dev = 0;
  cudaError_t status = cudaGetDevice(&dev);
  if (status != cudaSuccess) return status;
  std::lock_guard<std::mutex> lock(g_init_mu);
  if (dev < 64 && (g_init_mask >> dev) & 1ull) return cudaSuccess;
  status = raise_limits();
  if (status == cudaSuccess && dev < 64) g_init_mask |= 1ull << dev;
  return status;
}

static cudaError_t raise_limits() {
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
#define MYOS_SET_STREAM(EPI, NR)                 \
  MYOS_SET((k_gemv_stream<EPI, NR, 3>), gemv_max) \
  MYOS_SET((k_gemv_stream<EPI, NR, 4>), gemv_max) \
  MYOS_SET((k_gemv_stream<EPI, NR, 5>), gemv_max) \
  MYOS_SET((k_gemv_stream<EPI, NR, 6>), gemv_max) \
  MYOS_SET((k_gemv_stream<EPI, NR, 7>), gemv_max) \
  MYOS_SET((k_gemv_stream<EPI, NR, 8>), gemv_max)
  MYOS_SET_STREAM(EPI_STORE, 1)
  MYOS_SET_STREAM(EPI_BIAS, 1)
  MYOS_SET_STREAM(EPI_RESID, 1)
  MYOS_SET_STREAM(EPI_SWIGLU, 2)
  MYOS_SET_STREAM(EPI_ARGMAX, 1)
#undef MYOS_SET_STREAM
  MYOS_SET((k_attn_dec<float, 64>), attn_max)
  MYOS_SET((k_attn_dec<__nv_bfloat16, 64>), attn_max)
  MYOS_SET((k_attn_dec<float, 128>), attn_max)
  MYOS_SET((k_attn_dec<__nv_bfloat16, 128>), attn_max)
  MYOS_SET((k_attn_dec<float, 256>), attn_max)
  MYOS_SET((k_attn_dec<__nv_bfloat16, 256>), attn_max)
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
