// One token step of the Qwen2.5 block stack as a single persistent kernel.
//
// Why: every phase of a decode step (QKV, attention, o_proj, gate/up, down,
// head) depends on the whole output of the previous one, and as separate
// launches each boundary costs several microseconds of drain / launch /
// re-staging while HBM sits idle. Here one block per SM runs the whole step:
//
//   * a producer warp walks a static schedule of every weight stage this
//     block will consume in the step (all layers, all phases, then the head)
//     and streams them with 1-D bulk copies (the TMA engine) into an
//     nslot-deep shared-memory ring, gated only by free slots. Weights never
//     depend on activations, so HBM keeps streaming through phase boundaries;
//   * eight consumer warps run the phases in order. Between phases they wait
//     on a device-wide arrival counter (one per phase, zeroed before each
//     launch) instead of a kernel boundary;
//   * every wait (ring slots, phase counters) is bounded in polls and time;
//     a wait that gives up raises a bit in ctl->err, which makes every later
//     wait of every block return at once, so the launch always ends and the
//     host reports MYOS_ERR_TIMEOUT.
// The launch is cooperative (one block per SM, all resident), so the phase
// counters never wait on a block that cannot run.
//
// Arithmetic is the same as the multi-kernel path (kernels.cu): RMSNorm
// fused into input staging, f32 accumulation of bf16 weights, fixed-order
// reductions, epilogues for bias / residual / SiLU*up / argmax.
#include <math.h>

#include "common.cuh"
#include "step_kernel.h"

namespace myos {

namespace {

constexpr int kCW = 8;                  // consumer warps
constexpr int kCT = kCW * 32;           // consumer threads
constexpr int kStepThreads = kCT + 32;  // + producer warp
constexpr int kTile = 32;               // attention key tile
constexpr int kMaxG = 8;

enum Phase { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_HEAD = 5 };

struct PhaseW {
  const uint16_t* w0;
  const uint16_t* w1;
  int M, K, NR, rs;
};

MYOS_DEV int rows_per_stage(int K, int NR, int slot_bytes) {
  int r = 8;
  while (r > 1 && NR * r * K * 2 > slot_bytes) r >>= 1;
  return r;
}

// Weight matrix of phase p (layer l), or M = 0 for attention.
MYOS_DEV PhaseW phase_w(const MegaArgs& a, int kind, int l) {
  PhaseW w = {nullptr, nullptr, 0, 0, 1, 1};
  if (kind == PH_HEAD) {
    w.w0 = a.head_w;
    w.M = a.V;
    w.K = a.H;
  } else if (kind != PH_ATTN) {
    const MegaLayer& L = a.layers[l];
    if (kind == PH_QKV) {
      w.w0 = L.wqkv;
      w.M = a.qd + 2 * a.kvd;
      w.K = a.H;
    } else if (kind == PH_O) {
      w.w0 = L.wo;
      w.M = a.H;
      w.K = a.qd;
    } else if (kind == PH_GU) {
      w.w0 = L.wg;
      w.w1 = L.wu;
      w.M = a.I;
      w.K = a.H;
      w.NR = 2;
    } else {
      w.w0 = L.wd;
      w.M = a.H;
      w.K = a.I;
    }
  }
  if (w.M) w.rs = rows_per_stage(w.K, w.NR, a.slot_bytes);
  return w;
}

MYOS_DEV void block_rows(int M, int* r0, int* r1) {
  *r0 = (int)((long long)blockIdx.x * M / gridDim.x);
  *r1 = (int)((long long)(blockIdx.x + 1) * M / gridDim.x);
}

// ---------------------------------------------------------------- sync
MYOS_DEV uint32_t ld_acquire(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

MYOS_DEV uint32_t ld_volatile(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// Bounded ring wait that also gives up at once when another block failed.
MYOS_DEV void ring_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 255u) == 0) {
      if (ld_volatile(err)) return;
      if (global_ns() - t0 > 1000000000ull) break;
    }
  }
  atomicOr(err, code);
}

// Phase arrival: every consumer thread fences its writes, then one thread
// counts the block in.
MYOS_DEV uint32_t phase_arrive(unsigned* cnt) {
  __threadfence();
  named_sync(1, kCT);
  uint32_t prev = 0;
  if (threadIdx.x == 0) prev = atomicAdd(cnt, 1u);
  return prev;
}

MYOS_DEV void phase_wait(const unsigned* cnt, uint32_t target, uint32_t* err) {
  if (threadIdx.x == 0) {
    if (ld_acquire(cnt) < target) {
      const uint64_t t0 = global_ns();
      for (uint32_t i = 0;; ++i) {
        if (ld_acquire(cnt) >= target) break;
        if ((i & 63u) == 0) {
          if (ld_volatile(err)) break;
          if (i > kWaitLimit || global_ns() - t0 > 1000000000ull) {
            atomicOr(err, kErrPhase);
            break;
          }
        }
      }
    }
  }
  named_sync(1, kCT);
}

MYOS_DEV float csum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  named_sync(2, kCT);
  if (warp == 0) {
    float s = lane < kCW ? red[lane] : 0.0f;
    s = warp_sum(s);
    if (lane == 0) red[32] = s;
  }
  named_sync(2, kCT);
  const float s = red[32];
  named_sync(2, kCT);
  return s;
}

// ---------------------------------------------------------------- staging
// x (f32 activations, or a bf16 embedding row) into the split layout, with
// the optional RMSNorm gamma * (x * inv) of crates/tensor_core/src/bf16.rs:231-270.
__device__ __noinline__ void stage_c(float* xs, int K, const float* xf, const uint16_t* xb,
                                     const float* gamma,
                      float eps, float* x_store, float* red) {
  const int nchunk = K >> 3, half = K >> 1;
  float4* xlo = reinterpret_cast<float4*>(xs);
  float4* xhi = reinterpret_cast<float4*>(xs + half);
  constexpr int B = 4;
  for (int c0 = threadIdx.x; c0 < nchunk; c0 += kCT * B) {
    float4 lo[B], hi[B];
#pragma unroll
    for (int i = 0; i < B; ++i) {
      const int c = c0 + i * kCT;
      if (c < nchunk) {
        if (xb) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(xb) + c);
          lo[i] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
          hi[i] = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
        } else {
          lo[i] = __ldcg(reinterpret_cast<const float4*>(xf) + 2 * c);
          hi[i] = __ldcg(reinterpret_cast<const float4*>(xf) + 2 * c + 1);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < B; ++i) {
      const int c = c0 + i * kCT;
      if (c < nchunk) {
        xlo[c] = lo[i];
        xhi[c] = hi[i];
        if (x_store) {
          __stcg(reinterpret_cast<float4*>(x_store) + 2 * c, lo[i]);
          __stcg(reinterpret_cast<float4*>(x_store) + 2 * c + 1, hi[i]);
        }
      }
    }
  }
  named_sync(2, kCT);
  if (!gamma) return;
  float ss = 0.0f;
  for (int j = threadIdx.x; j < K; j += kCT) ss = fmaf(xs[j], xs[j], ss);
  ss = csum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
  for (int c = threadIdx.x; c < nchunk; c += kCT) {
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c);
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c + 1);
    float4 p = xlo[c], q = xhi[c];
    p = make_float4(__fmul_rn(g0.x, __fmul_rn(p.x, inv)), __fmul_rn(g0.y, __fmul_rn(p.y, inv)),
                    __fmul_rn(g0.z, __fmul_rn(p.z, inv)), __fmul_rn(g0.w, __fmul_rn(p.w, inv)));
    q = make_float4(__fmul_rn(g1.x, __fmul_rn(q.x, inv)), __fmul_rn(g1.y, __fmul_rn(q.y, inv)),
                    __fmul_rn(g1.z, __fmul_rn(q.z, inv)), __fmul_rn(g1.w, __fmul_rn(q.w, inv)));
    xlo[c] = p;
    xhi[c] = q;
  }
  named_sync(2, kCT);
}

MYOS_DEV float dot8s(const uint4& u, const float4& lo, const float4& hi, float acc) {
  return dot8(u, lo, hi, acc);
}

MYOS_DEV bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > -INFINITY && (v > bv || (v == bv && i < bi));
}

MYOS_DEV float silu_mul(float g, float u) {
  const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

// ---------------------------------------------------------------- attention
template <typename KT>
MYOS_DEV float4 kvl4(const KT* p);
template <>
MYOS_DEV float4 kvl4<float>(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}
template <>
MYOS_DEV float4 kvl4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p));
  return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
}
template <typename KT>
MYOS_DEV KT kv_round(float v);
template <>
MYOS_DEV float kv_round<float>(float v) {
  return v;
}
template <>
MYOS_DEV __nv_bfloat16 kv_round<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

MYOS_DEV float rope1(const float* x, int e, int d, const float* cs, const float* sn) {
  const int half = d >> 1;
  const int p = e < half ? e : e - half;
  const float x0 = x[p], x1 = x[p + half];
  return e < half ? __fsub_rn(__fmul_rn(x0, cs[p]), __fmul_rn(x1, sn[p]))
                  : __fadd_rn(__fmul_rn(x1, cs[p]), __fmul_rn(x0, sn[p]));
}

// Attention task (KV head g, key split s) for the decode position pos, by
// the 256 consumer threads, in the shared scratch sm. Same math as k_attn.
template <typename KT>
__device__ __noinline__ void attention_task(const MegaArgs& a, int layer, int g, int s, int pos,
                                            float* sm, int* flag) {
  const int d = a.d, G = a.G, half = d >> 1, ds = d + 4;
  float* qs = sm;
  float* ks = qs + G * d;
  float* vs = ks + kTile * ds;
  float* ps = vs + kTile * ds;
  float* corr = ps + G * kTile;
  float* knew = corr + kMaxG;
  float* vnew = knew + d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t kv_elt = sizeof(KT);
  KT* kc = reinterpret_cast<KT*>(reinterpret_cast<uint8_t*>(a.kcache) +
                                 (size_t)layer * a.kv_layer_elems * kv_elt) + (size_t)g * a.S * d;
  KT* vc = reinterpret_cast<KT*>(reinterpret_cast<uint8_t*>(a.vcache) +
                                 (size_t)layer * a.kv_layer_elems * kv_elt) + (size_t)g * a.S * d;
  const int nkeys = pos + 1;
  const int kb = s * a.chunk, ke = min(kb + a.chunk, nkeys);
  const bool has_new = pos >= kb && pos < ke;
  const float* cs = a.cos_t + (size_t)pos * half;
  const float* sn = a.sin_t + (size_t)pos * half;
  {
    float* qraw = ks;
    float* cst = vs;
    float* snt = vs + half;
    float* kraw = vs + d;
    float* vraw = vs + 2 * d;
    const int nq = G * d;
    const int ntot = nq + d + (has_new ? 2 * d : 0);
    const float* qsrc = a.qkv + (size_t)g * G * d;
    const float* ksrc = a.qkv + (size_t)a.Hq * d + (size_t)g * d;
    const float* vsrc = a.qkv + (size_t)(a.Hq + a.Hkv) * d + (size_t)g * d;
    constexpr int kJ = 12;
    float val[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int v = threadIdx.x + kCT * j;
      if (v < ntot) {
        if (v < nq) val[j] = __ldcg(qsrc + v);
        else if (v < nq + half) val[j] = __ldg(cs + (v - nq));
        else if (v < nq + d) val[j] = __ldg(sn + (v - nq - half));
        else if (v < nq + 2 * d) val[j] = __ldcg(ksrc + (v - nq - d));
        else val[j] = __ldcg(vsrc + (v - nq - 2 * d));
      }
    }
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int v = threadIdx.x + kCT * j;
      if (v < ntot) {
        if (v < nq) qraw[v] = val[j];
        else if (v < nq + half) cst[v - nq] = val[j];
        else if (v < nq + d) snt[v - nq - half] = val[j];
        else if (v < nq + 2 * d) kraw[v - nq - d] = val[j];
        else vraw[v - nq - 2 * d] = val[j];
      }
    }
    named_sync(2, kCT);
    for (int i = threadIdx.x; i < nq; i += kCT) {
      const int hh = i / d, e = i - hh * d;
      qs[i] = rope1(qraw + hh * d, e, d, cst, snt);
    }
    if (has_new) {
      for (int e = threadIdx.x; e < d; e += kCT) {
        const KT kq = kv_round<KT>(rope1(kraw, e, d, cst, snt));
        const KT vq = kv_round<KT>(vraw[e]);
        knew[e] = (float)kq;
        vnew[e] = (float)vq;
        kc[(size_t)pos * d + e] = kq;  // KvCache::store for this position
        vc[(size_t)pos * d + e] = vq;
      }
    }
  }
  constexpr int kMaxOut = kMaxG * 256 / kCT;
  float acc[kMaxOut];
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) acc[i] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  for (int t0 = kb; t0 < ke; t0 += kTile) {
    const int nk = min(kTile, ke - t0);
    named_sync(2, kCT);
    const int qpr = d >> 2, nqd = nk * qpr;
    constexpr int kQ = kTile * 64 / kCT;
    float4 kq[kQ], vq[kQ];
#pragma unroll
    for (int j = 0; j < kQ; ++j) {
      const int i = threadIdx.x + kCT * j;
      if (i < nqd) {
        const int tt = i / qpr, e = (i - tt * qpr) * 4;
        const int t = t0 + tt;
        if (!(has_new && t == pos)) {
          kq[j] = kvl4<KT>(kc + (size_t)t * d + e);
          vq[j] = kvl4<KT>(vc + (size_t)t * d + e);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kQ; ++j) {
      const int i = threadIdx.x + kCT * j;
      if (i < nqd) {
        const int tt = i / qpr, e = (i - tt * qpr) * 4;
        if (has_new && t0 + tt == pos) {
          kq[j] = make_float4(knew[e], knew[e + 1], knew[e + 2], knew[e + 3]);
          vq[j] = make_float4(vnew[e], vnew[e + 1], vnew[e + 2], vnew[e + 3]);
        }
        *reinterpret_cast<float4*>(ks + tt * ds + e) = kq[j];
        *reinterpret_cast<float4*>(vs + tt * ds + e) = vq[j];
      }
    }
    named_sync(2, kCT);
    for (int i = threadIdx.x; i < G * kTile; i += kCT) {
      const int hh = i / kTile, tt = i - hh * kTile;
      float sc = -INFINITY;
      if (tt < nk) {
        const float* qh = qs + hh * d;
        const float* kr = ks + tt * ds;
        float dot = 0.0f;
        for (int e = 0; e < d; e += 4) {
          const float4 qv = *reinterpret_cast<const float4*>(qh + e);
          const float4 kv = *reinterpret_cast<const float4*>(kr + e);
          dot = fmaf(qv.x, kv.x, dot);
          dot = fmaf(qv.y, kv.y, dot);
          dot = fmaf(qv.z, kv.z, dot);
          dot = fmaf(qv.w, kv.w, dot);
        }
        sc = __fmul_rn(dot, a.scale);
      }
      ps[hh * kTile + tt] = sc;
    }
    named_sync(2, kCT);
    if (warp < G) {
      const float sc = ps[warp * kTile + lane];
      const float mt = warp_max(sc);
      const float mn = fmaxf(m_run, mt);
      const float cf = expf(m_run - mn);
      const float p = lane < nk ? expf(sc - mn) : 0.0f;
      l_run = fmaf(l_run, cf, warp_sum(p));
      m_run = mn;
      ps[warp * kTile + lane] = p;
      if (lane == 0) corr[warp] = cf;
    }
    named_sync(2, kCT);
#pragma unroll
    for (int i = 0; i < kMaxOut; ++i) {
      const int o = threadIdx.x + kCT * i;
      if (o < G * d) {
        const int hh = o / d, e = o - hh * d;
        const float* ph = ps + hh * kTile;
        float v = acc[i] * corr[hh];
        for (int tt = 0; tt < nk; ++tt) v = fmaf(ph[tt], vs[tt * ds + e], v);
        acc[i] = v;
      }
    }
  }
  const size_t pbase = ((size_t)g * a.nsplit + s) * G;
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) {
    const int o = threadIdx.x + kCT * i;
    if (o < G * d) __stcg(a.part_o + pbase * d + o, acc[i]);
  }
  if (warp < G && lane == 0) {
    __stcg(a.part_m + pbase + warp, m_run);
    __stcg(a.part_l + pbase + warp, l_run);
  }
  __threadfence();
  named_sync(2, kCT);
  if (threadIdx.x == 0) *flag = atomicAdd(a.attn_cnt + g, 1u) == (unsigned)(a.nsplit - 1);
  named_sync(2, kCT);
  if (!*flag) return;
  __threadfence();
  float* fs = sm;
  float* ls = sm + a.nsplit * G;
  float* Ls = ls + a.nsplit * G;
  const size_t gbase = (size_t)g * a.nsplit * G;
  for (int i = threadIdx.x; i < a.nsplit * G; i += kCT) {
    fs[i] = __ldcg(a.part_m + gbase + i);
    ls[i] = __ldcg(a.part_l + gbase + i);
  }
  named_sync(2, kCT);
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
  named_sync(2, kCT);
  for (int o = threadIdx.x; o < G * d; o += kCT) {
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
    __stcg(a.attn + (size_t)g * G * d + o, __fdiv_rn(O, Ls[hh]));
  }
  if (threadIdx.x == 0) a.attn_cnt[g] = 0u;
  named_sync(2, kCT);
}

// ---------------------------------------------------------------- the kernel
template <typename KT>
__global__ void __launch_bounds__(kStepThreads, 1) k_step(MegaArgs a) {
  extern __shared__ float4 smem4[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(smem4);
  __shared__ float red[33];
  __shared__ float wbv[kCW];
  __shared__ uint32_t wbi[kCW];
  __shared__ int flag;

  float* scratch = reinterpret_cast<float*>(smem);  // staged x, or attention scratch
  uint8_t* ring = smem + a.scratch_bytes;
  float* part = reinterpret_cast<float*>(ring + (size_t)a.nslot * a.slot_bytes);  // [2][2][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(part + 2 * 2 * kCW);
  uint64_t* empty = full + a.nslot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nslot = a.nslot;
  uint32_t* err = &a.ctl->err;

  if (threadIdx.x == 0) {
    for (int i = 0; i < nslot; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  const int nphase = 5 * a.L + (a.head ? 1 : 0);

  if (warp == kCW) {
    // ------------------------------------------------ producer
    if (lane == 0) {
      // A second cursor runs `lookahead` stages ahead of the ring and pulls
      // those rows into L2, so each bulk copy is served from L2.
      int pp = 0, prow = 0, pr1 = 0;
      PhaseW pw = {};
      bool pvalid = false;
      auto pnext = [&]() {
        if (pvalid) {
          prow += pw.rs;
          if (prow < pr1) return;
          ++pp;
        }
        pvalid = false;
        for (; pp < nphase; ++pp) {
          const int kind = pp < 5 * a.L ? pp % 5 : PH_HEAD;
          if (kind == PH_ATTN) continue;
          pw = phase_w(a, kind, pp / 5);
          block_rows(pw.M, &prow, &pr1);
          if (prow < pr1) {
            pvalid = true;
            return;
          }
        }
      };
      auto pissue = [&]() {
        if (!pvalid) return;
        const uint32_t n = (uint32_t)min(pw.rs, pr1 - prow);
        const uint32_t bytes = n * (uint32_t)pw.K * 2u;
        prefetch_l2(pw.w0 + (size_t)prow * pw.K, bytes);
        if (pw.NR > 1) prefetch_l2(pw.w1 + (size_t)prow * pw.K, bytes);
        pnext();
      };
      pnext();
      for (int i = 0; i < a.lookahead; ++i) pissue();
      uint32_t seq = 0;
      for (int p = 0; p < nphase; ++p) {
        const int kind = p < 5 * a.L ? p % 5 : PH_HEAD;
        if (kind == PH_ATTN) continue;
        const PhaseW w = phase_w(a, kind, p / 5);
        int r0, r1;
        block_rows(w.M, &r0, &r1);
        const size_t row_bytes = (size_t)w.K * 2;
        if (a.trace) a.trace[((size_t)blockIdx.x * nphase + p) * 4 + 3] = global_ns();
        for (int row0 = r0; row0 < r1; row0 += w.rs, ++seq) {
          const int slot = (int)(seq % nslot);
          if (seq >= (uint32_t)nslot) ring_wait(&empty[slot], ((seq / nslot) - 1) & 1u, err, kErrWaitEmpty);
          const int n = min(w.rs, r1 - row0);
          const uint32_t bytes = (uint32_t)(n * row_bytes);
          mbar_arrive_expect_tx(&full[slot], w.NR * bytes);
          uint8_t* dst = ring + (size_t)slot * a.slot_bytes;
          bulk_g2s(dst, w.w0 + (size_t)row0 * w.K, bytes, &full[slot]);
          if (w.NR > 1)
            bulk_g2s(dst + (size_t)w.rs * row_bytes, w.w1 + (size_t)row0 * w.K, bytes, &full[slot]);
          pissue();
        }
      }
    }
    return;
  }

  // -------------------------------------------------- consumers (256 threads)
  const uint32_t pos = a.ctl->pos;
  const uint32_t step = a.ctl->step;
  const uint32_t tok = a.feed ? a.feed[step] : a.ctl->argmax;
  const uint32_t G = gridDim.x;
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  uint32_t seq = 0;
  for (int p = 0; p < nphase; ++p) {
    const int kind = p < 5 * a.L ? p % 5 : PH_HEAD;
    const int l = p / 5;
    if (p > 0) phase_wait(&a.bar[p - 1], G, err);
    uint64_t* tr = a.trace ? a.trace + ((size_t)blockIdx.x * nphase + p) * 4 : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = global_ns();
    if (kind == PH_ATTN) {
      const int T = a.Hkv * a.nsplit;
      if ((int)blockIdx.x < T)
        attention_task<KT>(a, l, (int)blockIdx.x / a.nsplit, (int)blockIdx.x % a.nsplit, (int)pos,
                           scratch, &flag);
      if (tr && threadIdx.x == 0) tr[1] = tr[2] = global_ns();
      phase_arrive(&a.bar[p]);
      continue;
    }
    const PhaseW w = phase_w(a, kind, l);
    const MegaLayer* Ly = kind == PH_HEAD ? nullptr : &a.layers[l];
    // stage the phase input
    if (kind == PH_QKV) {
      const bool emb = l == 0;
      stage_c(scratch, w.K, emb ? nullptr : a.resid, emb ? a.embed + (size_t)tok * a.H : nullptr,
              Ly->ln1, a.eps, (emb && blockIdx.x == 0) ? a.resid : nullptr, red);
    } else if (kind == PH_O) {
      stage_c(scratch, w.K, a.attn, nullptr, nullptr, 0.0f, nullptr, red);
    } else if (kind == PH_GU) {
      stage_c(scratch, w.K, a.resid, nullptr, Ly->ln2, a.eps, nullptr, red);
    } else if (kind == PH_DOWN) {
      stage_c(scratch, w.K, a.act, nullptr, nullptr, 0.0f, nullptr, red);
    } else {
      stage_c(scratch, w.K, a.resid, nullptr, a.final_norm, a.eps, nullptr, red);
    }
    if (tr && threadIdx.x == 0) tr[1] = global_ns();
    const float4* xlo = reinterpret_cast<const float4*>(scratch);
    const float4* xhi = reinterpret_cast<const float4*>(scratch + (w.K >> 1));
    int r0, r1;
    block_rows(w.M, &r0, &r1);
    const size_t row_bytes = (size_t)w.K * 2;
    const int spl = kCW / w.rs;
    const int rr = warp / spl, cs = warp - rr * spl;
    const int cps = (w.K >> 3) / spl, c0 = cs * cps;
    for (int row0 = r0; row0 < r1; row0 += w.rs, ++seq) {
      const int slot = (int)(seq % nslot);
      ring_wait(&full[slot], (seq / nslot) & 1u, err, kErrWaitFull);
      const int n = min(w.rs, r1 - row0);
      float acc0 = 0.0f, acc1 = 0.0f;
      if (rr < n) {
        const uint8_t* base = ring + (size_t)slot * a.slot_bytes + (size_t)rr * row_bytes;
        if (w.NR == 1) {
#pragma unroll 4
          for (int c = c0 + lane; c < c0 + cps; c += 32) {
            const uint4 u = *reinterpret_cast<const uint4*>(base + (size_t)c * 16);
            acc0 = dot8s(u, xlo[c], xhi[c], acc0);
          }
        } else {
          const uint8_t* base1 = base + (size_t)w.rs * row_bytes;
#pragma unroll 4
          for (int c = c0 + lane; c < c0 + cps; c += 32) {
            const float4 lo = xlo[c], hi = xhi[c];
            acc0 = dot8s(*reinterpret_cast<const uint4*>(base + (size_t)c * 16), lo, hi, acc0);
            acc1 = dot8s(*reinterpret_cast<const uint4*>(base1 + (size_t)c * 16), lo, hi, acc1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      acc0 = warp_sum(acc0);
      if (w.NR > 1) acc1 = warp_sum(acc1);
      int row = -1;
      if (spl == 1) {
        if (rr < n) row = row0 + rr;
      } else {
        float* pp = part + (seq & 1) * 2 * kCW;
        if (lane == 0) {
          pp[warp] = acc0;
          pp[kCW + warp] = acc1;
        }
        named_sync(3, kCT);
        if (cs == 0 && rr < n) {
          row = row0 + rr;
          acc0 = 0.0f;
          acc1 = 0.0f;
          for (int q = 0; q < spl; ++q) {
            acc0 += pp[rr * spl + q];
            acc1 += pp[kCW + rr * spl + q];
          }
        }
      }
      if (row >= 0) {
        if (kind == PH_HEAD && better(acc0, (uint32_t)row, bv, bi)) {
          bv = acc0;
          bi = (uint32_t)row;
        }
        if (lane == 0) {
          if (kind == PH_QKV) __stcg(a.qkv + row, __fadd_rn(acc0, __ldg(Ly->bqkv + row)));
          else if (kind == PH_O || kind == PH_DOWN)
            __stcg(a.resid + row, __fadd_rn(__ldcg(a.resid + row), acc0));
          else if (kind == PH_GU) __stcg(a.act + row, silu_mul(acc0, acc1));
          else __stcg(a.logits + row, acc0);
        }
      }
    }
    if (tr && threadIdx.x == 0) tr[2] = global_ns();
    if (kind != PH_HEAD) {
      const uint32_t prev = phase_arrive(&a.bar[p]);
      // Step without a head: the last block through the final phase advances
      // the cursor (every block has read the step control by then).
      if (!a.head && p == nphase - 1 && threadIdx.x == 0 && prev == G - 1) {
        a.ctl->pos = pos + 1;
        a.ctl->step = step + 1;
      }
    }
  }
  if (!a.head) return;
  // ---------------------------------------------------- argmax finalize
  if (lane == 0) {
    wbv[warp] = bv;
    wbi[warp] = bi;
  }
  named_sync(1, kCT);
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    for (int q = 0; q < kCW; ++q)
      if (better(wbv[q], wbi[q], v, i)) {
        v = wbv[q];
        i = wbi[q];
      }
    __stcg(a.part_val + blockIdx.x, v);
    __stcg(a.part_idx + blockIdx.x, i);
    __threadfence();
    const bool last = atomicAdd(a.head_cnt, 1u) == G - 1;
    if (last) {
      __threadfence();
      v = -INFINITY;
      i = 0xffffffffu;
      for (uint32_t q = 0; q < G; ++q) {
        const float pv = __ldcg(a.part_val + q);
        const uint32_t pi = __ldcg(a.part_idx + q);
        if (better(pv, pi, v, i)) {
          v = pv;
          i = pi;
        }
      }
      if (a.rec_fed) a.rec_fed[step] = tok;
      if (a.rec_argmax) a.rec_argmax[step] = a.ctl->argmax;
      a.ctl->argmax = i == 0xffffffffu ? 0u : i;
      a.ctl->pos = pos + 1;
      a.ctl->step = step + 1;
      *a.head_cnt = 0u;
    }
  }
}

}  // namespace

bool mega_supported(int H, int I, int qd, int kvd, int d, int G, int slot_bytes) {
  if (H % 256 || I % 256 || qd % 256) return false;
  if (d % 4 || d > 256 || G > kMaxG) return false;
  // a whole row of every matrix must fit one ring slot
  const int kmax = H > I ? (H > qd ? H : qd) : (I > qd ? I : qd);
  return kmax * 2 <= slot_bytes && 2 * H * 2 <= slot_bytes;
}

size_t mega_scratch_bytes(int H, int I, int qd, int d, int G) {
  size_t x = (size_t)(H > I ? (H > qd ? H : qd) : (I > qd ? I : qd)) * 4;
  size_t at = (size_t)(G * d + 2 * kTile * (d + 4) + G * kTile + kMaxG + 2 * d) * 4;
  size_t s = x > at ? x : at;
  return (s + 127) / 128 * 128;
}

int mega_threads() { return kStepThreads; }

cudaError_t mega_configure(MegaArgs* a, int max_smem) {
  // ring slots as large as the biggest stage, as many as fit
  const size_t fixed = a->scratch_bytes + 2 * 2 * kCW * 4 + 16;
  int n = (int)((max_smem - fixed) / (a->slot_bytes + 16));
  if (n > 16) n = 16;
  if (n < 2) return cudaErrorInvalidValue;
  a->nslot = n;
  return cudaSuccess;
}

size_t mega_smem_bytes(const MegaArgs& a) {
  return a.scratch_bytes + (size_t)a.nslot * a.slot_bytes + 2 * 2 * kCW * 4 + 16 * (size_t)a.nslot + 16;
}

cudaError_t launch_step_mega(const MegaArgs& a, cudaStream_t st) {
  // Raise the dynamic shared-memory limit to exactly what this launch uses
  // (once per device and size).
  static int configured_dev = -1;
  static size_t configured_smem = 0;
  const size_t smem = mega_smem_bytes(a);
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev || configured_smem < smem) {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_step<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem)) != cudaSuccess)
      return e;
    if ((e = cudaFuncSetAttribute(k_step<__nv_bfloat16>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
        cudaSuccess)
      return e;
    configured_dev = dev;
    configured_smem = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.kv_bf16) return cudaLaunchKernelEx(&cfg, k_step<__nv_bfloat16>, a);
  return cudaLaunchKernelEx(&cfg, k_step<float>, a);
}

}  // namespace myos
