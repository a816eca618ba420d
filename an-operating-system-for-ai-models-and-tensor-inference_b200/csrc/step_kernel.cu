// One token step of the Qwen2.5 block stack as a single persistent kernel.
//
// Why: every phase of a decode step (QKV, attention, o_proj, gate/up, down,
// head) depends on the whole output of the previous one. As separate
// launches each boundary costs several microseconds of drain, launch and
// re-staging with HBM idle, and a step has 5 * layers + 1 of them. Here one
// block per SM runs the whole step, and phases are separated by device-wide
// arrival counters (one per phase, zeroed before each launch):
//
//   * each of the 16 warps of a block owns rows of the block's row range of
//     every weight matrix and streams them with 16-byte loads, double
//     buffered in registers (the measured fastest way to pull HBM here; a
//     bulk-copy ring was throughput-limited per SM);
//   * the first weight batch of a phase is loaded BEFORE the phase's counter
//     wait, so its HBM latency hides behind the wait and the input staging;
//   * input staging (RMSNorm fused, crates/tensor_core/src/bf16.rs:231-270)
//     issues all its loads at once: one L2 round trip per phase;
//   * attention tasks (KV head, key split) preload their cached K/V tile
//     before the wait; with few splits their merge is folded into the o_proj
//     staging, otherwise the last task of a head group merges;
//   * every counter wait is bounded in polls and time; a wait that gives up
//     raises a bit in ctl->err, which ends every later wait of every block at
//     once, so the launch always finishes and the host reports
//     MYOS_ERR_TIMEOUT.
// The launch is cooperative (one block per SM, all resident), so a counter
// never waits on a block that cannot run.
#include <math.h>

#include "common.cuh"
#include "step_kernel.h"

namespace myos {

namespace {

constexpr int kW = 16;       // warps per block
constexpr int kT = kW * 32;  // threads per block
constexpr int kTile = 32;    // attention key tile
constexpr int kMaxG = 8;
constexpr int kCombineMax = 32;  // attention tasks merged in the o_proj staging

enum Phase { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_HEAD = 5 };

struct PhaseW {
  const uint16_t* w0;
  const uint16_t* w1;
  int M, K, NR;
};

MYOS_DEV PhaseW phase_w(const MegaArgs& a, int kind, int l) {
  PhaseW w = {nullptr, nullptr, 0, 0, 1};
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

// Phase arrival: every thread fences its writes, then one thread counts the
// block in. Returns the previous count (thread 0 only).
MYOS_DEV uint32_t phase_arrive(unsigned* cnt) {
  __threadfence();
  __syncthreads();
  uint32_t prev = 0;
  if (threadIdx.x == 0) prev = atomicAdd(cnt, 1u);
  return prev;
}

// Wait until every block arrived; bounded (polls and one second), and
// abandoned at once when another block already reported a failure.
MYOS_DEV void phase_wait(const unsigned* cnt, uint32_t target, uint32_t* err) {
  if (threadIdx.x == 0 && ld_acquire(cnt) < target) {
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
  __syncthreads();
}

MYOS_DEV float bsum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float s = lane < kW ? red[lane] : 0.0f;
    s = warp_sum(s);
    if (lane == 0) red[32] = s;
  }
  __syncthreads();
  const float s = red[32];
  __syncthreads();
  return s;
}

// ---------------------------------------------------------------- L2 prefetch
// Weight slices of phases ahead are requested into L2 while this block still
// waits on the dependency chain (counters, staging, attention), so HBM keeps
// streaming through the latency-bound phases. Block b's rows of a row-major
// matrix are one contiguous byte range.
MYOS_DEV void prefetch_line_range(const void* base, size_t bytes) {
  const uintptr_t a0 = (uintptr_t)base & ~(uintptr_t)127;
  const uintptr_t end = (uintptr_t)base + bytes;
  for (uintptr_t p = a0 + (uintptr_t)threadIdx.x * 128; p < end; p += (uintptr_t)kT * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

MYOS_DEV void prefetch_phase(const MegaArgs& a, int q) {
  const int nph = 5 * a.L + (a.head ? 1 : 0);
  if (q >= nph) return;
  const int kind = q < 5 * a.L ? q % 5 : PH_HEAD;
  if (kind == PH_ATTN) return;
  const PhaseW w = phase_w(a, kind, q / 5);
  int r0, r1;
  block_rows(w.M, &r0, &r1);
  size_t bytes = (size_t)(r1 - r0) * w.K * 2;
  const size_t cap = (size_t)a.pf_kb << 10;
  if (bytes > cap) bytes = cap;
  const uint16_t* m[2] = {w.w0, w.w1};
  for (int r = 0; r < w.NR; ++r) {
    const uint16_t* p = m[r] + (size_t)r0 * w.K;
    if (a.pf_mode) prefetch_line_range(p, bytes);
    else prefetch_range(p, bytes);
  }
}

// ---------------------------------------------------------------- staging
// Inputs land in shared memory through cp.async (no registers held, so the
// first weight batch stays in flight meanwhile), in the split layout the
// GEMV loop reads: chunk c of 8 values puts 4 at xs[4c] and 4 at
// xs[K/2 + 4c]. Each thread copies and later reads back only its own
// chunks, so its own cp.async wait orders them.
MYOS_DEV void cpa16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
MYOS_DEV void cpa_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Split-layout copy of K f32 values.
MYOS_DEV void copy_split(float* xs, const float* x, int K) {
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4* lo = reinterpret_cast<float4*>(xs);
  float4* hi = reinterpret_cast<float4*>(xs + (K >> 1));
  for (int c = threadIdx.x; c < (K >> 3); c += kT) {
    cpa16(lo + c, x4 + 2 * c);
    cpa16(hi + c, x4 + 2 * c + 1);
  }
}

// Embedding row (bf16) into the split layout via a raw copy in eb.
MYOS_DEV void copy_embed(float* xs, const uint16_t* row, int K, uint4* eb) {
  const uint4* r4 = reinterpret_cast<const uint4*>(row);
  for (int c = threadIdx.x; c < (K >> 3); c += kT) cpa16(eb + c, r4 + c);
  cpa_wait_all();
  float4* lo = reinterpret_cast<float4*>(xs);
  float4* hi = reinterpret_cast<float4*>(xs + (K >> 1));
  for (int c = threadIdx.x; c < (K >> 3); c += kT) {
    const uint4 u = eb[c];
    lo[c] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
    hi[c] = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
  }
}

// RMSNorm in place over the staged split layout, gamma staged the same way
// in gs: y = gamma * (x * inv), inv = 1 / sqrtf(mean(x^2) + eps)
// (crates/tensor_core/src/bf16.rs:231-270); optionally stores the raw x
// (natural order) to x_store first.
MYOS_DEV void norm_split(float* xs, const float* gs, int K, float eps, float* x_store, float* red) {
  const int half = K >> 1;
  float4* lo = reinterpret_cast<float4*>(xs);
  float4* hi = reinterpret_cast<float4*>(xs + half);
  const float4* glo = reinterpret_cast<const float4*>(gs);
  const float4* ghi = reinterpret_cast<const float4*>(gs + half);
  float ss = 0.0f;
  for (int c = threadIdx.x; c < (K >> 3); c += kT) {
    const float4 u = lo[c], v = hi[c];
    ss = fmaf(u.x, u.x, ss);
    ss = fmaf(u.y, u.y, ss);
    ss = fmaf(u.z, u.z, ss);
    ss = fmaf(u.w, u.w, ss);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = bsum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
  for (int c = threadIdx.x; c < (K >> 3); c += kT) {
    const float4 u = lo[c], v = hi[c], g = glo[c], h = ghi[c];
    if (x_store) {
      __stcg(reinterpret_cast<float4*>(x_store) + 2 * c, u);
      __stcg(reinterpret_cast<float4*>(x_store) + 2 * c + 1, v);
    }
    lo[c] = make_float4(__fmul_rn(g.x, __fmul_rn(u.x, inv)), __fmul_rn(g.y, __fmul_rn(u.y, inv)),
                        __fmul_rn(g.z, __fmul_rn(u.z, inv)), __fmul_rn(g.w, __fmul_rn(u.w, inv)));
    hi[c] = make_float4(__fmul_rn(h.x, __fmul_rn(v.x, inv)), __fmul_rn(h.y, __fmul_rn(v.y, inv)),
                        __fmul_rn(h.z, __fmul_rn(v.z, inv)), __fmul_rn(h.w, __fmul_rn(v.w, inv)));
  }
}

MYOS_DEV void put_split(float* xs, int K, int j, float v) {
  const int c = j >> 3, e = j & 7;
  xs[e < 4 ? (c * 4 + e) : ((K >> 1) + c * 4 + (e - 4))] = v;
}

// Per (head group, split) merge factors f = expf(m - M) and per-head sums
// L = sum l * f for head rows [h0, h0 + nh), from split partials m, l laid
// out [Hkv][nsplit][G]; fs is overwritten by the factors.
MYOS_DEV void merge_factors(const MegaArgs& a, float* fs, const float* ls, float* Ls, int h0,
                            int nh) {
  const int G = a.G, ns = a.nsplit;
  if (threadIdx.x < nh) {
    const int h = h0 + threadIdx.x, g = h / G, hh = h - g * G;
    float M = -INFINITY;
    for (int q = 0; q < ns; ++q) M = fmaxf(M, fs[(g * ns + q) * G + hh]);
    float L = 0.0f;
    for (int q = 0; q < ns; ++q) {
      const int i = (g * ns + q) * G + hh;
      const float mq = fs[i];
      const float f = mq == -INFINITY ? 0.0f : expf(mq - M);
      fs[i] = f;
      L = fmaf(ls[i], f, L);
    }
    Ls[threadIdx.x] = L;
  }
  __syncthreads();
}

// o_proj input from the split partials (few splits): every partial copied
// into shared memory at once, then out = sum_q part_o * f / L (the
// reference's e / sum, reassociated) written in the split layout.
MYOS_DEV void merge_stage(const MegaArgs& a, float* xs, int K, float* mb) {
  const int T = a.Hkv * a.nsplit, Tg = T * a.G, d = a.d, G = a.G, ns = a.nsplit;
  float* po = mb;             // [T][G][d]
  float* fs = po + Tg * d;    // [T][G]
  float* ls = fs + Tg;        // [T][G]
  float* Ls = ls + Tg;        // [Hq]
  const float4* s4 = reinterpret_cast<const float4*>(a.part_o);
  for (int i = threadIdx.x; i < (Tg * d) >> 2; i += kT) cpa16(reinterpret_cast<float4*>(po) + i, s4 + i);
  for (int i = threadIdx.x; i < Tg; i += kT) {
    fs[i] = __ldcg(a.part_m + i);
    ls[i] = __ldcg(a.part_l + i);
  }
  cpa_wait_all();
  __syncthreads();
  merge_factors(a, fs, ls, Ls, 0, a.Hq);
  for (int o = threadIdx.x; o < K; o += kT) {
    const int h = o / d, e = o - h * d, g = h / G, hh = h - g * G;
    float O = 0.0f;
    for (int q = 0; q < ns; ++q) {
      const int i = (g * ns + q) * G + hh;
      O = fmaf(po[i * d + e], fs[i], O);
    }
    put_split(xs, K, o, __fdiv_rn(O, Ls[h]));
  }
}

// Many splits: the merge of head group g from global partials, in groups of
// 2 outputs x 8 splits per load round.
MYOS_DEV void merge_group(const MegaArgs& a, int g, float* sm, float* att) {
  const int G = a.G, d = a.d, ns = a.nsplit, n = G * d;
  float* fs = sm;
  float* ls = fs + ns * G;
  float* Ls = ls + ns * G;
  for (int i = threadIdx.x; i < ns * G; i += kT) {
    fs[i] = __ldcg(a.part_m + (size_t)g * ns * G + i);
    ls[i] = __ldcg(a.part_l + (size_t)g * ns * G + i);
  }
  __syncthreads();
  // factors for this group's heads (local indices: group 0 of the tables)
  if (threadIdx.x < G) {
    const int hh = threadIdx.x;
    float M = -INFINITY;
    for (int q = 0; q < ns; ++q) M = fmaxf(M, fs[q * G + hh]);
    float L = 0.0f;
    for (int q = 0; q < ns; ++q) {
      const float mq = fs[q * G + hh];
      const float f = mq == -INFINITY ? 0.0f : expf(mq - M);
      fs[q * G + hh] = f;
      L = fmaf(ls[q * G + hh], f, L);
    }
    Ls[hh] = L;
  }
  __syncthreads();
  constexpr int kO = 2, kS = 8;
  for (int ob = 0; ob < n; ob += kO * kT) {
    float O[kO] = {0.0f, 0.0f};
    for (int q0 = 0; q0 < ns; q0 += kS) {
      float v[kO][kS];
#pragma unroll
      for (int k = 0; k < kO; ++k) {
        const int o = ob + threadIdx.x + kT * k, hh = o / d, e = o - hh * d;
#pragma unroll
        for (int u = 0; u < kS; ++u)
          v[k][u] = (o < n && q0 + u < ns)
                        ? __ldcg(a.part_o + (((size_t)g * ns + q0 + u) * G + hh) * d + e)
                        : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < kO; ++k) {
        const int o = ob + threadIdx.x + kT * k, hh = o / d;
#pragma unroll
        for (int u = 0; u < kS; ++u)
          if (o < n && q0 + u < ns) O[k] = fmaf(v[k][u], fs[(q0 + u) * G + hh], O[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < kO; ++k) {
      const int o = ob + threadIdx.x + kT * k;
      if (o < n) __stcg(att + o, __fdiv_rn(O[k], Ls[o / d]));
    }
  }
}

MYOS_DEV bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > -INFINITY && (v > bv || (v == bv && i < bi));
}

MYOS_DEV float silu_mul(float g, float u) {
  const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

// ---------------------------------------------------------------- GEMV phase
// One GEMV phase on this block's rows: the first weight batch is loaded,
// then the phase waits for its inputs and stages them, then streams the
// rest. Warp w owns rows r0 + w + kW*i; per row K/256 chunks of 16 bytes per
// lane, in batches of kU double-buffered in registers. One loop serves every
// phase kind (gate/up streams two matrices, the others one) so the kernel
// holds a single copy of it.
constexpr int kU = 4;

MYOS_DEV void gemv_phase(const MegaArgs& a, int p, int kind, uint32_t tok, float* xs, float* red,
                         float* bvp, uint32_t* bip) {
  const int l = p / 5;
  const PhaseW w = phase_w(a, kind, l);
  const bool two = w.NR == 2;
  uint64_t* tr = a.trace ? a.trace + ((size_t)blockIdx.x * (5 * a.L + 1) + p) * 4 : nullptr;
  int r0, r1;
  block_rows(w.M, &r0, &r1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = w.K, P = K >> 8, nbr = (P + kU - 1) / kU;
  const int nrw = r1 - r0 > warp ? (r1 - r0 - warp + kW - 1) / kW : 0;
  const int nb = nrw * nbr;
  uint4 cur[2][kU], nxt[2][kU];
  auto load = [&](uint4(&buf)[2][kU], int bt) {
    const int rb = bt / nbr, j0 = (bt - rb * nbr) * kU;
    const size_t off = (size_t)(r0 + warp + kW * rb) * K;
    const uint4* s0 = reinterpret_cast<const uint4*>(w.w0 + off) + lane;
    const uint4* s1 = reinterpret_cast<const uint4*>((two ? w.w1 : w.w0) + off) + lane;
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      const int j = j0 + i;
      buf[0][i] = j < P ? ld_stream(s0 + 32 * j) : make_uint4(0u, 0u, 0u, 0u);
      buf[1][i] = (two && j < P) ? ld_stream(s1 + 32 * j) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  if (nb > 0) load(cur, 0);
  // ---- inputs: gamma needs no wait; x does
  const MegaLayer* Ly = kind == PH_HEAD ? nullptr : &a.layers[l];
  const float* gamma = kind == PH_QKV ? Ly->ln1
                       : kind == PH_GU ? Ly->ln2
                       : kind == PH_HEAD ? a.final_norm
                                         : nullptr;
  float* gs = xs + a.x_floats;
  if (gamma) copy_split(gs, gamma, K);
  if (p > 0) phase_wait(&a.bar[p - 1], gridDim.x, &a.ctl->err);
  if (tr && threadIdx.x == 0) tr[0] = global_ns();
  if (kind == PH_QKV && l == 0) {
    copy_embed(xs, a.embed + (size_t)tok * a.H, K, reinterpret_cast<uint4*>(gs + a.H));
  } else if (kind == PH_O && a.merge_in_stage) {
    merge_stage(a, xs, K, gs);
  } else {
    copy_split(xs, kind == PH_O ? a.attn : kind == PH_DOWN ? a.act : a.resid, K);
  }
  cpa_wait_all();
  if (gamma)
    norm_split(xs, gs, K, a.eps, (kind == PH_QKV && l == 0 && blockIdx.x == 0) ? a.resid : nullptr,
               red);
  __syncthreads();
  if (tr && threadIdx.x == 0) tr[1] = global_ns();
  // ---- stream
  const float4* xlo = reinterpret_cast<const float4*>(xs);
  const float4* xhi = reinterpret_cast<const float4*>(xs + (K >> 1));
  float* const out = kind == PH_QKV ? a.qkv
                     : kind == PH_GU ? a.act
                     : kind == PH_HEAD ? a.logits
                                       : a.resid;
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  float acc0 = 0.0f, acc1 = 0.0f;
  for (int bt = 0; bt < nb; ++bt) {
    const int rb = bt / nbr, jb = bt - rb * nbr;
    if (bt + 1 < nb) load(nxt, bt + 1);
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      const int j = jb * kU + i;
      if (j < P) {
        const float4 lo = xlo[lane + 32 * j], hi = xhi[lane + 32 * j];
        acc0 = dot8(cur[0][i], lo, hi, acc0);
        if (two) acc1 = dot8(cur[1][i], lo, hi, acc1);
      }
    }
    if (jb == nbr - 1) {
      const int row = r0 + warp + kW * rb;
      const float v0 = warp_sum(acc0);
      const float v1 = two ? warp_sum(acc1) : 0.0f;
      acc0 = acc1 = 0.0f;
      if (kind == PH_HEAD && better(v0, (uint32_t)row, bv, bi)) {
        bv = v0;
        bi = (uint32_t)row;
      }
      if (lane == 0) {
        if (kind == PH_QKV) __stcg(out + row, __fadd_rn(v0, __ldg(Ly->bqkv + row)));
        else if (kind == PH_O || kind == PH_DOWN) __stcg(out + row, __fadd_rn(__ldcg(out + row), v0));
        else if (kind == PH_GU) __stcg(out + row, silu_mul(v0, v1));
        else __stcg(out + row, v0);
      }
    }
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      cur[0][i] = nxt[0][i];
      cur[1][i] = nxt[1][i];
    }
  }
  if (tr && threadIdx.x == 0) tr[2] = global_ns();
  if (kind == PH_HEAD && lane == 0) {
    bvp[warp] = bv;
    bip[warp] = bi;
  }
}

// ---------------------------------------------------------------- attention
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

struct AttnSmem {
  float *qs, *ks, *vs, *ps, *corr, *knew, *vnew, *cs, *sn;
  uint4* raw;  // bf16 tile rows before widening: [2][kTile][d / 8]
};

MYOS_DEV AttnSmem attn_smem(float* sm, int G, int d) {
  AttnSmem s;
  const int ds = d + 4;
  s.qs = sm;
  s.ks = s.qs + G * d;
  s.vs = s.ks + kTile * ds;
  s.ps = s.vs + kTile * ds;
  s.corr = s.ps + G * kTile;
  s.knew = s.corr + kMaxG;
  s.vnew = s.knew + d;
  s.cs = s.vnew + d;
  s.sn = s.cs + d / 2;
  s.raw = reinterpret_cast<uint4*>(s.sn + d / 2);  // 16-byte aligned: offsets are multiples of 4
  return s;
}

template <typename KT>
MYOS_DEV KT* kv_base(const MegaArgs& a, void* cache, int layer, int g) {
  return reinterpret_cast<KT*>(reinterpret_cast<uint8_t*>(cache) +
                               (size_t)layer * a.kv_layer_elems * sizeof(KT)) +
         (size_t)g * a.S * a.d;
}

// Cached rows [t0, t0 + nk) except `skip` (the new position) into the
// padded K/V tiles through cp.async: f32 rows straight into the tiles, bf16
// rows into a raw buffer that tile_finish widens. Each thread widens only
// the 16-byte pieces it copied itself, after its own cp.async wait.
template <typename KT>
MYOS_DEV void tile_issue(const KT* kc, const KT* vc, int d, int t0, int nk, int skip, float* ks,
                         float* vs, uint4* raw) {
  constexpr int per = 16 / sizeof(KT);  // elements per 16-byte piece
  const int ppr = d / per, n = nk * ppr, ds = d + 4;
  for (int i = threadIdx.x; i < n; i += kT) {
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

template <typename KT>
MYOS_DEV void tile_finish(int d, int t0, int nk, int skip, float* ks, float* vs, const uint4* raw) {
  cpa_wait_all();
  if (sizeof(KT) == 4) return;
  const int ppr = d / 8, n = nk * ppr, ds = d + 4;
  for (int i = threadIdx.x; i < n; i += kT) {
    const int tt = i / ppr, e = (i - tt * ppr) * 8;
    if (t0 + tt == skip) continue;
    const uint4 u = raw[i], v = raw[kTile * ppr + i];
    float4* kd = reinterpret_cast<float4*>(ks + tt * ds + e);
    float4* vd = reinterpret_cast<float4*>(vs + tt * ds + e);
    kd[0] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
    kd[1] = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
    vd[0] = make_float4(bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y));
    vd[1] = make_float4(bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w));
  }
}

// Attention task (KV head g, key split s) at decode position pos: scores,
// online softmax and value mix over the split's keys (the math of
// crates/tensor_core/src/gqa.rs:174-218 reassociated as flash decoding);
// writes the split's (sum e*v, max, sum e). The first tile of cached keys
// and the rotation table row are already in shared memory.
template <typename KT>
MYOS_DEV void attention_task(const MegaArgs& a, int layer, int g, int s, int pos, float* sm) {
  const int d = a.d, G = a.G, half = d >> 1, ds = d + 4;
  const AttnSmem S = attn_smem(sm, G, d);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  KT* kc = kv_base<KT>(a, a.kcache, layer, g);
  KT* vc = kv_base<KT>(a, a.vcache, layer, g);
  const int kb = s * a.chunk, ke = min(kb + a.chunk, pos + 1);
  const bool has_new = pos >= kb && pos < ke;
  {
    // q of the G heads, and this KV head's new k and v: one float4 each
    const int nq4 = G * d / 4, d4 = d / 4;
    const int ntot = nq4 + (has_new ? 2 * d4 : 0);
    const float4* qsrc = reinterpret_cast<const float4*>(a.qkv + (size_t)g * G * d);
    const float4* ksrc = reinterpret_cast<const float4*>(a.qkv + (size_t)a.Hq * d + (size_t)g * d);
    const float4* vsrc =
        reinterpret_cast<const float4*>(a.qkv + (size_t)(a.Hq + a.Hkv) * d + (size_t)g * d);
    constexpr int kJ = (kMaxG * 64 + 128 + kT - 1) / kT;
    float4 val[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int v = threadIdx.x + kT * j;
      if (v < ntot)
        val[j] = v < nq4 ? __ldcg(qsrc + v)
                         : (v < nq4 + d4 ? __ldcg(ksrc + (v - nq4)) : __ldcg(vsrc + (v - nq4 - d4)));
    }
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int v = threadIdx.x + kT * j;
      if (v < ntot) {
        float4* dst = v < nq4 ? reinterpret_cast<float4*>(S.qs) + v
                              : (v < nq4 + d4 ? reinterpret_cast<float4*>(S.knew) + (v - nq4)
                                              : reinterpret_cast<float4*>(S.vnew) + (v - nq4 - d4));
        *dst = val[j];
      }
    }
    __syncthreads();
    // NeoX rotation in place, one (lane i, lane i + d/2) pair per thread,
    // y0 = x0*c - x1*s, y1 = x1*c + x0*s (crates/tensor_core/src/rope.rs:145-184)
    const int npair = (G + (has_new ? 1 : 0)) * half;
    for (int i = threadIdx.x; i < npair; i += kT) {
      const int hh = i / half, p = i - hh * half;
      float* x = hh < G ? S.qs + hh * d : S.knew;
      const float x0 = x[p], x1 = x[p + half];
      const float c = S.cs[p], sv = S.sn[p];
      x[p] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sv));
      x[p + half] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sv));
    }
    __syncthreads();
    if (has_new) {
      for (int e = threadIdx.x; e < d; e += kT) {
        const KT kq = kv_round<KT>(S.knew[e]);
        const KT vq = kv_round<KT>(S.vnew[e]);
        kc[(size_t)pos * d + e] = kq;  // KvCache::store for this position
        vc[(size_t)pos * d + e] = vq;
        S.knew[e] = (float)kq;
        S.vnew[e] = (float)vq;
      }
    }
  }
  constexpr int kMaxOut = kMaxG * 256 / kT;
  float acc[kMaxOut];
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) acc[i] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  for (int t0 = kb; t0 < ke; t0 += kTile) {
    const int nk = min(kTile, ke - t0);
    if (t0 != kb) {  // later tiles (the first was preloaded)
      __syncthreads();
      tile_issue<KT>(kc, vc, d, t0, nk, has_new ? pos : -1, S.ks, S.vs, S.raw);
      tile_finish<KT>(d, t0, nk, has_new ? pos : -1, S.ks, S.vs, S.raw);
    }
    __syncthreads();
    if (has_new && pos >= t0 && pos < t0 + nk) {
      const int tt = pos - t0;
      for (int e = threadIdx.x; e < d; e += kT) {
        S.ks[tt * ds + e] = S.knew[e];
        S.vs[tt * ds + e] = S.vnew[e];
      }
      __syncthreads();
    }
    // scores: two threads per (head, key), halves of d summed by a shuffle
    for (int i = threadIdx.x; i < 2 * G * kTile; i += kT) {
      const int hk = i >> 1, part = i & 1;
      const int hh = hk / kTile, tt = hk - hh * kTile;
      float dot = 0.0f;
      if (tt < nk) {
        const float* qh = S.qs + hh * d + part * half;
        const float* kr = S.ks + tt * ds + part * half;
        for (int e = 0; e < half; e += 4) {
          const float4 qv = *reinterpret_cast<const float4*>(qh + e);
          const float4 kv = *reinterpret_cast<const float4*>(kr + e);
          dot = fmaf(qv.x, kv.x, dot);
          dot = fmaf(qv.y, kv.y, dot);
          dot = fmaf(qv.z, kv.z, dot);
          dot = fmaf(qv.w, kv.w, dot);
        }
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      if (part == 0) S.ps[hh * kTile + tt] = tt < nk ? __fmul_rn(dot, a.scale) : -INFINITY;
    }
    __syncthreads();
    if (warp < G) {
      const float sc = S.ps[warp * kTile + lane];
      const float mt = warp_max(sc);
      const float mn = fmaxf(m_run, mt);
      const float cf = expf(m_run - mn);
      const float pr = lane < nk ? expf(sc - mn) : 0.0f;
      l_run = fmaf(l_run, cf, warp_sum(pr));
      m_run = mn;
      S.ps[warp * kTile + lane] = pr;
      if (lane == 0) S.corr[warp] = cf;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxOut; ++i) {
      const int o = threadIdx.x + kT * i;
      if (o < G * d) {
        const int hh = o / d, e = o - hh * d;
        const float* ph = S.ps + hh * kTile;
        float v = acc[i] * S.corr[hh];
        for (int tt = 0; tt < nk; ++tt) v = fmaf(ph[tt], S.vs[tt * ds + e], v);
        acc[i] = v;
      }
    }
  }
  const size_t pbase = ((size_t)g * a.nsplit + s) * G;
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) {
    const int o = threadIdx.x + kT * i;
    if (o < G * d) __stcg(a.part_o + pbase * d + o, acc[i]);
  }
  if (warp < G && lane == 0) {
    __stcg(a.part_m + pbase + warp, m_run);
    __stcg(a.part_l + pbase + warp, l_run);
  }
}

// The attention phase: tasks (KV head g, split s) on blocks [0, Hkv*nsplit).
// With many splits, the last task of a head group (by arrival) merges the
// group's partials into a.attn; otherwise the o_proj staging merges.
template <typename KT>
MYOS_DEV void attn_phase(const MegaArgs& a, int p, int pos, float* sm, int* flag) {
  const int l = p / 5, T = a.Hkv * a.nsplit;
  uint64_t* tr = a.trace ? a.trace + ((size_t)blockIdx.x * (5 * a.L + 1) + p) * 4 : nullptr;
  const bool task = (int)blockIdx.x < T;
  const int g = (int)blockIdx.x / a.nsplit, s = (int)blockIdx.x % a.nsplit;
  const int kb = s * a.chunk, ke = min(kb + a.chunk, pos + 1);
  const AttnSmem S = attn_smem(sm, a.G, a.d);
  if (task && kb < ke) {  // inputs that do not depend on this step: before the wait
    tile_issue<KT>(kv_base<KT>(a, a.kcache, l, g), kv_base<KT>(a, a.vcache, l, g), a.d, kb,
                   min(kTile, ke - kb), pos, S.ks, S.vs, S.raw);
    const int half4 = a.d >> 3;  // rotation table row: d/2 floats each
    const float4* c4 = reinterpret_cast<const float4*>(a.cos_t + (size_t)pos * (a.d >> 1));
    const float4* s4 = reinterpret_cast<const float4*>(a.sin_t + (size_t)pos * (a.d >> 1));
    for (int i = threadIdx.x; i < half4; i += kT) {
      cpa16(reinterpret_cast<float4*>(S.cs) + i, c4 + i);
      cpa16(reinterpret_cast<float4*>(S.sn) + i, s4 + i);
    }
    tile_finish<KT>(a.d, kb, min(kTile, ke - kb), pos, S.ks, S.vs, S.raw);
  }
  phase_wait(&a.bar[p - 1], gridDim.x, &a.ctl->err);
  if (tr && threadIdx.x == 0) tr[0] = tr[1] = global_ns();
  if (task) {
    if (kb < ke) {
      attention_task<KT>(a, l, g, s, pos, sm);
    } else {  // empty split: neutral partial
      const size_t pbase = ((size_t)g * a.nsplit + s) * a.G;
      for (int i = threadIdx.x; i < a.G * a.d; i += kT) __stcg(a.part_o + pbase * a.d + i, 0.0f);
      if (threadIdx.x < a.G) {
        __stcg(a.part_m + pbase + threadIdx.x, -INFINITY);
        __stcg(a.part_l + pbase + threadIdx.x, 0.0f);
      }
    }
    if (!a.merge_in_stage) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) *flag = atomicAdd(a.attn_cnt + g, 1u) == (unsigned)(a.nsplit - 1);
      __syncthreads();
      if (*flag) {
        __threadfence();
        merge_group(a, g, sm, a.attn + (size_t)g * a.G * a.d);
        if (threadIdx.x == 0) a.attn_cnt[g] = 0u;
      }
    }
  }
  if (tr && threadIdx.x == 0) tr[2] = global_ns();
}

// ---------------------------------------------------------------- the kernel
template <typename KT>
__global__ void __launch_bounds__(kT, 1) k_step(MegaArgs a) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);  // staged input, or attention tiles
  __shared__ float red[33];
  __shared__ float wbv[kW];
  __shared__ uint32_t wbi[kW];
  __shared__ int flag;
  const uint32_t pos = a.ctl->pos;
  const uint32_t step = a.ctl->step;
  const uint32_t tok = a.feed ? a.feed[step] : a.ctl->argmax;
  const uint32_t G = gridDim.x;
  const int nphase = 5 * a.L + (a.head ? 1 : 0);
  int pf_next = 0;

  for (int p = 0; p < nphase; ++p) {
    const int kind = p < 5 * a.L ? p % 5 : PH_HEAD;
    for (; pf_next <= p + a.lookahead && pf_next < nphase; ++pf_next)
      if (pf_next > p) prefetch_phase(a, pf_next);
    if (kind == PH_ATTN) attn_phase<KT>(a, p, (int)pos, sm, &flag);
    else gemv_phase(a, p, kind, tok, sm, red, wbv, wbi);
    if (kind != PH_HEAD) {
      const uint32_t prev = phase_arrive(&a.bar[p]);  // includes a block barrier
      if (!a.head && p == nphase - 1 && threadIdx.x == 0 && prev == G - 1) {
        // Step without a head: the last block through the final phase
        // advances the cursor; every block has read the step control.
        a.ctl->pos = pos + 1;
        a.ctl->step = step + 1;
      }
    }
  }
  if (!a.head) return;
  // ---------------------------------------------------- argmax finalize
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    for (int q = 0; q < kW; ++q)
      if (better(wbv[q], wbi[q], v, i)) {
        v = wbv[q];
        i = wbi[q];
      }
    __stcg(a.part_val + blockIdx.x, v);
    __stcg(a.part_idx + blockIdx.x, i);
    __threadfence();
    if (atomicAdd(a.head_cnt, 1u) == G - 1) {
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

bool mega_supported(int H, int I, int qd, int kvd, int d, int G) {
  (void)kvd;
  if (H % 256 || I % 256 || qd % 256) return false;
  if (d % 8 || d > 256 || G > kMaxG || qd / d > kT) return false;
  return true;
}

int mega_threads() { return kT; }

cudaError_t mega_configure(MegaArgs* a, int max_smem) {
  const int kmax = a->H > a->I ? (a->H > a->qd ? a->H : a->qd) : (a->I > a->qd ? a->I : a->qd);
  a->x_floats = (kmax + 31) / 32 * 32;
  const int T = a->Hkv * a->nsplit, Tg = T * a->G;
  const size_t norm_area = (size_t)a->H + a->H / 2;            // gamma, raw embedding row
  const size_t merge_area = (size_t)Tg * a->d + 2 * Tg + a->Hq;  // partials, factors, sums
  const size_t tiles = (size_t)a->G * a->d + 2 * kTile * (a->d + 4) + a->G * kTile + kMaxG +
                       3 * a->d + 2 * kTile * a->d / 2;  // + raw bf16 rows
  const size_t mgroup = 2 * (size_t)a->nsplit * a->G + a->G;
  const size_t attn = tiles > mgroup ? tiles : mgroup;
  auto bytes = [&](size_t second) {
    const size_t x = (size_t)a->x_floats + second;
    return ((x > attn ? x : attn) * 4 + 127) / 128 * 128;
  };
  const size_t with_merge = bytes(norm_area > merge_area ? norm_area : merge_area);
  a->merge_in_stage = T <= kCombineMax && with_merge <= (size_t)max_smem;
  a->scratch_bytes = a->merge_in_stage ? with_merge : bytes(norm_area);
  return a->scratch_bytes <= (size_t)max_smem ? cudaSuccess : cudaErrorInvalidValue;
}

size_t mega_smem_bytes(const MegaArgs& a) { return a.scratch_bytes; }

cudaError_t launch_step_mega(const MegaArgs& a, cudaStream_t st) {
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
  cfg.blockDim = dim3(kT);
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
