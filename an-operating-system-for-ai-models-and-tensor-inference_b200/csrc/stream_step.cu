// Decode token steps as one persistent kernel with a continuous weight stream.
//
// A batch-1 decode step reads 3.09 GB of bf16 weights (Qwen2.5-1.5B) through
// 5 dependent phases per layer (QKV, attention, o_proj, gate/up, down) and
// the head. Launched per phase, every boundary drains HBM: the next kernel's
// first weight bytes arrive a DRAM latency after its dependency clears, and
// the small phases (QKV 6.3 MB, o_proj 4.7 MB) never reach streaming speed.
// Here the weight stream does not wait for phase boundaries:
//
//   * one CTA per SM (cooperative launch, so every CTA is resident); CTA b
//     owns a contiguous row range of every weight matrix;
//   * a producer warp copies the CTA's rows, matrix after matrix in step
//     order, with 1-D bulk copies (cp.async.bulk, the TMA engine) into a
//     4-slot shared-memory ring of ~45 KB slots. It waits for a free slot
//     and keeps few copies outstanding (every queued request in the memory
//     system delays the consumers' barrier and staging accesses), never for
//     activations: during a phase boundary (grid barrier, input staging,
//     attention) HBM keeps filling the ring with the next phases' weights;
//   * 15 consumer warps stage each phase's input vector in shared memory
//     with cp.async (RMSNorm fused, crates/tensor_core/src/bf16.rs:231-270),
//     dot every ring slot's rows against it (bf16 weights promoted exactly,
//     f32 FMA, fixed reduction order: deterministic) and apply the epilogue:
//     QKV bias (bf16.rs:147-158), residual add (qwen25_block.rs:172-178),
//     SiLU(gate) * up (swiglu.rs:113-131,254-261), logits and the
//     first-maximum argmax (model_core/src/lib.rs:157-167);
//   * attention (gqa.rs:174-307) runs as split-KV tasks (KV head, key range)
//     on the first CTAs, with RoPE (rope.rs:145-184) and the KV store
//     (kv_cache.rs:149-302) fused; the split partials are merged in the
//     o_proj input staging (few splits) or by the last task of a KV head;
//   * phases are separated by a grid barrier of per-CTA arrival flags
//     (monotonic counts, no atomics); every wait is bounded in time, and a
//     wait that gives up raises kErrStream in ctl->err and ends the launch;
//   * several token steps run per launch: the greedy token is reduced by
//     every CTA from the per-CTA head candidates, so the next step starts
//     without a host round trip or a relaunch.
// With most of shared memory taken by the ring, L1 is small: the kernel is
// written to keep its state in registers (no local-memory stack).
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "stream_step.h"

namespace myos {

namespace {

#ifndef MYOS_STREAM_WARPS
#define MYOS_STREAM_WARPS 15  // consumer warps (16 warps in all: 128 registers a thread)
#endif
constexpr int kNCW = MYOS_STREAM_WARPS;
constexpr int kCT = kNCW * 32;      // consumer threads
constexpr int kST = kCT + 32;       // plus the producer warp
constexpr int kNS = 4;              // ring slots
constexpr int kGMax = 8;            // query heads per KV head
constexpr int kD = 128;             // head dim of the supported shapes
constexpr int kBar = 1;             // named barrier of the consumer warps
constexpr int kMaxLayers = 128;

MYOS_DEV void csync() { named_sync(kBar, kCT); }

MYOS_DEV float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

MYOS_DEV void cpa16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
MYOS_DEV void cpa_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

MYOS_DEV uint32_t ld_acquire(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
MYOS_DEV void st_release(unsigned* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

MYOS_DEV float silu_mul(float g, float u) {
  // z / (1 + expf(-z)), then one multiply (swiglu.rs:113-115, 254-261)
  const float a = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(a, u);
}

// First maximum with strict >: NaN and -inf never win, ties keep the lower
// index (model_core/src/lib.rs:157-167).
MYOS_DEV bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > -INFINITY && (v > bv || (v == bv && i < bi));
}

// ---------------------------------------------------------------- shared state
// Dynamic shared memory: [ring: kNS x slot_bytes][scr][part][res][bias][layer
// table], at the offsets stream_configure puts in the arguments (no pointer
// table held in registers). Small fixed state is static.
__shared__ float s_red[64];            // reductions
__shared__ float s_wbv[kNCW];          // per-warp head candidates
__shared__ uint32_t s_wbi[kNCW];
__shared__ uint64_t s_full[kNS];       // ring: slot landed
__shared__ uint64_t s_empty[kNS];      // ring: slot consumed by every consumer warp
__shared__ volatile int s_abort;       // a wait gave up: every role stops
__shared__ uint32_t s_tok[2];          // reduced greedy token; last-task flag of a merge

MYOS_DEV uint8_t* smem_base() {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  return smem_raw;
}
MYOS_DEV uint8_t* ring_slot(const StreamArgs& a, int slot) {
  return smem_base() + (size_t)slot * a.slot_bytes;
}
MYOS_DEV float* scr(const StreamArgs& a) { return reinterpret_cast<float*>(smem_base() + a.off_scr); }
MYOS_DEV float* part(const StreamArgs& a) { return reinterpret_cast<float*>(smem_base() + a.off_part); }
MYOS_DEV float* resrows(const StreamArgs& a) { return reinterpret_cast<float*>(smem_base() + a.off_res); }
MYOS_DEV float* biasrows(const StreamArgs& a) {
  return reinterpret_cast<float*>(smem_base() + a.off_bias);
}
MYOS_DEV const StreamLayer& layer(const StreamArgs& a, int l) {
  return reinterpret_cast<const StreamLayer*>(smem_base() + a.off_lay)[l];
}

struct Geo {
  const uint16_t* w0;
  const uint16_t* w1;
  int M, K, NR, rps, wpr;
};

MYOS_DEV Geo geo(const StreamArgs& a, int kind, int l) {
  Geo g;
  g.w1 = nullptr;
  g.NR = 1;
  g.rps = a.rps[kind];
  g.wpr = a.wpr[kind];
  if (kind == SK_HEAD) {
    g.w0 = a.head_w;
    g.M = a.V;
    g.K = a.H;
    return g;
  }
  const StreamLayer& L = layer(a, l);
  if (kind == SK_QKV) {
    g.w0 = L.wqkv;
    g.M = a.qd + 2 * a.kvd;
    g.K = a.H;
  } else if (kind == SK_O) {
    g.w0 = L.wo;
    g.M = a.H;
    g.K = a.qd;
  } else if (kind == SK_GU) {
    g.w0 = L.wg;
    g.w1 = L.wu;
    g.M = a.I;
    g.K = a.H;
    g.NR = 2;
  } else {
    g.w0 = L.wd;
    g.M = a.H;
    g.K = a.I;
  }
  return g;
}

MYOS_DEV void rows_of(int M, int grid, int* r0, int* r1) {
  *r0 = (int)((long long)blockIdx.x * M / grid);
  *r1 = (int)((long long)(blockIdx.x + 1) * M / grid);
}

// Raise the error bit once and stop every role of this CTA.
MYOS_DEV void give_up(const StreamArgs& a) {
  if (!s_abort) {
    s_abort = 1;
    atomicOr(&a.ctl->err, kErrStream);
  }
}

// Bounded wait on a ring mbarrier phase; false when the CTA aborted or the
// bound passed.
MYOS_DEV bool ring_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (s_abort) return false;
      if (global_ns() - t0 > limit_ns) return false;
    }
  }
}

// ---------------------------------------------------------------- trace
MYOS_DEV uint64_t* trace_row(const StreamArgs& a, int t, int ph) {
  return (a.trace && t == a.nsteps - 1) ? a.trace + ((size_t)blockIdx.x * (5 * a.L + 1) + ph) * 8
                                        : nullptr;
}
MYOS_DEV void mark(uint64_t* row, int k) {
  if (row && threadIdx.x == 0) row[k] = global_ns();
}

// Optional per-slot stamps of the last step: [grid][kSlotTrace][4] =
// (producer issued, consumer warp 0 saw it landed, warp 0 released it, -).
constexpr int kSlotTrace = 640;
MYOS_DEV void slot_mark(const StreamArgs& a, uint32_t seq, int k) {
  if (!a.strace) return;
  const uint32_t base = a.strace_seq0;
  if (seq < base || seq - base >= (uint32_t)kSlotTrace) return;
  a.strace[((size_t)blockIdx.x * kSlotTrace + (seq - base)) * 4 + k] = global_ns();
}

// ---------------------------------------------------------------- producer
// Position in the stream of ring slots: token step t, layer l, matrix kind
// k, first row r of the slot (rows [r, min(r + rps, r1)) of this CTA).
struct Cursor {
  int t, l, k, r, r1;
};

MYOS_DEV void cur_phase(const StreamArgs& a, Cursor& c) {
  // first phase at or after (t, l, k) in which this CTA owns rows
  for (;;) {
    if (c.t >= a.nsteps) return;
    if (c.k > SK_DOWN && !(c.k == SK_HEAD && c.l == a.L && a.head)) {
      // past the layers' kinds: next layer, or the head, or the next step
      if (c.l + 1 < a.L) {
        c.l += 1;
        c.k = SK_QKV;
      } else if (c.l + 1 == a.L && a.head) {
        c.l = a.L;
        c.k = SK_HEAD;
      } else {
        c.t += 1;
        c.l = 0;
        c.k = SK_QKV;
      }
      continue;
    }
    const Geo g = geo(a, c.k, c.k == SK_HEAD ? 0 : c.l);
    int r0, r1;
    rows_of(g.M, a.grid, &r0, &r1);
    if (r0 < r1) {
      c.r = r0;
      c.r1 = r1;
      return;
    }
    c.k += 1;
  }
}

MYOS_DEV void cur_next(const StreamArgs& a, Cursor& c) {
  c.r += a.rps[c.k];
  if (c.r < c.r1) return;
  if (c.k == SK_HEAD) {
    c.t += 1;
    c.l = 0;
    c.k = SK_QKV;
  } else {
    c.k += 1;
  }
  cur_phase(a, c);
}

// Copy (or request into L2) the slot at c.
MYOS_DEV void cur_issue(const StreamArgs& a, const Cursor& c, int slot, bool to_l2) {
  const Geo g = geo(a, c.k, c.k == SK_HEAD ? 0 : c.l);
  const int n = min(g.rps, c.r1 - c.r);
  const uint32_t bytes = (uint32_t)((size_t)n * g.K * 2);
  const uint16_t* s0 = g.w0 + (size_t)c.r * g.K;
  if (to_l2) {
    prefetch_l2(s0, bytes);
    if (g.NR == 2) prefetch_l2(g.w1 + (size_t)c.r * g.K, bytes);
    return;
  }
  uint8_t* dst = ring_slot(a, slot);
  mbar_arrive_expect_tx(&s_full[slot], bytes * (uint32_t)g.NR);
  bulk_g2s(dst, s0, bytes, &s_full[slot]);
  if (g.NR == 2)
    bulk_g2s(dst + (size_t)g.rps * g.K * 2, g.w1 + (size_t)c.r * g.K, bytes, &s_full[slot]);
}

// At most a.inflight copies outstanding (issued, not landed): one ~45 KB
// copy per SM already keeps HBM streaming, and more only lengthen every
// queue. Landed slots wait in the ring for the consumers. With a.l2_la > 0
// the slot that many places ahead is also requested into L2.
MYOS_DEV void producer(const StreamArgs& a) {
  uint32_t seq = 0;
  bool ok = true;
  Cursor c = {0, 0, SK_QKV, 0, 0}, pf = {0, 0, SK_QKV, 0, 0};
  cur_phase(a, c);
  cur_phase(a, pf);
  for (int i = 0; i < a.l2_la && pf.t < a.nsteps; ++i) {
    cur_issue(a, pf, 0, true);
    cur_next(a, pf);
  }
  while (c.t < a.nsteps) {
    const int slot = (int)(seq % kNS);
    if (seq >= (uint32_t)kNS && !ring_wait(&s_empty[slot], ((seq / kNS) - 1u) & 1u, a.wait_ns)) {
      ok = false;
      break;
    }
    if (seq >= (uint32_t)a.inflight) {
      const uint32_t q = seq - (uint32_t)a.inflight;
      if (!ring_wait(&s_full[q % kNS], (q / kNS) & 1u, a.wait_ns)) {
        ok = false;
        break;
      }
    }
    cur_issue(a, c, slot, false);
    slot_mark(a, seq, 0);
    ++seq;
    cur_next(a, c);
    if (a.l2_la && pf.t < a.nsteps) {
      cur_issue(a, pf, 0, true);
      cur_next(a, pf);
    }
  }
  if (!ok) give_up(a);
  // Every copy issued must land before the CTA exits (the consumers wait for
  // all of them on the normal path; after an abort this drains them).
  const uint32_t first = seq > (uint32_t)kNS ? seq - kNS : 0u;
  for (uint32_t q = first; q < seq; ++q) mbar_wait(&s_full[q % kNS], (q / kNS) & 1u, nullptr, 0u);
}

// ---------------------------------------------------------------- grid barrier
// One 64-bit arrival counter per context, never reset: every CTA adds 1 per
// barrier, so after barrier n of this CTA (counting all launches, flags[b]
// holds the count at launch start) the counter reaches grid * n once every
// CTA has arrived. Arrival: the consumer barrier orders every consumer
// thread's writes before thread 0's release add (cumulative at gpu scope).
// One poller per CTA keeps the counter's line from being flooded.
MYOS_DEV void red_release_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
MYOS_DEV unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

MYOS_DEV void arrive(const StreamArgs& a, uint32_t count, uint64_t* tr = nullptr) {
  csync();
  if (threadIdx.x == 0) {
    mark(tr, 3);
    red_release_add(a.bar, 1ull);
    mark(tr, 4);
  }
  (void)count;
}

// Wait until every CTA arrived at `count` barriers. The outcome is read
// after the consumer barrier, so it is uniform.
MYOS_DEV bool wait_all(const StreamArgs& a, uint32_t count) {
  if (threadIdx.x == 0) {
    const unsigned long long target = (unsigned long long)a.grid * count;
    if (ld_acquire64(a.bar) < target) {
      const uint64_t t0 = global_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire64(a.bar) >= target) break;
        if ((i & 63u) == 0) {
          if (s_abort || (*(volatile uint32_t*)&a.ctl->err & kErrStream) ||
              global_ns() - t0 > a.wait_ns) {
            give_up(a);
            break;
          }
        }
      }
    }
  }
  csync();
  return !s_abort;
}

// ---------------------------------------------------------------- reductions
MYOS_DEV float cons_sum(float v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) s_red[warp] = v;
  csync();
  if (warp == 0) {
    float s = lane < kNCW ? s_red[lane] : 0.0f;
    s = warp_sum(s);
    if (lane == 0) s_red[32] = s;
  }
  csync();
  const float s = s_red[32];
  csync();
  return s;
}

// ---------------------------------------------------------------- staging
// Split layout (K % 8 == 0): chunk c's first four values at xs[4c], its last
// four at xs[K/2 + 4c]; a lane's two float4 reads hit distinct banks. The
// norm weight gamma [K] sits right after xs (gs = xs + K), the raw bf16
// embedding row after that.

// Before the phase's barrier: the norm weight depends on no kernel.
MYOS_DEV void gamma_issue(float* gs, const float* gamma, int K) {
  for (int c = threadIdx.x; c < (K >> 2); c += kCT) cpa16(gs + 4 * c, gamma + 4 * c);
}

// xs <- x (f32, written by other CTAs: cp.async reads through L2) or the
// bf16 embedding row erow; with norm, x = gamma * (x * inv), inv = 1 /
// sqrtf(mean(x^2) + eps) (gamma already issued into gs). raw_store (CTA 0 of
// the first layer): the un-normalised row is also written there (the
// residual stream starts as the embedding). keep: the un-normalised elements
// [k0, k1) also go there (this CTA's residual rows, for the o_proj and down
// epilogues, so they need no load of their own).
MYOS_DEV void stage(float* xs, int K, const float* x, const uint16_t* erow, bool norm, float eps,
                    float* raw_store, float* keep, int k0, int k1, uint64_t* tr) {
  const int nchunk = K >> 3, half = K >> 1;
  float* gs = xs + K;
  uint16_t* eb = reinterpret_cast<uint16_t*>(gs + K);
  for (int c = threadIdx.x; c < nchunk; c += kCT) {
    if (erow) {
      cpa16(eb + 8 * c, erow + 8 * c);
    } else {
      cpa16(xs + 4 * c, x + 8 * c);
      cpa16(xs + half + 4 * c, x + 8 * c + 4);
    }
  }
  cpa_wait_all();  // this thread's chunks (and its share of gamma)
  mark(tr, 5);
  float ss = 0.0f;
  for (int c = threadIdx.x; c < nchunk; c += kCT) {
    float4* lo = reinterpret_cast<float4*>(xs + 4 * c);
    float4* hi = reinterpret_cast<float4*>(xs + half + 4 * c);
    if (erow) {
      const uint4 u = *reinterpret_cast<const uint4*>(eb + 8 * c);
      *lo = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
      *hi = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
    }
    const float4 p = *lo, q = *hi;
    if (raw_store) {
      reinterpret_cast<float4*>(raw_store)[2 * c] = p;
      reinterpret_cast<float4*>(raw_store)[2 * c + 1] = q;
    }
    if (keep && 8 * c + 8 > k0 && 8 * c < k1) {
      const float v[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (8 * c + e >= k0 && 8 * c + e < k1) keep[8 * c + e - k0] = v[e];
    }
    if (norm) {
      ss = fmaf(p.x, p.x, ss);
      ss = fmaf(p.y, p.y, ss);
      ss = fmaf(p.z, p.z, ss);
      ss = fmaf(p.w, p.w, ss);
      ss = fmaf(q.x, q.x, ss);
      ss = fmaf(q.y, q.y, ss);
      ss = fmaf(q.z, q.z, ss);
      ss = fmaf(q.w, q.w, ss);
    }
  }
  if (norm) {
    ss = cons_sum(ss);
    mark(tr, 6);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
    for (int c = threadIdx.x; c < nchunk; c += kCT) {
      float4* lo = reinterpret_cast<float4*>(xs + 4 * c);
      float4* hi = reinterpret_cast<float4*>(xs + half + 4 * c);
      const float4 p = *lo, q = *hi;
      const float4 ga = *reinterpret_cast<const float4*>(gs + 8 * c);
      const float4 gb = *reinterpret_cast<const float4*>(gs + 8 * c + 4);
      *lo = make_float4(__fmul_rn(ga.x, __fmul_rn(p.x, inv)), __fmul_rn(ga.y, __fmul_rn(p.y, inv)),
                        __fmul_rn(ga.z, __fmul_rn(p.z, inv)), __fmul_rn(ga.w, __fmul_rn(p.w, inv)));
      *hi = make_float4(__fmul_rn(gb.x, __fmul_rn(q.x, inv)), __fmul_rn(gb.y, __fmul_rn(q.y, inv)),
                        __fmul_rn(gb.z, __fmul_rn(q.z, inv)), __fmul_rn(gb.w, __fmul_rn(q.w, inv)));
    }
  }
  csync();
}

// o_proj input as the merge of the split-KV partials of the splits holding
// keys 0..pos. Per head h (KV head g = h / G): M = max_q m_q, f_q =
// expf(m_q - M), L = sum_q l_q f_q, x = (sum_q o_q f_q) / L, sums in split
// order (the reference's e / sum, gqa.rs:283-307, reassociated).
MYOS_DEV void stage_merge(const StreamArgs& a, float* xs, int pos) {
  const int G = a.G, d = kD, ns = a.nsplit, Hq = a.Hq, Hkv = a.Hkv, K = a.qd;
  int ne = (pos + a.chunk) / a.chunk;
  if (ne > ns) ne = ns;
  float* po = xs + K;                         // [Hkv][ns][G][d] (valid splits)
  float* fs = po + (size_t)Hkv * ns * G * d;  // [Hkv][ns][G]
  float* ls = fs + Hkv * ns * G;
  float* Ls = ls + Hkv * ns * G;              // [Hq]
  const int per_g = ne * G * d;
  const int q4 = per_g >> 2;
  for (int i = threadIdx.x; i < Hkv * q4; i += kCT) {
    const int g = i / q4, r = i - g * q4;
    const size_t off = (size_t)g * ns * G * d + 4 * (size_t)r;
    cpa16(po + off, a.part_o + off);
  }
  const int per_m = ne * G;
  for (int i = threadIdx.x; i < Hkv * per_m; i += kCT) {
    const int g = i / per_m, r = i - g * per_m;
    const int off = g * ns * G + r;
    fs[off] = __ldcg(a.part_m + off);
    ls[off] = __ldcg(a.part_l + off);
  }
  cpa_wait_all();
  csync();
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
  csync();
  for (int o = threadIdx.x; o < K; o += kCT) {
    const int h = o / d, e = o - h * d, g = h / G, hh = h - g * G;
    float O = 0.0f;
    for (int q = 0; q < ne; ++q) {
      const int i = (g * ns + q) * G + hh;
      O = fmaf(po[(size_t)i * d + e], fs[i], O);
    }
    const float v = __fdiv_rn(O, Ls[h]);
    const int c = o >> 3, r = o & 7;
    xs[r < 4 ? (c * 4 + r) : ((K >> 1) + c * 4 + (r - 4))] = v;
  }
  csync();
}

// ---------------------------------------------------------------- GEMV over ring slots
// A warp keeps the same chunk columns of the input for every row it
// computes in a phase (chunks c = c0 + lane + 32 j, j < nj, of [c0, c1)), so
// its lanes hold those input values in registers for the whole phase and
// read only weights from the ring: shared-memory traffic is then the bulk
// copy in and one read of each weight (re-reading the f32 input per weight
// chunk would triple it and make the consumers bound by shared memory).
constexpr int kXMax = 8;  // input chunks a lane holds (K / warps-per-row / 256 <= 8)

struct XRegs {
  float4 lo[kXMax], hi[kXMax];
  int nj;     // chunks this lane holds
  int cbase;  // c0 + lane
};

MYOS_DEV void x_load(XRegs& x, const float* xs, int K, int c0, int c1, int lane) {
  const float4* xlo = reinterpret_cast<const float4*>(xs);
  const float4* xhi = reinterpret_cast<const float4*>(xs + (K >> 1));
  x.cbase = c0 + lane;
  x.nj = x.cbase < c1 ? (c1 - x.cbase + 31) / 32 : 0;
#pragma unroll
  for (int j = 0; j < kXMax; ++j) {
    if (j < x.nj) {
      x.lo[j] = xlo[x.cbase + 32 * j];
      x.hi[j] = xhi[x.cbase + 32 * j];
    }
  }
}

// Row i of a slot (NR matrices: rows of matrix r at offset r * rps * K * 2)
// against the lane's input chunks: weight loads of four chunks issued at
// once, two accumulators per matrix, then the warp's shuffle tree.
template <int NR>
MYOS_DEV void dot_row(const uint8_t* sp, int rps, int K, int i, const XRegs& x, float& o0,
                      float& o1) {
  const size_t rowb = (size_t)K * 2;
  const uint4* w0 = reinterpret_cast<const uint4*>(sp + (size_t)i * rowb) + x.cbase;
  const uint4* w1 = reinterpret_cast<const uint4*>(sp + (size_t)(rps + i) * rowb) + x.cbase;
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
  for (int h = 0; h < kXMax; h += 4) {
    uint4 u0[4], u1[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (h + j < x.nj) {
        u0[j] = w0[32 * (h + j)];
        if (NR == 2) u1[j] = w1[32 * (h + j)];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (h + j < x.nj) {
        if (j & 1) {
          a1 = dot8(u0[j], x.lo[h + j], x.hi[h + j], a1);
          if (NR == 2) b1 = dot8(u1[j], x.lo[h + j], x.hi[h + j], b1);
        } else {
          a0 = dot8(u0[j], x.lo[h + j], x.hi[h + j], a0);
          if (NR == 2) b0 = dot8(u1[j], x.lo[h + j], x.hi[h + j], b0);
        }
      }
    }
  }
  o0 = warp_sum(a0 + a1);
  if (NR == 2) o1 = warp_sum(b0 + b1);
}

struct Best {
  float v;
  uint32_t i;
};

MYOS_DEV void keep_best(Best& b, float v, uint32_t row) {
  if (better(v, row, b.v, b.i)) {
    b.v = v;
    b.i = row;
  }
}

// Epilogue of one finished row (one thread writes).
template <int KIND>
MYOS_DEV void epi_row(const StreamArgs& a, int row, int r0, float v, float u) {
  if (KIND == SK_QKV) a.qkv[row] = __fadd_rn(v, biasrows(a)[row - r0]);
  if (KIND == SK_O || KIND == SK_DOWN) a.resid[row] = __fadd_rn(resrows(a)[row - r0], v);
  if (KIND == SK_GU) a.act[row] = silu_mul(v, u);
  if (KIND == SK_HEAD) a.logits[row] = v;
}

// Consume this phase's ring slots. Rows with warps-per-row > 1 leave
// partials in shared memory, summed in part order after the last slot. A
// failed wait never skips a consumer barrier: the slot loop runs out, and
// the outcome is read from the shared abort flag after the final barrier,
// so every consumer thread returns the same answer.
template <int KIND>
MYOS_DEV bool consume_gemv(const StreamArgs& a, int l, uint32_t& seq, Best& best) {
  constexpr int NR = KIND == SK_GU ? 2 : 1;
  const Geo g = geo(a, KIND, l);
  int r0, r1;
  rows_of(g.M, a.grid, &r0, &r1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpr = g.wpr, rg = kNCW / wpr;
  const int rr = warp / wpr, pt = warp - rr * wpr;
  const int nchunk = g.K >> 3;
  const int c0 = pt * nchunk / wpr, c1 = (pt + 1) * nchunk / wpr;
  XRegs x;
  x_load(x, scr(a), g.K, c0, c1, lane);
  for (int r = r0; r < r1; r += g.rps) {
    const int n = min(g.rps, r1 - r);
    const int slot = (int)(seq % kNS);
    // every lane waits; the warp proceeds only if all saw the slot filled
    if (!__all_sync(0xffffffffu, ring_wait(&s_full[slot], (seq / kNS) & 1u, a.wait_ns))) {
      if (lane == 0) give_up(a);
      break;
    }
    if (warp == 0 && lane == 0) slot_mark(a, seq, 1);
    const uint8_t* sp = ring_slot(a, slot);
    if (rr < rg) {
      for (int i = rr; i < n; i += rg) {
        float o0, o1 = 0.f;
        dot_row<NR>(sp, g.rps, g.K, i, x, o0, o1);
        const int row = r + i;
        if (wpr == 1) {
          if (lane == 0) epi_row<KIND>(a, row, r0, o0, o1);
          if (KIND == SK_HEAD) keep_best(best, o0, (uint32_t)row);  // same value in every lane
        } else if (lane == 0) {
          float* pp = part(a) + ((size_t)(row - r0) * wpr + pt) * NR;
          pp[0] = o0;
          if (NR == 2) pp[1] = o1;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&s_empty[slot]);
    if (warp == 0 && lane == 0) slot_mark(a, seq, 2);
    ++seq;
  }
  csync();  // slots consumed (the staged input may be overwritten after this)
  if (s_abort) return false;
  if (wpr > 1) {
    for (int i = threadIdx.x; i < r1 - r0; i += kCT) {
      const float* pp = part(a) + (size_t)i * wpr * NR;
      float v = 0.f, u = 0.f;
      for (int p = 0; p < wpr; ++p) {
        v += pp[p * NR];
        if (NR == 2) u += pp[p * NR + 1];
      }
      epi_row<KIND>(a, r0 + i, r0, v, u);
      if (KIND == SK_HEAD) keep_best(best, v, (uint32_t)(r0 + i));
    }
  }
  return true;
}

// ---------------------------------------------------------------- attention
template <typename KT>
MYOS_DEV float4 ld4(const KT* p);
template <>
MYOS_DEV float4 ld4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
MYOS_DEV float4 ld4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
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

// Attention scratch: qs [G][d] f32, K and V tiles [tile][ds] of the cache
// type (row stride ds = d + 16 bytes of padding), new k / v [d], cos / sin
// [d/2].
template <typename KT>
struct AttnSm {
  float* qs;
  KT* kt;
  KT* vt;
  float* kn;
  float* vn;
  float* cs;
  float* sn;
  static constexpr int ds = kD + 16 / (int)sizeof(KT);
  MYOS_DEV AttnSm(float* base, int G, int tile) {
    qs = base;
    kt = reinterpret_cast<KT*>(qs + G * kD);
    vt = kt + (size_t)tile * ds;
    kn = reinterpret_cast<float*>(vt + (size_t)tile * ds);
    vn = kn + kD;
    cs = vn + kD;
    sn = cs + kD / 2;
  }
};

// Cached keys [t0, t0 + nk) of this task except `skip` (this step's slot)
// into the tile, 16 bytes per copy.
template <typename KT>
MYOS_DEV void tile_issue(const AttnSm<KT>& s, const KT* kc, const KT* vc, int t0, int nk, int skip) {
  constexpr int per = 16 / sizeof(KT), ppr = kD / per;
  for (int i = threadIdx.x; i < nk * ppr; i += kCT) {
    const int tt = i / ppr, e = (i - tt * ppr) * per;
    if (t0 + tt == skip) continue;
    cpa16(s.kt + tt * s.ds + e, kc + (size_t)(t0 + tt) * kD + e);
    cpa16(s.vt + tt * s.ds + e, vc + (size_t)(t0 + tt) * kD + e);
  }
}

// Before the QKV barrier: the first tile's cached keys and the rotation row
// depend on nothing this step computes.
template <typename KT>
MYOS_DEV void attn_prefetch(const StreamArgs& a, int l, int pos) {
  const int task = blockIdx.x, g = task / a.nsplit, s = task - g * a.nsplit;
  const int kb = s * a.chunk, ke = min(kb + a.chunk, pos + 1);
  if (kb >= ke) return;
  AttnSm<KT> at(scr(a), a.G, a.tile);
  const size_t lo = (size_t)l * a.kv_layer_elems + (size_t)g * a.S * kD;
  const KT* kc = reinterpret_cast<const KT*>(a.kcache) + lo;
  const KT* vc = reinterpret_cast<const KT*>(a.vcache) + lo;
  tile_issue<KT>(at, kc, vc, kb, min(a.tile, ke - kb), pos);
  const float4* c4 = reinterpret_cast<const float4*>(a.cos_t + (size_t)pos * (kD / 2));
  const float4* s4 = reinterpret_cast<const float4*>(a.sin_t + (size_t)pos * (kD / 2));
  for (int i = threadIdx.x; i < kD / 8; i += kCT) {
    cpa16(reinterpret_cast<float4*>(at.cs) + i, c4 + i);
    cpa16(reinterpret_cast<float4*>(at.sn) + i, s4 + i);
  }
}

// One warp merges one head over the splits q < ne (global partials):
// M = max m_q, f_q = expf(m_q - M), L = sum l_q f_q, out = (sum o_q f_q) / L
// in split order.
MYOS_DEV void merge_head_global(const StreamArgs& a, int g, int h, int ne, int lane, float* out) {
  const int ns = a.nsplit, G = a.G;
  const size_t base = (size_t)g * ns * G + h;
  float M = -INFINITY;
  for (int q0 = 0; q0 < ne; q0 += 32)
    M = fmaxf(M, warp_max(q0 + lane < ne ? __ldcg(a.part_m + base + (size_t)(q0 + lane) * G) : -INFINITY));
  float Lp = 0.0f;
  float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q0 = 0; q0 < ne; q0 += 32) {
    const int q = q0 + lane;
    const float mq = q < ne ? __ldcg(a.part_m + base + (size_t)q * G) : -INFINITY;
    const float f = mq == -INFINITY ? 0.0f : expf(mq - M);
    if (q < ne) Lp = fmaf(__ldcg(a.part_l + base + (size_t)q * G), f, Lp);
    const int nr = min(32, ne - q0);
    for (int u = 0; u < nr; ++u) {
      const float fu = __shfl_sync(0xffffffffu, f, u);
      const float4 po = ldcg4(a.part_o + (base + (size_t)(q0 + u) * G) * kD + 4 * lane);
      O.x = fmaf(po.x, fu, O.x);
      O.y = fmaf(po.y, fu, O.y);
      O.z = fmaf(po.z, fu, O.z);
      O.w = fmaf(po.w, fu, O.w);
    }
  }
  const float L = warp_sum(Lp);
  *reinterpret_cast<float4*>(out + 4 * lane) =
      make_float4(__fdiv_rn(O.x, L), __fdiv_rn(O.y, L), __fdiv_rn(O.z, L), __fdiv_rn(O.w, L));
}

// Split-KV task (KV head g, split s) of layer l at position pos: RoPE of q
// and the new key (rope.rs:145-184), the KV store at pos, then for each
// 32-key tile: scores (q . k) * scale (gqa.rs:189-191) lane per key, an
// online softmax per head (one warp each), p . v lane per 4 dims. Writes the
// task's (unnormalised output, max, sum) per head; without the staging
// merge the last task of the KV head merges them into attn.
template <typename KT>
MYOS_DEV void attn_task(const StreamArgs& a, int l, int pos) {
  const int task = blockIdx.x, G = a.G, ns = a.nsplit;
  const int g = task / ns, s = task - g * ns;
  const int kb = s * a.chunk, ke = min(kb + a.chunk, pos + 1);
  if (kb >= ke) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int half = kD / 2;
  AttnSm<KT> at(scr(a), G, a.tile);
  constexpr int ds = AttnSm<KT>::ds;
  const size_t lo = (size_t)l * a.kv_layer_elems + (size_t)g * a.S * kD;
  KT* kc = reinterpret_cast<KT*>(a.kcache) + lo;
  KT* vc = reinterpret_cast<KT*>(a.vcache) + lo;
  const bool has_new = pos >= kb && pos < ke;
  // q of the G heads; the new k and v when this split holds position pos
  const int nq4 = G * kD / 4, d4 = kD / 4;
  const float4* q4 = reinterpret_cast<const float4*>(a.qkv + (size_t)g * G * kD);
  const float4* k4 = reinterpret_cast<const float4*>(a.qkv + (size_t)(a.Hq + g) * kD);
  const float4* v4 = reinterpret_cast<const float4*>(a.qkv + (size_t)(a.Hq + a.Hkv + g) * kD);
  for (int i = threadIdx.x; i < nq4 + (has_new ? 2 * d4 : 0); i += kCT) {
    if (i < nq4) cpa16(reinterpret_cast<float4*>(at.qs) + i, q4 + i);
    else if (i < nq4 + d4) cpa16(reinterpret_cast<float4*>(at.kn) + (i - nq4), k4 + (i - nq4));
    else cpa16(reinterpret_cast<float4*>(at.vn) + (i - nq4 - d4), v4 + (i - nq4 - d4));
  }
  cpa_wait_all();
  csync();
  // NeoX rotation in place: y0 = x0*c - x1*s, y1 = x1*c + x0*s
  for (int i = threadIdx.x; i < (G + (has_new ? 1 : 0)) * half; i += kCT) {
    const int h = i / half, p = i - h * half;
    float* x = h < G ? at.qs + h * kD : at.kn;
    const float x0 = x[p], x1 = x[p + half];
    x[p] = __fsub_rn(__fmul_rn(x0, at.cs[p]), __fmul_rn(x1, at.sn[p]));
    x[p + half] = __fadd_rn(__fmul_rn(x1, at.cs[p]), __fmul_rn(x0, at.sn[p]));
  }
  csync();
  if (has_new) {  // KvCache::store for this position, then the tile copy of it
    for (int e = threadIdx.x; e < kD; e += kCT) {
      const KT kq = kv_from<KT>(at.kn[e]), vq = kv_from<KT>(at.vn[e]);
      kc[(size_t)pos * kD + e] = kq;
      vc[(size_t)pos * kD + e] = vq;
      if (pos - kb < a.tile) {
        at.kt[(pos - kb) * ds + e] = kq;
        at.vt[(pos - kb) * ds + e] = vq;
      }
    }
    csync();
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float m_run = -INFINITY, l_run = 0.0f;
  for (int t0 = kb; t0 < ke; t0 += a.tile) {
    const int nk = min(a.tile, ke - t0);
    if (t0 != kb) {  // later tiles (the first was prefetched)
      csync();
      tile_issue<KT>(at, kc, vc, t0, nk, pos);
      cpa_wait_all();
      if (has_new && pos >= t0 && pos < t0 + nk)
        for (int e = threadIdx.x; e < kD; e += kCT) {
          at.kt[(pos - t0) * ds + e] = kv_from<KT>(at.kn[e]);
          at.vt[(pos - t0) * ds + e] = kv_from<KT>(at.vn[e]);
        }
      csync();
    }
    if (warp < G) {
      const float* qh = at.qs + warp * kD;
      float sc = -INFINITY;
      if (lane < nk) {
        const KT* kr = at.kt + lane * ds;
        float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll 8
        for (int e = 0; e < kD; e += 4) {
          const float4 q = *reinterpret_cast<const float4*>(qh + e);
          const float4 k = ld4<KT>(kr + e);
          p0 = fmaf(q.x, k.x, p0);
          p1 = fmaf(q.y, k.y, p1);
          p2 = fmaf(q.z, k.z, p2);
          p3 = fmaf(q.w, k.w, p3);
        }
        sc = __fmul_rn((p0 + p1) + (p2 + p3), a.scale);
      }
      const float mn = fmaxf(m_run, warp_max(sc));
      const float cf = expf(m_run - mn);  // 0 on the first tile (m_run = -inf)
      const float p = lane < nk ? expf(sc - mn) : 0.0f;
      l_run = fmaf(l_run, cf, warp_sum(p));
      m_run = mn;
      acc.x *= cf;
      acc.y *= cf;
      acc.z *= cf;
      acc.w *= cf;
#pragma unroll 8
      for (int t = 0; t < nk; ++t) {
        const float pt = __shfl_sync(0xffffffffu, p, t);
        const float4 v = ld4<KT>(at.vt + t * ds + 4 * lane);
        acc.x = fmaf(pt, v.x, acc.x);
        acc.y = fmaf(pt, v.y, acc.y);
        acc.z = fmaf(pt, v.z, acc.z);
        acc.w = fmaf(pt, v.w, acc.w);
      }
    }
  }
  const size_t pb = ((size_t)g * ns + s) * G;  // partial row of (g, s, head 0)
  if (warp < G) {
    *reinterpret_cast<float4*>(a.part_o + (pb + warp) * kD + 4 * lane) = acc;
    if (lane == 0) {
      a.part_m[pb + warp] = m_run;
      a.part_l[pb + warp] = l_run;
    }
  }
  if (!a.merge_in_stage) {
    const int ne = min(ns, (pos + a.chunk) / a.chunk);  // splits holding keys
    csync();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(a.attn_cnt + g, 1u);
      s_tok[1] = prev == (unsigned)(ne - 1);  // this task is the last of KV head g
    }
    csync();
    if (s_tok[1]) {
      __threadfence();
      if (warp < G) merge_head_global(a, g, warp, ne, lane, a.attn + ((size_t)g * G + warp) * kD);
      if (threadIdx.x == 0) a.attn_cnt[g] = 0u;
    }
  }
}

// ---------------------------------------------------------------- head
// This CTA's first maximum goes to the candidates; after the barrier every
// CTA takes the first maximum over all candidates (the (value desc, index
// asc) order is total, so the order of comparisons does not matter).
MYOS_DEV void head_candidate(const StreamArgs& a, Best best) {
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, best.i, o);
    if (better(ov, oi, best.v, best.i)) {
      best.v = ov;
      best.i = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_wbv[warp] = best.v;
    s_wbi[warp] = best.i;
  }
  csync();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    for (int w = 0; w < kNCW; ++w)
      if (better(s_wbv[w], s_wbi[w], v, i)) {
        v = s_wbv[w];
        i = s_wbi[w];
      }
    a.cand_val[blockIdx.x] = v;
    a.cand_idx[blockIdx.x] = i;
  }
}

// The greedy token (0 when no logit qualifies).
MYOS_DEV uint32_t head_pick(const StreamArgs& a) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    for (int q = lane; q < a.grid; q += 32) {
      const float pv = __ldcg(a.cand_val + q);
      const uint32_t pi = __ldcg(a.cand_idx + q);
      if (better(pv, pi, v, i)) {
        v = pv;
        i = pi;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (better(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (lane == 0) s_tok[0] = i == 0xffffffffu ? 0u : i;
  }
  csync();
  const uint32_t tok = s_tok[0];
  csync();  // s_tok is rewritten by the next head
  return tok;
}

// ---------------------------------------------------------------- consumers
template <typename KT>
MYOS_DEV void consumers(const StreamArgs& a) {
  const uint32_t pos0 = a.ctl->pos, step0 = a.ctl->step;
  uint32_t argmax = a.ctl->argmax;
  uint32_t nbar = __ldcg(a.flags + blockIdx.x);  // barriers this CTA arrived at so far
  uint32_t seq = 0;
  const bool attn_cta = (int)blockIdx.x < a.Hkv * a.nsplit;
  uint32_t fed = 0;
  int hr0, hr1;  // this CTA's rows of the hidden-width outputs (o_proj, down)
  rows_of(a.H, a.grid, &hr0, &hr1);
  for (int t = 0; t < a.nsteps; ++t) {
    const int pos = (int)(pos0 + t);
    const uint32_t tok = a.feed ? a.feed[step0 + t] : argmax;
    fed = tok;
    for (int l = 0; l < a.L; ++l) {
      Best best = {-INFINITY, 0xffffffffu};
      // ---- QKV: RMSNorm(ln1) of the residual (layer 0: the token's embedding row)
      {
        uint64_t* tr = trace_row(a, t, 5 * l);
        gamma_issue(scr(a) + a.H, layer(a, l).ln1, a.H);
        {  // bias rows: depend on nothing, loaded before the barrier
          int q0, q1;
          rows_of(a.qd + 2 * a.kvd, a.grid, &q0, &q1);
          for (int i = threadIdx.x; i < q1 - q0; i += kCT)
            biasrows(a)[i] = __ldg(layer(a, l).bqkv + q0 + i);
        }
        if (t > 0 || l > 0) {
          if (!wait_all(a, nbar)) return;
        } else {
          csync();
        }
        mark(tr, 0);
        // the raw rows hr0..hr1 are the residual the o_proj epilogue adds to
        stage(scr(a), a.H, a.resid, l == 0 ? a.embed + (size_t)tok * a.H : nullptr, true, a.eps,
              (l == 0 && blockIdx.x == 0) ? a.resid : nullptr, resrows(a), hr0, hr1, tr);
        mark(tr, 1);
        if (!consume_gemv<SK_QKV>(a, l, seq, best)) return;
        mark(tr, 2);
        arrive(a, ++nbar, tr);
      }
      // ---- attention
      if (attn_cta) {
        uint64_t* tr = trace_row(a, t, 5 * l + 1);
        attn_prefetch<KT>(a, l, pos);
        if (!wait_all(a, nbar)) return;
        mark(tr, 0);
        attn_task<KT>(a, l, pos);
        mark(tr, 2);
      }
      arrive(a, ++nbar);
      // ---- o_proj: residual += W_o . attention output
      {
        uint64_t* tr = trace_row(a, t, 5 * l + 2);
        if (!wait_all(a, nbar)) return;
        mark(tr, 0);
        if (a.merge_in_stage) stage_merge(a, scr(a), pos);
        else stage(scr(a), a.qd, a.attn, nullptr, false, 0.f, nullptr, nullptr, 0, 0, tr);
        mark(tr, 1);
        if (!consume_gemv<SK_O>(a, l, seq, best)) return;
        mark(tr, 2);
        arrive(a, ++nbar, tr);
      }
      // ---- gate/up: RMSNorm(ln2), SiLU(gate) * up
      {
        uint64_t* tr = trace_row(a, t, 5 * l + 3);
        gamma_issue(scr(a) + a.H, layer(a, l).ln2, a.H);
        if (!wait_all(a, nbar)) return;
        mark(tr, 0);
        // the raw rows hr0..hr1 (after o_proj) are the residual of the down epilogue
        stage(scr(a), a.H, a.resid, nullptr, true, a.eps, nullptr, resrows(a), hr0, hr1, tr);
        mark(tr, 1);
        if (!consume_gemv<SK_GU>(a, l, seq, best)) return;
        mark(tr, 2);
        arrive(a, ++nbar, tr);
      }
      // ---- down: residual += W_down . act
      {
        uint64_t* tr = trace_row(a, t, 5 * l + 4);
        if (!wait_all(a, nbar)) return;
        mark(tr, 0);
        stage(scr(a), a.I, a.act, nullptr, false, 0.f, nullptr, nullptr, 0, 0, tr);
        mark(tr, 1);
        if (!consume_gemv<SK_DOWN>(a, l, seq, best)) return;
        mark(tr, 2);
        arrive(a, ++nbar, tr);
      }
    }
    // ---- head: final RMSNorm, logits, first maximum over the vocabulary
    if (a.head) {
      uint64_t* tr = trace_row(a, t, 5 * a.L);
      Best best = {-INFINITY, 0xffffffffu};
      gamma_issue(scr(a) + a.H, a.final_norm, a.H);
      if (!wait_all(a, nbar)) return;
      mark(tr, 0);
      stage(scr(a), a.H, a.resid, nullptr, true, a.eps, nullptr, nullptr, 0, 0, tr);
      mark(tr, 1);
      if (!consume_gemv<SK_HEAD>(a, 0, seq, best)) return;
      head_candidate(a, best);
      mark(tr, 2);
      arrive(a, ++nbar, tr);
      if (!wait_all(a, nbar)) return;
      const uint32_t next = head_pick(a);
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (a.rec_fed) a.rec_fed[step0 + t] = tok;
        if (a.rec_argmax) a.rec_argmax[step0 + t] = argmax;
      }
      argmax = next;
    }
  }
  // this CTA's barrier count for the next launch; cursor and greedy state
  if (threadIdx.x == 0) a.flags[blockIdx.x] = nbar;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    StepCtl* c = a.ctl;
    c->fed = fed;
    c->argmax = argmax;
    c->pos = pos0 + (uint32_t)a.nsteps;
    c->step = step0 + (uint32_t)a.nsteps;
  }
}

template <typename KT>
__global__ void __launch_bounds__(kST, 1) k_step_stream(const __grid_constant__ StreamArgs a) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < kNS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kNCW);
    }
    mbar_fence_init();
    s_abort = 0;
    s_tok[0] = s_tok[1] = 0u;
  }
  StreamLayer* lt = reinterpret_cast<StreamLayer*>(smem_base() + a.off_lay);
  for (int i = threadIdx.x; i < a.L; i += kST) lt[i] = a.layers[i];
  __syncthreads();
  if (threadIdx.x >= kCT) {
    if (threadIdx.x == kCT) producer(a);
    return;
  }
  consumers<KT>(a);
}

}  // namespace

int stream_threads() { return kST; }

size_t stream_smem_bytes(const StreamArgs& a) {
  return (size_t)a.off_lay + (size_t)a.L * sizeof(StreamLayer);
}

cudaError_t stream_configure(StreamArgs* a, int max_smem) {
  if (a->d != kD || a->G > kGMax || a->G < 1 || a->H % 256 || a->qd % 256 || a->I % 256 ||
      a->L > kMaxLayers || a->grid < 1 || a->grid > kCT || a->Hkv * a->nsplit > a->grid ||
      a->Hq > kCT)
    return cudaErrorNotSupported;
  const size_t kv = a->kv_bf16 ? 2 : 4;
  // scratch: the largest staged input (with gamma and the bf16 embedding row
  // after a hidden-width one), the attention tiles, the o_proj merge
  a->tile = 32;
  const size_t ds_bytes = kD * kv + 16;
  const size_t attn = (size_t)a->G * kD * 4 + 2 * (size_t)a->tile * ds_bytes + 3 * kD * 4;
  const size_t x = std::max((size_t)std::max(a->qd, a->I) * 4, (size_t)a->H * 10);
  const size_t merge = (size_t)a->qd * 4 + (size_t)a->Hkv * a->nsplit * a->G * (kD + 2) * 4 +
                       (size_t)a->Hq * 4;
  size_t scr = std::max(x, attn);
  if (a->merge_in_stage) scr = std::max(scr, merge);
  scr = (scr + 1023) / 1024 * 1024;
  // rows per slot for each matrix kind, then the split of rows over warps
  const int Ks[5] = {a->H, a->qd, a->H, a->I, a->H};
  const int NRs[5] = {1, 1, 2, 1, 1};
  const int Ms[5] = {a->qd + 2 * a->kvd, a->H, a->I, a->H, a->V};
  const size_t res = (size_t)(((a->H + a->grid - 1) / a->grid + 3) / 4 * 4) * 4;
  const size_t bia = (size_t)(((a->qd + 2 * a->kvd + a->grid - 1) / a->grid + 3) / 4 * 4) * 4;
  const size_t fixed = scr + res + bia + (size_t)a->L * sizeof(StreamLayer) + 2048;  // + static
  if ((size_t)max_smem <= fixed) return cudaErrorNotSupported;
  size_t slot = ((size_t)max_smem - fixed) / kNS;
  slot = slot / 1024 * 1024;
  size_t maxrow = 0;
  for (int k = 0; k < 5; ++k) maxrow = std::max(maxrow, (size_t)Ks[k] * 2 * NRs[k]);
  if (slot < maxrow) return cudaErrorNotSupported;
  int prt = 0;
  for (int k = 0; k < 5; ++k) {
    int r = (int)(slot / ((size_t)Ks[k] * 2 * NRs[k]));
    if (r > kNCW) r = kNCW;
    const int wpr = std::max(1, kNCW / r);
    // every lane holds at most kXMax input chunks of its part of a row
    if ((Ks[k] / 8 + wpr - 1) / wpr > 32 * kXMax) return cudaErrorNotSupported;
    a->rps[k] = r;
    a->wpr[k] = wpr;
    if (wpr > 1) prt = std::max(prt, ((Ms[k] + a->grid - 1) / a->grid) * wpr * NRs[k]);
  }
  // the slots shrink to what the kinds use (whole rows), in 1 KiB steps
  size_t used = 0;
  for (int k = 0; k < 5; ++k) used = std::max(used, (size_t)a->rps[k] * Ks[k] * 2 * NRs[k]);
  a->slot_bytes = (int)((used + 1023) / 1024 * 1024);
  a->ns = kNS;
  a->scr_bytes = (int)scr;
  a->part_floats = (prt + 3) / 4 * 4;
  a->off_scr = kNS * a->slot_bytes;
  a->off_part = a->off_scr + a->scr_bytes;
  a->off_res = a->off_part + a->part_floats * 4;
  a->off_bias = a->off_res + (int)res;
  a->off_lay = a->off_bias + (int)bia;
  const size_t smem = stream_smem_bytes(*a);
  if (smem + 2048 > (size_t)max_smem) return cudaErrorNotSupported;
  cudaError_t e = a->kv_bf16 ? cudaFuncSetAttribute(k_step_stream<__nv_bfloat16>,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                             : cudaFuncSetAttribute(k_step_stream<float>,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return e;
}

cudaError_t launch_step_stream(const StreamArgs& a, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(kST);
  cfg.dynamicSmemBytes = stream_smem_bytes(a);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.kv_bf16) return cudaLaunchKernelEx(&cfg, k_step_stream<__nv_bfloat16>, a);
  return cudaLaunchKernelEx(&cfg, k_step_stream<float>, a);
}

}  // namespace myos
