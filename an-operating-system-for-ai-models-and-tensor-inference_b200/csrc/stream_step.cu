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
//     4-slot shared-memory ring of ~45 KB slots. It waits only for a free
//     slot and keeps few copies outstanding (every queued request in the
//     memory system delays the consumers' dependent accesses), never for
//     activations, so HBM keeps filling the ring while the consumers wait on
//     the previous phase or run attention;
//   * consumer warps stage each phase's input vector in shared memory
//     (RMSNorm fused, crates/tensor_core/src/bf16.rs:231-270), dot every
//     ring slot's rows against it (bf16 weights promoted exactly, f32 FMA,
//     fixed reduction order: deterministic) and apply the epilogue: QKV bias
//     (bf16.rs:147-158), residual add (qwen25_block.rs:172-178), SiLU(gate)
//     * up (swiglu.rs:113-131,254-261), logits and the first-maximum argmax
//     (model_core/src/lib.rs:157-167);
//   * attention (gqa.rs:174-307) runs as split-KV tasks (KV head, key range)
//     on the first CTAs, with RoPE (rope.rs:145-184) and the KV store
//     (kv_cache.rs:149-302) fused; the tasks of a KV head then merge its
//     query heads' split partials among themselves;
//   * there is no grid barrier: every vector a phase hands to the next (q|k|v,
//     split partials, attention output, residual, activations, head
//     candidates) is stored as 8-byte words (value bits, epoch), where the
//     epoch numbers the producing phase. An aligned 8-byte store is seen
//     whole, so a reader polls the words it needs until each carries the
//     expected epoch: the data is its own flag, with no fence, counter or
//     separate staging round trip. Every phase needs the whole output of the
//     one before, so no word is rewritten while a reader may still want its
//     previous value. Every wait is bounded in time; a wait that gives up
//     raises kErrStream in ctl->err and ends the launch;
//   * several token steps run per launch: every CTA reduces the greedy token
//     from the per-CTA head candidates, so the next step starts without a
//     host round trip or a relaunch.
// With most of shared memory taken by the ring, L1 is small: the kernel keeps
// its state in registers (no local-memory stack).
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "stream_step.h"

namespace myos {

namespace {

#ifndef MYOS_STREAM_WARPS
#define MYOS_STREAM_WARPS 11  // consumer warps (12 warps in all: 168 registers a thread)
#endif
constexpr int kNCW = MYOS_STREAM_WARPS;
constexpr int kCT = kNCW * 32;      // consumer threads
constexpr int kST = kCT + 32;       // plus the producer warp
constexpr int kNS = 4;              // ring slots
constexpr int kGMax = 8;            // query heads per KV head
constexpr int kD = 128;             // head dim of the supported shapes
constexpr int kBar = 1;             // named barrier of the consumer warps
constexpr int kMaxLayers = 128;
constexpr int kDotBatch = 4;        // slot chunks a lane loads before its FMAs
constexpr int kStageMax = 3;        // 8-value chunks a consumer thread stages per round

MYOS_DEV void csync() { named_sync(kBar, kCT); }

MYOS_DEV void cpa16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
MYOS_DEV void cpa_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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

// ---------------------------------------------------------------- epoch words
MYOS_DEV uint64_t word(float v, uint32_t e) {
  return ((uint64_t)e << 32) | __float_as_uint(v);
}
MYOS_DEV float word_val(uint64_t w) { return __uint_as_float((uint32_t)w); }
MYOS_DEV uint32_t word_epoch(uint64_t w) { return (uint32_t)(w >> 32); }

MYOS_DEV void put_word(uint64_t* p, uint64_t w) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
MYOS_DEV void put_words2(uint64_t* p, uint64_t a, uint64_t b) {  // p 16-byte aligned
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
MYOS_DEV void get_words2(const uint64_t* p, uint64_t& a, uint64_t& b) {  // p 16-byte aligned
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
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
__shared__ uint32_t s_tok;             // reduced greedy token

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

// A word poll gave up (time bound, this CTA aborted, or another CTA raised
// the error bit): raise the bit here too.
MYOS_DEV bool poll_failed(const StreamArgs& a, uint64_t t0) {
  if (s_abort || (*(volatile uint32_t*)&a.ctl->err & kErrStream) || global_ns() - t0 > a.wait_ns) {
    give_up(a);
    return true;
  }
  return false;
}

// Two adjacent words (16-byte aligned) once both carry epoch e.
MYOS_DEV bool poll2(const StreamArgs& a, const uint64_t* p, uint32_t e, uint64_t& w0, uint64_t& w1) {
  get_words2(p, w0, w1);
  if (word_epoch(w0) == e && word_epoch(w1) == e) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    get_words2(p, w0, w1);
    if (word_epoch(w0) == e && word_epoch(w1) == e) return true;
    if ((i & 31u) == 0 && poll_failed(a, t0)) return false;
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

// At most a.inflight copies outstanding (issued, not landed): more only
// lengthen every queue. Landed slots wait in the ring for the consumers.
// With a.l2_la > 0 the slot that many places ahead is also requested into L2.
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

// The norm weight depends on no earlier phase: copied while the input is
// still being produced.
MYOS_DEV void gamma_issue(float* gs, const float* gamma, int K) {
  for (int c = threadIdx.x; c < (K >> 2); c += kCT) cpa16(gs + 4 * c, gamma + 4 * c);
}

// xs <- the words w[0..K) of epoch e (every thread polls its own chunks of 8
// values, all of its loads in flight at once, then reloads only stale pairs
// until each carries e), or the bf16 embedding row erow; with norm, x =
// gamma * (x * inv), inv = 1 / sqrtf(mean(x^2) + eps) (gamma already issued
// into gs). keep: the un-normalised elements [k0, k1) also go there (this
// CTA's residual rows, for the o_proj and down epilogues). Each thread
// reads back only the chunks it wrote, so no barrier is needed before the
// final one. Returns false (uniformly) when a poll gave up.
MYOS_DEV bool stage(const StreamArgs& a, float* xs, int K, const uint64_t* w, uint32_t e,
                    const uint16_t* erow, bool norm, float* keep, int k0, int k1, uint64_t* tr) {
  const int nchunk = K >> 3, half = K >> 1;
  float* gs = xs + K;
  uint16_t* eb = reinterpret_cast<uint16_t*>(gs + K);
  if (erow) {
    for (int c = threadIdx.x; c < nchunk; c += kCT) cpa16(eb + 8 * c, erow + 8 * c);
    cpa_wait_all();  // this thread's chunks (and its share of gamma)
    for (int c = threadIdx.x; c < nchunk; c += kCT) {
      const uint4 u = *reinterpret_cast<const uint4*>(eb + 8 * c);
      reinterpret_cast<float4*>(xs)[c] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
      reinterpret_cast<float4*>(xs + half)[c] = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
    }
  } else {
    // rounds of kStageMax chunks per thread (every load of a round in flight)
    const uint64_t t0 = global_ns();
    for (int base = 0; base < nchunk; base += kStageMax * kCT) {
      uint64_t v[kStageMax][8];
#pragma unroll
      for (int i = 0; i < kStageMax; ++i) {
        const int c = base + threadIdx.x + i * kCT;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c < nchunk) get_words2(w + 8 * c + 2 * j, v[i][2 * j], v[i][2 * j + 1]);
          else v[i][2 * j] = v[i][2 * j + 1] = (uint64_t)e << 32;
      }
      for (uint32_t it = 1;; ++it) {
        bool stale = false;
#pragma unroll
        for (int i = 0; i < kStageMax; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (word_epoch(v[i][2 * j]) != e || word_epoch(v[i][2 * j + 1]) != e) {
              stale = true;
              get_words2(w + 8 * (base + threadIdx.x + i * kCT) + 2 * j, v[i][2 * j], v[i][2 * j + 1]);
            }
        if (!stale) break;
        if ((it & 31u) == 0 && poll_failed(a, t0)) break;
      }
#pragma unroll
      for (int i = 0; i < kStageMax; ++i) {
        const int c = base + threadIdx.x + i * kCT;
        if (c < nchunk) {
          reinterpret_cast<float4*>(xs)[c] =
              make_float4(word_val(v[i][0]), word_val(v[i][1]), word_val(v[i][2]), word_val(v[i][3]));
          reinterpret_cast<float4*>(xs + half)[c] =
              make_float4(word_val(v[i][4]), word_val(v[i][5]), word_val(v[i][6]), word_val(v[i][7]));
        }
      }
      if (s_abort) break;
    }
    cpa_wait_all();  // this thread's share of gamma
  }
  mark(tr, 5);
  float ss = 0.0f;
  for (int c = threadIdx.x; c < nchunk; c += kCT) {
    const float4 p = reinterpret_cast<const float4*>(xs)[c];
    const float4 q = reinterpret_cast<const float4*>(xs + half)[c];
    if (keep && 8 * c + 8 > k0 && 8 * c < k1) {
      const float vv[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (8 * c + k >= k0 && 8 * c + k < k1) keep[8 * c + k - k0] = vv[k];
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
    ss = cons_sum(ss);  // gamma of every thread is in shared memory after this barrier
    mark(tr, 6);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
    for (int c = threadIdx.x; c < nchunk; c += kCT) {
      float4* lo = reinterpret_cast<float4*>(xs) + c;
      float4* hi = reinterpret_cast<float4*>(xs + half) + c;
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
  return !s_abort;
}

// ---------------------------------------------------------------- GEMV over ring slots
// Row i of a slot (NR matrices: rows of matrix r at offset r * rps * K * 2),
// chunks [c0, c1) of 16 bytes: lane-strided, loads of kDotBatch chunks
// issued at once, two accumulators per matrix, then the warp's shuffle tree.
template <int NR>
MYOS_DEV void dot_part(const uint8_t* sp, int rps, int K, int i, int c0, int c1, const float4* xlo,
                       const float4* xhi, int lane, float& o0, float& o1) {
  const size_t rowb = (size_t)K * 2;
  const uint4* w0 = reinterpret_cast<const uint4*>(sp + (size_t)i * rowb);
  const uint4* w1 = reinterpret_cast<const uint4*>(sp + (size_t)(rps + i) * rowb);
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
  for (int cb = c0 + lane; cb < c1; cb += 32 * kDotBatch) {
    uint4 u0[kDotBatch], u1[kDotBatch];
#pragma unroll
    for (int j = 0; j < kDotBatch; ++j) {
      const int c = cb + 32 * j;
      if (c < c1) {
        u0[j] = w0[c];
        if (NR == 2) u1[j] = w1[c];
      }
    }
#pragma unroll
    for (int j = 0; j < kDotBatch; ++j) {
      const int c = cb + 32 * j;
      if (c < c1) {
        const float4 lo = xlo[c], hi = xhi[c];
        if (j & 1) {
          a1 = dot8(u0[j], lo, hi, a1);
          if (NR == 2) b1 = dot8(u1[j], lo, hi, b1);
        } else {
          a0 = dot8(u0[j], lo, hi, a0);
          if (NR == 2) b0 = dot8(u1[j], lo, hi, b0);
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

// Epilogue of one finished row (one thread writes); e is this phase's epoch.
template <int KIND>
MYOS_DEV void epi_row(const StreamArgs& a, int row, int r0, float v, float u, uint32_t e) {
  if (KIND == SK_QKV) put_word(a.w_qkv + row, word(__fadd_rn(v, biasrows(a)[row - r0]), e));
  if (KIND == SK_O || KIND == SK_DOWN)
    put_word(a.w_resid + row, word(__fadd_rn(resrows(a)[row - r0], v), e));
  if (KIND == SK_GU) put_word(a.w_act + row, word(silu_mul(v, u), e));
  if (KIND == SK_HEAD) a.logits[row] = v;
}

// Consume this phase's ring slots. Rows with warps-per-row > 1 leave
// partials in shared memory, summed in part order after the last slot. A
// failed wait never skips a consumer barrier: the slot loop runs out, and
// the outcome is read from the shared abort flag after the final barrier,
// so every consumer thread returns the same answer.
template <int KIND>
MYOS_DEV bool consume_gemv(const StreamArgs& a, int l, uint32_t& seq, Best& best, uint32_t e) {
  constexpr int NR = KIND == SK_GU ? 2 : 1;
  const Geo g = geo(a, KIND, l);
  int r0, r1;
  rows_of(g.M, a.grid, &r0, &r1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpr = g.wpr, rg = kNCW / wpr;
  const int rr = warp / wpr, pt = warp - rr * wpr;
  const int nchunk = g.K >> 3;
  const int c0 = pt * nchunk / wpr, c1 = (pt + 1) * nchunk / wpr;
  const float4* xlo = reinterpret_cast<const float4*>(scr(a));
  const float4* xhi = reinterpret_cast<const float4*>(scr(a) + (g.K >> 1));
  for (int r = r0; r < r1; r += g.rps) {
    const int n = min(g.rps, r1 - r);
    const int slot = (int)(seq % kNS);
    // every lane waits; the warp proceeds only if all saw the slot filled
    if (!__all_sync(0xffffffffu, ring_wait(&s_full[slot], (seq / kNS) & 1u, a.wait_ns))) {
      if (lane == 0) give_up(a);
      break;
    }
    const uint8_t* sp = ring_slot(a, slot);
    if (rr < rg) {
      for (int i = rr; i < n; i += rg) {
        float o0, o1 = 0.f;
        dot_part<NR>(sp, g.rps, g.K, i, c0, c1, xlo, xhi, lane, o0, o1);
        const int row = r + i;
        if (wpr == 1) {
          if (lane == 0) epi_row<KIND>(a, row, r0, o0, o1, e);
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
      epi_row<KIND>(a, r0 + i, r0, v, u, e);
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

// Words of split partial (g, s, head h): o [d] then m, l.
MYOS_DEV uint64_t* part_words(const StreamArgs& a, int g, int s, int h) {
  return a.w_part + (((size_t)g * a.nsplit + s) * a.G + h) * (kD + 2);
}

// Split-KV task (KV head g, split s) of layer l at position pos: RoPE of q
// and the new key (rope.rs:145-184), the KV store at pos, then for each
// 32-key tile: scores (q . k) * scale (gqa.rs:189-191) lane per key, an
// online softmax per head (one warp each), p . v lane per 4 dims. Writes the
// task's (unnormalised output, max, sum) per head as words of epoch e; then
// the tasks that hold keys merge the KV head's query heads among themselves
// (head h by task h mod ne): M = max m_q, f_q = expf(m_q - M), L = sum l_q
// f_q, out = (sum o_q f_q) / L in split order (the reference's e / sum,
// gqa.rs:283-307, reassociated), written as attention-output words.
template <typename KT>
MYOS_DEV bool attn_task(const StreamArgs& a, int l, int pos, uint32_t e_qkv, uint32_t e) {
  const int task = blockIdx.x, G = a.G, ns = a.nsplit;
  const int g = task / ns, s = task - g * ns;
  const int kb = s * a.chunk, ke = min(kb + a.chunk, pos + 1);
  if (kb >= ke) return true;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int half = kD / 2;
  AttnSm<KT> at(scr(a), G, a.tile);
  constexpr int ds = AttnSm<KT>::ds;
  const size_t lo = (size_t)l * a.kv_layer_elems + (size_t)g * a.S * kD;
  KT* kc = reinterpret_cast<KT*>(a.kcache) + lo;
  KT* vc = reinterpret_cast<KT*>(a.vcache) + lo;
  const bool has_new = pos >= kb && pos < ke;
  // the first tile's cached keys and the rotation row depend on nothing this
  // step computes: in flight while q, k and v are polled
  tile_issue<KT>(at, kc, vc, kb, min(a.tile, ke - kb), pos);
  {
    const float4* c4 = reinterpret_cast<const float4*>(a.cos_t + (size_t)pos * half);
    const float4* s4 = reinterpret_cast<const float4*>(a.sin_t + (size_t)pos * half);
    for (int i = threadIdx.x; i < half / 4; i += kCT) {
      cpa16(reinterpret_cast<float4*>(at.cs) + i, c4 + i);
      cpa16(reinterpret_cast<float4*>(at.sn) + i, s4 + i);
    }
  }
  // q of the G heads; the new k and v when this split holds position pos:
  // every pair's load in flight at once, then only stale pairs reloaded
  {
    const int nq = G * kD, npair = (nq + (has_new ? 2 * kD : 0)) / 2;
    constexpr int kPairs = 4;  // (kGMax + 2) * kD / 2 pairs over the consumer threads
    uint64_t v[kPairs][2];
    const uint64_t* src[kPairs];
#pragma unroll
    for (int r = 0; r < kPairs; ++r) {
      const int i = 2 * ((int)threadIdx.x + r * kCT);
      src[r] = i < nq ? a.w_qkv + (size_t)g * G * kD + i
                      : (i < nq + kD ? a.w_qkv + (size_t)(a.Hq + g) * kD + (i - nq)
                                     : a.w_qkv + (size_t)(a.Hq + a.Hkv + g) * kD + (i - nq - kD));
      if (i / 2 < npair) get_words2(src[r], v[r][0], v[r][1]);
      else v[r][0] = v[r][1] = (uint64_t)e_qkv << 32;
    }
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
      bool stale = false;
#pragma unroll
      for (int r = 0; r < kPairs; ++r)
        if (word_epoch(v[r][0]) != e_qkv || word_epoch(v[r][1]) != e_qkv) {
          stale = true;
          get_words2(src[r], v[r][0], v[r][1]);
        }
      if (!stale) break;
      if ((it & 31u) == 0 && poll_failed(a, t0)) break;
    }
#pragma unroll
    for (int r = 0; r < kPairs; ++r) {
      const int i = 2 * ((int)threadIdx.x + r * kCT);
      if (i / 2 < npair) {
        float* dst = i < nq ? at.qs + i : (i < nq + kD ? at.kn + (i - nq) : at.vn + (i - nq - kD));
        dst[0] = word_val(v[r][0]);
        dst[1] = word_val(v[r][1]);
      }
    }
  }
  cpa_wait_all();
  csync();
  if (s_abort) return false;
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
    for (int i = threadIdx.x; i < kD; i += kCT) {
      const KT kq = kv_from<KT>(at.kn[i]), vq = kv_from<KT>(at.vn[i]);
      kc[(size_t)pos * kD + i] = kq;
      vc[(size_t)pos * kD + i] = vq;
      if (pos - kb < a.tile) {
        at.kt[(pos - kb) * ds + i] = kq;
        at.vt[(pos - kb) * ds + i] = vq;
      }
    }
    csync();
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float m_run = -INFINITY, l_run = 0.0f;
  for (int t0 = kb; t0 < ke; t0 += a.tile) {
    const int nk = min(a.tile, ke - t0);
    if (t0 != kb) {  // later tiles
      csync();
      tile_issue<KT>(at, kc, vc, t0, nk, pos);
      cpa_wait_all();
      if (has_new && pos >= t0 && pos < t0 + nk)
        for (int i = threadIdx.x; i < kD; i += kCT) {
          at.kt[(pos - t0) * ds + i] = kv_from<KT>(at.kn[i]);
          at.vt[(pos - t0) * ds + i] = kv_from<KT>(at.vn[i]);
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
        for (int i = 0; i < kD; i += 4) {
          const float4 q = *reinterpret_cast<const float4*>(qh + i);
          const float4 k = ld4<KT>(kr + i);
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
  if (warp < G) {
    uint64_t* pw = part_words(a, g, s, warp);
    put_words2(pw + 4 * lane, word(acc.x, e), word(acc.y, e));
    put_words2(pw + 4 * lane + 2, word(acc.z, e), word(acc.w, e));
    if (lane == 0) put_words2(pw + kD, word(m_run, e), word(l_run, e));
  }
  // merge: this task takes heads h = s, s + ne, ... of KV head g, one warp
  // each; every split's words of a round in flight at once
  const int ne = min(ns, (pos + a.chunk) / a.chunk);  // splits holding keys
  bool ok = true;
  for (int h = s + ne * warp; h < G && ok; h += ne * kNCW) {
    float M = -INFINITY, Lp = 0.0f, f = 0.0f;
    if (ne <= 32) {  // every split's (max, sum) in one round, lane q holding split q
      uint64_t wm = (uint64_t)e << 32, wl = (uint64_t)e << 32;
      if (lane < ne) ok = poll2(a, part_words(a, g, lane, h) + kD, e, wm, wl);
      ok = __all_sync(0xffffffffu, ok);
      const float mq = lane < ne ? word_val(wm) : -INFINITY;
      M = warp_max(mq);
      f = mq == -INFINITY ? 0.0f : expf(mq - M);
      if (lane < ne) Lp = word_val(wl) * f;
    } else {  // more splits than lanes: the maxima first, then the factors per round
      for (int q0 = 0; q0 < ne && ok; q0 += 32) {
        uint64_t wm = (uint64_t)e << 32, wl = (uint64_t)e << 32;
        if (q0 + lane < ne) ok = poll2(a, part_words(a, g, q0 + lane, h) + kD, e, wm, wl);
        ok = __all_sync(0xffffffffu, ok);
        M = fmaxf(M, warp_max(q0 + lane < ne ? word_val(wm) : -INFINITY));
      }
    }
    if (!ok) break;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int kB = 4;  // splits per round of o loads
    for (int q0 = 0; q0 < ne && ok; q0 += 32) {
      if (ne > 32) {
        uint64_t wm = (uint64_t)e << 32, wl = (uint64_t)e << 32;
        if (q0 + lane < ne) ok = poll2(a, part_words(a, g, q0 + lane, h) + kD, e, wm, wl);
        ok = __all_sync(0xffffffffu, ok);
        const float mq = q0 + lane < ne ? word_val(wm) : -INFINITY;
        f = mq == -INFINITY ? 0.0f : expf(mq - M);
        if (q0 + lane < ne) Lp = fmaf(word_val(wl), f, Lp);
      }
      const int nr = min(32, ne - q0);
      for (int u0 = 0; u0 < nr && ok; u0 += kB) {
        uint64_t o[kB][4];
#pragma unroll
        for (int u = 0; u < kB; ++u) {
          const uint64_t* po = part_words(a, g, q0 + u0 + u, h) + 4 * lane;
          if (u0 + u < nr) {
            get_words2(po, o[u][0], o[u][1]);
            get_words2(po + 2, o[u][2], o[u][3]);
          } else {
            o[u][0] = o[u][1] = o[u][2] = o[u][3] = (uint64_t)e << 32;
          }
        }
        const uint64_t t0 = global_ns();
        for (uint32_t it = 1;; ++it) {
          bool stale = false;
#pragma unroll
          for (int u = 0; u < kB; ++u) {
            const uint64_t* po = part_words(a, g, q0 + u0 + u, h) + 4 * lane;
            if (word_epoch(o[u][0]) != e || word_epoch(o[u][1]) != e) {
              stale = true;
              get_words2(po, o[u][0], o[u][1]);
            }
            if (word_epoch(o[u][2]) != e || word_epoch(o[u][3]) != e) {
              stale = true;
              get_words2(po + 2, o[u][2], o[u][3]);
            }
          }
          if (!stale) break;
          if ((it & 31u) == 0 && poll_failed(a, t0)) {
            ok = false;
            break;
          }
        }
#pragma unroll
        for (int u = 0; u < kB; ++u) {
          const float fu = __shfl_sync(0xffffffffu, f, (u0 + u) & 31);
          if (u0 + u < nr) {
            O.x = fmaf(word_val(o[u][0]), fu, O.x);
            O.y = fmaf(word_val(o[u][1]), fu, O.y);
            O.z = fmaf(word_val(o[u][2]), fu, O.z);
            O.w = fmaf(word_val(o[u][3]), fu, O.w);
          }
        }
        ok = __all_sync(0xffffffffu, ok);
      }
    }
    if (!ok) break;
    const float L = warp_sum(Lp);
    uint64_t* out = a.w_attn + ((size_t)g * G + h) * kD + 4 * lane;
    put_words2(out, word(__fdiv_rn(O.x, L), e), word(__fdiv_rn(O.y, L), e));
    put_words2(out + 2, word(__fdiv_rn(O.z, L), e), word(__fdiv_rn(O.w, L), e));
  }
  csync();
  return !s_abort;
}

// ---------------------------------------------------------------- head
// This CTA's first maximum goes to the candidate words; every CTA then takes
// the first maximum over all candidates (the (value desc, index asc) order
// is total, so the order of comparisons does not matter).
MYOS_DEV void head_candidate(const StreamArgs& a, Best best, uint32_t e) {
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
    put_words2(a.w_cand + 2 * blockIdx.x, word(v, e), word(__uint_as_float(i), e));
  }
}

// The greedy token (0 when no logit qualifies); false when a poll gave up.
MYOS_DEV bool head_pick(const StreamArgs& a, uint32_t e, uint32_t& tok) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    bool ok = true;
    for (int q = lane; q < a.grid && ok; q += 32) {
      uint64_t wv, wi;
      ok = poll2(a, a.w_cand + 2 * q, e, wv, wi);
      const float pv = word_val(wv);
      const uint32_t pi = (uint32_t)wi;
      if (ok && better(pv, pi, v, i)) {
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
    if (lane == 0) s_tok = i == 0xffffffffu ? 0u : i;
  }
  csync();
  tok = s_tok;
  csync();  // s_tok is rewritten by the next head
  return !s_abort;
}

// ---------------------------------------------------------------- consumers
template <typename KT>
MYOS_DEV void consumers(const StreamArgs& a) {
  const uint32_t pos0 = a.ctl->pos, step0 = a.ctl->step;
  uint32_t argmax = a.ctl->argmax;
  uint32_t ph = a.flags[blockIdx.x];  // phases this CTA has run (epoch of the last one)
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
        const uint32_t e_in = ph;  // the last down phase (layer 0: none)
        ++ph;
        gamma_issue(scr(a) + a.H, layer(a, l).ln1, a.H);
        {  // bias rows: depend on nothing
          int q0, q1;
          rows_of(a.qd + 2 * a.kvd, a.grid, &q0, &q1);
          for (int i = threadIdx.x; i < q1 - q0; i += kCT)
            biasrows(a)[i] = __ldg(layer(a, l).bqkv + q0 + i);
        }
        mark(tr, 0);
        // the raw rows hr0..hr1 are the residual the o_proj epilogue adds to
        if (!stage(a, scr(a), a.H, a.w_resid, e_in, l == 0 ? a.embed + (size_t)tok * a.H : nullptr,
                   true, resrows(a), hr0, hr1, tr))
          return;
        mark(tr, 1);
        if (!consume_gemv<SK_QKV>(a, l, seq, best, ph)) return;
        mark(tr, 2);
      }
      // ---- attention
      const uint32_t e_qkv = ph;
      ++ph;
      if (attn_cta) {
        uint64_t* tr = trace_row(a, t, 5 * l + 1);
        mark(tr, 0);
        if (!attn_task<KT>(a, l, pos, e_qkv, ph)) return;
        mark(tr, 2);
      }
      // ---- o_proj: residual += W_o . attention output
      {
        uint64_t* tr = trace_row(a, t, 5 * l + 2);
        const uint32_t e_in = ph;
        ++ph;
        mark(tr, 0);
        if (!stage(a, scr(a), a.qd, a.w_attn, e_in, nullptr, false, nullptr, 0, 0, tr)) return;
        mark(tr, 1);
        if (!consume_gemv<SK_O>(a, l, seq, best, ph)) return;
        mark(tr, 2);
      }
      // ---- gate/up: RMSNorm(ln2), SiLU(gate) * up
      {
        uint64_t* tr = trace_row(a, t, 5 * l + 3);
        const uint32_t e_in = ph;
        ++ph;
        gamma_issue(scr(a) + a.H, layer(a, l).ln2, a.H);
        mark(tr, 0);
        // the raw rows hr0..hr1 (after o_proj) are the residual of the down epilogue
        if (!stage(a, scr(a), a.H, a.w_resid, e_in, nullptr, true, resrows(a), hr0, hr1, tr)) return;
        mark(tr, 1);
        if (!consume_gemv<SK_GU>(a, l, seq, best, ph)) return;
        mark(tr, 2);
      }
      // ---- down: residual += W_down . act
      {
        uint64_t* tr = trace_row(a, t, 5 * l + 4);
        const uint32_t e_in = ph;
        ++ph;
        mark(tr, 0);
        if (!stage(a, scr(a), a.I, a.w_act, e_in, nullptr, false, nullptr, 0, 0, tr)) return;
        mark(tr, 1);
        if (!consume_gemv<SK_DOWN>(a, l, seq, best, ph)) return;
        mark(tr, 2);
      }
    }
    // ---- head: final RMSNorm, logits, first maximum over the vocabulary
    if (a.head) {
      uint64_t* tr = trace_row(a, t, 5 * a.L);
      Best best = {-INFINITY, 0xffffffffu};
      const uint32_t e_in = ph;
      ++ph;
      gamma_issue(scr(a) + a.H, a.final_norm, a.H);
      mark(tr, 0);
      if (!stage(a, scr(a), a.H, a.w_resid, e_in, nullptr, true, nullptr, 0, 0, tr)) return;
      mark(tr, 1);
      if (!consume_gemv<SK_HEAD>(a, 0, seq, best, ph)) return;
      head_candidate(a, best, ph);
      mark(tr, 2);
      uint32_t next;
      if (!head_pick(a, ph, next)) return;
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (a.rec_fed) a.rec_fed[step0 + t] = tok;
        if (a.rec_argmax) a.rec_argmax[step0 + t] = argmax;
      }
      argmax = next;
    }
  }
  // this CTA's phase count for the next launch; cursor and greedy state
  if (threadIdx.x == 0) a.flags[blockIdx.x] = ph;
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
    s_tok = 0u;
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

size_t stream_word_count(const StreamArgs& a) {
  return (size_t)a.H + (size_t)(a.qd + 2 * a.kvd) + (size_t)a.Hkv * a.nsplit * a.G * (kD + 2) +
         (size_t)a.qd + (size_t)a.I + 2 * (size_t)a.grid;
}

void stream_set_words(StreamArgs* a, uint64_t* base) {
  a->w_resid = base;
  a->w_qkv = a->w_resid + a->H;
  a->w_part = a->w_qkv + (a->qd + 2 * a->kvd);
  a->w_attn = a->w_part + (size_t)a->Hkv * a->nsplit * a->G * (kD + 2);
  a->w_act = a->w_attn + a->qd;
  a->w_cand = a->w_act + a->I;
}

cudaError_t stream_configure(StreamArgs* a, int max_smem) {
  if (a->d != kD || a->G > kGMax || a->G < 1 || a->H % 256 || a->qd % 256 || a->I % 256 ||
      a->L > kMaxLayers || a->grid < 1 || a->grid > kCT || a->Hkv * a->nsplit > a->grid ||
      a->Hq > kCT || a->kvd % 256)
    return cudaErrorNotSupported;
  const size_t kv = a->kv_bf16 ? 2 : 4;
  // scratch: the largest staged input (with gamma and the bf16 embedding row
  // after a hidden-width one), the attention tiles
  a->tile = 32;
  const size_t ds_bytes = kD * kv + 16;
  const size_t attn = (size_t)a->G * kD * 4 + 2 * (size_t)a->tile * ds_bytes + 3 * kD * 4;
  const size_t x = std::max((size_t)std::max(a->qd, a->I) * 4, (size_t)a->H * 10);
  size_t scr = std::max(x, attn);
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
  if (a.kv_bf16) return counted(cudaLaunchKernelEx(&cfg, k_step_stream<__nv_bfloat16>, a));
  return counted(cudaLaunchKernelEx(&cfg, k_step_stream<float>, a));
}

}  // namespace myos
