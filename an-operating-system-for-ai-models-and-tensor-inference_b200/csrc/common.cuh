// Device helpers shared by the sm_100a kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MYOS_DEV __device__ __forceinline__

namespace myos {

constexpr int kWarp = 32;

// BF16 is the top half of an f32 (crates/tensor_core/src/bf16.rs:61-63), so
// promotion is a shift or a mask: exact, no rounding.
MYOS_DEV float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
MYOS_DEV float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
MYOS_DEV float bf16_at(const uint16_t* p) { return __uint_as_float((uint32_t)(*p) << 16); }

// Weights are read once per token: stream them past L1.
MYOS_DEV uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

MYOS_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

MYOS_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch. wait: block until the preceding grid in the
// stream has completed and its writes are visible (a no-op when the launch
// carried no programmatic edge). launch: allow the next grid to be scheduled.
MYOS_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MYOS_DEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Fire-and-forget bulk prefetch of [p, p+bytes) into L2. p and bytes must be
// 16-byte multiples; callers round.
MYOS_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch a byte range from one thread, in <=64 KiB pieces.
MYOS_DEV void prefetch_range_1(const void* base, size_t bytes) {
  uintptr_t a = (uintptr_t)base;
  uintptr_t p = (a + 15) & ~(uintptr_t)15;
  const uintptr_t end = (a + bytes) & ~(uintptr_t)15;
  for (; p < end; p += 65536) prefetch_l2((const void*)p, (uint32_t)(end - p < 65536 ? end - p : 65536));
}

// Prefetch a byte range split into <=64 KiB pieces across the block's threads.
MYOS_DEV void prefetch_range(const void* base, size_t bytes) {
  uintptr_t a = (uintptr_t)base;
  uintptr_t start = (a + 15) & ~(uintptr_t)15;
  uintptr_t end = (a + bytes) & ~(uintptr_t)15;
  if (end <= start) return;
  const size_t piece = 65536;
  size_t n = (end - start + piece - 1) / piece;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
    uintptr_t p = start + i * piece;
    uintptr_t q = p + piece < end ? p + piece : end;
    prefetch_l2((const void*)p, (uint32_t)(q - p));
  }
}

// ---------------------------------------------------------------- mbarrier + bulk copy
// Shared-memory mbarriers track the bulk (TMA-engine) copies of weight
// stages. Every wait is bounded: after kWaitLimit polls it gives up, raises
// a bit in *err and returns false, so a broken pipeline ends the kernel with
// an error the host reads instead of hanging the GPU.
constexpr uint32_t kWaitLimit = 1u << 25;
constexpr uint32_t kErrWaitFull = 1u, kErrWaitEmpty = 2u;

MYOS_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MYOS_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

MYOS_DEV void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

MYOS_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

MYOS_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

MYOS_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

MYOS_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity to complete: gives up
// after kWaitLimit polls or one second, whichever comes first.
MYOS_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 0 && global_ns() - t0 > 1000000000ull) break;
  }
  if (err) atomicOr(err, code);
  return false;
}

// ---------------------------------------------------------------- tensor-parallel peers
// Ranks of a tensor-parallel group are processes on different GPUs. A rank
// stores each value of its part of a result straight into every rank's
// inbox (peer memory over NVLink) as one 8-byte word (value bits, epoch):
// an aligned 8-byte store is seen whole or not at all, so the word carries
// its own validity and needs no fence or counter. The consumer polls each
// word until its epoch is the current one. Epochs count the exchanges of a
// context (every rank makes the same ones in the same order). Another rank
// may reach the same step later than this one (its host enqueued later), so
// a wait is bounded in time rather than in polls; once one wait has given
// up, later waits of the context return at once with the error bit set.
constexpr uint32_t kErrTpWait = 4u;
constexpr uint64_t kTpWaitNs = 60000000000ull;  // 60 s (default bound)

MYOS_DEV void tp_store(float* slot, float v, unsigned epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(slot), "l"(w) : "memory");
}

MYOS_DEV unsigned long long tp_load(const float* slot) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(slot) : "memory");
  return w;
}

// The value of word `slot` once it carries `epoch`; false (and the error bit)
// when `limit_ns` passes first (0: kTpWaitNs), or an earlier wait gave up.
MYOS_DEV bool tp_wait_word(const float* slot, unsigned epoch, uint32_t* err, float* v,
                           uint64_t limit_ns = 0) {
  if (limit_ns == 0) limit_ns = kTpWaitNs;
  unsigned long long w = tp_load(slot);
  if ((unsigned)(w >> 32) != epoch) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
      if ((i & 63u) == 0) {
        if (*(volatile uint32_t*)err & kErrTpWait) return false;
        if (global_ns() - t0 > limit_ns) {
          atomicOr(err, kErrTpWait);
          return false;
        }
      }
      w = tp_load(slot);
      if ((unsigned)(w >> 32) == epoch) break;
    }
  }
  *v = __uint_as_float((unsigned)w);
  return true;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on bar.
// dst, src 16-byte aligned; bytes a multiple of 16.
MYOS_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Named barrier over the first nthreads threads of the block (id 1..15).
MYOS_DEV void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Sum over the block in a fixed order (deterministic). red holds >= 33 floats.
MYOS_DEV float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float s = lane < nwarps ? red[lane] : 0.0f;
    s = warp_sum(s);
    if (lane == 0) red[32] = s;
  }
  __syncthreads();
  float s = red[32];
  __syncthreads();
  return s;
}

// 8 promoted weights (one 16-byte chunk) against 8 staged activations.
MYOS_DEV float dot8(const uint4& u, const float4& lo, const float4& hi, float acc) {
  acc = fmaf(bf16_lo(u.x), lo.x, acc);
  acc = fmaf(bf16_hi(u.x), lo.y, acc);
  acc = fmaf(bf16_lo(u.y), lo.z, acc);
  acc = fmaf(bf16_hi(u.y), lo.w, acc);
  acc = fmaf(bf16_lo(u.z), hi.x, acc);
  acc = fmaf(bf16_hi(u.z), hi.y, acc);
  acc = fmaf(bf16_lo(u.w), hi.z, acc);
  acc = fmaf(bf16_hi(u.w), hi.w, acc);
  return acc;
}

}  // namespace myos
