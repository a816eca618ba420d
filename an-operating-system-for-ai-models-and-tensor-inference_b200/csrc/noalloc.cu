// Split-KV decode attention on caller-held device buffers that allocates
// nothing: the kernel's scratch (per-split partials and the merge counters)
// is carved from one fixed file-scope device array instead of cudaMalloc.
//
// Scratch layout inside g_scratch (each region 256-byte aligned):
//   counters [Hkv] u32      MUST be zero when the kernel starts: the last
//                           split of a head group to arrive merges, and
//                           finds itself last by counting. The kernel puts
//                           each counter back to zero after its merge, the
//                           array starts zeroed at module load, and each
//                           call also clears them on its stream first
//                           (cudaMemsetAsync, which allocates nothing), so
//                           an earlier failed launch cannot leave them set.
//   part_m, part_l [Hkv][nsplit][G] f32, part_o [Hkv][nsplit][G][d] f32:
//                           written before they are read; no initial value.
//
// Calls share the one array per device: two calls whose kernels overlap in
// time (different streams, or different host threads without ordering) race
// on it and corrupt each other's results. Issue them on one stream, or order
// them.
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "../../include/myos_cuda.h"
#include "kernels.h"

using namespace myos;

namespace {

constexpr size_t kScratchBytes = MYOS_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

// Device address of g_scratch on the current device. Resolved once per
// device (cudaGetSymbolAddress may load the module on first use, so that
// first call belongs outside any stream capture) and cached.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MYOS_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_scratch);
    if (rc != cudaSuccess || !p) return MYOS_ERR_CUDA;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return MYOS_OK;
}

}  // namespace

extern "C" int myos_dev_gqa_attn_f32_noalloc(float* d_y, const float* d_q, const float* d_k,
                                             const float* d_v, size_t hq, size_t hkv, size_t d,
                                             size_t seq, int32_t mask_kind, size_t query_pos,
                                             void* stream) {
  if (!d_y || !d_q || !d_k || !d_v) return MYOS_ERR_ARG;
  // GqaMask has two variants: Full (0) and Causal (1).
  if (mask_kind != 0 && mask_kind != 1) return MYOS_ERR_ARG;
  // Every buffer holds f32 (4-byte aligned); with d % 4 == 0 the kernel reads
  // K and V rows as 16-byte vectors, so those two start on 16 bytes. A
  // misaligned pointer is refused here, before any device work, instead of
  // faulting the caller's context.
  const uintptr_t any = (uintptr_t)d_y | (uintptr_t)d_q | (uintptr_t)d_k | (uintptr_t)d_v;
  if ((any & 3) != 0) return MYOS_ERR_ARG;
  if (d % 4 == 0 && (((uintptr_t)d_k | (uintptr_t)d_v) & 15) != 0) return MYOS_ERR_ARG;
  // Shape rules of tensor_core::gqa_attn_f32 (gqa.rs:174-218), as the
  // host-slice entry point applies them.
  if (hq == 0 || hkv == 0 || d == 0 || seq == 0 || hq % hkv != 0) return MYOS_ERR_SHAPE;
  const size_t G = hq / hkv;
  if (G > 8 || d > 256 || seq > 0x7fffffff) return MYOS_ERR_SHAPE;
  // hq * (2 + d) * 4 bytes of partials at the least: past the reserve
  if (hq > ((size_t)1 << 20)) return MYOS_ERR_SCRATCH_LIMIT;
  size_t nkeys = seq;
  if (mask_kind == 1 && query_pos < seq - 1) nkeys = query_pos + 1;
  // Same split geometry as the host-slice entry point, so both run the same
  // reduction order.
  size_t nsplit = (nkeys + 31) / 32;
  if (nsplit > 64) nsplit = 64;
  const size_t chunk = (nkeys + nsplit - 1) / nsplit;
  const size_t ml = hkv * nsplit * G;  // <= 2^20 * 64 entries
  const size_t off_m = a256(hkv * sizeof(unsigned));
  const size_t off_l = off_m + a256(ml * sizeof(float));
  const size_t off_o = off_l + a256(ml * sizeof(float));
  const size_t need = off_o + a256(ml * d * sizeof(float));
  if (need > kScratchBytes) return MYOS_ERR_SCRATCH_LIMIT;  // before any device work

  if (kernels_init() != cudaSuccess) return MYOS_ERR_CUDA;
  void* base = nullptr;
  if (int st = scratch_address(&base)) return st;
  uint8_t* s = static_cast<uint8_t*>(base);
  const cudaStream_t cs = (cudaStream_t)stream;
  if (cudaMemsetAsync(s, 0, hkv * sizeof(unsigned), cs) != cudaSuccess) return MYOS_ERR_CUDA;
  AttnArgs a = {};
  a.q = d_q;
  a.kc = const_cast<float*>(d_k);
  a.vc = const_cast<float*>(d_v);
  a.S = (int)seq;
  a.Hq = (int)hq;
  a.Hkv = (int)hkv;
  a.d = (int)d;
  a.G = (int)G;
  a.nkeys_fixed = (int)nkeys;
  a.chunk = (int)chunk;
  a.nsplit = (int)nsplit;
  a.scale = 1.0f / sqrtf((float)d);
  a.counters = reinterpret_cast<unsigned*>(s);
  a.part_m = reinterpret_cast<float*>(s + off_m);
  a.part_l = reinterpret_cast<float*>(s + off_l);
  a.part_o = reinterpret_cast<float*>(s + off_o);
  a.out = d_y;
  a.decode = 0;
  if (launch_attention(a, 0, cs, false) != cudaSuccess) return MYOS_ERR_CUDA;
  return MYOS_OK;
}
