// Persistent one-launch-per-token step kernel (see step_kernel.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "kernels.h"

namespace myos {

constexpr uint32_t kErrPhase = 4u;  // a phase counter wait gave up

struct MegaLayer {
  const uint16_t *wqkv, *wo, *wg, *wu, *wd;
  const float *bqkv, *ln1, *ln2;
};

struct MegaArgs {
  int L, H, I, V, qd, kvd, Hq, Hkv, d, G;
  float eps, scale;
  const uint16_t* embed;
  const uint16_t* head_w;
  const float* final_norm;
  const MegaLayer* layers;  // device array [L]
  StepCtl* ctl;
  const uint32_t* feed;     // token source: feed[ctl->step], else ctl->argmax
  uint32_t* rec_fed;
  uint32_t* rec_argmax;
  float *resid, *qkv, *attn, *act, *logits;
  void *kcache, *vcache;
  size_t kv_layer_elems;
  int S;
  int kv_bf16;
  const float *cos_t, *sin_t;
  int nsplit, chunk;
  float *part_o, *part_m, *part_l;
  unsigned* attn_cnt;       // [Hkv], zero between launches
  unsigned* bar;            // [5L] phase counters, zeroed before each launch
  unsigned* head_cnt;
  float* part_val;          // [grid]
  uint32_t* part_idx;
  int head;                 // 1: final norm + head + argmax, else only advance
  int grid;
  size_t scratch_bytes;
  int slot_bytes;
  int nslot;
  uint64_t* trace;          // optional [grid][nphase][4] global-timer stamps
  int lookahead;            // stages the producer prefetches into L2 ahead of the ring
};

bool mega_supported(int H, int I, int qd, int kvd, int d, int G, int slot_bytes);
size_t mega_scratch_bytes(int H, int I, int qd, int d, int G);
int mega_threads();
cudaError_t mega_configure(MegaArgs* a, int max_smem);
size_t mega_smem_bytes(const MegaArgs& a);
cudaError_t launch_step_mega(const MegaArgs& a, cudaStream_t st);

}  // namespace myos
