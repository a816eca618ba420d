// Persistent one-launch-per-token step kernel (kernel and design notes in
// step_kernel.cu).
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
  size_t scratch_bytes;     // dynamic shared memory of the launch
  int x_floats;             // staged-input region; gamma / embedding / merge area follows
  int merge_in_stage;       // 1: o_proj staging merges the attention splits
  uint64_t* trace;          // optional [grid][nphase][4] global-timer stamps
  int lookahead;            // phases whose weight slices are prefetched into L2 ahead
  int pf_kb;                // cap of one block's prefetch per phase, KiB
  int pf_mode;              // 0: bulk prefetch (TMA engine), 1: per-line prefetch
};

bool mega_supported(int H, int I, int qd, int kvd, int d, int G);
int mega_threads();
// Shared-memory layout from the shape fields of *a (H, I, qd, Hq, Hkv, d, G,
// nsplit): fills scratch_bytes, x_floats and merge_in_stage; fails when the
// layout exceeds max_smem.
cudaError_t mega_configure(MegaArgs* a, int max_smem);
size_t mega_smem_bytes(const MegaArgs& a);
cudaError_t launch_step_mega(const MegaArgs& a, cudaStream_t st);

}  // namespace myos
