// Persistent decode kernel with a continuous weight stream (kernel and
// design notes in stream_step.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "kernels.h"

namespace myos {

constexpr uint32_t kErrStream = 8u;  // a wait of the streaming step kernel gave up

struct StreamLayer {
  const uint16_t *wqkv, *wo, *wg, *wu, *wd;
  const float *bqkv, *ln1, *ln2;
};

// Matrix kinds of a token step, in stream order per layer, then the head.
enum StreamKind { SK_QKV = 0, SK_O = 1, SK_GU = 2, SK_DOWN = 3, SK_HEAD = 4 };

struct StreamArgs {
  // shape
  int L, H, I, V, qd, kvd, Hq, Hkv, d, G;
  float eps, scale;  // scale = 1/sqrtf(d), computed on the host as the reference does
  // weights
  const uint16_t* embed;
  const uint16_t* head_w;
  const float* final_norm;
  const StreamLayer* layers;  // device array [L]
  // step control: nsteps token steps per launch, greedy (feed null) or fed
  StepCtl* ctl;
  const uint32_t* feed;       // token of step s: feed[ctl->step + s]
  uint32_t* rec_fed;
  uint32_t* rec_argmax;
  int nsteps;
  int head;                   // 0: no head (prompt steps), the cursor still advances
  // activations (f32)
  float *resid, *qkv, *attn, *act, *logits;
  // KV cache [L][Hkv][S][d] of K and V, f32 or bf16
  void *kcache, *vcache;
  size_t kv_layer_elems;
  int S, kv_bf16;
  const float *cos_t, *sin_t;  // [S][d/2], host-built with libm
  // split-KV attention: tasks (KV head, split) on CTAs 0..Hkv*nsplit-1
  int nsplit, chunk, tile;
  // phase hand-over words (value bits, epoch): residual [H], q|k|v [qd+2kvd],
  // split partials [Hkv][nsplit][G][d+2], attention output [qd], activations
  // [I], head candidates [grid][2]; one allocation of stream_word_count
  // words, zeroed before first use and after a failed launch
  uint64_t *w_resid, *w_qkv, *w_part, *w_attn, *w_act, *w_cand;
  // flags[b] = phases CTA b had run when its last launch ended (the epoch base)
  unsigned* flags;
  // geometry (stream_configure)
  int grid, ns, slot_bytes, scr_bytes, part_floats;
  int off_scr, off_part, off_res, off_bias, off_lay;  // dynamic shared memory layout
  int rps[5], wpr[5];         // rows per ring slot and warps per row, per kind
  uint64_t wait_ns;           // bound of each wait
  int inflight;               // ring copies outstanding at once (issued, not landed)
  int l2_la;                  // slots ahead also requested into L2 (0: none)
  uint64_t* trace;            // optional [grid][5L+1][8] %globaltimer stamps (last step)
  uint64_t* strace;           // optional per-slot stamps (diagnostics)
  uint32_t strace_seq0;       // first slot index recorded
};

// Fills grid-dependent geometry (ns, slot_bytes, scr_bytes, part_floats,
// rps, wpr, tile) from the shape fields; fails when the layout does not fit
// max_smem bytes of shared memory.
cudaError_t stream_configure(StreamArgs* a, int max_smem);
// Words of the hand-over buffers, and their layout from one base pointer.
size_t stream_word_count(const StreamArgs& a);
void stream_set_words(StreamArgs* a, uint64_t* base);
size_t stream_smem_bytes(const StreamArgs& a);
int stream_threads();
cudaError_t launch_step_stream(const StreamArgs& a, cudaStream_t st);

}  // namespace myos
