// Kernel argument blocks and host-side launchers for the decode step.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace myos {

// Device-resident step control. Kernels read it only after their
// programmatic-dependency wait, so a whole token step (or several) can run
// from a CUDA graph with no host round trip.
struct StepCtl {
  uint32_t pos;     // KV slot this step writes (KvCache cursor)
  uint32_t step;    // index of this step within the current call
  uint32_t argmax;  // first maximum of the most recent logits
  uint32_t fed;     // token embedded by this step
  uint32_t err;     // sticky error bits
  uint32_t pad[3];
};

// Optional launch timeline (diagnostics): per (step mod kTraceSteps, slot)
// kTraceWidth u64 %globaltimer stamps: earliest block start, earliest return
// from the dependency wait, latest block end, then kernel-specific latest
// stage marks. Null buf disables it.
constexpr int kTraceSteps = 64;
constexpr int kTraceWidth = 8;
struct KTrace {
  uint64_t* buf;
  int slot, nslot;
};

// How a GEMV block stages its input vector in shared memory.
struct GemvInput {
  const float* x;         // f32 [K] (ignored in embed mode)
  const uint16_t* embed;  // embed mode: x[j] = bf16(embed[token*K + j])
  const uint32_t* feed;   // embed mode token: feed[ctl->step], else ctl->argmax
  StepCtl* ctl;
  float* x_store;         // embed mode: block 0 writes the gathered row here
  const float* gamma;     // RMSNorm weight (promoted f32) or null
  float eps;
  // Attention-merge mode (o_proj input, decode): x is the merge of the
  // split-KV partials [Hkv][nsplit][G][d] of the splits that hold keys
  // 0..ctl->pos; the staging does the merge the attention kernel deferred.
  const float* part_o;    // non-null selects this mode
  const float* part_m;
  const float* part_l;
  int m_G, m_d, m_nsplit, m_chunk;
};

enum EpiKind { EPI_STORE = 0, EPI_BIAS = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4 };

// Tensor-parallel push (peer memory): out[p] is this rank's slot in rank
// p's inbox (8-byte words: value, epoch), seq this rank's exchange counter
// (the push uses epoch *seq + 1).
constexpr int kMaxTp = 8;
struct TpPush {
  int n;  // ranks; 0: no push
  float* out[kMaxTp];
  const unsigned* seq;
};

// Sum of the ranks' pushed parts: out[i] = sum over ranks p = 0..n-1, in
// rank order, of inbox word p * H + i once it carries epoch *seq + 1; then
// *seq is advanced (by the last of the kernel's blocks).
struct TpReduceArgs {
  int n, H;
  const float* inbox;
  unsigned* seq;
  unsigned* done;  // blocks finished (reset by the last one)
  float* out;
  uint32_t* err;
  uint64_t wait_ns;  // bound on each word's wait (0: 60 s)
};
cudaError_t launch_tp_reduce(const TpReduceArgs& r, cudaStream_t st, bool pdl);

struct GemvArgs {
  const uint16_t* w;   // [M, K] row-major bf16
  const uint16_t* w2;  // EPI_SWIGLU: up_proj [M, K]
  int M, K;
  GemvInput in;
  float* y;            // output [M]; EPI_RESID: residual updated in place
  const float* bias;   // EPI_BIAS
  size_t prefetch_cap; // bytes of this block's rows to pull into L2 before the wait
  // EPI_ARGMAX
  float* part_val;
  uint32_t* part_idx;
  unsigned* counter;
  uint32_t* rec_fed;
  uint32_t* rec_argmax;
  uint32_t* err;       // bounded-wait failure bits (nullable)
  KTrace tr;
  // Weights of a later kernel to pull into L2 while this one waits on its
  // inputs (pf_mode 1): the ranges pf_ptr[m] + i * pf_stride of pf_bytes[0]
  // bytes for m < 2 and i < pf_n, one bulk prefetch sequence per range,
  // spread over the blocks.
  const void* pf_ptr[2];
  size_t pf_bytes[1];
  int pf_mode;
  size_t pf_stride;
  int pf_n;
  // Tensor parallel. EPI_RESID: y[row] = base + v with base = res[row] (res
  // set), y[row] (res null: in place), or 0 (res_zero: a partial sum for the
  // allreduce). EPI_ARGMAX with tp_cand: the block-reduced first maximum goes
  // to tp_cand as (value, row0 + row), the step control is left alone.
  // With push.n > 0 the EPI_RESID rows (or the EPI_ARGMAX candidate) go to
  // every rank's inbox instead, as (value, epoch) words of epoch *push.seq + 1.
  const float* res;
  int res_zero;
  float* tp_cand;
  uint32_t row0;
  TpPush push;
  int warps;  // streaming kernel: warps per block (0: the full block); gemv_warps
};

// Global first maximum over the tensor-parallel ranks' candidates
// [(value, index)] x n, then the step control advanced (tp pick). With seq
// non-null the candidates arrive by push (words of epoch *seq + 1, two per
// rank) and *seq is advanced after.
cudaError_t launch_tp_pick(const float* cands, int n, unsigned* seq, StepCtl* ctl,
                           uint32_t* rec_fed, uint32_t* rec_argmax, cudaStream_t st);

struct AttnArgs {
  const float* q;        // decode: qkv buffer [q | k | v] before RoPE; op: q [Hq*d]
  void* kc;              // this layer's K: [Hkv][S][d] of the cache type
  void* vc;
  int S;                 // slot stride (max_seq)
  int Hq, Hkv, d, G;
  int nkeys_fixed;       // op mode: keys 0..nkeys_fixed-1
  StepCtl* ctl;          // decode mode: keys 0..ctl->pos, new key at ctl->pos
  const float* cos_t;    // [S][d/2], host-built with libm
  const float* sin_t;
  int chunk, nsplit;
  float scale;           // 1/sqrtf(d), computed on the host as the reference does
  float* part_o;         // [Hkv][nsplit][G][d]
  float* part_m;         // [Hkv][nsplit][G]
  float* part_l;
  unsigned* counters;    // [Hkv], zero between launches
  // decode, more than 8 splits: arrivals per KV head (monotonic; each launch
  // adds nsplit), the last G blocks to arrive each merge one query head
  unsigned long long* arrive;
  float* out;            // [Hq*d]
  int decode;
  int defer_merge;       // decode: write the split partials only; the o_proj
                         // staging merges them (GemvInput attention-merge mode)
  int cluster;           // decode, nsplit <= 8: the splits of a KV head form one
                         // thread-block cluster and merge through shared memory
  KTrace tr;
};

// Shared memory of the attention-merge staging beyond the staged input.
size_t merge_smem_bytes(int Hq, int nsplit, int d);

// Fused MLP of one decode layer (qwen25_block.rs:250-287: RMSNorm(ln2),
// gate|up, SiLU(gate)*up, down_proj, residual add) in one launch. Block b
// owns the intermediate columns [64b, 64b + 64): it computes their
// activations from RMSNorm(resid) and their share of every down_proj output
// row, W_down[:, 64b:64b+64] . act[64b:64b+64], into part[row][b]. After
// every block has arrived (a grid-wide count; all blocks are resident, one
// per SM), block b sums the shares of its output rows in block order and
// adds them to the residual. The intermediate vector never leaves the SM
// and down_proj needs no staging of it.
constexpr int kMlpSlice = 64;     // intermediate columns per block
constexpr uint32_t kErrMlpWait = 16u;
constexpr uint32_t kErrAttnWait = 32u;  // a split-merge arrival wait gave up
struct MlpArgs {
  const uint16_t *wg, *wu, *wd;  // gate, up [I][H]; down [H][I]
  // down_proj re-laid out by block, [grid][H][64] (mlp_relayout), so a block
  // streams one contiguous range; null: read wd's columns in place
  const uint16_t* wd_slices;
  const float* gamma;            // ln2, promoted f32
  float eps;
  int H, I;
  float* resid;                  // [H], updated in place
  float* part;                   // [H][grid] per-block shares of the down rows
  unsigned long long* arrive;    // arrivals so far; a multiple of the grid between launches
  StepCtl* ctl;
  uint32_t* err;
  uint64_t wait_ns;              // bound of the arrival wait
  KTrace tr;
};
// Blocks of the fused MLP for this shape, or 0 when it does not apply
// (hidden not 1024/1280/1536, I not a multiple of 64, or I/64 outside
// [3/4, 1] of the SM count).
int mlp_grid(int H, int I, int num_sms);
cudaError_t launch_mlp(const MlpArgs& a, int grid, cudaStream_t st, bool pdl);
// dst[b][r][c] = wd[r][64 b + c] for the I / 64 column slices of a [H][I] matrix.
cudaError_t launch_mlp_relayout(const uint16_t* wd, uint16_t* dst, int H, int I, cudaStream_t st);

// Launchers. pdl=true attaches a programmatic-serialization edge to the
// previous launch in the stream.
cudaError_t launch_gemv(int epi, const GemvArgs& a, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_attention(const AttnArgs& a, int kv_bf16, cudaStream_t st, bool pdl);
cudaError_t launch_step_end(StepCtl* ctl, cudaStream_t st, bool pdl);
cudaError_t launch_argmax(const float* v, int n, float* part_val, uint32_t* part_idx,
                          unsigned* counter, uint32_t* out, int grid, cudaStream_t st);
cudaError_t launch_swiglu_mul(float* h, const float* gate, const float* up, int n, cudaStream_t st);
cudaError_t launch_rope(float* y, const float* x, int len, int head_dim, const float* cos_row,
                        const float* sin_row, cudaStream_t st);
cudaError_t launch_rmsnorm(float* y, const float* x, const float* gamma, int n, float eps,
                           cudaStream_t st);
cudaError_t kernels_init();  // raises dynamic shared-memory limits once per device

// Kernel launches the library has enqueued in this process (diagnostics):
// every launcher counts a successful launch; a CUDA graph replay counts the
// kernels captured in it, the capture itself counts none.
cudaError_t counted(cudaError_t e, uint64_t n = 1);
void launches_uncount(uint64_t n);
uint64_t launches_total();

size_t gemv_smem_bytes(int K);
// Grid for an M x K GEMV (NR = 2 for gate|up): up to two blocks per SM.
int gemv_grid(int M, int K, int NR, int num_sms);
// Warps per block of the streaming kernel for that grid: rows spread evenly
// over the warps, and at least enough threads to stage the input in one trip.
int gemv_warps(int M, int K, int NR, bool has_gamma, int grid);
size_t attn_smem_bytes(int G, int d);
int attn_dpl(int d);

}  // namespace myos
