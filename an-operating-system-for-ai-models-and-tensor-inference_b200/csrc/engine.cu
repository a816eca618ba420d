// Engine: HBM weight arena, KV cache, token-step orchestration and the C ABI.
//
// A token step (model_core::forward_token, qwen25_block.rs:220-304) is 5
// kernels per layer plus the head:
//   QKV   fused RMSNorm(input_layernorm) -> [q|k|v] GEMV -> +bias
//         (layer 0 also gathers the embedding row of the step's token)
//   ATTN  RoPE(q,k) -> KV write at pos -> split-KV GQA -> combine
//   O     o_proj GEMV -> residual += (attn_wire.rs:286-312)
//   GU    fused RMSNorm(post_attention_layernorm) -> gate,up GEMV -> SiLU*up
//   DOWN  down_proj GEMV -> residual += (qwen25_block.rs:280-288)
//   HEAD  final RMSNorm -> tied/untied head GEMV -> logits + argmax ->
//         advance the cursor (KvCache::advance once per token)
// Every launch carries a programmatic-dependency edge so each kernel's
// weight prefetch overlaps its predecessor; steps are replayed from CUDA
// graphs, with token and position living in device memory (StepCtl).
#include <fcntl.h>
#include <math.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/myos_cuda.h"
#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"
#include "prefill.h"
#include "safetensors.h"
#include "tp.h"

using namespace myos;

namespace {

constexpr int kSuffixes = 12;
const char* kSuffix[kSuffixes] = {
    "input_layernorm.weight",  "self_attn.q_proj.weight", "self_attn.q_proj.bias",
    "self_attn.k_proj.weight", "self_attn.k_proj.bias",   "self_attn.v_proj.weight",
    "self_attn.v_proj.bias",   "self_attn.o_proj.weight", "post_attention_layernorm.weight",
    "mlp.gate_proj.weight",    "mlp.up_proj.weight",      "mlp.down_proj.weight"};
const char* kEmbed = "model.embed_tokens.weight";
const char* kFinalNorm = "model.norm.weight";
const char* kLmHead = "lm_head.weight";

struct LayerW {
  uint16_t *wqkv, *wo, *wg, *wu, *wd;
  float *bqkv, *ln1, *ln2;
};

enum GraphKind { G_FEED_NOHEAD = 0, G_FEED_HEAD = 1, G_ARGMAX_HEAD = 2 };

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

struct myos_ctx {
  myos_shape s;  // this rank's slice of the model (the whole model without tensor parallelism)
  myos_opts o;
  int device = 0;
  int num_sms = 148;
  cudaStream_t st = nullptr, copy_st = nullptr;
  std::string err;
  size_t qd = 0, kvd = 0, G = 1;
  size_t qd_pad = 0;  // o_proj input width: qd, or (tensor parallel) qd rounded up to 256
  // HBM
  uint8_t* warena = nullptr;
  size_t warena_bytes = 0;
  uint16_t *embed = nullptr, *lm_head = nullptr;
  float* final_norm = nullptr;
  std::vector<LayerW> layers;
  void *kcache = nullptr, *vcache = nullptr;
  size_t kv_layer_elems = 0;
  float *resid = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr;
  float *part_val = nullptr, *part_o = nullptr, *part_m = nullptr, *part_l = nullptr;
  uint32_t* part_idx = nullptr;
  unsigned* counters = nullptr;  // [0] head, [1..Hkv] attention
  unsigned long long* attn_arrive = nullptr;  // [Hkv] split arrivals (distributed merge)
  StepCtl* ctl = nullptr;
  uint32_t *feed = nullptr, *rec_fed = nullptr, *rec_argmax = nullptr;
  float *cos_t = nullptr, *sin_t = nullptr;
  // pinned staging
  uint8_t* pin[2] = {nullptr, nullptr};
  size_t pin_bytes = 0;
  cudaEvent_t pin_ev[2] = {nullptr, nullptr};
  int pin_slot = 0;
  cudaEvent_t load_ev = nullptr;  // recorded on copy_st after each load
  StepCtl* ctl_host = nullptr;  // pinned mirror for uploads
  // launch geometry
  int grid_qkv = 0, grid_o = 0, grid_gu = 0, grid_down = 0, grid_head = 0;
  int warps_qkv = 0, warps_o = 0, warps_gu = 0, warps_down = 0, warps_head = 0;
  int attn_chunk = 0, attn_nsplit = 0;
  int defer_merge = 0;  // o_proj staging merges the attention splits
  int attn_cluster = 0; // attention splits merge across a thread-block cluster
  // fused MLP (k_mlp: gate|up, SwiGLU and down_proj in one launch per layer)
  // when the shape allows and MYOS_MLP is not 0; grid 0 keeps the two GEMVs
  int grid_mlp = 0;
  float* mlp_part = nullptr;                  // [hidden][grid_mlp] down_proj shares
  unsigned long long* mlp_arrive = nullptr;   // grid-wide arrival count
  uint16_t* mlp_wd = nullptr;  // [L][grid_mlp][hidden][64] down_proj by block (null: in place)
  int mlp_pf_rows = 0;  // MYOS_MLP_PF (default 64): gate/up rows per MLP block that o_proj pulls into L2
  // GEMM prefill (chunks of pf_chunk prompt tokens through the tensor cores)
  bool pf_ok = false;
  int pf_chunk = 0;
  float *pf_X = nullptr, *pf_D = nullptr, *pf_Q = nullptr;
  uint16_t* pf_A = nullptr;
  void* pf_ws = nullptr;
  size_t pf_ws_bytes = 0;
  size_t pf_D_elems = 0;  // capacity of pf_D in floats
  bool pf_splitk = true;  // MYOS_SPLITK=0: one K slice per projection
  bool pf_m64 = true;     // MYOS_GEMM_M64=0: 128-row tiles only
  // batched decode (myos_batch_generate): per-sequence KV slabs and buffers
  void *bt_k = nullptr, *bt_v = nullptr;
  size_t bt_kv_bytes = 0;
  float *bt_X = nullptr, *bt_D = nullptr;
  size_t bt_D_bytes = 0;
  int *bt_pos = nullptr, *bt_rows = nullptr;
  uint32_t *bt_tok = nullptr, *bt_out = nullptr, *bt_ids = nullptr, *bt_feed = nullptr;
  int* bt_step = nullptr;  // device step index of the batched step graph
  size_t bt_feed_bytes = 0;
  float* at_o = nullptr;     // split attention partials of the GEMM path (o)
  float2* at_ml = nullptr;   // ... and their (max, sum of exponentials)
  size_t at_o_bytes = 0, at_ml_bytes = 0;
  unsigned* at_arrive = nullptr;  // per (row, KV head) split arrivals (zero between launches)
  size_t at_arrive_bytes = 0;
  unsigned* at_work = nullptr;    // the split attention's item queue (zero between launches)
  size_t at_work_bytes = 0;
  float2* bt_amax = nullptr;  // per-chunk argmax candidates of the batched head
  size_t bt_amax_bytes = 0;
  size_t bt_out_n = 0, bt_ids_n = 0;
  size_t prefetch_total = 0;  // bulk L2 prefetch (MYOS_PREFETCH_MB); measured slower, off
  // loaded-tensor bookkeeping
  std::vector<uint8_t> have;  // per layer x suffix, then embed, final norm, lm_head
  size_t len = 0;             // KV cursor (host mirror of ctl->pos)
  std::map<std::pair<int, int>, cudaGraphExec_t> graphs;
  std::map<std::pair<int, int>, uint64_t> graph_kernels;  // kernels captured in each graph
  cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev2 = nullptr;
  float prefill_ms = 0.f, decode_ms = 0.f;
  int steps_per_graph = 16;
  bool profiling = false;
  uint64_t* ktrace = nullptr;  // MYOS_KTRACE_FILE: launch timeline of the per-kernel step
  std::string ktrace_file;
  std::vector<uint64_t> ktrace_init;
  // tensor parallelism (myos_ctx_create_tp): heads, MLP columns and head rows
  // split over tp_size ranks; residual updates summed over NCCL
  int tp_size = 1, tp_rank = 0;
  myos_shape full = {};      // the whole model (the loader checks tensors against it)
  uint32_t i_cut = 0;        // MLP columns of this rank before padding to s.intermediate
  uint32_t head_rows = 0, head_row0 = 0;  // this rank's vocabulary rows of the head
  ncclComm_t comm = nullptr;
  float* tp_part = nullptr;  // [hidden] this rank's partial residual update
  float* tp_cand = nullptr;  // [2] this rank's (value, index), then [2 * tp_size] all ranks'
  // Peer-memory exchange (default when every rank can map every other's
  // memory; MYOS_TP_COMM=nccl uses NCCL collectives instead): the o_proj and
  // down_proj epilogues push their rows into every rank's inbox, a one-block
  // kernel sums them; the head pushes its candidate the same way.
  bool tp_p2p = false;
  uint8_t* tp_link = nullptr;         // this rank's inboxes, epoch and block counters
  void* tp_peer[kMaxTp] = {};         // every rank's tp_link as mapped here
  TpPush push_o = {}, push_d = {}, push_c = {};
  float *inbox_o = nullptr, *inbox_d = nullptr, *inbox_c = nullptr;  // 8-byte words
  unsigned* tp_seq = nullptr;         // [0] exchanges completed by this rank, [1] reduce blocks done
};

namespace {

// Tensor name -> (layer, suffix) or global (0 embed, 1 final norm, 2
// lm_head) for the model shape s; false for names the model never reads
// (qwen25_layout.rs:15-207 keys).
bool parse_tensor_name(const myos_shape& s, const std::string& n, int* layer, int* suffix,
                       int* global) {
  *layer = *suffix = *global = -1;
  if (n == kEmbed) {
    *global = 0;
  } else if (n == kFinalNorm) {
    *global = 1;
  } else if (n == kLmHead) {
    if (s.tied_head) return false;
    *global = 2;
  } else if (n.compare(0, 13, "model.layers.") == 0) {
    const size_t dot = n.find('.', 13);
    if (dot == std::string::npos) return false;
    const std::string idx = n.substr(13, dot - 13);
    if (idx.empty() || idx.find_first_not_of("0123456789") != std::string::npos) return false;
    if (idx.size() > 1 && idx[0] == '0') return false;
    const unsigned long li = strtoul(idx.c_str(), nullptr, 10);
    if (li >= s.num_layers) return false;
    const std::string suf = n.substr(dot + 1);
    for (int k = 0; k < kSuffixes; ++k)
      if (suf == kSuffix[k]) *suffix = k;
    if (*suffix < 0) return false;
    *layer = (int)li;
  } else {
    return false;
  }
  return true;
}

// How rank rk of N holds a tensor of the whole model f: heads (q/k/v rows,
// o_proj columns), MLP columns (gate/up rows, down_proj columns) and head
// vocabulary rows are split in rank order; the o_proj input and MLP widths
// are padded to multiples of 256 with zeros; everything else is replicated.
// The loader and myos_tp_slice both use it.
myos_tp_part tp_part(const myos_shape& f, uint32_t N, uint32_t rk, int global, int suffix) {
  const uint64_t H = f.hidden, I = f.intermediate, V = f.vocab;
  const uint64_t qd = (uint64_t)f.num_q_heads * f.head_dim, kvd = (uint64_t)f.num_kv_heads * f.head_dim;
  const uint64_t qdl = qd / N, kvdl = kvd / N, Ic = I / N, Vl = V / N;
  const uint64_t Il = N > 1 ? (Ic + 255) / 256 * 256 : Ic, qdp = N > 1 ? (qdl + 255) / 256 * 256 : qdl;
  myos_tp_part p = {};
  auto whole = [&](uint64_t r, uint64_t cl, bool mtx) {
    p.rows = r;
    p.cols = cl;
    p.nrows = p.store_rows = r;
    p.ncols = p.store_cols = cl;
    p.matrix = mtx ? 1 : 0;
    p.kept = 1;
  };
  auto rowpart = [&](uint64_t r, uint64_t cl, bool mtx, uint64_t r0, uint64_t nr, uint64_t sr) {
    whole(r, cl, mtx);
    p.row0 = r0;
    p.nrows = nr;
    p.store_rows = sr;
  };
  auto colpart = [&](uint64_t r, uint64_t cl, uint64_t c0, uint64_t nc, uint64_t sc) {
    whole(r, cl, true);
    p.col0 = c0;
    p.ncols = nc;
    p.store_cols = sc;
  };
  if (global == 0) whole(V, H, true);
  else if (global == 1) whole(H, 1, false);
  else if (global == 2) rowpart(V, H, true, rk * Vl, Vl, Vl);
  else switch (suffix) {
    case 0: case 8: whole(H, 1, false); break;
    case 1: rowpart(qd, H, true, rk * qdl, qdl, qdl); break;
    case 2: rowpart(qd, 1, false, rk * qdl, qdl, qdl); break;
    case 3: case 5: rowpart(kvd, H, true, rk * kvdl, kvdl, kvdl); break;
    case 4: case 6: rowpart(kvd, 1, false, rk * kvdl, kvdl, kvdl); break;
    case 7: colpart(H, qd, rk * qdl, qdl, qdp); break;
    case 9: case 10: rowpart(I, H, true, rk * Ic, Ic, Il); break;
    case 11: colpart(H, I, rk * Ic, Ic, Il); break;
  }
  return p;
}

int fail(myos_ctx* c, int code, const std::string& msg) {
  if (c) c->err = msg;
  return code;
}

#define CK(call)                                                                   \
  do {                                                                             \
    cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess)                                                         \
      return fail(c, MYOS_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

size_t have_index(const myos_ctx* c, int layer, int suffix) {
  return (size_t)layer * kSuffixes + suffix;
}
size_t have_embed(const myos_ctx* c) { return (size_t)c->s.num_layers * kSuffixes; }

size_t prefetch_cap(const myos_ctx* c, int grid) {
  if (c->prefetch_total == 0) return 0;
  return (c->prefetch_total / (size_t)grid + 15) & ~(size_t)15;
}

// Host-built RoPE table: cos/sin of f32(pos) * (1 / powf(theta, 2i/d)) with
// glibc libm, exactly rope.rs:186-194, so the device applies bit-identical
// rotations.
void rope_table(const myos_shape& s, size_t max_seq, std::vector<float>* cs,
                std::vector<float>* sn) {
  size_t half = s.head_dim / 2;
  cs->assign(max_seq * half, 0.f);
  sn->assign(max_seq * half, 0.f);
  std::vector<float> inv(half);
  for (size_t i = 0; i < half; ++i) {
    volatile float exponent = (float)(2 * i) / (float)s.head_dim;
    inv[i] = 1.0f / powf(s.rope_theta, exponent);
  }
  for (size_t p = 0; p < max_seq; ++p)
    for (size_t i = 0; i < half; ++i) {
      volatile float angle = (float)p * inv[i];
      (*cs)[p * half + i] = cosf(angle);
      (*sn)[p * half + i] = sinf(angle);
    }
}

int check_shape(const myos_shape& s) {
  if (s.hidden == 0 || s.num_q_heads == 0 || s.num_kv_heads == 0 || s.head_dim == 0 ||
      s.head_dim % 2 != 0 || s.num_q_heads % s.num_kv_heads != 0 || s.intermediate == 0 ||
      s.vocab == 0 || s.num_layers == 0)
    return MYOS_ERR_SHAPE;
  if (s.num_q_heads / s.num_kv_heads > 8 || s.head_dim > 256) return MYOS_ERR_SHAPE;
  return MYOS_OK;
}

// Copy host bytes to device through the pinned ring (double-buffered).
int stage_h2d(myos_ctx* c, void* dst, const void* src, size_t n) {
  const uint8_t* s = (const uint8_t*)src;
  uint8_t* d = (uint8_t*)dst;
  int& slot = c->pin_slot;
  while (n) {
    size_t chunk = n < c->pin_bytes ? n : c->pin_bytes;
    CK(cudaEventSynchronize(c->pin_ev[slot]));
    memcpy(c->pin[slot], s, chunk);
    CK(cudaMemcpyAsync(d, c->pin[slot], chunk, cudaMemcpyHostToDevice, c->copy_st));
    CK(cudaEventRecord(c->pin_ev[slot], c->copy_st));
    slot ^= 1;
    s += chunk;
    d += chunk;
    n -= chunk;
  }
  return MYOS_OK;
}

int stage_bf16_as_f32(myos_ctx* c, float* dst, const void* src, size_t n) {
  std::vector<float> tmp(n);
  const uint8_t* b = (const uint8_t*)src;
  for (size_t i = 0; i < n; ++i) {
    uint32_t bits = ((uint32_t)b[2 * i] | ((uint32_t)b[2 * i + 1] << 8)) << 16;
    memcpy(&tmp[i], &bits, 4);
  }
  return stage_h2d(c, dst, tmp.data(), n * 4);
}

int sync_copies(myos_ctx* c) {
  CK(cudaStreamSynchronize(c->copy_st));
  return MYOS_OK;
}

// ---------------------------------------------------------------- step enqueue
enum KernelKind { K_QKV = 0, K_ATTN = 1, K_O = 2, K_GU = 3, K_DOWN = 4, K_HEAD = 5, K_END = 6 };

KTrace ktrace_at(const myos_ctx* c, int slot) {
  KTrace t = {};
  if (c->ktrace && !c->profiling) {
    t.buf = c->ktrace;
    t.slot = slot;
    t.nslot = 5 * (int)c->s.num_layers + 1;
  }
  return t;
}

// Tensor parallel residual update: each rank's projection writes its partial
// sum to tp_part (rank 0 adds the residual), then the ranks' parts are summed
// into every rank's residual.
void tp_partial(const myos_ctx* c, GemvArgs* a, int kind) {
  if (c->tp_size == 1) return;
  a->y = c->tp_part;
  a->res = c->tp_rank == 0 ? c->resid : nullptr;
  a->res_zero = c->tp_rank == 0 ? 0 : 1;
  if (c->tp_p2p) a->push = kind == K_O ? c->push_o : c->push_d;
}

int tp_sum_resid(myos_ctx* c, int kind) {
  if (c->tp_size == 1) return MYOS_OK;
  if (c->tp_p2p) {
    TpReduceArgs r = {};
    r.n = c->tp_size;
    r.H = (int)c->s.hidden;
    r.inbox = kind == K_O ? c->inbox_o : c->inbox_d;
    r.seq = c->tp_seq;
    r.done = c->tp_seq + 1;
    r.out = c->resid;
    r.err = &c->ctl->err;
    CK(launch_tp_reduce(r, c->st, true));
    return MYOS_OK;
  }
  if (!tp_allreduce_sum(c->tp_part, c->resid, c->s.hidden, c->comm, c->st))
    return fail(c, MYOS_ERR_NCCL, "allreduce of the residual update failed");
  return MYOS_OK;
}

// After a head pass, every rank's logits slice to every rank (in place).
int tp_gather_logits(myos_ctx* c) {
  if (c->tp_size == 1) return MYOS_OK;
  if (!tp_allgather(c->logits + c->head_row0, c->logits, (size_t)c->head_rows * 4, c->comm, c->st))
    return fail(c, MYOS_ERR_NCCL, "allgather of the logits failed");
  return MYOS_OK;
}

int launch_kind(myos_ctx* c, int kind, int l, const uint32_t* feed, bool pdl, bool embed_l0) {
  const myos_shape& s = c->s;
  const int H = (int)s.hidden, I = (int)s.intermediate;
  const int kv_bf16 = c->o.kv_dtype == MYOS_KV_BF16;
  const size_t kv_elt = kv_bf16 ? 2 : 4;
  if (kind == K_END) {
    CK(launch_step_end(c->ctl, c->st, pdl));
    return MYOS_OK;
  }
  if (kind == K_HEAD) {
    GemvArgs h = {};
    h.w = s.tied_head ? c->embed + (size_t)c->head_row0 * H : c->lm_head;
    h.M = (int)c->head_rows;
    h.K = H;
    h.in.x = c->resid;
    h.in.ctl = c->ctl;
    h.in.gamma = c->final_norm;
    h.in.eps = s.rms_eps;
    h.y = c->logits + c->head_row0;
    h.prefetch_cap = prefetch_cap(c, c->grid_head);
    h.part_val = c->part_val;
    h.part_idx = c->part_idx;
    h.counter = c->counters;
    // While profiling, the head runs many times per step index: no records.
    h.err = &c->ctl->err;
    h.rec_fed = c->profiling ? nullptr : c->rec_fed;
    h.rec_argmax = c->profiling ? nullptr : c->rec_argmax;
    h.tr = ktrace_at(c, 5 * (int)s.num_layers);
    h.warps = c->warps_head;
    if (c->tp_size > 1) {
      h.row0 = c->head_row0;
      if (c->tp_p2p) h.push = c->push_c;
      else h.tp_cand = c->tp_cand;
    }
    CK(launch_gemv(EPI_ARGMAX, h, c->grid_head, c->st, pdl));
    if (c->tp_size > 1) {  // every rank's slice maximum, then the first global one
      uint32_t* rf = c->profiling ? nullptr : c->rec_fed;
      uint32_t* ra = c->profiling ? nullptr : c->rec_argmax;
      if (c->tp_p2p) {
        CK(launch_tp_pick(c->inbox_c, c->tp_size, c->tp_seq, c->ctl, rf, ra, c->st));
      } else {
        if (!tp_allgather(c->tp_cand, c->tp_cand + 2, 8, c->comm, c->st))
          return fail(c, MYOS_ERR_NCCL, "allgather of the head candidates failed");
        CK(launch_tp_pick(c->tp_cand + 2, c->tp_size, nullptr, c->ctl, rf, ra, c->st));
      }
    }
    return MYOS_OK;
  }
  const LayerW& w = c->layers[l];
  if (kind == K_QKV) {
    GemvArgs q = {};
    q.w = w.wqkv;
    q.M = (int)(c->qd + 2 * c->kvd);
    q.K = H;
    q.in.x = c->resid;
    q.in.embed = (l == 0 && embed_l0) ? c->embed : nullptr;
    q.in.feed = feed;
    q.in.ctl = c->ctl;
    q.in.x_store = (l == 0 && embed_l0) ? c->resid : nullptr;
    q.in.gamma = w.ln1;
    q.in.eps = s.rms_eps;
    q.y = c->qkv;
    q.bias = w.bqkv;
    q.err = &c->ctl->err;
    q.prefetch_cap = prefetch_cap(c, c->grid_qkv);
    q.tr = ktrace_at(c, 5 * l + K_QKV);
    q.warps = c->warps_qkv;
    CK(launch_gemv(EPI_BIAS, q, c->grid_qkv, c->st, pdl));
  } else if (kind == K_ATTN) {
    AttnArgs at = {};
    at.q = c->qkv;
    at.kc = (uint8_t*)c->kcache + (size_t)l * c->kv_layer_elems * kv_elt;
    at.vc = (uint8_t*)c->vcache + (size_t)l * c->kv_layer_elems * kv_elt;
    at.S = (int)c->o.max_seq;
    at.Hq = (int)s.num_q_heads;
    at.Hkv = (int)s.num_kv_heads;
    at.d = (int)s.head_dim;
    at.G = (int)c->G;
    at.ctl = c->ctl;
    at.cos_t = c->cos_t;
    at.sin_t = c->sin_t;
    at.chunk = c->attn_chunk;
    at.nsplit = c->attn_nsplit;
    at.scale = 1.0f / sqrtf((float)s.head_dim);
    at.part_o = c->part_o;
    at.part_m = c->part_m;
    at.part_l = c->part_l;
    at.counters = c->counters + 1;
    at.arrive = c->attn_arrive;
    at.out = c->attn;
    at.decode = 1;
    at.defer_merge = c->defer_merge;
    at.cluster = c->attn_cluster;
    at.tr = ktrace_at(c, 5 * l + K_ATTN);

    CK(launch_attention(at, kv_bf16, c->st, pdl));
  } else if (kind == K_O) {
    GemvArgs o = {};
    o.w = w.wo;
    o.M = H;
    o.K = (int)c->qd_pad;
    o.in.x = c->attn;
    o.in.ctl = c->ctl;
    if (c->defer_merge) {  // the staging merges the attention splits
      o.in.part_o = c->part_o;
      o.in.part_m = c->part_m;
      o.in.part_l = c->part_l;
      o.in.m_G = (int)c->G;
      o.in.m_d = (int)s.head_dim;
      o.in.m_nsplit = c->attn_nsplit;
      o.in.m_chunk = c->attn_chunk;
    }
    o.y = c->resid;
    o.err = &c->ctl->err;
    o.prefetch_cap = prefetch_cap(c, c->grid_o);
    o.tr = ktrace_at(c, 5 * l + K_O);
    o.warps = c->warps_o;
    if (c->grid_mlp && c->mlp_pf_rows > 0) {  // the first gate/up rows of every MLP block
      o.pf_ptr[0] = w.wg;
      o.pf_ptr[1] = w.wu;
      o.pf_bytes[0] = (size_t)c->mlp_pf_rows * H * 2;
      o.pf_stride = (size_t)kMlpSlice * H * 2;
      o.pf_n = c->grid_mlp;
      o.pf_mode = 1;
    }
    tp_partial(c, &o, K_O);
    CK(launch_gemv(EPI_RESID, o, c->grid_o, c->st, pdl));
    if (int st = tp_sum_resid(c, K_O)) return st;
  } else if (kind == K_GU && c->grid_mlp) {
    MlpArgs m = {};
    m.wg = w.wg;
    m.wu = w.wu;
    m.wd = w.wd;
    m.wd_slices = c->mlp_wd ? c->mlp_wd + (size_t)l * H * I : nullptr;
    m.gamma = w.ln2;
    m.eps = s.rms_eps;
    m.H = H;
    m.I = I;
    m.resid = c->resid;
    m.part = c->mlp_part;
    m.arrive = c->mlp_arrive;
    m.ctl = c->ctl;
    m.err = &c->ctl->err;
    m.wait_ns = 1000000000ull;
    m.tr = ktrace_at(c, 5 * l + K_GU);
    CK(launch_mlp(m, c->grid_mlp, c->st, pdl));
  } else if (kind == K_DOWN && c->grid_mlp) {
    // part of the fused MLP launch
  } else if (kind == K_GU) {
    GemvArgs gu = {};
    gu.w = w.wg;
    gu.w2 = w.wu;
    gu.M = I;
    gu.K = H;
    gu.in.x = c->resid;
    gu.in.ctl = c->ctl;
    gu.in.gamma = w.ln2;
    gu.in.eps = s.rms_eps;
    gu.y = c->act;
    gu.err = &c->ctl->err;
    gu.prefetch_cap = prefetch_cap(c, c->grid_gu);
    gu.tr = ktrace_at(c, 5 * l + K_GU);
    gu.warps = c->warps_gu;
    CK(launch_gemv(EPI_SWIGLU, gu, c->grid_gu, c->st, pdl));
  } else if (kind == K_DOWN) {
    GemvArgs dn = {};
    dn.w = w.wd;
    dn.M = H;
    dn.K = I;
    dn.in.x = c->act;
    dn.in.ctl = c->ctl;
    dn.y = c->resid;
    dn.err = &c->ctl->err;
    dn.prefetch_cap = prefetch_cap(c, c->grid_down);
    dn.tr = ktrace_at(c, 5 * l + K_DOWN);
    dn.warps = c->warps_down;
    tp_partial(c, &dn, K_DOWN);
    CK(launch_gemv(EPI_RESID, dn, c->grid_down, c->st, pdl));
    if (int st = tp_sum_resid(c, K_DOWN)) return st;
  }
  return MYOS_OK;
}

int enqueue_step(myos_ctx* c, bool head, const uint32_t* feed, bool first_pdl) {
  const int L = (int)c->s.num_layers;
  for (int l = 0; l < L; ++l) {
    for (int k = K_QKV; k <= K_DOWN; ++k) {
      int st = launch_kind(c, k, l, feed, (l > 0 || k > K_QKV) || first_pdl, true);
      if (st) return st;
    }
  }
  return launch_kind(c, head ? K_HEAD : K_END, 0, feed, true, true);
}

// Algorithmic bytes of one launch of each kind (weights + activations + KV).
double kind_bytes(const myos_ctx* c, int kind) {
  const myos_shape& s = c->s;
  const double H = s.hidden, I = s.intermediate, V = s.vocab, qd = c->qd, kvd = c->kvd;
  const double kv_elt = c->o.kv_dtype == MYOS_KV_BF16 ? 2 : 4;
  switch (kind) {
    case K_QKV: return (qd + 2 * kvd) * H * 2 + (qd + 2 * kvd) * 8 + H * 8;
    case K_ATTN: return 2.0 * s.num_kv_heads * (double)(c->len + 1) * s.head_dim * kv_elt +
                        (qd + 2 * kvd) * 4 + qd * 4;
    case K_O: return H * qd * 2 + qd * 4 + H * 8;
    case K_GU:  // the fused MLP: gate, up and down weights, the residual read and written
      if (c->grid_mlp) return 3 * I * H * 2 + H * 8;
      return 2 * I * H * 2 + H * 8 + I * 4;
    case K_DOWN: return c->grid_mlp ? 0 : H * I * 2 + I * 4 + H * 8;
    case K_HEAD: return V * H * 2 + H * 8 + V * 4;
  }
  return 0;
}

int run_steps(myos_ctx* c, int kind, size_t nsteps) {
  const bool head = kind != G_FEED_NOHEAD;
  const uint32_t* feed = kind == G_ARGMAX_HEAD ? nullptr : c->feed;
  if (!c->o.use_graphs) {
    for (size_t i = 0; i < nsteps; ++i) {
      int st = enqueue_step(c, head, feed, i > 0);
      if (st) return st;
    }
    return MYOS_OK;
  }
  size_t done = 0;
  while (done < nsteps) {
    int chunk = (int)((nsteps - done) >= (size_t)c->steps_per_graph ? c->steps_per_graph : 1);
    auto key = std::make_pair(kind, chunk);
    auto it = c->graphs.find(key);
    if (it == c->graphs.end()) {
      cudaGraph_t g;
      CK(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
      int st = MYOS_OK;
      const uint64_t before = launches_total();  // a capture launches nothing
      for (int i = 0; i < chunk && st == MYOS_OK; ++i) st = enqueue_step(c, head, feed, i > 0);
      const uint64_t captured = launches_total() - before;
      launches_uncount(captured);
      c->graph_kernels[key] = captured;
      cudaError_t ce = cudaStreamEndCapture(c->st, &g);
      if (st) return st;
      if (ce != cudaSuccess)
        return fail(c, MYOS_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
      cudaGraphExec_t ge;
      ce = cudaGraphInstantiate(&ge, g, 0);
      cudaGraphDestroy(g);
      if (ce != cudaSuccess)
        return fail(c, MYOS_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
      it = c->graphs.emplace(key, ge).first;
    }
    CK(counted(cudaGraphLaunch(it->second, c->st), c->graph_kernels[key]));
    done += (size_t)chunk;
  }
  return MYOS_OK;
}

// Upload ctl.step = 0 (and pos when asked) before a call.
int set_ctl(myos_ctx* c, bool set_pos) {
  CK(cudaStreamWaitEvent(c->st, c->load_ev, 0));
  // Peer-memory waits are bounded in time: start every rank's call together
  // (a one-float NCCL allreduce holds each GPU until all ranks are here).
  if (c->tp_p2p && !tp_allreduce_sum(c->tp_cand, c->tp_cand, 1, c->comm, c->st))
    return fail(c, MYOS_ERR_NCCL, "tensor-parallel call alignment failed");
  if (c->ktrace)
    CK(cudaMemcpyAsync(c->ktrace, c->ktrace_init.data(), c->ktrace_init.size() * 8,
                       cudaMemcpyHostToDevice, c->st));
  c->ctl_host->step = 0;
  c->ctl_host->pos = (uint32_t)c->len;
  if (set_pos) {
    CK(cudaMemcpyAsync(c->ctl, c->ctl_host, 8, cudaMemcpyHostToDevice, c->st));
  } else {
    CK(cudaMemcpyAsync(&c->ctl->step, &c->ctl_host->step, 4, cudaMemcpyHostToDevice, c->st));
  }
  return MYOS_OK;
}

int finish(myos_ctx* c) {
  cudaError_t e = cudaMemcpyAsync(&c->ctl_host->err, &c->ctl->err, 4, cudaMemcpyDeviceToHost, c->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);
  if (e != cudaSuccess) return fail(c, MYOS_ERR_CUDA, std::string("step: ") + cudaGetErrorString(e));
  if (c->ktrace) {  // launch timeline of the last call, for offline analysis
    const size_t nt = (size_t)kTraceSteps * (5 * c->s.num_layers + 1) * kTraceWidth;
    std::vector<uint64_t> h(nt);
    if (cudaMemcpy(h.data(), c->ktrace, nt * 8, cudaMemcpyDeviceToHost) == cudaSuccess) {
      if (FILE* f = fopen(c->ktrace_file.c_str(), "wb")) {
        fwrite(h.data(), 8, nt, f);
        fclose(f);
      }
    }
  }
  if (c->ctl_host->err) {
    const uint32_t bits = c->ctl_host->err;
    c->ctl_host->err = 0;
    cudaMemcpy(&c->ctl->err, &c->ctl_host->err, 4, cudaMemcpyHostToDevice);
    // an arrival count left partway would misplace the next MLP launch's target
    if (c->mlp_arrive) cudaMemset(c->mlp_arrive, 0, sizeof(unsigned long long));
    cudaMemset(c->counters, 0, (1 + c->s.num_kv_heads) * 4);
    // arrival counts left partway would misplace the next launch's targets
    cudaMemset(c->attn_arrive, 0, c->s.num_kv_heads * sizeof(unsigned long long));
    return fail(c, MYOS_ERR_TIMEOUT,
                "a bounded device wait gave up (bits " + std::to_string(bits) + ")");
  }
  return MYOS_OK;
}

int missing_weight(myos_ctx* c) {
  const myos_shape& s = c->s;
  if (!c->have[have_embed(c)]) return fail(c, MYOS_ERR_WEIGHT_MISSING, std::string("tensor not found: ") + kEmbed);
  if (!c->have[have_embed(c) + 1])
    return fail(c, MYOS_ERR_WEIGHT_MISSING, std::string("tensor not found: ") + kFinalNorm);
  for (uint32_t l = 0; l < s.num_layers; ++l)
    for (int k = 0; k < kSuffixes; ++k)
      if (!c->have[have_index(c, (int)l, k)])
        return fail(c, MYOS_ERR_WEIGHT_MISSING, "tensor not found: model.layers." +
                                                   std::to_string(l) + "." + kSuffix[k]);
  if (!s.tied_head && !c->have[have_embed(c) + 2])
    return fail(c, MYOS_ERR_WEIGHT_MISSING, std::string("tensor not found: ") + kLmHead);
  return MYOS_OK;
}

}  // namespace

// ================================================================ C ABI
// (Re)allocates *p to at least `need` bytes; keeps a large enough buffer.
template <class T>
static int grow(myos_ctx* c, T** p, size_t* have, size_t need) {
  if (*have >= need && *p) return MYOS_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  CK(cudaMalloc(p, need));
  *have = need;
  return MYOS_OK;
}

extern "C" {

const char* myos_version(void) { return "myos-b200 0.1 (sm_100a)"; }

myos_shape myos_shape_qwen25_1_5b(void) {
  myos_shape s;
  s.hidden = 1536;
  s.num_q_heads = 12;
  s.num_kv_heads = 2;
  s.head_dim = 128;
  s.rope_theta = 1000000.0f;
  s.intermediate = 8960;
  s.vocab = 151936;
  s.num_layers = 28;
  s.rms_eps = 1e-6f;
  s.tied_head = 1;
  return s;
}

myos_shape myos_shape_qwen25_14b(void) {
  myos_shape s;
  s.hidden = 5120;
  s.num_q_heads = 40;
  s.num_kv_heads = 8;
  s.head_dim = 128;
  s.rope_theta = 1000000.0f;
  s.intermediate = 13824;
  s.vocab = 152064;
  s.num_layers = 48;
  s.rms_eps = 1e-6f;
  s.tied_head = 0;
  return s;
}

const char* myos_last_error(const myos_ctx* c) { return c ? c->err.c_str() : "null context"; }

// Peer-memory exchange for a tensor-parallel context: every rank's inboxes
// and counters in one allocation, its IPC handle and device UUID gathered
// over NCCL, every other rank's allocation mapped here. The ranks agree on
// the outcome (all map every peer, or all keep the NCCL collectives).
static int setup_tp_p2p(myos_ctx* c) {
  const int n = c->tp_size, me = c->tp_rank;
  const size_t H = c->s.hidden;
  const size_t in_bytes = align256((size_t)n * H * 8);  // one (value, epoch) word per row
  const size_t off_c = 2 * in_bytes, off_f = off_c + 256, total = off_f + 256;
  CK(cudaMalloc(&c->tp_link, total));
  CK(cudaMemset(c->tp_link, 0, total));
  struct Card {
    cudaIpcMemHandle_t h;
    uint8_t uuid[16];
    int32_t ok;
    uint8_t pad[12];
  };
  Card mine = {};
  mine.ok = cudaIpcGetMemHandle(&mine.h, c->tp_link) == cudaSuccess;
  cudaGetLastError();
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, c->device));
  memcpy(mine.uuid, &prop.uuid, 16);
  std::vector<Card> all(n);
  Card* d = nullptr;
  CK(cudaMalloc(&d, n * sizeof(Card)));
  CK(cudaMemcpy(d + me, &mine, sizeof(Card), cudaMemcpyHostToDevice));
  const bool sent = tp_allgather(d + me, d, sizeof(Card), c->comm, c->st);
  cudaError_t e = cudaStreamSynchronize(c->st);
  if (e == cudaSuccess) e = cudaMemcpy(all.data(), d, n * sizeof(Card), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (!sent) return fail(c, MYOS_ERR_NCCL, "exchange of peer handles failed");
  CK(e);
  // the bounded waits assume each rank has a GPU of its own
  for (int p = 0; p < n; ++p)
    for (int q = p + 1; q < n; ++q)
      if (memcmp(all[p].uuid, all[q].uuid, 16) == 0)
        return fail(c, MYOS_ERR_ARG, "two tensor-parallel ranks share one GPU");
  bool ok = true;
  for (int p = 0; p < n; ++p) ok = ok && all[p].ok;
  for (int p = 0; p < n && ok; ++p) {
    if (p == me) continue;
    if (cudaIpcOpenMemHandle(&c->tp_peer[p], all[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      c->tp_peer[p] = nullptr;
      ok = false;
    }
  }
  // every rank mapped every peer?
  const float one = ok ? 1.0f : 0.0f;
  CK(cudaMemcpy(c->tp_cand, &one, 4, cudaMemcpyHostToDevice));
  if (!tp_allreduce_sum(c->tp_cand, c->tp_cand, 1, c->comm, c->st))
    return fail(c, MYOS_ERR_NCCL, "peer-mapping agreement failed");
  float agreed = 0.0f;
  CK(cudaStreamSynchronize(c->st));
  CK(cudaMemcpy(&agreed, c->tp_cand, 4, cudaMemcpyDeviceToHost));
  if (agreed != (float)n) {  // keep the NCCL collectives
    for (int p = 0; p < n; ++p)
      if (p != me && c->tp_peer[p]) cudaIpcCloseMemHandle(c->tp_peer[p]);
    memset(c->tp_peer, 0, sizeof c->tp_peer);
    return MYOS_OK;
  }
  c->tp_peer[me] = c->tp_link;
  c->tp_seq = (unsigned*)(c->tp_link + off_f);
  for (int p = 0; p < n; ++p) {
    uint8_t* base = (uint8_t*)c->tp_peer[p];
    c->push_o.out[p] = (float*)base + 2 * (size_t)me * H;
    c->push_d.out[p] = (float*)(base + in_bytes) + 2 * (size_t)me * H;
    c->push_c.out[p] = (float*)(base + off_c) + 4 * me;  // two words per rank
  }
  c->push_o.n = c->push_d.n = c->push_c.n = n;
  c->push_o.seq = c->push_d.seq = c->push_c.seq = c->tp_seq;
  c->inbox_o = (float*)c->tp_link;
  c->inbox_d = (float*)(c->tp_link + in_bytes);
  c->inbox_c = (float*)(c->tp_link + off_c);
  c->tp_p2p = true;
  return MYOS_OK;
}

static int create_impl(myos_ctx* c, const myos_shape* shape, const myos_opts* opts,
                       const myos_tp* tp) {
  c->full = *shape;
  c->s = *shape;
  c->o = *opts;
  c->i_cut = shape->intermediate;
  c->head_rows = shape->vocab;
  if (tp && tp->size > 1) {  // this rank's slice (divisibility checked by the caller)
    const uint32_t N = (uint32_t)tp->size;
    c->tp_size = tp->size;
    c->tp_rank = tp->rank;
    c->s.num_q_heads /= N;
    c->s.num_kv_heads /= N;
    c->i_cut = shape->intermediate / N;
    c->s.intermediate = (c->i_cut + 255) / 256 * 256;  // zero rows/columns pad the GEMV width
    c->head_rows = shape->vocab / N;
    c->head_row0 = (uint32_t)tp->rank * c->head_rows;
  }
  c->device = opts->device;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= opts->device || opts->device < 0) {
    cudaGetLastError();
    return fail(c, MYOS_ERR_CUDA, "no CUDA device with this ordinal");
  }
  CK(cudaSetDevice(opts->device));
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, opts->device));
  if (prop.major != 10) return fail(c, MYOS_ERR_CUDA, "device is not sm_100 (B200)");
  c->num_sms = prop.multiProcessorCount;
  CK(kernels_init());
  if (const char* e = getenv("MYOS_PREFETCH_MB")) c->prefetch_total = (size_t)atol(e) << 20;
  if (const char* e = getenv("MYOS_STEPS_PER_GRAPH")) c->steps_per_graph = atoi(e) > 0 ? atoi(e) : 1;
  const myos_shape& s = c->s;
  c->qd = (size_t)s.num_q_heads * s.head_dim;
  c->kvd = (size_t)s.num_kv_heads * s.head_dim;
  // A tensor-parallel rank's o_proj slice is zero-padded to a multiple of
  // 256 columns (the streaming GEMV's width), fed by a zero-padded attention
  // output (14B at 8 ranks: 5 heads x 128 = 640 -> 768).
  c->qd_pad = c->tp_size > 1 ? (c->qd + 255) / 256 * 256 : c->qd;
  c->G = s.num_q_heads / s.num_kv_heads;
  const size_t H = s.hidden, I = s.intermediate, V = s.vocab, L = s.num_layers;
  // weight arena
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  size_t o_embed = take(V * H * 2);
  size_t o_lm = s.tied_head ? 0 : take((size_t)c->head_rows * H * 2);
  size_t o_fn = take(H * 4);
  std::vector<size_t> lo(L * 8);
  for (size_t l = 0; l < L; ++l) {
    lo[l * 8 + 0] = take((c->qd + 2 * c->kvd) * H * 2);
    lo[l * 8 + 1] = take(H * c->qd_pad * 2);
    lo[l * 8 + 2] = take(I * H * 2);
    lo[l * 8 + 3] = take(I * H * 2);
    lo[l * 8 + 4] = take(H * I * 2);
    lo[l * 8 + 5] = take((c->qd + 2 * c->kvd) * 4);
    lo[l * 8 + 6] = take(H * 4);
    lo[l * 8 + 7] = take(H * 4);
  }
  c->warena_bytes = off;
  CK(cudaMalloc(&c->warena, c->warena_bytes));
  CK(cudaMemset(c->warena, 0, c->warena_bytes));
  c->embed = (uint16_t*)(c->warena + o_embed);
  c->lm_head = s.tied_head ? nullptr : (uint16_t*)(c->warena + o_lm);
  c->final_norm = (float*)(c->warena + o_fn);
  c->layers.resize(L);
  for (size_t l = 0; l < L; ++l) {
    LayerW& w = c->layers[l];
    w.wqkv = (uint16_t*)(c->warena + lo[l * 8 + 0]);
    w.wo = (uint16_t*)(c->warena + lo[l * 8 + 1]);
    w.wg = (uint16_t*)(c->warena + lo[l * 8 + 2]);
    w.wu = (uint16_t*)(c->warena + lo[l * 8 + 3]);
    w.wd = (uint16_t*)(c->warena + lo[l * 8 + 4]);
    w.bqkv = (float*)(c->warena + lo[l * 8 + 5]);
    w.ln1 = (float*)(c->warena + lo[l * 8 + 6]);
    w.ln2 = (float*)(c->warena + lo[l * 8 + 7]);
  }
  c->have.assign(L * kSuffixes + 3, 0);
  // KV cache [L][Hkv][max_seq][d]
  const size_t S = opts->max_seq, d = s.head_dim, kv_elt = opts->kv_dtype == MYOS_KV_BF16 ? 2 : 4;
  c->kv_layer_elems = (size_t)s.num_kv_heads * S * d;
  CK(cudaMalloc(&c->kcache, L * c->kv_layer_elems * kv_elt));
  CK(cudaMalloc(&c->vcache, L * c->kv_layer_elems * kv_elt));
  CK(cudaMemset(c->kcache, 0, L * c->kv_layer_elems * kv_elt));
  CK(cudaMemset(c->vcache, 0, L * c->kv_layer_elems * kv_elt));
  // geometry
  c->grid_qkv = gemv_grid((int)(c->qd + 2 * c->kvd), (int)H, 1, c->num_sms);
  c->grid_o = gemv_grid((int)H, (int)c->qd_pad, 1, c->num_sms);
  c->grid_gu = gemv_grid((int)I, (int)H, 2, c->num_sms);
  c->grid_down = gemv_grid((int)H, (int)I, 1, c->num_sms);
  c->grid_head = gemv_grid((int)c->head_rows, (int)H, 1, c->num_sms);
  c->warps_qkv = gemv_warps((int)(c->qd + 2 * c->kvd), (int)H, 1, true, c->grid_qkv);
  c->warps_o = gemv_warps((int)H, (int)c->qd_pad, 1, false, c->grid_o);
  c->warps_gu = gemv_warps((int)I, (int)H, 2, true, c->grid_gu);
  c->warps_down = gemv_warps((int)H, (int)I, 1, false, c->grid_down);
  c->warps_head = gemv_warps((int)c->head_rows, (int)H, 1, true, c->grid_head);
  size_t nsplit = (S + 31) / 32;
  size_t cap = (size_t)c->num_sms / s.num_kv_heads;
  if (cap > 160) cap = 160;  // the split merge takes at most 160 splits
  if (cap < 1) cap = 1;
  if (nsplit > cap) nsplit = cap;
  c->attn_nsplit = (int)nsplit;
  c->attn_chunk = (int)((S + nsplit - 1) / nsplit);
  {
    // MYOS_DEFER_MERGE=1: merge the attention splits in the o_proj staging
    // (saves the attention kernel's fence and counter, but every o_proj block
    // then reads all partials; measured slower for the 1.5B step).
    const char* e = getenv("MYOS_DEFER_MERGE");
    const bool want = e && e[0] == '1';
    c->defer_merge = want && c->qd_pad == c->qd && s.num_q_heads <= 256 &&
                     merge_smem_bytes((int)s.num_q_heads, (int)nsplit, (int)d) <= (96u << 10);
    // MYOS_ATTN_CLUSTER=0 keeps the global-memory last-block merge
    const char* ce = getenv("MYOS_ATTN_CLUSTER");
    c->attn_cluster = !(ce && ce[0] == '0') && !c->defer_merge && nsplit <= 8 && d % 8 == 0;
  }
  // workspace
  CK(cudaMalloc(&c->resid, H * 4));
  CK(cudaMalloc(&c->qkv, (c->qd + 2 * c->kvd) * 4));
  CK(cudaMalloc(&c->attn, c->qd_pad * 4));
  CK(cudaMemset(c->attn, 0, c->qd_pad * 4));  // the padding stays zero
  CK(cudaMalloc(&c->act, I * 4));
  CK(cudaMalloc(&c->logits, V * 4));
  CK(cudaMemset(c->logits, 0, V * 4));
  CK(cudaMemset(c->resid, 0, H * 4));
  CK(cudaMalloc(&c->part_val, (size_t)c->grid_head * 4));
  CK(cudaMalloc(&c->part_idx, (size_t)c->grid_head * 4));
  CK(cudaMalloc(&c->part_o, (size_t)s.num_kv_heads * nsplit * c->G * d * 4));
  CK(cudaMalloc(&c->part_m, (size_t)s.num_kv_heads * nsplit * c->G * 4));
  CK(cudaMalloc(&c->part_l, (size_t)s.num_kv_heads * nsplit * c->G * 4));
  CK(cudaMalloc(&c->counters, (1 + s.num_kv_heads) * 4));
  CK(cudaMemset(c->counters, 0, (1 + s.num_kv_heads) * 4));
  CK(cudaMalloc(&c->attn_arrive, s.num_kv_heads * sizeof(unsigned long long)));
  CK(cudaMemset(c->attn_arrive, 0, s.num_kv_heads * sizeof(unsigned long long)));
  {
    const char* e = getenv("MYOS_MLP");
    if (c->tp_size == 1 && !(e && e[0] == '0')) c->grid_mlp = mlp_grid((int)H, (int)I, c->num_sms);
    if (c->grid_mlp) {
      CK(cudaMalloc(&c->mlp_part, (size_t)H * c->grid_mlp * 4));
      CK(cudaMalloc(&c->mlp_arrive, sizeof(unsigned long long)));
      CK(cudaMemset(c->mlp_arrive, 0, sizeof(unsigned long long)));
      // a second copy of down_proj, by block (MYOS_MLP=i reads it in place)
      if (!(e && e[0] == 'i')) CK(cudaMalloc(&c->mlp_wd, (size_t)L * H * I * 2));
      const char* pe = getenv("MYOS_MLP_PF");
      c->mlp_pf_rows = pe ? atoi(pe) : kMlpSlice;
      if (c->mlp_pf_rows < 0 || c->mlp_pf_rows > kMlpSlice) c->mlp_pf_rows = 0;
    }
  }
  CK(cudaMalloc(&c->ctl, sizeof(StepCtl)));
  CK(cudaMemset(c->ctl, 0, sizeof(StepCtl)));
  CK(cudaMalloc(&c->feed, (S + 1) * 4));
  CK(cudaMalloc(&c->rec_fed, (S + 1) * 4));
  CK(cudaMalloc(&c->rec_argmax, (S + 1) * 4));
  std::vector<float> cs, sn;
  rope_table(s, S, &cs, &sn);
  CK(cudaMalloc(&c->cos_t, cs.size() * 4));
  CK(cudaMalloc(&c->sin_t, sn.size() * 4));
  CK(cudaMemcpy(c->cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(c->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  {
    // GEMM prefill: hidden, q and MLP widths 16-byte aligned for TMA, gate and
    // up rows adjacent (one [2I, H] projection), a supported head dim.
    const char* e = getenv("MYOS_PREFILL");
    const bool want = !(e && e[0] == 's');
    bool ok = want && pf_attn_supported((int)d, (int)c->G) && H % 64 == 0 && I % 64 == 0 &&
              c->qd % 64 == 0 && (c->qd + 2 * c->kvd) % 64 == 0;
    for (size_t l = 0; ok && l < L; ++l) ok = c->layers[l].wu == c->layers[l].wg + I * H;
    if (ok) {
      // prompt tokens per chunk (MYOS_PF_CHUNK: 64..512, a multiple of 64).
      // 256: each chunk reads the weights once for twice the tokens of 128
      // (M = 768 rows: six full 128-row tiles)
      int nc = 256;
      if (const char* pc = getenv("MYOS_PF_CHUNK")) {
        const int v = atoi(pc);
        if (v >= 64 && v <= 512 && v % 64 == 0) nc = v;
      }
      const size_t M = kSplitParts * (size_t)nc;
      const size_t kmax = std::max(H, std::max((size_t)c->qd, I));
      const size_t nmax = std::max(c->qd + 2 * c->kvd, std::max(H, 2 * I));
      const int shapes[4][2] = {{(int)(c->qd + 2 * c->kvd), (int)H}, {(int)H, (int)c->qd},
                                {(int)(2 * I), (int)H}, {(int)H, (int)I}};
      size_t ws = 256;
      for (auto& sh : shapes) ws = std::max(ws, gemm_workspace_bytes((int)M, sh[0], sh[1]));
      CK(cudaMalloc(&c->pf_X, (size_t)nc * H * 4));
      CK(cudaMalloc(&c->pf_A, M * kmax * 2));
      CK(cudaMalloc(&c->pf_D, M * nmax * 4));
      c->pf_D_elems = M * nmax;
      const char* sk = getenv("MYOS_SPLITK");
      c->pf_splitk = !(sk && sk[0] == '0');
      const char* m64 = getenv("MYOS_GEMM_M64");
      c->pf_m64 = !(m64 && m64[0] == '0');
      CK(cudaMalloc(&c->pf_Q, (size_t)nc * (c->qd + 2 * c->kvd) * 4));
      CK(cudaMalloc(&c->pf_ws, ws));
      c->pf_ws_bytes = ws;
      c->pf_chunk = nc;
      CK(pf_init());
      c->pf_ok = true;
    }
  }
  if (const char* kf = getenv("MYOS_KTRACE_FILE")) {
    c->ktrace_file = kf;
    const size_t rows = (size_t)kTraceSteps * (5 * L + 1);
    c->ktrace_init.assign(rows * kTraceWidth, 0);  // max fields start at 0
    for (size_t r = 0; r < rows; ++r)
      c->ktrace_init[kTraceWidth * r] = c->ktrace_init[kTraceWidth * r + 1] = ~0ull;  // min fields
    CK(cudaMalloc(&c->ktrace, rows * kTraceWidth * 8));
  }
  // streams, staging
  CK(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking));
  CK(cudaStreamCreateWithFlags(&c->copy_st, cudaStreamNonBlocking));
  c->pin_bytes = 32ull << 20;
  for (int i = 0; i < 2; ++i) {
    CK(cudaHostAlloc(&c->pin[i], c->pin_bytes, cudaHostAllocDefault));
    CK(cudaEventCreateWithFlags(&c->pin_ev[i], cudaEventDisableTiming));
    CK(cudaEventRecord(c->pin_ev[i], c->copy_st));
  }
  CK(cudaHostAlloc(&c->ctl_host, sizeof(StepCtl), cudaHostAllocDefault));
  memset(c->ctl_host, 0, sizeof(StepCtl));
  CK(cudaEventCreateWithFlags(&c->load_ev, cudaEventDisableTiming));
  CK(cudaEventRecord(c->load_ev, c->copy_st));
  CK(cudaEventCreate(&c->ev0));
  CK(cudaEventCreate(&c->ev1));
  CK(cudaEventCreate(&c->ev2));
  if (c->tp_size > 1) {
    CK(cudaMalloc(&c->tp_part, H * 4));
    CK(cudaMalloc(&c->tp_cand, (2 + 2 * (size_t)c->tp_size) * 4));
    CK(cudaMemset(c->tp_cand, 0, (2 + 2 * (size_t)c->tp_size) * 4));
  }
  CK(cudaDeviceSynchronize());
  if (c->tp_size > 1) {  // blocks until every rank has joined
    std::string why;
    if (!tp_comm_init(&c->comm, c->tp_size, c->tp_rank, tp->unique_id, &why))
      return fail(c, MYOS_ERR_NCCL, "tensor-parallel communicator: " + why);
    const char* m = getenv("MYOS_TP_COMM");
    if (!(m && strcmp(m, "nccl") == 0)) {
      int st = setup_tp_p2p(c);
      if (st) return st;
    }
  }
  return MYOS_OK;
}

int myos_ctx_create(const myos_shape* shape, const myos_opts* opts, myos_ctx** out) {
  return myos_ctx_create_tp(shape, opts, nullptr, out);
}

int myos_tp_unique_id(uint8_t out[128]) {
  if (!out) return MYOS_ERR_ARG;
  std::string why;
  return tp_unique_id(out, &why) ? MYOS_OK : MYOS_ERR_NCCL;
}

int myos_tp_reduce_selftest(int32_t device, uint32_t n, uint32_t H, int32_t fill,
                            uint32_t timeout_ms, float* out) {
  if (n < 1 || n > (uint32_t)kMaxTp || H == 0 || H > (1u << 20) || (fill && !out) ||
      timeout_ms == 0 || timeout_ms > 10000)
    return MYOS_ERR_ARG;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return MYOS_ERR_CUDA;
  }
  if (cudaSetDevice(device) != cudaSuccess || kernels_init() != cudaSuccess) return MYOS_ERR_CUDA;
  const size_t words = (size_t)n * H;
  // inbox words (value bits, epoch) for ranks 0..n-1, then seq, done, err
  std::vector<uint64_t> host(words, 0);
  if (fill)
    for (size_t p = 0; p < n; ++p)
      for (size_t i = 0; i < H; ++i) {
        const float v = 0.25f * (float)(p + 1) + (float)i * (1.0f / 1024.0f);
        uint32_t bits;
        memcpy(&bits, &v, 4);
        host[p * H + i] = (1ull << 32) | bits;  // epoch 1: the first exchange
      }
  uint8_t* buf = nullptr;
  float* d_out = nullptr;
  int rc = MYOS_OK;
  uint32_t ctl[3] = {0, 0, 0};
  if (cudaMalloc(&buf, words * 8 + 256) != cudaSuccess || cudaMalloc(&d_out, (size_t)H * 4) != cudaSuccess) {
    rc = MYOS_ERR_CUDA;
  } else if (cudaMemcpy(buf, host.data(), words * 8, cudaMemcpyHostToDevice) != cudaSuccess ||
             cudaMemset(buf + words * 8, 0, 256) != cudaSuccess) {
    rc = MYOS_ERR_CUDA;
  } else {
    TpReduceArgs r = {};
    r.n = (int)n;
    r.H = (int)H;
    r.inbox = (const float*)buf;
    r.seq = (unsigned*)(buf + words * 8);
    r.done = r.seq + 1;
    r.err = (uint32_t*)(r.seq + 2);
    r.out = d_out;
    r.wait_ns = (uint64_t)timeout_ms * 1000000ull;
    if (launch_tp_reduce(r, 0, false) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(ctl, r.seq, sizeof ctl, cudaMemcpyDeviceToHost) != cudaSuccess ||
        (fill && cudaMemcpy(out, d_out, (size_t)H * 4, cudaMemcpyDeviceToHost) != cudaSuccess))
      rc = MYOS_ERR_CUDA;
    else if (ctl[2] & kErrTpWait)
      rc = MYOS_ERR_TIMEOUT;
    else if (ctl[0] != 1u || ctl[1] != 0u)  // epoch advanced once, block count reset
      rc = MYOS_ERR_CUDA;
  }
  if (buf) cudaFree(buf);
  if (d_out) cudaFree(d_out);
  cudaGetLastError();
  return rc;
}

int myos_ctx_create_tp(const myos_shape* shape, const myos_opts* opts, const myos_tp* tp,
                       myos_ctx** out) {
  if (!shape || !opts || !out) return MYOS_ERR_ARG;
  *out = nullptr;
  if (check_shape(*shape)) return MYOS_ERR_SHAPE;
  if (opts->max_seq == 0) return MYOS_ERR_SHAPE;
  if (opts->kv_dtype != MYOS_KV_F32 && opts->kv_dtype != MYOS_KV_BF16) return MYOS_ERR_ARG;
  if (tp) {
    if (tp->size < 1 || tp->size > kMaxTp || tp->rank < 0 || tp->rank >= tp->size)
      return MYOS_ERR_ARG;
    const uint32_t N = (uint32_t)tp->size;
    if (shape->num_q_heads % N || shape->num_kv_heads % N || shape->intermediate % N ||
        shape->vocab % N || ((shape->num_q_heads / N) * shape->head_dim) % 8)
      return MYOS_ERR_SHAPE;
  }
  myos_ctx* c = new myos_ctx();
  int st = create_impl(c, shape, opts, tp);
  if (st) {
    myos_ctx_destroy(c);
    return st;
  }
  *out = c;
  return MYOS_OK;
}

void myos_ctx_destroy(myos_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->st) cudaStreamSynchronize(c->st);
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);  // they hold NCCL calls
  c->graphs.clear();
  for (int p = 0; p < kMaxTp; ++p)
    if (c->tp_peer[p] && c->tp_peer[p] != c->tp_link) cudaIpcCloseMemHandle(c->tp_peer[p]);
  tp_comm_destroy(c->comm);
  void* dev[] = {c->warena, c->kcache, c->vcache, c->resid, c->qkv, c->attn, c->act, c->logits,
                 c->part_val, c->part_idx, c->part_o, c->part_m, c->part_l, c->counters, (void*)c->attn_arrive, c->ctl,
                 c->feed, c->rec_fed, c->rec_argmax, c->cos_t, c->sin_t, c->mlp_part, c->mlp_arrive, c->mlp_wd,
                 (void*)c->ktrace, c->pf_X, c->pf_D, c->pf_Q, c->pf_A, c->pf_ws,
                 c->bt_k, c->bt_v, c->bt_X, c->bt_D, c->bt_pos, c->bt_rows, c->bt_tok,
                 c->bt_out, c->bt_ids, c->bt_feed, c->tp_part, c->tp_cand, c->tp_link,
                 c->at_o, (void*)c->at_ml, (void*)c->at_arrive, (void*)c->at_work, (void*)c->bt_amax, c->bt_step};
  for (void* p : dev)
    if (p) cudaFree(p);
  for (int i = 0; i < 2; ++i) {
    if (c->pin[i]) cudaFreeHost(c->pin[i]);
    if (c->pin_ev[i]) cudaEventDestroy(c->pin_ev[i]);
  }
  if (c->ctl_host) cudaFreeHost(c->ctl_host);
  if (c->load_ev) cudaEventDestroy(c->load_ev);
  if (c->ev0) cudaEventDestroy(c->ev0);
  if (c->ev1) cudaEventDestroy(c->ev1);
  if (c->ev2) cudaEventDestroy(c->ev2);
  if (c->st) cudaStreamDestroy(c->st);
  if (c->copy_st) cudaStreamDestroy(c->copy_st);
  delete c;
}

int myos_load_tensor(myos_ctx* c, const char* name, int32_t dtype, const int64_t* shape,
                     int32_t rank, const void* bytes, size_t nbytes) {
  if (!c) return MYOS_ERR_ARG;
  if (!name || !*name) return fail(c, MYOS_ERR_EMPTY_NAME, "tensor name is empty");
  if (rank < 0 || (rank > 0 && !shape) || (nbytes && !bytes)) return fail(c, MYOS_ERR_ARG, "bad tensor arguments");
  CK(cudaSetDevice(c->device));
  const myos_shape& s = c->full;  // tensors arrive whole; a tensor-parallel rank keeps its slice
  const uint64_t H = s.hidden, I = s.intermediate, V = s.vocab;
  const uint64_t qd = (uint64_t)s.num_q_heads * s.head_dim, kvd = (uint64_t)s.num_kv_heads * s.head_dim;
  std::string n(name);
  int layer = -1, suffix = -1, global = -1;  // global: 0 embed, 1 final norm, 2 lm_head
  // names the model never reads (e.g. o_proj.bias, the tied model's lm_head:
  // qwen25_block.rs:290-301) are accepted and skipped
  if (!parse_tensor_name(s, n, &layer, &suffix, &global)) return MYOS_OK;
  const myos_tp_part p = tp_part(s, (uint32_t)c->tp_size, (uint32_t)c->tp_rank, global, suffix);
  std::vector<uint64_t> expect = {p.rows};
  if (p.matrix) expect.push_back(p.cols);
  if (dtype != MYOS_BF16)
    return fail(c, MYOS_ERR_WEIGHT_DTYPE, "tensor dtype is not bf16: " + n);
  unsigned __int128 numel = 1;
  for (int i = 0; i < rank; ++i) {
    if (shape[i] < 0) return fail(c, MYOS_ERR_WEIGHT_SHAPE, "negative dimension: " + n);
    numel *= (unsigned __int128)shape[i];
  }
  if (numel * 2 != (unsigned __int128)nbytes)
    return fail(c, MYOS_ERR_WEIGHT_LENGTH, "tensor byte length does not match shape: " + n);
  bool same = (size_t)rank == expect.size();
  for (int i = 0; same && i < rank; ++i) same = (uint64_t)shape[i] == expect[i];
  if (!same) return fail(c, MYOS_ERR_WEIGHT_SHAPE, "tensor shape does not match the layout: " + n);
  // This rank's slice: rows [r0, r0 + nr) of a row-major tensor, or columns
  // [c0, c0 + nc) of every row stored at a row stride of `ld` elements (the
  // padding columns stay zero from the arena's initial clear).
  const uint8_t* src = (const uint8_t*)bytes;
  auto rows = [&](void* dst, uint64_t r0, uint64_t nr, uint64_t row_elems) {
    return stage_h2d(c, dst, src + r0 * row_elems * 2, nr * row_elems * 2);
  };
  auto cols = [&](uint16_t* dst, uint64_t nrows, uint64_t ncols, uint64_t c0, uint64_t nc,
                  uint64_t ld) {
    if (c0 == 0 && nc == ncols && ld == ncols) return stage_h2d(c, dst, src, nrows * ncols * 2);
    std::vector<uint16_t> tmp(nrows * ld, 0);
    for (uint64_t r = 0; r < nrows; ++r) memcpy(&tmp[r * ld], src + (r * ncols + c0) * 2, nc * 2);
    return stage_h2d(c, dst, tmp.data(), tmp.size() * 2);
  };
  auto vec = [&](float* dst) { return stage_bf16_as_f32(c, dst, src + p.row0 * 2, p.nrows); };
  auto mat = [&](void* dst) {
    if (p.col0 == 0 && p.ncols == p.cols) return rows(dst, p.row0, p.nrows, p.cols);
    return cols((uint16_t*)dst, p.rows, p.cols, p.col0, p.ncols, p.store_cols);
  };
  const uint64_t qdl = c->qd, kvdl = c->kvd;
  int st = MYOS_OK;
  if (global == 0) st = mat(c->embed);
  else if (global == 1) st = vec(c->final_norm);
  else if (global == 2) st = mat(c->lm_head);
  else {
    const LayerW& w = c->layers[layer];
    switch (suffix) {
      case 0: st = vec(w.ln1); break;
      case 1: st = mat(w.wqkv); break;
      case 2: st = vec(w.bqkv); break;
      case 3: st = mat(w.wqkv + qdl * H); break;
      case 4: st = vec(w.bqkv + qdl); break;
      case 5: st = mat(w.wqkv + (qdl + kvdl) * H); break;
      case 6: st = vec(w.bqkv + qdl + kvdl); break;
      case 7: st = mat(w.wo); break;
      case 8: st = vec(w.ln2); break;
      case 9: st = mat(w.wg); break;
      case 10: st = mat(w.wu); break;
      case 11:
        st = mat(w.wd);
        if (!st && c->mlp_wd)  // the fused MLP's copy, by block
          CK(launch_mlp_relayout(w.wd, c->mlp_wd + (size_t)layer * H * I, (int)H, (int)I, c->copy_st));
        break;
    }
  }
  if (st) return st;
  CK(cudaEventRecord(c->load_ev, c->copy_st));
  if (global >= 0) c->have[have_embed(c) + global] = 1;
  else c->have[have_index(c, layer, suffix)] = 1;
  return MYOS_OK;
}

int myos_load_safetensors(myos_ctx* c, const char* path) {
  if (!c || !path) return MYOS_ERR_ARG;
  int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(c, MYOS_ERR_IO, std::string(path) + ": " + strerror(errno));
  struct stat stbuf;
  if (fstat(fd, &stbuf) != 0) {
    int e = errno;
    close(fd);
    return fail(c, MYOS_ERR_IO, std::string(path) + ": " + strerror(e));
  }
  size_t len = (size_t)stbuf.st_size;
  const uint8_t* buf = nullptr;
  void* map = nullptr;
  if (len > 0) {
    map = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
      int e = errno;
      close(fd);
      return fail(c, MYOS_ERR_IO, std::string(path) + ": " + strerror(e));
    }
    buf = (const uint8_t*)map;
    madvise(map, len, MADV_SEQUENTIAL);
  }
  close(fd);
  std::vector<StTensor> ts;
  size_t data_off = 0;
  std::string why;
  int rc = MYOS_OK;
  if (st_parse(buf, len, &ts, &data_off, &why)) {
    rc = fail(c, MYOS_ERR_PARSE, "weight buffer could not be parsed: " + why);
  } else {
    for (auto& t : ts)
      if (t.dtype != "F32" && t.dtype != "F16" && t.dtype != "BF16") {
        rc = fail(c, MYOS_ERR_UNSUPPORTED, "tensor dtype is not supported: " + t.name);
        break;
      }
    for (size_t i = 0; rc == MYOS_OK && i < ts.size(); ++i)
      if (ts[i].name.empty()) rc = fail(c, MYOS_ERR_EMPTY_NAME, "tensor name is empty");
    for (size_t i = 0; rc == MYOS_OK && i < ts.size(); ++i) {
      const StTensor& t = ts[i];
      int dt = t.dtype == "F32" ? MYOS_F32 : t.dtype == "F16" ? MYOS_F16 : MYOS_BF16;
      rc = myos_load_tensor(c, t.name.c_str(), dt, t.shape.data(), (int32_t)t.shape.size(),
                            buf + data_off + t.begin, t.end - t.begin);
    }
    if (rc == MYOS_OK) rc = sync_copies(c);
  }
  if (map) munmap(map, len);
  return rc;
}

int myos_check_safetensors(const char* path, size_t* n_tensors, char* err, size_t err_len) {
  auto say = [&](int code, const std::string& msg) {
    if (err && err_len) {
      size_t n = msg.size() < err_len - 1 ? msg.size() : err_len - 1;
      memcpy(err, msg.data(), n);
      err[n] = 0;
    }
    return code;
  };
  if (!path) return MYOS_ERR_ARG;
  int fd = open(path, O_RDONLY);
  if (fd < 0) return say(MYOS_ERR_IO, std::string(path) + ": " + strerror(errno));
  struct stat stbuf;
  if (fstat(fd, &stbuf) != 0) {
    int e = errno;
    close(fd);
    return say(MYOS_ERR_IO, std::string(path) + ": " + strerror(e));
  }
  size_t len = (size_t)stbuf.st_size;
  void* map = nullptr;
  if (len > 0) {
    map = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
      int e = errno;
      close(fd);
      return say(MYOS_ERR_IO, std::string(path) + ": " + strerror(e));
    }
  }
  close(fd);
  std::vector<StTensor> ts;
  size_t data_off = 0;
  std::string why;
  int rc = MYOS_OK;
  if (st_parse((const uint8_t*)map, len, &ts, &data_off, &why)) {
    rc = say(MYOS_ERR_PARSE, "weight buffer could not be parsed: " + why);
  } else {
    for (auto& t : ts) {
      if (t.dtype != "F32" && t.dtype != "F16" && t.dtype != "BF16") {
        rc = say(MYOS_ERR_UNSUPPORTED, "tensor dtype is not supported: " + t.name);
        break;
      }
      if (t.name.empty()) {
        rc = say(MYOS_ERR_EMPTY_NAME, "tensor name is empty");
        break;
      }
    }
  }
  if (rc == MYOS_OK && n_tensors) *n_tensors = ts.size();
  if (map) munmap(map, len);
  return rc;
}

int myos_weights_ready(myos_ctx* c) {
  if (!c) return 0;
  return missing_weight(c) == MYOS_OK ? 1 : 0;
}

int myos_kv_len(const myos_ctx* c, size_t* len) {
  if (!c || !len) return MYOS_ERR_ARG;
  *len = c->len;
  return MYOS_OK;
}

int myos_reset(myos_ctx* c) {
  if (!c) return MYOS_ERR_ARG;
  CK(cudaSetDevice(c->device));
  c->len = 0;
  int st = set_ctl(c, true);
  if (st) return st;
  return finish(c);
}

int myos_logits(myos_ctx* c, float* out) {
  if (!c || !out) return MYOS_ERR_ARG;
  CK(cudaSetDevice(c->device));
  CK(cudaMemcpyAsync(out, c->logits, (size_t)c->s.vocab * 4, cudaMemcpyDeviceToHost, c->st));
  return finish(c);
}

int myos_profile_kernels(myos_ctx* c, int iters, float* ms_out, double* bytes_out) {
  if (!c || !ms_out || iters <= 0) return MYOS_ERR_ARG;
  if (c->tp_size > 1) return fail(c, MYOS_ERR_UNSUPPORTED, "kernel profiling is single-GPU only");
  CK(cudaSetDevice(c->device));
  int st = missing_weight(c);
  if (st) return st;
  if (c->len >= c->o.max_seq) return fail(c, MYOS_ERR_CACHE_FULL, "kv cache is full");
  CK(cudaStreamWaitEvent(c->st, c->load_ev, 0));
  StepCtl saved;
  CK(cudaMemcpyAsync(&saved, c->ctl, sizeof saved, cudaMemcpyDeviceToHost, c->st));
  std::vector<float> saved_logits(c->s.vocab);
  CK(cudaMemcpyAsync(saved_logits.data(), c->logits, c->s.vocab * 4, cudaMemcpyDeviceToHost, c->st));
  if ((st = finish(c))) return st;
  const int L = (int)c->s.num_layers;
  c->profiling = true;
  for (int kind = K_QKV; kind <= K_HEAD; ++kind) {
    if (kind_bytes(c, kind) == 0.0) {  // runs inside a fused launch (timed with it)
      ms_out[kind] = 0.f;
      if (bytes_out) bytes_out[kind] = 0.0;
      continue;
    }
    // one untimed pass to warm instruction caches and the launch path
    for (int l = 0; l < L; ++l)
      if ((st = launch_kind(c, kind, l, nullptr, false, false))) break;
    // back to back with programmatic dependent launch, as inside the step:
    // each launch's pre-wait prologue overlaps the previous launch's tail
    CK(cudaEventRecord(c->ev0, c->st));
    int n = 0;
    for (int it = 0; it < iters && !st; ++it)
      for (int l = 0; l < L && !st; ++l, ++n) st = launch_kind(c, kind, l, nullptr, n > 0, false);
    CK(cudaEventRecord(c->ev1, c->st));
    if (!st) st = finish(c);
    if (st) {
      c->profiling = false;
      return st;
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    ms_out[kind] = ms / (float)n;
    if (bytes_out) bytes_out[kind] = kind_bytes(c, kind);
  }
  c->profiling = false;
  CK(cudaMemcpyAsync(c->ctl, &saved, sizeof saved, cudaMemcpyHostToDevice, c->st));
  CK(cudaMemcpyAsync(c->logits, saved_logits.data(), c->s.vocab * 4, cudaMemcpyHostToDevice, c->st));
  return finish(c);
}

int myos_tp_slice(const myos_shape* shape, int32_t size, int32_t rank, const char* name,
                  myos_tp_part* out) {
  if (!shape || !name || !out) return MYOS_ERR_ARG;
  if (size < 1 || size > kMaxTp || rank < 0 || rank >= size) return MYOS_ERR_ARG;
  if (check_shape(*shape)) return MYOS_ERR_SHAPE;
  const uint32_t N = (uint32_t)size;
  if (shape->num_q_heads % N || shape->num_kv_heads % N || shape->intermediate % N ||
      shape->vocab % N || ((shape->num_q_heads / N) * shape->head_dim) % 8)
    return MYOS_ERR_SHAPE;
  *out = myos_tp_part{};
  int layer, suffix, global;
  if (!parse_tensor_name(*shape, name, &layer, &suffix, &global)) return MYOS_OK;  // kept = 0
  *out = tp_part(*shape, N, (uint32_t)rank, global, suffix);
  return MYOS_OK;
}

int myos_launch_count(uint64_t* out) {
  if (!out) return MYOS_ERR_ARG;
  *out = launches_total();
  return MYOS_OK;
}

int myos_last_timing(const myos_ctx* c, float* prefill_ms, float* decode_ms) {
  if (!c) return MYOS_ERR_ARG;
  if (prefill_ms) *prefill_ms = c->prefill_ms;
  if (decode_ms) *decode_ms = c->decode_ms;
  return MYOS_OK;
}

int myos_kv_head(myos_ctx* c, uint32_t layer, uint32_t head, size_t pos, float* k, float* v) {
  if (!c || !k || !v) return MYOS_ERR_ARG;
  if (layer >= c->s.num_layers || head >= c->s.num_kv_heads || pos >= c->o.max_seq)
    return fail(c, MYOS_ERR_CACHE_RANGE, "kv index is out of range");
  CK(cudaSetDevice(c->device));
  const size_t d = c->s.head_dim;
  const size_t off = ((size_t)layer * c->s.num_kv_heads + head) * c->o.max_seq * d + pos * d;
  if (c->o.kv_dtype == MYOS_KV_F32) {
    CK(cudaMemcpyAsync(k, (float*)c->kcache + off, d * 4, cudaMemcpyDeviceToHost, c->st));
    CK(cudaMemcpyAsync(v, (float*)c->vcache + off, d * 4, cudaMemcpyDeviceToHost, c->st));
    return finish(c);
  }
  std::vector<uint16_t> kb(d), vb(d);
  CK(cudaMemcpyAsync(kb.data(), (uint16_t*)c->kcache + off, d * 2, cudaMemcpyDeviceToHost, c->st));
  CK(cudaMemcpyAsync(vb.data(), (uint16_t*)c->vcache + off, d * 2, cudaMemcpyDeviceToHost, c->st));
  int st = finish(c);
  if (st) return st;
  for (size_t i = 0; i < d; ++i) {
    uint32_t kb32 = (uint32_t)kb[i] << 16, vb32 = (uint32_t)vb[i] << 16;
    memcpy(&k[i], &kb32, 4);
    memcpy(&v[i], &vb32, 4);
  }
  return MYOS_OK;
}

int myos_forward_token(myos_ctx* c, uint32_t token, size_t pos, float* logits) {
  if (!c) return MYOS_ERR_ARG;
  CK(cudaSetDevice(c->device));
  if (pos != c->len) return fail(c, MYOS_ERR_POSITION, "block position does not match the kv cursor");
  if (pos >= c->o.max_seq) return fail(c, MYOS_ERR_CACHE_FULL, "kv cache is full");
  int st = missing_weight(c);
  if (st) return st;
  if (token >= c->s.vocab) return fail(c, MYOS_ERR_TOKEN, "token id is out of range");
  CK(cudaMemcpyAsync(c->feed, &token, 4, cudaMemcpyHostToDevice, c->st));
  if ((st = set_ctl(c, false))) return st;
  CK(cudaEventRecord(c->ev0, c->st));
  if ((st = run_steps(c, G_FEED_HEAD, 1))) return st;
  CK(cudaEventRecord(c->ev1, c->st));
  if ((st = tp_gather_logits(c))) return st;
  if (logits) CK(cudaMemcpyAsync(logits, c->logits, (size_t)c->s.vocab * 4, cudaMemcpyDeviceToHost, c->st));
  if ((st = finish(c))) return st;
  cudaEventElapsedTime(&c->decode_ms, c->ev0, c->ev1);
  c->len += 1;
  return MYOS_OK;
}

// Split-attention partials for `rows` rows of up to max_keys keys each.
static int attn_scratch(myos_ctx* c, int rows, int max_keys) {
  int ch = 0;
  const size_t ns = (size_t)pf_attn_splits(max_keys, &ch);
  const size_t heads = (size_t)rows * c->s.num_q_heads * ns;
  int st = grow(c, &c->at_o, &c->at_o_bytes, heads * c->s.head_dim * 4);
  if (!st) st = grow(c, &c->at_ml, &c->at_ml_bytes, heads * sizeof(float2));
  const size_t had = c->at_arrive_bytes;
  if (!st) st = grow(c, &c->at_arrive, &c->at_arrive_bytes,
                     (size_t)rows * c->s.num_kv_heads * sizeof(unsigned));
  if (!st && c->at_arrive_bytes != had) CK(cudaMemsetAsync(c->at_arrive, 0, c->at_arrive_bytes, c->st));
  if (!st && !c->at_work) {
    st = grow(c, &c->at_work, &c->at_work_bytes, 2 * sizeof(unsigned));
    if (!st) CK(cudaMemsetAsync(c->at_work, 0, c->at_work_bytes, c->st));
  }
  return st;
}

// K slices for an [M, N, K] projection of the GEMM path: enough to put an
// output tile (or slice) on every SM, bounded by pf_D's room for partials.
static int pf_splits(const myos_ctx* c, int M, int N, int K) {
  if (!c->pf_splitk) return 1;
  int sp = gemm_pick_splits(M, N, K, c->num_sms, c->pf_m64);
  while (sp > 1 && ((size_t)sp * M * N > c->pf_D_elems || (K / 64) % sp)) --sp;
  return sp;
}

// One projection of the GEMM path: D = pf_A x W^T with K slices when its
// tiles would leave SMs idle (sp null: never sliced, D holds one [M, N]
// block); *sp receives the slices now in D.
static cudaError_t pf_gemm(const myos_ctx* c, int M, int N, int K, const uint16_t* W, float* D,
                           cudaStream_t st, int ldw, int* sp) {
  int one = 1;
  if (!sp) sp = &one;
  else *sp = pf_splits(c, M, N, K);
  return gemm_bf16_f32(M, N, K, c->pf_A, W, nullptr, D, 0.0f, c->pf_ws, c->pf_ws_bytes, st, ldw,
                       *sp, pf_pdl(), c->pf_m64);
}

// One chunk of n prompt tokens at positions p0.. through every layer
// (GEMM prefill); leaves the chunk's residual rows in pf_X and their K/V in
// the cache.
int prefill_chunk(myos_ctx* c, const uint32_t* d_ids, int n, int p0, void* kcache = nullptr,
                  void* vcache = nullptr, int S_ = 0) {
  // default: the context's own cache; batched decode passes a sequence's slab
  const myos_shape& s = c->s;
  const int H = (int)s.hidden, I = (int)s.intermediate, qd = (int)c->qd;
  const int Nq = (int)(c->qd + 2 * c->kvd), Hq = (int)s.num_q_heads, Hkv = (int)s.num_kv_heads;
  const int d = (int)s.head_dim, S = S_ ? S_ : (int)c->o.max_seq, M = kSplitParts * n;
  if (!kcache) {
    kcache = c->kcache;
    vcache = c->vcache;
  }
  const size_t layer_elems = (size_t)Hkv * S * d;
  const int kv_bf16 = c->o.kv_dtype == MYOS_KV_BF16;
  const size_t kv_elt = kv_bf16 ? 2 : 4;
  const float scale = 1.0f / sqrtf((float)d);
  cudaStream_t st = c->st;
  // sp: the K slices of the projection now in pf_D (split-K when its output
  // tiles would leave SMs idle and pf_D has room for the partials)
  int sp = 1;
  auto gemm = [&](int N, int K, const uint16_t* W, int ldw = 0) {
    const cudaError_t e = pf_gemm(c, M, N, K, W, c->pf_D, st, ldw, &sp);
    return e == cudaSuccess ? MYOS_OK : fail(c, MYOS_ERR_CUDA, std::string("prefill gemm: ") + cudaGetErrorString(e));
  };
  // residual += the projection (the partial rows of pf_D), then the next
  // RMSNorm's split input from the updated rows (gamma null: none); under
  // tensor parallelism each rank's part (rank 0's with the residual) is
  // summed over the ranks with one NCCL allreduce of the chunk's rows
  auto resid = [&](int rows, int N, const float* gamma) -> int {
    if (c->tp_size == 1) {
      CK(pf_resid_norm(c->pf_X, c->pf_D, sp, gamma, c->pf_A, rows, N, s.rms_eps, st));
      return MYOS_OK;
    }
    CK(pf_resid_part(c->pf_D, c->tp_rank == 0 ? c->pf_X : nullptr, rows, N, sp, st));
    if (!tp_allreduce_sum(c->pf_D, c->pf_X, (size_t)rows * N, c->comm, st))
      return fail(c, MYOS_ERR_NCCL, "allreduce of the prefill residual failed");
    if (gamma) CK(pf_norm_split(c->pf_A, c->pf_X, gamma, rows, N, s.rms_eps, st));
    return MYOS_OK;
  };
  int rc;
  if ((rc = attn_scratch(c, n, p0 + n))) return rc;
  CK(pf_embed(c->pf_X, c->embed, d_ids, n, H, st));
  CK(pf_norm_split(c->pf_A, c->pf_X, c->layers[0].ln1, n, H, s.rms_eps, st));
  for (int l = 0; l < (int)s.num_layers; ++l) {
    const LayerW& w = c->layers[l];
    void* kc = (uint8_t*)kcache + (size_t)l * layer_elems * kv_elt;
    void* vc = (uint8_t*)vcache + (size_t)l * layer_elems * kv_elt;
    if ((rc = gemm(Nq, H, w.wqkv))) return rc;
    CK(pf_qkv_post(c->pf_Q, c->pf_D, sp, w.bqkv, kc, vc, kv_bf16, c->cos_t, c->sin_t, p0, n, Hq,
                   Hkv, d, S, st));
    CK(pf_attn(c->pf_A, c->at_o, c->at_ml, c->pf_Q, kc, vc, kv_bf16, p0, n, Hq, Hkv, d, S, scale,
               p0 + n, c->num_sms, st, nullptr, 0, c->at_arrive, c->at_work));
    if ((rc = gemm(H, qd, w.wo, (int)c->qd_pad))) return rc;
    if ((rc = resid(n, H, w.ln2))) return rc;
    if ((rc = gemm(2 * I, H, w.wg))) return rc;  // gate rows then up rows
    CK(pf_swiglu_split(c->pf_A, c->pf_D, n, I, sp, st));
    if ((rc = gemm(H, I, w.wd))) return rc;
    if ((rc = resid(n, H, l + 1 < (int)s.num_layers ? c->layers[l + 1].ln1 : nullptr))) return rc;
  }
  return MYOS_OK;
}

// Batched decode of independent sequences: greedy (feed null: each step's
// token is the argmax of the sequence's current logits) or teacher-forced
// (feed [nseq][steps]: step s embeds feed[b][s]); out_ids[b][s] is the
// argmax of sequence b's logits before step s either way. logits, when
// non-null, receives each sequence's final logits [nseq][vocab].
static int batch_run(myos_ctx* c, size_t nseq, const uint32_t* ids, const uint32_t* lens,
                     size_t steps, const uint32_t* feed, uint32_t* out_ids, float* logits) {
  if (!c || !ids || !lens || (steps && !out_ids)) return MYOS_ERR_ARG;
  if (c->tp_size > 1) return fail(c, MYOS_ERR_UNSUPPORTED, "batched decode is single-GPU only");
  if (!c->pf_ok) return fail(c, MYOS_ERR_SHAPE, "batched decode needs the tensor-core path's shape");
  if (nseq == 0 || nseq > (size_t)c->pf_chunk)
    return fail(c, MYOS_ERR_SHAPE, "batch size must be 1.." + std::to_string(c->pf_chunk));
  const myos_shape& s = c->s;
  size_t total = 0, maxlen = 0;
  for (size_t b = 0; b < nseq; ++b) {
    if (lens[b] == 0) return fail(c, MYOS_ERR_SHAPE, "block shape does not match the buffers");
    total += lens[b];
    maxlen = std::max(maxlen, (size_t)lens[b]);
  }
  for (size_t i = 0; i < total; ++i)
    if (ids[i] >= s.vocab) return fail(c, MYOS_ERR_TOKEN, "token id is out of range");
  if (feed)
    for (size_t i = 0; i < nseq * steps; ++i)
      if (feed[i] >= s.vocab) return fail(c, MYOS_ERR_TOKEN, "token id is out of range");
  if (maxlen + steps > c->o.max_seq) return fail(c, MYOS_ERR_CACHE_FULL, "kv cache is full");
  int st = missing_weight(c);
  if (st) return st;
  CK(cudaSetDevice(c->device));
  const int B = (int)nseq, H = (int)s.hidden, I = (int)s.intermediate, qd = (int)c->qd;
  const int Nq = (int)(c->qd + 2 * c->kvd), Hq = (int)s.num_q_heads, Hkv = (int)s.num_kv_heads;
  const int d = (int)s.head_dim, V = (int)s.vocab, L = (int)s.num_layers, M = kSplitParts * B;
  const int Sb = (int)(maxlen + steps);  // slots per sequence
  const int kv_bf16 = c->o.kv_dtype == MYOS_KV_BF16;
  const size_t kv_elt = kv_bf16 ? 2 : 4;
  const size_t layer_elems = (size_t)Hkv * Sb * d, seq_elems = (size_t)L * layer_elems;
  const float scale = 1.0f / sqrtf((float)d);
  const uint16_t* head_w = s.tied_head ? c->embed : c->lm_head;
  cudaStream_t stq = c->st;
  // buffers (kept for later calls of the same or smaller size)
  size_t have_k = c->bt_kv_bytes, have_v = c->bt_kv_bytes;
  if ((st = grow(c, &c->bt_k, &have_k, (size_t)B * seq_elems * kv_elt))) return st;
  if ((st = grow(c, &c->bt_v, &have_v, (size_t)B * seq_elems * kv_elt))) return st;
  c->bt_kv_bytes = std::min(have_k, have_v);
  size_t have_x = c->bt_X ? (size_t)c->pf_chunk * H * 4 : 0;
  if ((st = grow(c, &c->bt_X, &have_x, (size_t)c->pf_chunk * H * 4))) return st;
  if ((st = grow(c, &c->bt_D, &c->bt_D_bytes, (size_t)M * V * 4))) return st;
  size_t have_small = c->bt_pos ? (size_t)c->pf_chunk * 4 : 0;
  size_t h2 = have_small, h3 = have_small, h4 = have_small;
  if ((st = grow(c, &c->bt_pos, &have_small, (size_t)c->pf_chunk * 4))) return st;
  if ((st = grow(c, &c->bt_rows, &h2, (size_t)c->pf_chunk * 4))) return st;
  if ((st = grow(c, &c->bt_tok, &h3, (size_t)c->pf_chunk * 4))) return st;
  size_t have_step = c->bt_step ? sizeof(int) : 0;
  if ((st = grow(c, &c->bt_step, &have_step, sizeof(int)))) return st;
  (void)h4;
  size_t have_out = c->bt_out_n * 4, have_ids = c->bt_ids_n * 4;
  if ((st = grow(c, &c->bt_out, &have_out, std::max<size_t>(1, (size_t)B * steps) * 4))) return st;
  c->bt_out_n = have_out / 4;
  if ((st = grow(c, &c->bt_ids, &have_ids, total * 4))) return st;
  c->bt_ids_n = have_ids / 4;
  if ((st = grow(c, &c->bt_amax, &c->bt_amax_bytes,
                 (size_t)B * pf_argmax_chunks(V) * sizeof(float2))))
    return st;
  const int max_keys = (int)(maxlen + steps);  // keys of the last step's longest row
  if (steps && (st = attn_scratch(c, B, max_keys))) return st;
  const size_t ws = gemm_workspace_bytes(M, V, H);
  if (ws > c->pf_ws_bytes && (st = grow(c, &c->pf_ws, &c->pf_ws_bytes, ws))) return st;
  // teacher-forced tokens, transposed to [steps][nseq] so each step's column
  // is one contiguous copy
  std::vector<uint32_t> feed_t;
  if (feed && steps) {
    if ((st = grow(c, &c->bt_feed, &c->bt_feed_bytes, nseq * steps * 4))) return st;
    feed_t.resize(nseq * steps);
    for (size_t b = 0; b < nseq; ++b)
      for (size_t t = 0; t < steps; ++t) feed_t[t * nseq + b] = feed[b * steps + t];
  }

  CK(cudaStreamWaitEvent(stq, c->load_ev, 0));
  CK(cudaMemcpyAsync(c->bt_ids, ids, total * 4, cudaMemcpyHostToDevice, stq));
  if (!feed_t.empty())
    CK(cudaMemcpyAsync(c->bt_feed, feed_t.data(), feed_t.size() * 4, cudaMemcpyHostToDevice, stq));
  std::vector<int> pos(B);
  CK(cudaEventRecord(c->ev0, stq));
  // 1. each prompt through the GEMM prefill into its own slab; its last
  //    residual row becomes row b of the batch
  size_t off = 0;
  for (int b = 0; b < B; ++b) {
    void* kb = (uint8_t*)c->bt_k + (size_t)b * seq_elems * kv_elt;
    void* vb = (uint8_t*)c->bt_v + (size_t)b * seq_elems * kv_elt;
    for (size_t c0 = 0; c0 < lens[b]; c0 += (size_t)c->pf_chunk) {
      const int nc = (int)std::min((size_t)c->pf_chunk, lens[b] - c0);
      if ((st = prefill_chunk(c, c->bt_ids + off + c0, nc, (int)c0, kb, vb, Sb))) return st;
      if (c0 + nc == lens[b])
        CK(cudaMemcpyAsync(c->bt_X + (size_t)b * H, c->pf_X + (size_t)(nc - 1) * H, (size_t)H * 4,
                           cudaMemcpyDeviceToDevice, stq));
    }
    off += lens[b];
    pos[b] = (int)lens[b];
  }
  CK(cudaMemcpyAsync(c->bt_pos, pos.data(), (size_t)B * 4, cudaMemcpyHostToDevice, stq));
  CK(cudaEventRecord(c->ev2, stq));  // prompts done: prefill_ms ends, decode_ms starts
  auto head = [&](int step, bool normed) -> int {
    if (!normed) CK(pf_norm_split(c->pf_A, c->bt_X, c->final_norm, B, H, s.rms_eps, stq));
    const cudaError_t e = pf_gemm(c, M, V, H, head_w, c->bt_D, stq, 0, nullptr);
    if (e != cudaSuccess) return fail(c, MYOS_ERR_CUDA, std::string("batch head gemm: ") + cudaGetErrorString(e));
    CK(pf_row_argmax(c->bt_tok, step < (int)steps ? c->bt_out : nullptr, (int)steps, step, c->bt_D,
                     c->bt_amax, B, V, stq));
    return MYOS_OK;
  };
  int sp = 1;  // K slices of the projection now in pf_D
  auto gemm = [&](int N, int K, const uint16_t* W) -> int {
    const cudaError_t e = pf_gemm(c, M, N, K, W, c->pf_D, stq, 0, &sp);
    return e == cudaSuccess ? MYOS_OK : fail(c, MYOS_ERR_CUDA, std::string("batch gemm: ") + cudaGetErrorString(e));
  };
  // 2. greedy: token s of every sequence is the argmax of its current
  //    logits; each is then forwarded (model_core greedy_decode, per sequence)
  if ((st = head(0, false))) return st;
  // One step reads everything that changes from step to step on the device
  // (positions, tokens, the step index bt_step), so the same launches serve
  // every step: captured once as a CUDA graph and replayed.
  CK(cudaMemsetAsync(c->bt_step, 0, sizeof(int), stq));
  auto step_body = [&]() -> int {
    if (feed)  // teacher-forced: this step embeds the given token, not the argmax
      CK(pf_feed(c->bt_tok, c->bt_feed, c->bt_step, B, stq));
    CK(pf_embed(c->bt_X, c->embed, c->bt_tok, B, H, stq));
    CK(pf_norm_split(c->pf_A, c->bt_X, c->layers[0].ln1, B, H, s.rms_eps, stq));
    for (int l = 0; l < L; ++l) {
      const LayerW& w = c->layers[l];
      void* kc = (uint8_t*)c->bt_k + (size_t)l * layer_elems * kv_elt;
      void* vc = (uint8_t*)c->bt_v + (size_t)l * layer_elems * kv_elt;
      if ((st = gemm(Nq, H, w.wqkv))) return st;
      CK(pf_qkv_post(c->pf_Q, c->pf_D, sp, w.bqkv, kc, vc, kv_bf16, c->cos_t, c->sin_t, 0, B, Hq,
                     Hkv, d, Sb, stq, c->bt_pos, seq_elems));
      CK(pf_attn(c->pf_A, c->at_o, c->at_ml, c->pf_Q, kc, vc, kv_bf16, 0, B, Hq, Hkv, d, Sb, scale,
                 max_keys, c->num_sms, stq, c->bt_pos, seq_elems, c->at_arrive, c->at_work));
      if ((st = gemm(H, qd, w.wo))) return st;
      CK(pf_resid_norm(c->bt_X, c->pf_D, sp, w.ln2, c->pf_A, B, H, s.rms_eps, stq));
      if ((st = gemm(2 * I, H, w.wg))) return st;
      CK(pf_swiglu_split(c->pf_A, c->pf_D, B, I, sp, stq));
      if ((st = gemm(H, I, w.wd))) return st;
      // the last layer's update goes on to the final norm of the head
      CK(pf_resid_norm(c->bt_X, c->pf_D, sp, l + 1 < L ? c->layers[l + 1].ln1 : c->final_norm,
                       c->pf_A, B, H, s.rms_eps, stq));
    }
    CK(pf_pos_advance(c->bt_pos, B, stq, c->bt_step));  // bt_step: this step + 1
    const cudaError_t e = pf_gemm(c, M, V, H, head_w, c->bt_D, stq, 0, nullptr);
    if (e != cudaSuccess)
      return fail(c, MYOS_ERR_CUDA, std::string("batch head gemm: ") + cudaGetErrorString(e));
    CK(pf_row_argmax(c->bt_tok, c->bt_out, (int)steps, 0, c->bt_D, c->bt_amax, B, V, stq,
                     c->bt_step));
    return MYOS_OK;
  };
  if (c->o.use_graphs && steps > 1) {
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(stq, cudaStreamCaptureModeRelaxed));
    const uint64_t before = launches_total();  // a capture launches nothing
    st = step_body();
    const uint64_t captured = launches_total() - before;
    launches_uncount(captured);
    cudaError_t ce = cudaStreamEndCapture(stq, &g);
    if (st) return st;
    if (ce != cudaSuccess)
      return fail(c, MYOS_ERR_CUDA, std::string("batch graph capture: ") + cudaGetErrorString(ce));
    cudaGraphExec_t ge;
    ce = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess)
      return fail(c, MYOS_ERR_CUDA, std::string("batch graph instantiate: ") + cudaGetErrorString(ce));
    for (size_t step = 0; step < steps && ce == cudaSuccess; ++step)
      ce = counted(cudaGraphLaunch(ge, stq), captured);
    cudaGraphExecDestroy(ge);  // released once its replays complete
    CK(ce);
  } else {
    for (size_t step = 0; step < steps; ++step)
      if ((st = step_body())) return st;
  }
  CK(cudaEventRecord(c->ev1, stq));
  if (steps)
    CK(cudaMemcpyAsync(out_ids, c->bt_out, (size_t)B * steps * 4, cudaMemcpyDeviceToHost, stq));
  std::vector<float> parts;
  if (logits) {  // final logits: the three partial rows of the head GEMM summed
    parts.resize((size_t)M * V);
    CK(cudaMemcpyAsync(parts.data(), c->bt_D, parts.size() * 4, cudaMemcpyDeviceToHost, stq));
  }
  if ((st = finish(c))) return st;
  for (size_t b = 0; logits && b < (size_t)B; ++b)
    for (size_t v = 0; v < (size_t)V; ++v)
      logits[b * V + v] = (parts[b * V + v] + parts[(B + b) * (size_t)V + v]) +
                          parts[(2 * B + b) * (size_t)V + v];
  cudaEventElapsedTime(&c->prefill_ms, c->ev0, c->ev2);
  cudaEventElapsedTime(&c->decode_ms, c->ev2, c->ev1);
  return MYOS_OK;
}

int myos_batch_generate(myos_ctx* c, size_t nseq, const uint32_t* ids, const uint32_t* lens,
                        size_t steps, uint32_t* out_ids) {
  return batch_run(c, nseq, ids, lens, steps, nullptr, out_ids, nullptr);
}

int myos_batch_forced_decode(myos_ctx* c, size_t nseq, const uint32_t* ids, const uint32_t* lens,
                             size_t steps, const uint32_t* feed, uint32_t* argmax_out,
                             float* logits) {
  if (steps && !feed) return MYOS_ERR_ARG;
  return batch_run(c, nseq, ids, lens, steps, feed, argmax_out, logits);
}

int myos_prefill(myos_ctx* c, const uint32_t* ids, size_t n, float* logits) {
  if (!c) return MYOS_ERR_ARG;
  if (n == 0 || !ids) return fail(c, MYOS_ERR_SHAPE, "block shape does not match the buffers");
  CK(cudaSetDevice(c->device));
  size_t start = c->len;
  if (start >= c->o.max_seq || start + n > c->o.max_seq) return fail(c, MYOS_ERR_CACHE_FULL, "kv cache is full");
  for (size_t i = 0; i < n; ++i)
    if (ids[i] >= c->s.vocab) return fail(c, MYOS_ERR_TOKEN, "token id is out of range");
  int st = missing_weight(c);
  if (st) return st;
  CK(cudaMemcpyAsync(c->feed, ids, n * 4, cudaMemcpyHostToDevice, c->st));
  if ((st = set_ctl(c, false))) return st;
  CK(cudaEventRecord(c->ev0, c->st));
  if (c->pf_ok && n > 1) {
    // all prompt tokens through the GEMM path; the head on the last one
    for (size_t c0 = 0; c0 < n; c0 += (size_t)c->pf_chunk) {
      const int nc = (int)std::min((size_t)c->pf_chunk, n - c0);
      if ((st = prefill_chunk(c, c->feed + c0, nc, (int)(start + c0)))) return st;
      if (c0 + nc == n)
        CK(cudaMemcpyAsync(c->resid, c->pf_X + (size_t)(nc - 1) * c->s.hidden, c->s.hidden * 4,
                           cudaMemcpyDeviceToDevice, c->st));
    }
    c->ctl_host->pos = (uint32_t)(start + n - 1);
    CK(cudaMemcpyAsync(&c->ctl->pos, &c->ctl_host->pos, 4, cudaMemcpyHostToDevice, c->st));
    if ((st = launch_kind(c, K_HEAD, 0, nullptr, false, false))) return st;
  } else {
    if (n > 1 && (st = run_steps(c, G_FEED_NOHEAD, n - 1))) return st;
    if ((st = run_steps(c, G_FEED_HEAD, 1))) return st;
  }
  CK(cudaEventRecord(c->ev1, c->st));
  if ((st = tp_gather_logits(c))) return st;
  if (logits) CK(cudaMemcpyAsync(logits, c->logits, (size_t)c->s.vocab * 4, cudaMemcpyDeviceToHost, c->st));
  if ((st = finish(c))) return st;
  cudaEventElapsedTime(&c->prefill_ms, c->ev0, c->ev1);
  c->len += n;
  return MYOS_OK;
}

int myos_greedy_decode(myos_ctx* c, size_t steps, uint32_t* out_ids) {
  if (!c || (steps && !out_ids)) return MYOS_ERR_ARG;
  CK(cudaSetDevice(c->device));
  int st = missing_weight(c);
  if (st) return st;
  size_t room = c->len < c->o.max_seq ? c->o.max_seq - c->len : 0;
  size_t run = steps < room ? steps : room;
  if ((st = set_ctl(c, false))) return st;
  CK(cudaEventRecord(c->ev0, c->st));
  if (run && (st = run_steps(c, G_ARGMAX_HEAD, run))) return st;
  CK(cudaEventRecord(c->ev1, c->st));
  if (run && (st = tp_gather_logits(c))) return st;
  if (run) CK(cudaMemcpyAsync(out_ids, c->rec_fed, run * 4, cudaMemcpyDeviceToHost, c->st));
  if ((st = finish(c))) return st;
  cudaEventElapsedTime(&c->decode_ms, c->ev0, c->ev1);
  c->len += run;
  if (run < steps) return fail(c, MYOS_ERR_CACHE_FULL, "kv cache is full");
  return MYOS_OK;
}

int myos_forced_decode(myos_ctx* c, const uint32_t* ids, size_t steps, uint32_t* argmax_out) {
  if (!c || (steps && (!ids || !argmax_out))) return MYOS_ERR_ARG;
  CK(cudaSetDevice(c->device));
  int st = missing_weight(c);
  if (st) return st;
  if (c->len + steps > c->o.max_seq) return fail(c, MYOS_ERR_CACHE_FULL, "kv cache is full");
  for (size_t i = 0; i < steps; ++i)
    if (ids[i] >= c->s.vocab) return fail(c, MYOS_ERR_TOKEN, "token id is out of range");
  if (!steps) return MYOS_OK;
  CK(cudaMemcpyAsync(c->feed, ids, steps * 4, cudaMemcpyHostToDevice, c->st));
  if ((st = set_ctl(c, false))) return st;
  CK(cudaEventRecord(c->ev0, c->st));
  if ((st = run_steps(c, G_FEED_HEAD, steps))) return st;
  CK(cudaEventRecord(c->ev1, c->st));
  if ((st = tp_gather_logits(c))) return st;
  CK(cudaMemcpyAsync(argmax_out, c->rec_argmax, steps * 4, cudaMemcpyDeviceToHost, c->st));
  if ((st = finish(c))) return st;
  cudaEventElapsedTime(&c->decode_ms, c->ev0, c->ev1);
  c->len += steps;
  return MYOS_OK;
}

}  // extern "C"
