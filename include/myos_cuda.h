/*
 * myos_cuda.h — C ABI of the B200 (sm_100a) Qwen2.5 BF16 token loop.
 *
 * This is the drop-in boundary for the MyOS reference's decode path. Each
 * entry point names the reference interface it stands in for (paths are
 * relative to the reference project). Plain pointers and sizes only; no
 * PyTorch or C++ types cross it. All numeric work runs on the GPU: there is
 * no CPU fallback, and every call fails with MYOS_ERR_CUDA when no usable
 * sm_100 device is present.
 *
 * Numerics contract (same as the reference): weights are little-endian BF16,
 * promoted to f32 inside the kernels; every activation, accumulator and the
 * logits are f32. Reductions run in a fixed parallel order (deterministic
 * run to run) instead of the reference's serial left-to-right chain, so
 * results agree to within float reassociation, not bit for bit. Elementwise
 * steps (RMSNorm scaling, bias, RoPE with a host-built libm cos/sin table,
 * residual adds, SiLU's division form, softmax's e/sum) use the reference's
 * operation order without contraction.
 *
 * Error contract: every int-returning call returns MYOS_OK (0) or a status
 * below; on error the KV cursor and the logits are unchanged
 * (crates/model_core/src/qwen25_block.rs:129-134) and myos_last_error()
 * holds a one-line message. One context drives one device stream and is not
 * thread-safe; separate contexts may be used from separate threads.
 */
#ifndef MYOS_CUDA_H
#define MYOS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. Names follow the reference's error enums. */
enum myos_status {
  MYOS_OK = 0,
  MYOS_ERR_SHAPE = 1,          /* BlockError::Shape, Bf16OpError::Shape, GqaError::Shape */
  MYOS_ERR_TOKEN = 2,          /* BlockError::Token, Bf16OpError::TokenOutOfBounds */
  MYOS_ERR_ROW_OOB = 3,        /* Bf16OpError::RowOutOfBounds */
  MYOS_ERR_POSITION = 4,       /* BlockError::Position */
  MYOS_ERR_CACHE_FULL = 5,     /* KvError::Full */
  MYOS_ERR_CACHE_RANGE = 6,    /* KvError::Range */
  MYOS_ERR_WEIGHT_MISSING = 7, /* QwenBf16Error::Missing */
  MYOS_ERR_WEIGHT_DTYPE = 8,   /* QwenBf16Error::DType */
  MYOS_ERR_WEIGHT_SHAPE = 9,   /* QwenBf16Error::Shape */
  MYOS_ERR_WEIGHT_LENGTH = 10, /* QwenBf16Error::Length, WeightError::LengthMismatch */
  MYOS_ERR_DUPLICATE = 11,     /* WeightError::Duplicate */
  MYOS_ERR_EMPTY_NAME = 12,    /* WeightError::EmptyName */
  MYOS_ERR_PARSE = 13,         /* WeightError::Parse */
  MYOS_ERR_UNSUPPORTED = 14,   /* WeightError::UnsupportedDType */
  MYOS_ERR_IO = 15,            /* WeightFileError::Io */
  MYOS_ERR_CUDA = 16,          /* CUDA runtime failure or no sm_100 device */
  MYOS_ERR_NCCL = 17,          /* collective failure (tensor-parallel contexts) */
  MYOS_ERR_TIMEOUT = 18,       /* a bounded device-side wait gave up */
  MYOS_ERR_ARG = 19,           /* null pointer or invalid option */
  MYOS_ERR_SCRATCH_LIMIT = 20, /* request needs more than the fixed no-allocation scratch
                                  (MYOS_NOALLOC_SCRATCH_BYTES); no reference counterpart */
};

/* Tensor storage tags, weight_loader::DType (crates/weight_loader/src/lib.rs:36-49). */
enum myos_dtype { MYOS_F32 = 0, MYOS_F16 = 1, MYOS_BF16 = 2 };

/* KV-cache element type. The reference cache is f32
 * (crates/model_core/src/kv_cache.rs:89-125); bf16 halves its HBM traffic. */
enum myos_kv_dtype { MYOS_KV_F32 = 0, MYOS_KV_BF16 = 1 };

/* model_core::BlockShape + AttnShape (crates/model_core/src/qwen25_block.rs:53-75,
 * crates/model_core/src/attn_wire.rs:44-63). tied_head = 1 uses
 * model.embed_tokens.weight as the output projection (the reference's only
 * mode, qwen25_block.rs:290-301); 0 reads lm_head.weight (Qwen2.5-14B). */
typedef struct myos_shape {
  uint32_t hidden;
  uint32_t num_q_heads;
  uint32_t num_kv_heads;
  uint32_t head_dim;
  float rope_theta;
  uint32_t intermediate;
  uint32_t vocab;
  uint32_t num_layers;
  float rms_eps;
  uint32_t tied_head;
} myos_shape;

/* Context options. max_seq is KvShape::max_seq
 * (crates/model_core/src/kv_cache.rs:28-45); the reference CLI passes
 * n_prompt + steps (crates/runtime/src/main.rs:549-555). */
typedef struct myos_opts {
  int32_t device;      /* CUDA ordinal */
  uint32_t max_seq;    /* KV slots per layer */
  int32_t kv_dtype;    /* enum myos_kv_dtype */
  int32_t use_graphs;  /* 1: replay each token step as one CUDA graph */
} myos_opts;

typedef struct myos_ctx myos_ctx;

/* BlockShape::qwen25_1_5b() (qwen25_block.rs:63-74) and the 14B geometry. */
myos_shape myos_shape_qwen25_1_5b(void);
myos_shape myos_shape_qwen25_14b(void);

/* Allocates the weight arena, KV cache (KvCache::new, kv_cache.rs:99-125) and
 * the workspace (BlockWorkspace::new, qwen25_block.rs:96-114) in HBM. */
int myos_ctx_create(const myos_shape* shape, const myos_opts* opts, myos_ctx** out);
void myos_ctx_destroy(myos_ctx* ctx);

/* Tensor parallelism over `size` GPUs, one process (and one context) per
 * GPU. The reference runs one process on one device and has no sharded
 * mode; this splits the same token step: q/k/v rows and attention by head,
 * o_proj and down_proj by input column (each projection's epilogue stores
 * its rows into every rank's inbox over peer memory and a small kernel
 * sums the ranks' parts in rank order; MYOS_TP_COMM=nccl, or GPUs that
 * cannot map each other's memory, use NCCL allreduce instead), gate/up by
 * row, and the output head by vocabulary row with a global first-maximum
 * pick. A rank's device waits on the others are bounded in time (60 s) and
 * end the call with MYOS_ERR_TIMEOUT; the context is not usable after that.
 * Weights are passed
 * whole to myos_load_tensor / myos_load_safetensors on every rank; each
 * rank keeps its slice. Every rank makes the same calls with the same
 * arguments, in the same order (host output pointers may be null on ranks
 * that do not read them). Needs size | num_q_heads, num_kv_heads,
 * intermediate and vocab (MYOS_ERR_SHAPE otherwise); a rank's MLP rows and
 * o_proj input columns are zero-padded to multiples of 256. The tensor-core prefill sums each chunk's
 * residual parts with an NCCL allreduce. Batched decode, the persistent step
 * kernel and myos_profile_kernels are single-GPU paths (MYOS_ERR_UNSUPPORTED).
 * At most 8 ranks (MYOS_ERR_ARG otherwise). */
typedef struct myos_tp {
  int32_t size;
  int32_t rank;
  uint8_t unique_id[128]; /* from myos_tp_unique_id on one rank, sent to all */
} myos_tp;

/* A fresh NCCL unique id (the rendezvous token every rank passes in). */
int myos_tp_unique_id(uint8_t out[128]);

/* Diagnostics of the tensor-parallel exchange on ONE GPU (no peers, no
 * NCCL): runs the exchange's reduce kernel over an inbox of n ranks x H
 * words. fill = 1: the host first writes every word as the first exchange's
 * (value 0.25 * (p + 1) + i / 1024 for rank p, element i) and out receives
 * the sums over p in rank order (f32 adds). fill = 0: nothing writes the
 * inbox, so the kernel's bounded wait must give up after timeout_ms
 * (1..10000) and the call returns MYOS_ERR_TIMEOUT. No reference
 * counterpart. */
int myos_tp_reduce_selftest(int32_t device, uint32_t n, uint32_t H, int32_t fill,
                            uint32_t timeout_ms, float* out);

/* How a tensor-parallel rank holds one named tensor of the whole model:
 * of the [rows, cols] tensor (matrix = 0: a vector, cols = 1) it keeps rows
 * [row0, row0 + nrows) and columns [col0, col0 + ncols), stored in an
 * extent of store_rows x store_cols whose extra rows/columns are zero (the
 * o_proj input and MLP widths are padded to multiples of 256). Heads (q/k/v
 * rows, o_proj columns), MLP columns (gate/up rows, down_proj columns) and
 * the untied head's vocabulary rows are split in rank order; embedding and
 * norms are whole on every rank. kept = 0: the model never reads the
 * tensor. This is the slicing myos_load_tensor applies to the whole tensor
 * it is given, so a loader can produce just the kept part (the rest of the
 * buffer it passes is not read). No counterpart in the reference, which
 * runs the whole model in one process. */
typedef struct myos_tp_part {
  uint64_t rows;
  uint64_t cols;
  uint64_t row0;
  uint64_t nrows;
  uint64_t col0;
  uint64_t ncols;
  uint64_t store_rows;
  uint64_t store_cols;
  int32_t matrix;
  int32_t kept;
} myos_tp_part;
int myos_tp_slice(const myos_shape* shape, int32_t size, int32_t rank, const char* name,
                  myos_tp_part* out);
int myos_ctx_create_tp(const myos_shape* shape, const myos_opts* opts, const myos_tp* tp,
                       myos_ctx** out);
const char* myos_last_error(const myos_ctx* ctx);

/* One named tensor from any WeightMap-shaped source
 * (weight_loader::WeightMap::tensor_info/tensor_bytes, lib.rs:137-146, with
 * the per-name dtype/shape checks of model_core::qwen25_bf16::bf16_tensor,
 * qwen25_bf16.rs:72-82). Bytes are copied to HBM through pinned staging; the
 * caller may free them on return. Unknown names are ignored (the reference
 * never looks them up), and only BF16 is accepted for known names. */
int myos_load_tensor(myos_ctx* ctx, const char* name, int32_t dtype, const int64_t* shape,
                     int32_t rank, const void* bytes, size_t nbytes);

/* SafeTensorsMmap::open + parse (crates/weight_loader/src/mmap.rs:82-100,
 * safe_tensors.rs:30-43): maps the file read-only, validates the header the
 * way the safetensors crate does, and stages every known tensor into HBM. */
int myos_load_safetensors(myos_ctx* ctx, const char* path);

/* Host-only: SafeTensorsMmap::open + parse without a context or a GPU (the
 * reference CLI's check_safetensors, crates/runtime/src/main.rs:452-458).
 * n_tensors (nullable) receives the tensor count. err (nullable, err_len
 * bytes) receives the failure message. */
int myos_check_safetensors(const char* path, size_t* n_tensors, char* err, size_t err_len);

/* 1 when every tensor the shape needs has been loaded (preflight_weights,
 * qwen25_block.rs:599-643); otherwise 0 and myos_last_error names the first
 * missing key. */
int myos_weights_ready(myos_ctx* ctx);

/* model_core::prefill (qwen25_block.rs:323-543): the prompt at positions
 * kv_len.., KV written for every position, head on the last id only. logits
 * (nullable) receives vocab floats. Advances the cursor by n on success. */
int myos_prefill(myos_ctx* ctx, const uint32_t* ids, size_t n, float* logits);

/* model_core::forward_token (qwen25_block.rs:220-304): pos must equal
 * kv_len. logits (nullable) receives vocab floats. */
int myos_forward_token(myos_ctx* ctx, uint32_t token, size_t pos, float* logits);

/* model_core::greedy_decode (qwen25_block.rs:765-780): steps tokens, each
 * the first maximum of the current logits (greedy_token,
 * crates/model_core/src/lib.rs:157-167), fed back on the device. */
int myos_greedy_decode(myos_ctx* ctx, size_t steps, uint32_t* out_ids);

/* Teacher-forced decode: feeds ids[i] at step i (not the argmax) and writes
 * the argmax of the logits seen before each feed into argmax_out[i]. Used
 * by the parity protocol so every step stays comparable after a divergence. */
int myos_forced_decode(myos_ctx* ctx, const uint32_t* ids, size_t steps, uint32_t* argmax_out);

/* KvCache::len / clear (kv_cache.rs:140-142, 234-237). */
int myos_kv_len(const myos_ctx* ctx, size_t* len);
int myos_reset(myos_ctx* ctx);

/* KvCache::key_head / value_head (kv_cache.rs:239-252): head_dim f32 each.
 * In a tensor-parallel context `head` counts this rank's KV heads
 * (global head rank * num_kv_heads / size + head). */
int myos_kv_head(myos_ctx* ctx, uint32_t layer, uint32_t head, size_t pos, float* k, float* v);

/* BlockWorkspace::logits (qwen25_block.rs:118-125): vocab floats. */
int myos_logits(myos_ctx* ctx, float* out);

/* Times each decode-step kernel alone with CUDA events on the context's
 * stream. Kinds: 0 QKV (RMSNorm + q|k|v GEMV + bias), 1 attention, 2 o_proj
 * (+ residual), 3 gate/up (RMSNorm + GEMV + SiLU*up), 4 down (+ residual),
 * 5 head (final norm + GEMV + argmax). A pass launches each kind once per
 * layer, each launch on that layer's weights, so the weights a pass touches
 * exceed L2; launches follow each other with programmatic dependent launch
 * as inside a token step; ms_out[6] gets the mean device time of one launch
 * over iters passes, bytes_out[6] the algorithmic bytes one launch moves (weights +
 * activations + KV read at the current length). Needs kv_len < max_seq;
 * the KV cursor, logits and argmax are left as they were. */
int myos_profile_kernels(myos_ctx* ctx, int iters, float* ms_out, double* bytes_out);

/* Device time of the last prefill / decode call, from CUDA events (ms). */
int myos_last_timing(const myos_ctx* ctx, float* prefill_ms, float* decode_ms);

/* Kernel launches this library has enqueued in the calling process, all
 * contexts and devices together (a CUDA graph replay adds the kernels
 * captured in it). Diagnostics for benchmarks; no counterpart in the
 * reference, which runs on the CPU. */
int myos_launch_count(uint64_t* out);

/* ---------------------------------------------------------------------------
 * tensor_core operators on host slices (crates/tensor_core/src/lib.rs:54-74).
 * Same argument meaning and error behaviour as the Rust functions; the work
 * runs on the current CUDA device through the same kernels the engine uses.
 * ------------------------------------------------------------------------- */

/* tensor_core::gemv_bf16 (bf16.rs:80-122): y[i] = sum_j bf16(W[i,j]) * x[j]. */
int myos_gemv_bf16(float* y, size_t y_len, const uint8_t* w, size_t w_len, const float* x,
                   size_t x_len, size_t m, size_t k);
/* tensor_core::rmsnorm_bf16_weight (bf16.rs:231-249). */
int myos_rmsnorm_bf16_weight(float* y, size_t y_len, const uint8_t* w, size_t w_len,
                             const float* x, size_t x_len, float eps);
/* tensor_core::gqa_attn_f32 (gqa.rs:174-218). mask_kind 0 = Full, 1 = Causal (any
 * other value: MYOS_ERR_ARG). */
int myos_gqa_attn_f32(float* y, size_t y_len, const float* q, size_t q_len, const float* k,
                      size_t k_len, const float* v, size_t v_len, size_t num_q_heads,
                      size_t num_kv_heads, size_t head_dim, size_t seq_len, int32_t mask_kind,
                      size_t query_pos);
/* tensor_core::swiglu_mul_f32 (swiglu.rs:125-131). */
int myos_swiglu_mul_f32(float* h, size_t h_len, const float* gate, size_t gate_len,
                        const float* up, size_t up_len);
/* tensor_core::rope_f32 (rope.rs:107-115), one position for every head. */
int myos_rope_f32(float* y, size_t y_len, const float* x, size_t x_len, uint32_t position,
                  size_t head_dim, float theta);
/* model_core::greedy_token (lib.rs:157-167) as the two-stage device argmax. */
int myos_greedy_token(const float* logits, size_t n, uint32_t* out);

/* ---------------------------------------------------------------------------
 * Device-pointer kernels (for callers that already hold HBM buffers, and the
 * isolated GEMV microbench). stream may be 0. No allocation, no sync.
 * ------------------------------------------------------------------------- */

/* y[m] (f32) = W[m,k] (bf16, row-major, 16-byte aligned rows when k%8==0) x[k] (f32). */
int myos_dev_gemv_bf16(float* d_y, const void* d_w, const float* d_x, size_t m, size_t k,
                       void* stream);

/* Greedy generation for nseq independent sequences at once. No direct
 * counterpart in the reference, which decodes one sequence per process
 * (model_core greedy_decode, qwen25_block.rs:765-780): this stands in for
 * running greedy_decode on each prompt. Sequence b's prompt is
 * ids[off_b .. off_b + lens[b]) (prompts concatenated in order);
 * out_ids[b * steps + s] receives its s-th generated id. Every prompt runs
 * through the tensor-core prefill into its own KV slab; each decode step then
 * runs the projections and the head of all sequences as GEMMs (each f32
 * activation as three stacked bf16 terms that sum to it exactly,
 * M = 3 nseq). 1 <= nseq <= 128 and
 * lens[b] + steps <= max_seq; needs a shape the GEMM prefill supports
 * (MYOS_ERR_SHAPE otherwise). The context's own cache and cursor are not
 * touched. */
int myos_batch_generate(myos_ctx* ctx, size_t nseq, const uint32_t* ids, const uint32_t* lens,
                        size_t steps, uint32_t* out_ids);

/* The teacher-forced form of myos_batch_generate (the per-sequence
 * myos_forced_decode, model_core forward_token fed given ids, for a batch):
 * step s of sequence b embeds feed[b*steps + s] instead of the argmax, and
 * argmax_out[b*steps + s] receives the argmax of b's logits before step s
 * (the prediction the fed token is scored against). logits, when non-null,
 * receives every sequence's final logits [nseq][vocab]. Same rules and
 * errors as myos_batch_generate; feed ids must be < vocab. */
int myos_batch_forced_decode(myos_ctx* ctx, size_t nseq, const uint32_t* ids, const uint32_t* lens,
                             size_t steps, const uint32_t* feed, uint32_t* argmax_out,
                             float* logits);

/* Size of the fixed device array that myos_dev_gqa_attn_f32_noalloc takes its
 * scratch from (one per device). */
#define MYOS_NOALLOC_SCRATCH_BYTES (2u << 20)

/* No counterpart in the reference (its attention runs on the host). The same
 * split-KV attention as myos_gqa_attn_f32 (tensor_core::gqa_attn_f32,
 * crates/tensor_core/src/gqa.rs:174-218; same arguments and shape rules, same
 * split geometry and so the same results) on caller-held device buffers
 * y[hq*d], q[hq*d], k[hkv][seq][d], v[hkv][seq][d], for callers that must not
 * allocate: code running while a device-memory budget is fixed (an allocator
 * that owns all free HBM, a pool sized at start-up) or on a path that may not
 * call cudaMalloc/cudaFree, which synchronize the device. It allocates
 * nothing: the split partials and merge counters live in one static device
 * array of MYOS_NOALLOC_SCRATCH_BYTES (2 MiB); a request needing more
 * ((hkv*4 + hq*nsplit*(d+2)*4 bytes, each part rounded up to 256, with
 * nsplit = min(64, ceil(keys/32))) returns MYOS_ERR_SCRATCH_LIMIT before any
 * device work. The counters must be zero at kernel start; each call clears
 * them on its stream first. The first call on a device resolves the array's
 * address (cudaGetSymbolAddress); make that call before any stream capture.
 * Calls share the array: calls that run concurrently (different streams or
 * unordered threads) race and corrupt each other's results. Every pointer
 * must be 4-byte aligned, and with d % 4 == 0 d_k and d_v 16-byte aligned
 * (their rows are read as 16-byte vectors); mask_kind is 0 (Full) or 1
 * (Causal). Other values return MYOS_ERR_ARG before any device work.
 * stream may be 0; asynchronous (no sync). */
int myos_dev_gqa_attn_f32_noalloc(float* d_y, const float* d_q, const float* d_k,
                                  const float* d_v, size_t hq, size_t hkv, size_t d, size_t seq,
                                  int32_t mask_kind, size_t query_pos, void* stream);

/* Library version string and the build's target architecture. */
const char* myos_version(void);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif
