/*
 * CPU ORACLE — test infrastructure only.
 *
 * A statement-for-statement C++ restatement of the MyOS reference's CPU
 * numerics (crates/tensor_core, crates/model_core). It exists to check the
 * CUDA library and to time the reference's --threads path as the CPU
 * baseline. Nothing in the product library links, loads or calls it; only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg do.
 *
 * Parity pin: the reference's own known-answer tests (bit patterns from
 * bf16.rs, gemv_bf16_kernel.rs, gqa.rs, rope.rs, swiglu.rs, qwen25_block.rs)
 * are ported to tests/test_oracle_pins.py and must pass bit for bit.
 *
 * Every reduction is serial, left to right, multiply then add (no FMA; the
 * file is compiled with -ffp-contract=off). libm expf/sqrtf/powf/sinf/cosf
 * are called directly, as the reference does through extern "C".
 */
#ifndef MYOS_ORACLE_H
#define MYOS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 0 = Ok. Values mirror the reference error enums. */
enum {
  ORC_OK = 0,
  ORC_SHAPE = 1,          /* Bf16OpError::Shape, GqaError::Shape, BlockError::Shape ... */
  ORC_TOKEN = 2,          /* TokenOutOfBounds / BlockError::Token */
  ORC_ROW_OOB = 3,        /* Bf16OpError::RowOutOfBounds */
  ORC_POSITION = 4,       /* BlockError::Position */
  ORC_CACHE_FULL = 5,     /* KvError::Full */
  ORC_CACHE_RANGE = 6,    /* KvError::Range */
  ORC_W_MISSING = 7,      /* QwenBf16Error::Missing */
  ORC_W_DTYPE = 8,        /* QwenBf16Error::DType */
  ORC_W_SHAPE = 9,        /* QwenBf16Error::Shape */
  ORC_W_LENGTH = 10,      /* QwenBf16Error::Length */
  ORC_DUPLICATE = 11,     /* WeightError::Duplicate */
  ORC_EMPTY_NAME = 12,    /* WeightError::EmptyName */
  ORC_PARSE = 13,         /* WeightError::Parse */
  ORC_UNSUPPORTED = 14,   /* WeightError::UnsupportedDType */
};

/* DType tags (weight_loader/src/lib.rs:36-49). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };

/* ---------------- tensor_core ops (host slices) ---------------- */
float orc_bf16_le_to_f32(const uint8_t le[2]);
int orc_gemv_bf16(float* y, size_t y_len, const uint8_t* w, size_t w_len, const float* x,
                  size_t x_len, size_t m, size_t k, int threads);
int orc_add_bf16_bias(float* y, size_t y_len, const uint8_t* bias, size_t bias_len);
int orc_embed_gather_bf16(float* out, size_t out_len, const uint8_t* table, size_t table_len,
                          const size_t* shape, size_t rank, uint32_t token);
int orc_rmsnorm_f32(float* y, size_t y_len, const float* w, size_t w_len, const float* x,
                    size_t x_len, float eps);
int orc_rmsnorm_bf16_weight(float* y, size_t y_len, const uint8_t* w, size_t w_len,
                            const float* x, size_t x_len, float eps);
int orc_attn_scale_f32(size_t head_dim, float* out);
/* mask_kind 0 = Full, 1 = Causal{query_pos} */
int orc_gqa_attn_f32(float* y, size_t y_len, const float* q, size_t q_len, const float* k,
                     size_t k_len, const float* v, size_t v_len, float* probs, size_t probs_len,
                     size_t num_q_heads, size_t num_kv_heads, size_t head_dim, size_t seq_len,
                     int mask_kind, size_t query_pos);
int orc_rope_inv_freqs(float* inv_freq, size_t len, size_t head_dim, float theta);
int orc_rope_f32(float* y, size_t y_len, const float* x, size_t x_len, uint32_t position,
                 size_t head_dim, float theta);
int orc_rope_f32_inplace(float* x, size_t len, uint32_t position, size_t head_dim, float theta);
float orc_silu_f32(float z);
int orc_swiglu_mul_f32(float* h, size_t h_len, const float* gate, size_t gate_len,
                       const float* up, size_t up_len);
int orc_swiglu_bf16(float* y, size_t y_len, const float* x, size_t x_len, const uint8_t* gate_w,
                    size_t gate_w_len, const uint8_t* up_w, size_t up_w_len,
                    const uint8_t* down_w, size_t down_w_len, float* gate, size_t gate_len,
                    float* up, size_t up_len, float* h, size_t h_len, size_t hidden,
                    size_t intermediate);
int orc_gemm_bf16(float* y, size_t y_len, const uint8_t* w, size_t w_len, const float* x,
                  size_t x_len, size_t batch, size_t m, size_t k, int threads);
uint32_t orc_greedy_token(const float* logits, size_t n);
/* gemv_row_spans: writes up to 64 (start,end) pairs into spans, returns count. */
size_t orc_gemv_row_spans(size_t m, size_t threads, size_t* spans);

/* Process-wide worker count used by orc_gemv_bf16/orc_gemm_bf16 when threads<=0. */
void orc_set_threads(int n);
int orc_get_threads(void);

/* ---------------- weight map ---------------- */
typedef struct orc_map orc_map;
orc_map* orc_map_new(void);
void orc_map_free(orc_map*);
/* Borrowed: bytes must stay alive while the map is used. copy!=0 copies them. */
int orc_map_insert(orc_map*, const char* name, int dtype, const size_t* shape, size_t rank,
                   const void* bytes, size_t nbytes, int copy);
/* SafeTensors header parse over a caller buffer (borrowed payloads). */
int orc_map_parse_safetensors(orc_map*, const uint8_t* file, size_t len);
size_t orc_map_len(const orc_map*);

/* ---------------- model_core ---------------- */
typedef struct {
  size_t hidden, num_q_heads, num_kv_heads, head_dim;
  float rope_theta;
  size_t intermediate, vocab, num_layers;
  float rms_eps;
  int tied_head; /* 1: embed_tokens is the head (reference). 0: lm_head.weight (extension). */
} orc_shape;

typedef struct orc_model orc_model;
orc_model* orc_model_new(const orc_shape* shape, size_t max_seq, int* status);
void orc_model_free(orc_model*);
int orc_forward_token(orc_model*, const orc_map*, uint32_t token, size_t pos);
int orc_prefill(orc_model*, const orc_map*, const uint32_t* tokens, size_t n);
/* Greedy decode; optional per-step logits dump (steps*vocab floats) and top-2 gaps. */
int orc_greedy_decode(orc_model*, const orc_map*, size_t steps, uint32_t* out, float* logits_dump,
                      float* top2_gap);
/* Teacher-forced decode: feed the given ids (not the argmax), record argmax and gap. */
int orc_forced_decode(orc_model*, const orc_map*, const uint32_t* feed, size_t steps,
                      uint32_t* argmax_out, float* top2_gap, float* logits_dump);
const float* orc_model_logits(const orc_model*);
size_t orc_kv_len(const orc_model*);
void orc_kv_clear(orc_model*);
int orc_kv_head(const orc_model*, size_t layer, size_t head, size_t pos, float* k_out,
                float* v_out);
/* Residual stream after the last forward/prefill (BlockWorkspace x). */
const float* orc_model_residual(const orc_model*);

#ifdef __cplusplus
}
#endif
#endif
