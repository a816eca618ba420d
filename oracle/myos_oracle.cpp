// CPU ORACLE — test infrastructure only (see myos_oracle.h).
//
// Restates, function by function, the MyOS reference's CPU path:
//   crates/tensor_core/src/bf16.rs            (bf16 promote, bias, embed, RMSNorm)
//   crates/tensor_core/src/gemv_bf16_kernel.rs (row spans, serial chain, AVX2 32-row panels)
//   crates/tensor_core/src/gemv_pool.rs        (row-span worker pool)
//   crates/tensor_core/src/gemm_bf16.rs        (prompt-chunk GEMM, same chain as GEMV)
//   crates/tensor_core/src/gqa.rs              (GQA scores / softmax / value mix)
//   crates/tensor_core/src/rope.rs             (NeoX half-rotate RoPE)
//   crates/tensor_core/src/swiglu.rs           (SiLU division form, SwiGLU)
//   crates/model_core/src/kv_cache.rs          (KvCache slots and cursor)
//   crates/model_core/src/attn_wire.rs         (attention_layer)
//   crates/model_core/src/qwen25_block.rs      (forward_token, prefill, greedy_decode)
//   crates/model_core/src/lib.rs:157-167       (greedy_token)
// Compiled with -O2 -ffp-contract=off -fno-fast-math: no FMA contraction, so
// every `acc += a * b` is a multiply then an add, as in the Rust source.
#include "myos_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr size_t kThreadsMax = 64;  // GEMV_THREADS_MAX, gemv_bf16_kernel.rs:34
constexpr size_t kRowPanel = 32;    // ROW_PANEL, gemv_bf16_kernel.rs:37
constexpr size_t kGemmRowBlock = 16;  // GEMM_ROW_BLOCK, gemm_bf16.rs:27
constexpr size_t kGemmJBlock = 64;    // GEMM_J_BLOCK, gemm_bf16.rs:30

std::atomic<int> g_threads{8};  // SHOWDOWN_THREADS default, gemv_bf16_kernel.rs:31,46

inline float bf16_at(const uint8_t* p) {
  // bf16.rs:61-63: u16 little-endian, shifted into the top half of an f32.
  uint32_t bits = (uint32_t)((uint32_t)p[0] | ((uint32_t)p[1] << 8)) << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

bool checked_mul(size_t a, size_t b, size_t* out) {
  return !__builtin_mul_overflow(a, b, out);
}

// ---------------------------------------------------------------- row spans
// gemv_bf16_kernel.rs:119-162
size_t row_spans(size_t m, size_t threads, size_t* spans /* 2*64 */) {
  if (m == 0) return 0;
  threads = std::min(std::max<size_t>(threads, 1), kThreadsMax);
  threads = std::min(threads, m);
  size_t n = 0;
  size_t panels = m / kRowPanel;
  if (panels >= threads) {
    size_t base = panels / threads, extra = panels % threads, tail = m % kRowPanel;
    size_t row = 0;
    for (size_t t = 0; t < threads; ++t) {
      size_t n_rows = (base + (t < extra ? 1 : 0)) * kRowPanel;
      if (t + 1 == threads) n_rows += tail;
      spans[2 * n] = row;
      spans[2 * n + 1] = row + n_rows;
      ++n;
      row += n_rows;
    }
    return n;
  }
  size_t base = m / threads, rem = m % threads, row = 0;
  for (size_t t = 0; t < threads; ++t) {
    size_t cnt = base + (t < rem ? 1 : 0);
    if (cnt == 0) break;
    spans[2 * n] = row;
    spans[2 * n + 1] = row + cnt;
    ++n;
    row += cnt;
  }
  return n;
}

// ---------------------------------------------------------------- worker pool
// gemv_pool.rs:130-189: span 0 runs on the caller, span i+1 on worker i.
class Pool {
 public:
  static Pool& get() {
    static Pool* p = new Pool();  // leaked on purpose: workers outlive static dtors
    return *p;
  }
  void run(size_t n_tasks, const std::function<void(size_t)>& fn) {
    if (n_tasks <= 1) {
      if (n_tasks == 1) fn(0);
      return;
    }
    std::lock_guard<std::mutex> call_lock(call_mu_);
    ensure(n_tasks - 1);
    {
      std::lock_guard<std::mutex> lk(mu_);
      job_ = &fn;
      active_ = n_tasks - 1;
      pending_ = n_tasks - 1;
      ++gen_;
    }
    cv_.notify_all();
    fn(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void ensure(size_t workers) {
    while (threads_.size() < workers) {
      size_t idx = threads_.size();
      threads_.emplace_back([this, idx] { loop(idx); });
    }
  }
  void loop(size_t idx) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(size_t)>* job;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (idx >= active_) continue;
        job = job_;
      }
      (*job)(idx + 1);
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (--pending_ == 0) done_cv_.notify_one();
      }
    }
  }
  std::mutex call_mu_, mu_;
  std::condition_variable cv_, done_cv_;
  std::vector<std::thread> threads_;
  const std::function<void(size_t)>* job_ = nullptr;
  size_t active_ = 0, pending_ = 0;
  uint64_t gen_ = 0;
};

// ---------------------------------------------------------------- GEMV kernels
// One row, left to right: the reference every fast path matches
// (gemv_bf16_kernel.rs:196-204, dot_row).
float dot_row(const uint8_t* row, const float* x, size_t k) {
  float acc = 0.0f;
  for (size_t j = 0; j < k; ++j) acc += bf16_at(row + 2 * j) * x[j];
  return acc;
}

bool have_avx2() {
  static int cached = -1;
  if (cached < 0) cached = __builtin_cpu_supports("avx2") ? 1 : 0;
  return cached == 1;
}

// 8x8 transpose of 16-bit lanes: column t, lane r = row r, column j+t.
// Same shuffle network as cols_8x8 (gemv_bf16_kernel.rs:440-490).
__attribute__((target("avx2"))) inline void cols8x8(const uint8_t* const* rows, size_t off,
                                                    __m128i* col) {
  __m128i r0 = _mm_loadu_si128((const __m128i*)(rows[0] + off));
  __m128i r1 = _mm_loadu_si128((const __m128i*)(rows[1] + off));
  __m128i r2 = _mm_loadu_si128((const __m128i*)(rows[2] + off));
  __m128i r3 = _mm_loadu_si128((const __m128i*)(rows[3] + off));
  __m128i r4 = _mm_loadu_si128((const __m128i*)(rows[4] + off));
  __m128i r5 = _mm_loadu_si128((const __m128i*)(rows[5] + off));
  __m128i r6 = _mm_loadu_si128((const __m128i*)(rows[6] + off));
  __m128i r7 = _mm_loadu_si128((const __m128i*)(rows[7] + off));
  __m128i a0 = _mm_unpacklo_epi16(r0, r1), a1 = _mm_unpackhi_epi16(r0, r1);
  __m128i a2 = _mm_unpacklo_epi16(r2, r3), a3 = _mm_unpackhi_epi16(r2, r3);
  __m128i a4 = _mm_unpacklo_epi16(r4, r5), a5 = _mm_unpackhi_epi16(r4, r5);
  __m128i a6 = _mm_unpacklo_epi16(r6, r7), a7 = _mm_unpackhi_epi16(r6, r7);
  __m128i b0 = _mm_unpacklo_epi32(a0, a2), b1 = _mm_unpackhi_epi32(a0, a2);
  __m128i b2 = _mm_unpacklo_epi32(a1, a3), b3 = _mm_unpackhi_epi32(a1, a3);
  __m128i b4 = _mm_unpacklo_epi32(a4, a6), b5 = _mm_unpackhi_epi32(a4, a6);
  __m128i b6 = _mm_unpacklo_epi32(a5, a7), b7 = _mm_unpackhi_epi32(a5, a7);
  col[0] = _mm_unpacklo_epi64(b0, b4);
  col[1] = _mm_unpackhi_epi64(b0, b4);
  col[2] = _mm_unpacklo_epi64(b1, b5);
  col[3] = _mm_unpackhi_epi64(b1, b5);
  col[4] = _mm_unpacklo_epi64(b2, b6);
  col[5] = _mm_unpackhi_epi64(b2, b6);
  col[6] = _mm_unpacklo_epi64(b3, b7);
  col[7] = _mm_unpackhi_epi64(b3, b7);
}

// acc += promote(col) * x (vmulps then vaddps, not vfmadd): madd8, :566-579.
__attribute__((target("avx2"))) inline __m256 madd8(__m256 acc, __m128i col, const float* x) {
  __m256 w = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(col), 16));
  return _mm256_add_ps(acc, _mm256_mul_ps(w, _mm256_broadcast_ss(x)));
}

// 32-row panels (dot_rows32_intrin, :583-651); remaining rows as serial chains.
__attribute__((target("avx2"))) void gemv_rows_avx2(float* y, const uint8_t* w, const float* x,
                                                    size_t m, size_t k) {
  const size_t row_bytes = 2 * k;
  size_t row = 0;
  for (; row + 32 <= m; row += 32) {
    const uint8_t* rows[32];
    for (int r = 0; r < 32; ++r) rows[r] = w + (row + r) * row_bytes;
    __m256 a[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                   _mm256_setzero_ps()};
    size_t j = 0, k8 = k & ~(size_t)7;
    __m128i c[8];
    for (; j < k8; j += 8) {
      for (int g = 0; g < 4; ++g) {
        cols8x8(rows + 8 * g, 2 * j, c);
        for (int t = 0; t < 8; ++t) a[g] = madd8(a[g], c[t], x + j + t);
      }
    }
    float tmp[32];
    for (int g = 0; g < 4; ++g) _mm256_storeu_ps(tmp + 8 * g, a[g]);
    for (; j < k; ++j) {
      float xj = x[j];
      for (int r = 0; r < 32; ++r) tmp[r] += bf16_at(rows[r] + 2 * j) * xj;
    }
    memcpy(y + row, tmp, sizeof tmp);
  }
  for (; row < m; ++row) y[row] = dot_row(w + row * row_bytes, x, k);
}

void gemv_rows(float* y, const uint8_t* w, const float* x, size_t m, size_t k) {
  if (m == 0) return;
  if (have_avx2()) {
    gemv_rows_avx2(y, w, x, m, k);
    return;
  }
  for (size_t r = 0; r < m; ++r) y[r] = dot_row(w + r * 2 * k, x, k);
}

// gemv_pool.rs:130-189 over gemv_row_spans.
void gemv_parallel(float* y, const uint8_t* w, const float* x, size_t m, size_t k,
                   size_t threads) {
  size_t spans[2 * kThreadsMax];
  size_t n = row_spans(m, threads, spans);
  if (n <= 1) {
    gemv_rows(y, w, x, m, k);
    return;
  }
  Pool::get().run(n, [&](size_t s) {
    size_t a = spans[2 * s], b = spans[2 * s + 1];
    gemv_rows(y + a, w + a * 2 * k, x, b - a, k);
  });
}

size_t resolve_threads(int threads) {
  int t = threads > 0 ? threads : g_threads.load();
  return (size_t)std::min(std::max(t, 1), (int)kThreadsMax);
}

// ---------------------------------------------------------------- GEMM (prefill)
// gemm_bf16.rs:297-430: per (token b, row i) one serial chain over j. X is
// staged [k, batch]; 16-row blocks; 64-column tiles; AVX2 over token lanes.
__attribute__((target("avx2"))) void accumulate_row(float* acc, const float* wf, size_t jb,
                                                    const float* stage, size_t batch, size_t j0) {
  size_t t = 0;
  if (have_avx2()) {
    for (; t + 8 <= batch; t += 8) {
      __m256 a0 = _mm256_loadu_ps(acc + t);
      for (size_t j = 0; j < jb; ++j) {
        __m256 wv = _mm256_broadcast_ss(wf + j);
        a0 = _mm256_add_ps(a0, _mm256_mul_ps(wv, _mm256_loadu_ps(stage + (j0 + j) * batch + t)));
      }
      _mm256_storeu_ps(acc + t, a0);
    }
  }
  for (size_t j = 0; j < jb; ++j) {
    const float* xcol = stage + (j0 + j) * batch;
    for (size_t b = t; b < batch; ++b) acc[b] += wf[j] * xcol[b];
  }
}

void gemm_rows(float* y, const uint8_t* w, const float* stage, float* acc, size_t batch,
               size_t m, size_t k, size_t row0, size_t row1) {
  const size_t row_bytes = 2 * k;
  float wf[kGemmJBlock];
  for (size_t row = row0; row < row1;) {
    size_t rb = std::min(row1 - row, kGemmRowBlock);
    std::fill(acc, acc + rb * batch, 0.0f);
    for (size_t j0 = 0; j0 < k;) {
      size_t jb = std::min(k - j0, kGemmJBlock);
      for (size_t r = 0; r < rb; ++r) {
        const uint8_t* wrow = w + (row + r) * row_bytes + 2 * j0;
        for (size_t j = 0; j < jb; ++j) wf[j] = bf16_at(wrow + 2 * j);
        accumulate_row(acc + r * batch, wf, jb, stage, batch, j0);
      }
      j0 += jb;
    }
    for (size_t r = 0; r < rb; ++r)
      for (size_t b = 0; b < batch; ++b) y[b * m + row + r] = acc[r * batch + b];
    row += rb;
  }
}

void gemm_impl(float* y, const uint8_t* w, const float* x, size_t batch, size_t m, size_t k,
               size_t threads) {
  std::vector<float> stage(k * batch);
  for (size_t b = 0; b < batch; ++b)
    for (size_t j = 0; j < k; ++j) stage[j * batch + b] = x[b * k + j];
  size_t spans[2 * kThreadsMax];
  size_t n = row_spans(m, threads, spans);
  std::vector<float> acc(std::max<size_t>(n, 1) * kGemmRowBlock * batch);
  if (n <= 1) {
    gemm_rows(y, w, stage.data(), acc.data(), batch, m, k, 0, m);
    return;
  }
  Pool::get().run(n, [&](size_t s) {
    gemm_rows(y, w, stage.data(), acc.data() + s * kGemmRowBlock * batch, batch, m, k,
              spans[2 * s], spans[2 * s + 1]);
  });
}

// ---------------------------------------------------------------- small ops
float inv_rms_serial(const float* x, size_t n, float eps) {
  // bf16.rs:263-270
  float sum_sq = 0.0f;
  for (size_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
  float mean = sum_sq / (float)n;
  return 1.0f / sqrtf(mean + eps);
}

void rmsnorm_bf16(float* y, const uint8_t* w, const float* x, size_t n, float eps) {
  // bf16.rs:231-249
  float inv = inv_rms_serial(x, n, eps);
  for (size_t i = 0; i < n; ++i) y[i] = bf16_at(w + 2 * i) * (x[i] * inv);
}

void add_bias(float* y, const uint8_t* b, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] += bf16_at(b + 2 * i);  // bf16.rs:147-158
}

float inv_freq_at(size_t pair, size_t head_dim, float theta) {
  // rope.rs:186-189
  float exponent = (float)(2 * pair) / (float)head_dim;
  return 1.0f / powf(theta, exponent);
}

// rope.rs:145-184. src==nullptr: in place.
void rotate(float* y, const float* src, size_t len, uint32_t position, size_t head_dim,
            float theta) {
  size_t n_heads = len / head_dim, n_pairs = head_dim / 2;
  float pos = (float)position;
  for (size_t pair = 0; pair < n_pairs; ++pair) {
    float angle = pos * inv_freq_at(pair, head_dim, theta);
    float c = cosf(angle), s = sinf(angle);
    for (size_t h = 0; h < n_heads; ++h) {
      size_t i0 = h * head_dim + pair, i1 = i0 + n_pairs;
      float x0 = src ? src[i0] : y[i0];
      float x1 = src ? src[i1] : y[i1];
      float x0c = x0 * c, x1s = x1 * s, x1c = x1 * c, x0s = x0 * s;
      y[i0] = x0c - x1s;
      y[i1] = x1c + x0s;
    }
  }
}

float silu(float z) { return z / (1.0f + expf(-z)); }  // swiglu.rs:113-115

void mul_ltr(float* h, const float* gate, const float* up, size_t n) {
  for (size_t i = 0; i < n; ++i) {  // swiglu.rs:254-261
    float a = silu(gate[i]);
    h[i] = a * up[i];
  }
}

inline bool key_kept(size_t t, int mask_kind, size_t query_pos) {
  return mask_kind == 0 || t <= query_pos;  // gqa.rs:225-230
}

// gqa.rs:174-218 + softmax_kept :283-307.
void gqa_impl(float* y, const float* q, const float* k, const float* v, float* probs, size_t hq,
              size_t hkv, size_t d, size_t seq, int mask_kind, size_t qpos) {
  size_t q_per_kv = hq / hkv;
  float scale = 1.0f / sqrtf((float)d);
  for (size_t h = 0; h < hq; ++h) {
    size_t g = h / q_per_kv;
    const float* qrow = q + h * d;
    for (size_t t = 0; t < seq; ++t) {
      if (!key_kept(t, mask_kind, qpos)) continue;
      const float* krow = k + (g * seq + t) * d;
      float acc = 0.0f;
      for (size_t i = 0; i < d; ++i) acc += qrow[i] * krow[i];
      probs[t] = acc * scale;
    }
    float mx = probs[0];
    for (size_t t = 1; t < seq; ++t)
      if (key_kept(t, mask_kind, qpos) && probs[t] > mx) mx = probs[t];
    float sum = 0.0f;
    for (size_t t = 0; t < seq; ++t) {
      if (!key_kept(t, mask_kind, qpos)) continue;
      float e = expf(probs[t] - mx);
      probs[t] = e;
      sum += e;
    }
    for (size_t t = 0; t < seq; ++t) {
      if (key_kept(t, mask_kind, qpos))
        probs[t] /= sum;
      else
        probs[t] = 0.0f;
    }
    float* yrow = y + h * d;
    for (size_t i = 0; i < d; ++i) {
      float acc = 0.0f;
      for (size_t t = 0; t < seq; ++t) {
        if (!key_kept(t, mask_kind, qpos)) continue;
        acc += probs[t] * v[(g * seq + t) * d + i];
      }
      yrow[i] = acc;
    }
  }
}

}  // namespace

// ================================================================= C ABI: ops
extern "C" {

float orc_bf16_le_to_f32(const uint8_t le[2]) { return bf16_at(le); }

void orc_set_threads(int n) { g_threads.store(std::min(std::max(n, 1), (int)kThreadsMax)); }
int orc_get_threads(void) { return g_threads.load(); }

size_t orc_gemv_row_spans(size_t m, size_t threads, size_t* spans) {
  return row_spans(m, threads, spans);
}

// bf16.rs:80-122 (gemv_bf16 / gemv_bf16_at_threads).
int orc_gemv_bf16(float* y, size_t y_len, const uint8_t* w, size_t w_len, const float* x,
                  size_t x_len, size_t m, size_t k, int threads) {
  if (y_len != m || x_len != k) return ORC_SHAPE;
  if (k == 0) {
    if (w_len != 0) return ORC_SHAPE;
    std::fill(y, y + m, 0.0f);
    return ORC_OK;
  }
  size_t row_bytes;
  if (!checked_mul(k, 2, &row_bytes)) return ORC_SHAPE;
  if (w_len / row_bytes < m) return ORC_ROW_OOB;
  size_t need;
  if (!checked_mul(row_bytes, m, &need)) return ORC_SHAPE;
  if (w_len != need) return ORC_SHAPE;
  gemv_parallel(y, w, x, m, k, resolve_threads(threads));
  return ORC_OK;
}

int orc_add_bf16_bias(float* y, size_t y_len, const uint8_t* bias, size_t bias_len) {
  if (bias_len != 2 * y_len) return ORC_SHAPE;
  add_bias(y, bias, y_len);
  return ORC_OK;
}

// bf16.rs:165-198
int orc_embed_gather_bf16(float* out, size_t out_len, const uint8_t* table, size_t table_len,
                          const size_t* shape, size_t rank, uint32_t token) {
  if (rank != 2) return ORC_SHAPE;
  size_t vocab = shape[0], hidden = shape[1];
  if (out_len != hidden) return ORC_SHAPE;
  if ((size_t)token >= vocab) return ORC_TOKEN;
  size_t row_bytes, start, end, need;
  if (!checked_mul(hidden, 2, &row_bytes)) return ORC_SHAPE;
  if (!checked_mul((size_t)token, row_bytes, &start)) return ORC_SHAPE;
  if (__builtin_add_overflow(start, row_bytes, &end)) return ORC_SHAPE;
  if (end > table_len) return ORC_ROW_OOB;
  if (!checked_mul(row_bytes, vocab, &need)) return ORC_SHAPE;
  if (table_len != need) return ORC_SHAPE;
  for (size_t j = 0; j < hidden; ++j) out[j] = bf16_at(table + start + 2 * j);
  return ORC_OK;
}

int orc_rmsnorm_f32(float* y, size_t y_len, const float* w, size_t w_len, const float* x,
                    size_t x_len, float eps) {
  if (x_len == 0 || y_len != x_len || w_len != x_len) return ORC_SHAPE;
  float inv = inv_rms_serial(x, x_len, eps);
  for (size_t i = 0; i < x_len; ++i) y[i] = w[i] * (x[i] * inv);
  return ORC_OK;
}

int orc_rmsnorm_bf16_weight(float* y, size_t y_len, const uint8_t* w, size_t w_len,
                            const float* x, size_t x_len, float eps) {
  if (x_len == 0 || y_len != x_len) return ORC_SHAPE;
  if (w_len != 2 * x_len) return ORC_SHAPE;
  rmsnorm_bf16(y, w, x, x_len, eps);
  return ORC_OK;
}

int orc_attn_scale_f32(size_t head_dim, float* out) {
  if (head_dim == 0) return ORC_SHAPE;  // gqa.rs:158-163
  *out = 1.0f / sqrtf((float)head_dim);
  return ORC_OK;
}

int orc_gqa_attn_f32(float* y, size_t y_len, const float* q, size_t q_len, const float* k,
                     size_t k_len, const float* v, size_t v_len, float* probs, size_t probs_len,
                     size_t hq, size_t hkv, size_t d, size_t seq, int mask_kind,
                     size_t query_pos) {
  // checked_shape, gqa.rs:232-266
  if (hq == 0 || hkv == 0 || d == 0 || seq == 0) return ORC_SHAPE;
  if (hq % hkv != 0) return ORC_SHAPE;
  size_t q_elems, kv_elems;
  if (!checked_mul(hq, d, &q_elems)) return ORC_SHAPE;
  if (!checked_mul(hkv, seq, &kv_elems) || !checked_mul(kv_elems, d, &kv_elems)) return ORC_SHAPE;
  if (y_len != q_elems || q_len != q_elems || k_len != kv_elems || v_len != kv_elems)
    return ORC_SHAPE;
  if (probs_len != seq) return ORC_SHAPE;
  gqa_impl(y, q, k, v, probs, hq, hkv, d, seq, mask_kind, query_pos);
  return ORC_OK;
}

int orc_rope_inv_freqs(float* inv_freq, size_t len, size_t head_dim, float theta) {
  if (head_dim == 0 || head_dim % 2 != 0) return ORC_SHAPE;  // rope.rs:82-92
  if (len != head_dim / 2) return ORC_SHAPE;
  for (size_t i = 0; i < len; ++i) inv_freq[i] = inv_freq_at(i, head_dim, theta);
  return ORC_OK;
}

static int rope_check(size_t len, size_t head_dim) {
  if (head_dim == 0 || head_dim % 2 != 0) return ORC_SHAPE;  // rope.rs:128-142
  if (len == 0 || len % head_dim != 0) return ORC_SHAPE;
  return ORC_OK;
}

int orc_rope_f32(float* y, size_t y_len, const float* x, size_t x_len, uint32_t position,
                 size_t head_dim, float theta) {
  if (x_len != y_len) return ORC_SHAPE;
  int st = rope_check(y_len, head_dim);
  if (st) return st;
  rotate(y, x, y_len, position, head_dim, theta);
  return ORC_OK;
}

int orc_rope_f32_inplace(float* x, size_t len, uint32_t position, size_t head_dim, float theta) {
  int st = rope_check(len, head_dim);
  if (st) return st;
  rotate(x, nullptr, len, position, head_dim, theta);
  return ORC_OK;
}

float orc_silu_f32(float z) { return silu(z); }

int orc_swiglu_mul_f32(float* h, size_t h_len, const float* gate, size_t gate_len,
                       const float* up, size_t up_len) {
  if (gate_len == 0 || up_len != gate_len || h_len != gate_len) return ORC_SHAPE;
  mul_ltr(h, gate, up, gate_len);
  return ORC_OK;
}

// swiglu.rs:184-213
int orc_swiglu_bf16(float* y, size_t y_len, const float* x, size_t x_len, const uint8_t* gate_w,
                    size_t gate_w_len, const uint8_t* up_w, size_t up_w_len,
                    const uint8_t* down_w, size_t down_w_len, float* gate, size_t gate_len,
                    float* up, size_t up_len, float* h, size_t h_len, size_t hidden,
                    size_t inter) {
  if (hidden == 0 || inter == 0) return ORC_SHAPE;
  if (y_len != hidden || x_len != hidden) return ORC_SHAPE;
  if (gate_len != inter || up_len != inter || h_len != inter) return ORC_SHAPE;
  size_t gb, db;
  if (!checked_mul(hidden, 2, &gb) || !checked_mul(gb, inter, &gb)) return ORC_SHAPE;
  if (!checked_mul(inter, 2, &db) || !checked_mul(db, hidden, &db)) return ORC_SHAPE;
  if (gate_w_len != gb || up_w_len != gb || down_w_len != db) return ORC_SHAPE;
  size_t t = resolve_threads(0);
  gemv_parallel(gate, gate_w, x, inter, hidden, t);
  gemv_parallel(up, up_w, x, inter, hidden, t);
  mul_ltr(h, gate, up, inter);
  gemv_parallel(y, down_w, h, hidden, inter, t);
  return ORC_OK;
}

// gemm_bf16.rs:73-110
int orc_gemm_bf16(float* y, size_t y_len, const uint8_t* w, size_t w_len, const float* x,
                  size_t x_len, size_t batch, size_t m, size_t k, int threads) {
  size_t yn, xn, wn;
  if (!checked_mul(batch, m, &yn) || !checked_mul(batch, k, &xn)) return ORC_SHAPE;
  if (!checked_mul(m, k, &wn) || !checked_mul(wn, 2, &wn)) return ORC_SHAPE;
  if (y_len != yn || x_len != xn || w_len != wn) return ORC_SHAPE;
  if (m == 0 || batch == 0) return ORC_OK;
  if (k == 0) {
    std::fill(y, y + yn, 0.0f);
    return ORC_OK;
  }
  gemm_impl(y, w, x, batch, m, k, resolve_threads(threads));
  return ORC_OK;
}

// model_core/src/lib.rs:157-167: first maximum, strict `>`, from -inf.
uint32_t orc_greedy_token(const float* logits, size_t n) {
  size_t best_i = 0;
  float best = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    if (logits[i] > best) {
      best = logits[i];
      best_i = i;
    }
  }
  return (uint32_t)best_i;
}

}  // extern "C"

// ================================================================= weight map
struct orc_map {
  struct Entry {
    int dtype;
    std::vector<size_t> shape;
    const uint8_t* bytes;
    size_t nbytes;
    std::vector<uint8_t> owned;
  };
  std::map<std::string, Entry> index;
};

static size_t dtype_size(int dt) { return dt == ORC_F32 ? 4 : 2; }

extern "C" {

orc_map* orc_map_new(void) { return new orc_map(); }
void orc_map_free(orc_map* m) { delete m; }
size_t orc_map_len(const orc_map* m) { return m->index.size(); }

// MmapWeights::insert_bytes, weight_loader/src/lib.rs:224-256
int orc_map_insert(orc_map* m, const char* name, int dtype, const size_t* shape, size_t rank,
                   const void* bytes, size_t nbytes, int copy) {
  if (!name || !*name) return ORC_EMPTY_NAME;
  if (m->index.count(name)) return ORC_DUPLICATE;
  if (dtype != ORC_F32 && dtype != ORC_F16 && dtype != ORC_BF16) return ORC_UNSUPPORTED;
  size_t numel = 1;
  for (size_t i = 0; i < rank; ++i)
    if (!checked_mul(numel, shape[i], &numel)) return ORC_W_LENGTH;
  size_t need;
  if (!checked_mul(numel, dtype_size(dtype), &need)) return ORC_W_LENGTH;
  if (need != nbytes) return ORC_W_LENGTH;
  orc_map::Entry e;
  e.dtype = dtype;
  e.shape.assign(shape, shape + rank);
  e.nbytes = nbytes;
  if (copy) {
    e.owned.assign((const uint8_t*)bytes, (const uint8_t*)bytes + nbytes);
    e.bytes = e.owned.data();
  } else {
    e.bytes = (const uint8_t*)bytes;
  }
  auto it = m->index.emplace(name, std::move(e)).first;
  if (copy) it->second.bytes = it->second.owned.data();
  return ORC_OK;
}

}  // extern "C"

// ================================================================= model_core
namespace {

struct View {
  const uint8_t* bytes;
  size_t nbytes;
};

// qwen25_bf16.rs:72-82 (bf16_tensor) over weight_loader::bf16_view (lib.rs:99-113).
int bf16_tensor(const orc_map* m, const std::string& name, std::initializer_list<size_t> expect,
                View* out) {
  auto it = m->index.find(name);
  if (it == m->index.end()) return ORC_W_MISSING;
  const auto& e = it->second;
  if (e.dtype != ORC_BF16) return ORC_W_DTYPE;
  size_t numel = 1;
  for (size_t d : e.shape) numel *= d;
  if (numel * 2 != e.nbytes) return ORC_W_LENGTH;
  if (e.shape.size() != expect.size() || !std::equal(e.shape.begin(), e.shape.end(), expect.begin()))
    return ORC_W_SHAPE;
  out->bytes = e.bytes;
  out->nbytes = e.nbytes;
  return ORC_OK;
}

std::string layer_key(size_t layer, const char* suffix) {  // qwen25_layout.rs:121-123
  return "model.layers." + std::to_string(layer) + "." + suffix;
}

const char* kEmbed = "model.embed_tokens.weight";
const char* kFinalNorm = "model.norm.weight";
const char* kLmHead = "lm_head.weight";

}  // namespace

struct orc_model {
  orc_shape s;
  size_t max_seq;
  size_t q_dim, kv_dim;
  size_t len = 0;             // KvCache cursor
  std::vector<float> kc, vc;  // [L][Hkv][max_seq][d]
  // BlockWorkspace / AttnWorkspace
  std::vector<float> x, normed, mlp, gate, up, act, logits;
  std::vector<float> q, k, v, att, proj, probs, pack_k, pack_v;

  size_t slot(size_t layer, size_t head, size_t pos) const {
    return ((layer * s.num_kv_heads + head) * max_seq + pos) * s.head_dim;
  }
  void store_at(size_t layer, size_t pos, const float* key, const float* val) {
    size_t d = s.head_dim;
    for (size_t h = 0; h < s.num_kv_heads; ++h) {
      memcpy(&kc[slot(layer, h, pos)], key + h * d, d * 4);
      memcpy(&vc[slot(layer, h, pos)], val + h * d, d * 4);
    }
  }
};

namespace {

int head_view(const orc_model* md, const orc_map* m, View* out) {
  const orc_shape& s = md->s;
  if (s.tied_head) return bf16_tensor(m, kEmbed, {s.vocab, s.hidden}, out);
  return bf16_tensor(m, kLmHead, {s.vocab, s.hidden}, out);  // untied extension
}

// attn_wire.rs:207-313
int attention_layer(orc_model* md, const orc_map* m, size_t layer, size_t pos) {
  const orc_shape& s = md->s;
  const size_t H = s.hidden, qd = md->q_dim, kvd = md->kv_dim, d = s.head_dim;
  View qw, qb, kw, kb, vw, vb, ow;
  int st;
  if ((st = bf16_tensor(m, layer_key(layer, "self_attn.q_proj.weight"), {qd, H}, &qw))) return st;
  if ((st = bf16_tensor(m, layer_key(layer, "self_attn.q_proj.bias"), {qd}, &qb))) return st;
  if ((st = bf16_tensor(m, layer_key(layer, "self_attn.k_proj.weight"), {kvd, H}, &kw))) return st;
  if ((st = bf16_tensor(m, layer_key(layer, "self_attn.k_proj.bias"), {kvd}, &kb))) return st;
  if ((st = bf16_tensor(m, layer_key(layer, "self_attn.v_proj.weight"), {kvd, H}, &vw))) return st;
  if ((st = bf16_tensor(m, layer_key(layer, "self_attn.v_proj.bias"), {kvd}, &vb))) return st;
  if ((st = bf16_tensor(m, layer_key(layer, "self_attn.o_proj.weight"), {H, qd}, &ow))) return st;
  size_t t = resolve_threads(0);
  gemv_parallel(md->q.data(), qw.bytes, md->normed.data(), qd, H, t);
  add_bias(md->q.data(), qb.bytes, qd);
  gemv_parallel(md->k.data(), kw.bytes, md->normed.data(), kvd, H, t);
  add_bias(md->k.data(), kb.bytes, kvd);
  gemv_parallel(md->v.data(), vw.bytes, md->normed.data(), kvd, H, t);
  add_bias(md->v.data(), vb.bytes, kvd);
  rotate(md->q.data(), nullptr, qd, (uint32_t)pos, d, s.rope_theta);
  rotate(md->k.data(), nullptr, kvd, (uint32_t)pos, d, s.rope_theta);
  // pack_prefix_with_token, kv_cache.rs:259-302
  size_t seq = pos + 1;
  for (size_t h = 0; h < s.num_kv_heads; ++h) {
    for (size_t tt = 0; tt < pos; ++tt) {
      memcpy(&md->pack_k[(h * seq + tt) * d], &md->kc[md->slot(layer, h, tt)], d * 4);
      memcpy(&md->pack_v[(h * seq + tt) * d], &md->vc[md->slot(layer, h, tt)], d * 4);
    }
    memcpy(&md->pack_k[(h * seq + pos) * d], &md->k[h * d], d * 4);
    memcpy(&md->pack_v[(h * seq + pos) * d], &md->v[h * d], d * 4);
  }
  gqa_impl(md->att.data(), md->q.data(), md->pack_k.data(), md->pack_v.data(), md->probs.data(),
           s.num_q_heads, s.num_kv_heads, d, seq, 0, 0);
  gemv_parallel(md->proj.data(), ow.bytes, md->att.data(), H, qd, t);
  md->store_at(layer, pos, md->k.data(), md->v.data());  // cache.store after attention
  for (size_t i = 0; i < H; ++i) md->x[i] += md->proj[i];
  return ORC_OK;
}

int check_ready(const orc_model* md, size_t pos) {  // qwen25_block.rs:185-208
  if (pos != md->len) return ORC_POSITION;
  if (pos >= md->max_seq) return ORC_CACHE_FULL;
  return ORC_OK;
}

int forward_token_impl(orc_model* md, const orc_map* m, uint32_t token, size_t pos) {
  // qwen25_block.rs:220-304
  int st = check_ready(md, pos);
  if (st) return st;
  const orc_shape& s = md->s;
  const size_t H = s.hidden, I = s.intermediate;
  View emb;
  if ((st = bf16_tensor(m, kEmbed, {s.vocab, H}, &emb))) return st;
  if ((size_t)token >= s.vocab) return ORC_TOKEN;
  for (size_t j = 0; j < H; ++j) md->x[j] = bf16_at(emb.bytes + ((size_t)token * H + j) * 2);
  size_t t = resolve_threads(0);
  for (size_t layer = 0; layer < s.num_layers; ++layer) {
    View ln, post, gw, uw, dw;
    if ((st = bf16_tensor(m, layer_key(layer, "input_layernorm.weight"), {H}, &ln))) return st;
    rmsnorm_bf16(md->normed.data(), ln.bytes, md->x.data(), H, s.rms_eps);
    if ((st = attention_layer(md, m, layer, pos))) return st;
    if ((st = bf16_tensor(m, layer_key(layer, "post_attention_layernorm.weight"), {H}, &post)))
      return st;
    rmsnorm_bf16(md->normed.data(), post.bytes, md->x.data(), H, s.rms_eps);
    if ((st = bf16_tensor(m, layer_key(layer, "mlp.gate_proj.weight"), {I, H}, &gw))) return st;
    if ((st = bf16_tensor(m, layer_key(layer, "mlp.up_proj.weight"), {I, H}, &uw))) return st;
    if ((st = bf16_tensor(m, layer_key(layer, "mlp.down_proj.weight"), {H, I}, &dw))) return st;
    gemv_parallel(md->gate.data(), gw.bytes, md->normed.data(), I, H, t);
    gemv_parallel(md->up.data(), uw.bytes, md->normed.data(), I, H, t);
    mul_ltr(md->act.data(), md->gate.data(), md->up.data(), I);
    gemv_parallel(md->mlp.data(), dw.bytes, md->act.data(), H, I, t);
    for (size_t i = 0; i < H; ++i) md->x[i] += md->mlp[i];
  }
  View fn, head;
  if ((st = bf16_tensor(m, kFinalNorm, {H}, &fn))) return st;
  rmsnorm_bf16(md->normed.data(), fn.bytes, md->x.data(), H, s.rms_eps);
  if ((st = head_view(md, m, &head))) return st;
  gemv_parallel(md->logits.data(), head.bytes, md->normed.data(), s.vocab, H, t);
  md->len += 1;  // cache.advance()
  return ORC_OK;
}

// qwen25_block.rs:599-643
int preflight(const orc_model* md, const orc_map* m) {
  const orc_shape& s = md->s;
  const size_t H = s.hidden, I = s.intermediate, qd = md->q_dim, kvd = md->kv_dim;
  View v;
  int st;
  if ((st = bf16_tensor(m, kEmbed, {s.vocab, H}, &v))) return st;
  if ((st = bf16_tensor(m, kFinalNorm, {H}, &v))) return st;
  for (size_t l = 0; l < s.num_layers; ++l) {
    if ((st = bf16_tensor(m, layer_key(l, "input_layernorm.weight"), {H}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "self_attn.q_proj.weight"), {qd, H}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "self_attn.q_proj.bias"), {qd}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "self_attn.k_proj.weight"), {kvd, H}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "self_attn.k_proj.bias"), {kvd}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "self_attn.v_proj.weight"), {kvd, H}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "self_attn.v_proj.bias"), {kvd}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "self_attn.o_proj.weight"), {H, qd}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "post_attention_layernorm.weight"), {H}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "mlp.gate_proj.weight"), {I, H}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "mlp.up_proj.weight"), {I, H}, &v))) return st;
    if ((st = bf16_tensor(m, layer_key(l, "mlp.down_proj.weight"), {H, I}, &v))) return st;
  }
  if (!s.tied_head && (st = bf16_tensor(m, kLmHead, {s.vocab, H}, &v))) return st;
  return ORC_OK;
}

// qwen25_block.rs:323-543
int prefill_impl(orc_model* md, const orc_map* m, const uint32_t* tokens, size_t n) {
  if (n == 0) return ORC_SHAPE;
  const orc_shape& s = md->s;
  size_t start = md->len;
  int st = check_ready(md, start);
  if (st) return st;
  size_t end = start + n;
  if (end > md->max_seq) return ORC_CACHE_FULL;
  const size_t H = s.hidden, I = s.intermediate, qd = md->q_dim, kvd = md->kv_dim,
               d = s.head_dim;
  for (size_t i = 0; i < n; ++i)
    if ((size_t)tokens[i] >= s.vocab) return ORC_TOKEN;
  if ((st = preflight(md, m))) return st;
  std::vector<float> x(n * H), normed(n * H), q(n * qd), k(n * kvd), v(n * kvd), att(n * qd),
      proj(n * H), gate(n * I), up(n * I), act(n * I), pk(s.num_kv_heads * end * d),
      pv(s.num_kv_heads * end * d), probs(end);
  View emb;
  bf16_tensor(m, kEmbed, {s.vocab, H}, &emb);
  for (size_t i = 0; i < n; ++i)
    for (size_t j = 0; j < H; ++j) x[i * H + j] = bf16_at(emb.bytes + ((size_t)tokens[i] * H + j) * 2);
  size_t t = resolve_threads(0);
  for (size_t l = 0; l < s.num_layers; ++l) {
    View ln, qw, kw, vw, qb, kb, vb, ow, post, gw, uw, dw;
    bf16_tensor(m, layer_key(l, "input_layernorm.weight"), {H}, &ln);
    bf16_tensor(m, layer_key(l, "self_attn.q_proj.weight"), {qd, H}, &qw);
    bf16_tensor(m, layer_key(l, "self_attn.k_proj.weight"), {kvd, H}, &kw);
    bf16_tensor(m, layer_key(l, "self_attn.v_proj.weight"), {kvd, H}, &vw);
    bf16_tensor(m, layer_key(l, "self_attn.q_proj.bias"), {qd}, &qb);
    bf16_tensor(m, layer_key(l, "self_attn.k_proj.bias"), {kvd}, &kb);
    bf16_tensor(m, layer_key(l, "self_attn.v_proj.bias"), {kvd}, &vb);
    bf16_tensor(m, layer_key(l, "self_attn.o_proj.weight"), {H, qd}, &ow);
    for (size_t i = 0; i < n; ++i) rmsnorm_bf16(&normed[i * H], ln.bytes, &x[i * H], H, s.rms_eps);
    gemm_impl(q.data(), qw.bytes, normed.data(), n, qd, H, t);
    gemm_impl(k.data(), kw.bytes, normed.data(), n, kvd, H, t);
    gemm_impl(v.data(), vw.bytes, normed.data(), n, kvd, H, t);
    for (size_t i = 0; i < n; ++i) {  // bias_rope_store, :679-712
      add_bias(&q[i * qd], qb.bytes, qd);
      add_bias(&k[i * kvd], kb.bytes, kvd);
      add_bias(&v[i * kvd], vb.bytes, kvd);
      rotate(&q[i * qd], nullptr, qd, (uint32_t)(start + i), d, s.rope_theta);
      rotate(&k[i * kvd], nullptr, kvd, (uint32_t)(start + i), d, s.rope_theta);
      md->store_at(l, start + i, &k[i * kvd], &v[i * kvd]);
    }
    // attend_chunk, :714-758: pack_prefix(end) then Causal{start+i} per query.
    for (size_t h = 0; h < s.num_kv_heads; ++h)
      for (size_t tt = 0; tt < end; ++tt) {
        memcpy(&pk[(h * end + tt) * d], &md->kc[md->slot(l, h, tt)], d * 4);
        memcpy(&pv[(h * end + tt) * d], &md->vc[md->slot(l, h, tt)], d * 4);
      }
    for (size_t i = 0; i < n; ++i)
      gqa_impl(&att[i * qd], &q[i * qd], pk.data(), pv.data(), probs.data(), s.num_q_heads,
               s.num_kv_heads, d, end, 1, start + i);
    gemm_impl(proj.data(), ow.bytes, att.data(), n, H, qd, t);
    for (size_t i = 0; i < n * H; ++i) x[i] += proj[i];
    bf16_tensor(m, layer_key(l, "post_attention_layernorm.weight"), {H}, &post);
    bf16_tensor(m, layer_key(l, "mlp.gate_proj.weight"), {I, H}, &gw);
    bf16_tensor(m, layer_key(l, "mlp.up_proj.weight"), {I, H}, &uw);
    bf16_tensor(m, layer_key(l, "mlp.down_proj.weight"), {H, I}, &dw);
    for (size_t i = 0; i < n; ++i)
      rmsnorm_bf16(&normed[i * H], post.bytes, &x[i * H], H, s.rms_eps);
    gemm_impl(gate.data(), gw.bytes, normed.data(), n, I, H, t);
    gemm_impl(up.data(), uw.bytes, normed.data(), n, I, H, t);
    for (size_t i = 0; i < n; ++i) mul_ltr(&act[i * I], &gate[i * I], &up[i * I], I);
    gemm_impl(proj.data(), dw.bytes, act.data(), n, H, I, t);
    for (size_t i = 0; i < n * H; ++i) x[i] += proj[i];
  }
  View fn, head;
  bf16_tensor(m, kFinalNorm, {H}, &fn);
  size_t last = (n - 1) * H;
  rmsnorm_bf16(md->normed.data(), fn.bytes, &x[last], H, s.rms_eps);
  memcpy(md->x.data(), &x[last], H * 4);
  if ((st = head_view(md, m, &head))) return st;
  gemv_parallel(md->logits.data(), head.bytes, md->normed.data(), s.vocab, H, t);
  md->len += n;
  return ORC_OK;
}

float top2_gap(const float* v, size_t n) {
  float a = -INFINITY, b = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    if (v[i] > a) {
      b = a;
      a = v[i];
    } else if (v[i] > b) {
      b = v[i];
    }
  }
  return a - b;
}

}  // namespace

extern "C" {

orc_model* orc_model_new(const orc_shape* shape, size_t max_seq, int* status) {
  const orc_shape& s = *shape;
  // BlockWorkspace::new / AttnWorkspace::new / KvCache::new checks.
  if (s.intermediate == 0 || s.vocab == 0 || s.num_layers == 0 || s.hidden == 0 ||
      s.num_q_heads == 0 || s.num_kv_heads == 0 || s.head_dim == 0 || s.head_dim % 2 != 0 ||
      s.num_q_heads % s.num_kv_heads != 0 || max_seq == 0) {
    if (status) *status = ORC_SHAPE;
    return nullptr;
  }
  orc_model* md = new orc_model();
  md->s = s;
  md->max_seq = max_seq;
  md->q_dim = s.num_q_heads * s.head_dim;
  md->kv_dim = s.num_kv_heads * s.head_dim;
  size_t kv_total = s.num_layers * s.num_kv_heads * max_seq * s.head_dim;
  md->kc.assign(kv_total, 0.0f);
  md->vc.assign(kv_total, 0.0f);
  md->x.assign(s.hidden, 0.0f);
  md->normed.assign(s.hidden, 0.0f);
  md->mlp.assign(s.hidden, 0.0f);
  md->gate.assign(s.intermediate, 0.0f);
  md->up.assign(s.intermediate, 0.0f);
  md->act.assign(s.intermediate, 0.0f);
  md->logits.assign(s.vocab, 0.0f);
  md->q.assign(md->q_dim, 0.0f);
  md->k.assign(md->kv_dim, 0.0f);
  md->v.assign(md->kv_dim, 0.0f);
  md->att.assign(md->q_dim, 0.0f);
  md->proj.assign(s.hidden, 0.0f);
  md->probs.assign(max_seq, 0.0f);
  md->pack_k.assign(s.num_kv_heads * max_seq * s.head_dim, 0.0f);
  md->pack_v.assign(s.num_kv_heads * max_seq * s.head_dim, 0.0f);
  if (status) *status = ORC_OK;
  return md;
}

void orc_model_free(orc_model* md) { delete md; }

int orc_forward_token(orc_model* md, const orc_map* m, uint32_t token, size_t pos) {
  // Logits are written only by the head GEMV after every layer succeeded, so
  // an error leaves them as they were (qwen25_block.rs:129-134).
  return forward_token_impl(md, m, token, pos);
}

int orc_prefill(orc_model* md, const orc_map* m, const uint32_t* tokens, size_t n) {
  return prefill_impl(md, m, tokens, n);
}

// qwen25_block.rs:765-780
int orc_greedy_decode(orc_model* md, const orc_map* m, size_t steps, uint32_t* out,
                      float* logits_dump, float* gap) {
  for (size_t i = 0; i < steps; ++i) {
    // gap[i] belongs to the logits that chose out[i] (before this forward).
    uint32_t tok = orc_greedy_token(md->logits.data(), md->s.vocab);
    if (gap) gap[i] = top2_gap(md->logits.data(), md->s.vocab);
    int st = orc_forward_token(md, m, tok, md->len);
    if (st) return st;
    out[i] = tok;
    if (logits_dump) memcpy(logits_dump + i * md->s.vocab, md->logits.data(), md->s.vocab * 4);
  }
  return ORC_OK;
}

int orc_forced_decode(orc_model* md, const orc_map* m, const uint32_t* feed, size_t steps,
                      uint32_t* argmax_out, float* gap, float* logits_dump) {
  for (size_t i = 0; i < steps; ++i) {
    if (argmax_out) argmax_out[i] = orc_greedy_token(md->logits.data(), md->s.vocab);
    if (gap) gap[i] = top2_gap(md->logits.data(), md->s.vocab);
    int st = orc_forward_token(md, m, feed[i], md->len);
    if (st) return st;
    if (logits_dump) memcpy(logits_dump + i * md->s.vocab, md->logits.data(), md->s.vocab * 4);
  }
  return ORC_OK;
}

const float* orc_model_logits(const orc_model* md) { return md->logits.data(); }
const float* orc_model_residual(const orc_model* md) { return md->x.data(); }
size_t orc_kv_len(const orc_model* md) { return md->len; }
void orc_kv_clear(orc_model* md) { md->len = 0; }

int orc_kv_head(const orc_model* md, size_t layer, size_t head, size_t pos, float* k_out,
                float* v_out) {
  if (layer >= md->s.num_layers || head >= md->s.num_kv_heads || pos >= md->max_seq)
    return ORC_CACHE_RANGE;
  size_t off = md->slot(layer, head, pos);
  memcpy(k_out, &md->kc[off], md->s.head_dim * 4);
  memcpy(v_out, &md->vc[off], md->s.head_dim * 4);
  return ORC_OK;
}

}  // extern "C"
