// tensor_core operators on host slices, and the device-pointer GEMV.
//
// Each host-slice entry point checks its arguments exactly as the Rust
// function it mirrors (returning before any write on error), copies the
// inputs to the current device, runs the same kernel the engine uses, and
// copies the result back. They exist for drop-in callers of the op-level
// API and for the per-kernel parity tests.
#include <math.h>
#include <string.h>

#include <vector>

#include "../../include/myos_cuda.h"
#include "kernels.h"

using namespace myos;

namespace {

// Scoped device buffer for the host-slice operators.
struct DBuf {
  void* p = nullptr;
  cudaError_t e = cudaSuccess;
  explicit DBuf(size_t n) { e = cudaMalloc(&p, n ? n : 16); }
  ~DBuf() {
    if (p) cudaFree(p);
  }
  template <class T>
  T* as() const {
    return (T*)p;
  }
};

bool mul_ok(size_t a, size_t b, size_t* out) { return !__builtin_mul_overflow(a, b, out); }

int num_sms() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

#define OPCK(call)                             \
  do {                                         \
    if ((call) != cudaSuccess) return MYOS_ERR_CUDA; \
  } while (0)

int gemv_device(float* y, const uint16_t* w, const float* x, size_t m, size_t k,
                cudaStream_t st) {
  GemvArgs a = {};
  a.w = w;
  a.M = (int)m;
  a.K = (int)k;
  a.in.x = x;
  a.y = y;
  OPCK(launch_gemv(EPI_STORE, a, gemv_grid((int)m, (int)k, 1, num_sms()), st, false));
  return MYOS_OK;
}

}  // namespace

extern "C" {

int myos_dev_gemv_bf16(float* d_y, const void* d_w, const float* d_x, size_t m, size_t k,
                       void* stream) {
  if (!d_y || !d_w || !d_x) return MYOS_ERR_ARG;
  if (m == 0) return MYOS_OK;
  if (k == 0 || m > 0x7fffffff || k > 50000) return MYOS_ERR_SHAPE;
  OPCK(kernels_init());
  return gemv_device(d_y, (const uint16_t*)d_w, d_x, m, k, (cudaStream_t)stream);
}

// tensor_core::gemv_bf16 (crates/tensor_core/src/bf16.rs:80-122).
int myos_gemv_bf16(float* y, size_t y_len, const uint8_t* w, size_t w_len, const float* x,
                   size_t x_len, size_t m, size_t k) {
  if (y_len != m || x_len != k) return MYOS_ERR_SHAPE;
  if (k == 0) {
    if (w_len != 0) return MYOS_ERR_SHAPE;
    for (size_t i = 0; i < m; ++i) y[i] = 0.0f;
    return MYOS_OK;
  }
  size_t row_bytes, need;
  if (!mul_ok(k, 2, &row_bytes)) return MYOS_ERR_SHAPE;
  if (w_len / row_bytes < m) return MYOS_ERR_ROW_OOB;
  if (!mul_ok(row_bytes, m, &need) || w_len != need) return MYOS_ERR_SHAPE;
  if (m == 0) return MYOS_OK;
  if (m > 0x7fffffff || k > 50000) return MYOS_ERR_SHAPE;
  OPCK(kernels_init());
  DBuf dw(w_len), dx(k * 4), dy(m * 4);
  if (dw.e || dx.e || dy.e) return MYOS_ERR_CUDA;
  OPCK(cudaMemcpy(dw.p, w, w_len, cudaMemcpyHostToDevice));
  OPCK(cudaMemcpy(dx.p, x, k * 4, cudaMemcpyHostToDevice));
  int st = gemv_device(dy.as<float>(), dw.as<uint16_t>(), dx.as<float>(), m, k, 0);
  if (st) return st;
  OPCK(cudaMemcpy(y, dy.p, m * 4, cudaMemcpyDeviceToHost));
  return MYOS_OK;
}

// tensor_core::rmsnorm_bf16_weight (bf16.rs:231-249).
int myos_rmsnorm_bf16_weight(float* y, size_t y_len, const uint8_t* w, size_t w_len,
                             const float* x, size_t x_len, float eps) {
  if (x_len == 0 || y_len != x_len || w_len != 2 * x_len) return MYOS_ERR_SHAPE;
  std::vector<float> g(x_len);
  for (size_t i = 0; i < x_len; ++i) {
    uint32_t b = ((uint32_t)w[2 * i] | ((uint32_t)w[2 * i + 1] << 8)) << 16;
    memcpy(&g[i], &b, 4);
  }
  OPCK(kernels_init());
  DBuf dg(x_len * 4), dx(x_len * 4), dy(x_len * 4);
  if (dg.e || dx.e || dy.e) return MYOS_ERR_CUDA;
  OPCK(cudaMemcpy(dg.p, g.data(), x_len * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemcpy(dx.p, x, x_len * 4, cudaMemcpyHostToDevice));
  OPCK(launch_rmsnorm(dy.as<float>(), dx.as<float>(), dg.as<float>(), (int)x_len, eps, 0));
  OPCK(cudaMemcpy(y, dy.p, x_len * 4, cudaMemcpyDeviceToHost));
  return MYOS_OK;
}

// tensor_core::gqa_attn_f32 (gqa.rs:174-218) without the probs scratch.
int myos_gqa_attn_f32(float* y, size_t y_len, const float* q, size_t q_len, const float* k,
                      size_t k_len, const float* v, size_t v_len, size_t hq, size_t hkv,
                      size_t d, size_t seq, int32_t mask_kind, size_t query_pos) {
  if (mask_kind != 0 && mask_kind != 1) return MYOS_ERR_ARG;  // GqaMask: Full or Causal
  if (hq == 0 || hkv == 0 || d == 0 || seq == 0 || hq % hkv != 0) return MYOS_ERR_SHAPE;
  size_t qe, kve;
  if (!mul_ok(hq, d, &qe) || !mul_ok(hkv, seq, &kve) || !mul_ok(kve, d, &kve)) return MYOS_ERR_SHAPE;
  if (y_len != qe || q_len != qe || k_len != kve || v_len != kve) return MYOS_ERR_SHAPE;
  const size_t G = hq / hkv;
  if (G > 8 || d > 256 || seq > 0x7fffffff) return MYOS_ERR_SHAPE;
  size_t nkeys = seq;
  if (mask_kind == 1 && query_pos < seq - 1) nkeys = query_pos + 1;
  OPCK(kernels_init());
  size_t nsplit = (nkeys + 31) / 32;
  if (nsplit > 64) nsplit = 64;
  const size_t chunk = (nkeys + nsplit - 1) / nsplit;
  DBuf dq(qe * 4), dk(kve * 4), dv(kve * 4), dy(qe * 4), po(hkv * nsplit * G * d * 4),
      pm(hkv * nsplit * G * 4), pl(hkv * nsplit * G * 4), cnt(hkv * 4);
  if (dq.e || dk.e || dv.e || dy.e || po.e || pm.e || pl.e || cnt.e) return MYOS_ERR_CUDA;
  OPCK(cudaMemcpy(dq.p, q, qe * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemcpy(dk.p, k, kve * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemcpy(dv.p, v, kve * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemset(cnt.p, 0, hkv * 4));
  AttnArgs a = {};
  a.q = dq.as<float>();
  a.kc = dk.p;
  a.vc = dv.p;
  a.S = (int)seq;
  a.Hq = (int)hq;
  a.Hkv = (int)hkv;
  a.d = (int)d;
  a.G = (int)G;
  a.nkeys_fixed = (int)nkeys;
  a.chunk = (int)chunk;
  a.nsplit = (int)nsplit;
  a.scale = 1.0f / sqrtf((float)d);
  a.part_o = po.as<float>();
  a.part_m = pm.as<float>();
  a.part_l = pl.as<float>();
  a.counters = cnt.as<unsigned>();
  a.out = dy.as<float>();
  a.decode = 0;
  OPCK(launch_attention(a, 0, 0, false));
  OPCK(cudaMemcpy(y, dy.p, qe * 4, cudaMemcpyDeviceToHost));
  return MYOS_OK;
}

// tensor_core::swiglu_mul_f32 (swiglu.rs:125-131).
int myos_swiglu_mul_f32(float* h, size_t h_len, const float* gate, size_t gate_len,
                        const float* up, size_t up_len) {
  if (gate_len == 0 || up_len != gate_len || h_len != gate_len) return MYOS_ERR_SHAPE;
  if (gate_len > 0x7fffffff) return MYOS_ERR_SHAPE;
  OPCK(kernels_init());
  DBuf dg(gate_len * 4), du(gate_len * 4), dh(gate_len * 4);
  if (dg.e || du.e || dh.e) return MYOS_ERR_CUDA;
  OPCK(cudaMemcpy(dg.p, gate, gate_len * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemcpy(du.p, up, gate_len * 4, cudaMemcpyHostToDevice));
  OPCK(launch_swiglu_mul(dh.as<float>(), dg.as<float>(), du.as<float>(), (int)gate_len, 0));
  OPCK(cudaMemcpy(h, dh.p, gate_len * 4, cudaMemcpyDeviceToHost));
  return MYOS_OK;
}

// tensor_core::rope_f32 (rope.rs:107-115). The cos/sin row is built on the
// host with libm exactly as rope.rs:186-194; the device applies it.
int myos_rope_f32(float* y, size_t y_len, const float* x, size_t x_len, uint32_t position,
                  size_t head_dim, float theta) {
  if (x_len != y_len) return MYOS_ERR_SHAPE;
  if (head_dim == 0 || head_dim % 2 != 0 || y_len == 0 || y_len % head_dim != 0)
    return MYOS_ERR_SHAPE;
  if (y_len > 0x7fffffff) return MYOS_ERR_SHAPE;
  const size_t half = head_dim / 2;
  std::vector<float> cs(half), sn(half);
  for (size_t i = 0; i < half; ++i) {
    volatile float exponent = (float)(2 * i) / (float)head_dim;
    volatile float inv = 1.0f / powf(theta, exponent);
    volatile float angle = (float)position * inv;
    cs[i] = cosf(angle);
    sn[i] = sinf(angle);
  }
  OPCK(kernels_init());
  DBuf dx(x_len * 4), dy(y_len * 4), dc(half * 4), ds(half * 4);
  if (dx.e || dy.e || dc.e || ds.e) return MYOS_ERR_CUDA;
  OPCK(cudaMemcpy(dx.p, x, x_len * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemcpy(dc.p, cs.data(), half * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemcpy(ds.p, sn.data(), half * 4, cudaMemcpyHostToDevice));
  OPCK(launch_rope(dy.as<float>(), dx.as<float>(), (int)y_len, (int)head_dim, dc.as<float>(),
                   ds.as<float>(), 0));
  OPCK(cudaMemcpy(y, dy.p, y_len * 4, cudaMemcpyDeviceToHost));
  return MYOS_OK;
}

// model_core::greedy_token (crates/model_core/src/lib.rs:157-167).
int myos_greedy_token(const float* logits, size_t n, uint32_t* out) {
  if (!out) return MYOS_ERR_ARG;
  if (n == 0) {
    *out = 0;
    return MYOS_OK;
  }
  if (n > 0x7fffffff) return MYOS_ERR_SHAPE;
  OPCK(kernels_init());
  int grid = (int)((n + 4095) / 4096);
  if (grid > 296) grid = 296;
  DBuf dv(n * 4), pv(grid * 4), pi(grid * 4), cnt(4), dout(4);
  if (dv.e || pv.e || pi.e || cnt.e || dout.e) return MYOS_ERR_CUDA;
  OPCK(cudaMemcpy(dv.p, logits, n * 4, cudaMemcpyHostToDevice));
  OPCK(cudaMemset(cnt.p, 0, 4));
  OPCK(launch_argmax(dv.as<float>(), (int)n, pv.as<float>(), pi.as<uint32_t>(), cnt.as<unsigned>(),
                     dout.as<uint32_t>(), grid, 0));
  OPCK(cudaMemcpy(out, dout.p, 4, cudaMemcpyDeviceToHost));
  return MYOS_OK;
}

}  // extern "C"
