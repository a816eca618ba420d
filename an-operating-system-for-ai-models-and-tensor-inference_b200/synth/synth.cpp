// Seeded synthetic weights and prompts for the Qwen2.5 configs.
//
// Counter-based: element i of stream s under seed k is a pure function of
// (k, s, i), so any thread split gives the same bytes and the CPU oracle and
// the CUDA engine always see identical inputs. Generator: Philox4x32-10
// (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011) -> two 53-bit uniforms -> Box-Muller (double precision) -> f32 ->
// bf16 round-to-nearest-even.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

namespace {

struct Block {
  uint32_t v[4];
};

inline void mulhilo(uint32_t a, uint32_t b, uint32_t* hi, uint32_t* lo) {
  uint64_t p = (uint64_t)a * (uint64_t)b;
  *hi = (uint32_t)(p >> 32);
  *lo = (uint32_t)p;
}

// Philox4x32 with 10 rounds; multipliers and Weyl key increments as published.
Block philox(uint64_t counter, uint64_t stream, uint64_t seed) {
  uint32_t c0 = (uint32_t)counter, c1 = (uint32_t)(counter >> 32);
  uint32_t c2 = (uint32_t)stream, c3 = (uint32_t)(stream >> 32);
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(0xD2511F53u, c0, &hi0, &lo0);
    mulhilo(0xCD9E8D57u, c2, &hi1, &lo1);
    uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
    c0 = n0;
    c1 = n1;
    c2 = n2;
    c3 = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return Block{{c0, c1, c2, c3}};
}

// (0, 1] from 53 bits, so log() never sees 0.
inline double unit_open0(uint32_t a, uint32_t b) {
  uint64_t m = ((uint64_t)a << 21) ^ (uint64_t)(b >> 11);
  m &= (1ull << 53) - 1;
  return ((double)m + 1.0) * (1.0 / 9007199254740992.0);
}

inline void normal_pair(uint64_t idx, uint64_t stream, uint64_t seed, double* z0, double* z1) {
  Block b = philox(idx, stream, seed);
  double u1 = unit_open0(b.v[0], b.v[1]);
  double u2 = unit_open0(b.v[2], b.v[3]);
  double r = sqrt(-2.0 * log(u1));
  double t = 6.283185307179586 * u2;
  *z0 = r * cos(t);
  *z1 = r * sin(t);
}

inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// fn(a, b) over [0, n) split across threads; `work` (default n) is the
// amount of work behind the n items, and below 2^16 of it one thread runs all.
template <class F>
void parallel_for(size_t n, int threads, F&& fn, size_t work = 0) {
  if (threads <= 1 || (work ? work : n) < (1u << 16)) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> ts;
  size_t per = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    size_t a = std::min(n, per * t), b = std::min(n, per * (t + 1));
    if (a < b) ts.emplace_back([=, &fn] { fn(a, b); });
  }
  for (auto& th : ts) th.join();
}

int default_threads(int threads) {
  if (threads > 0) return threads;
  unsigned hc = std::thread::hardware_concurrency();
  return (int)std::max(1u, std::min(hc, 64u));
}

}  // namespace

extern "C" {

// out[i] = bf16(mean + std * N(0,1)), element i of (seed, stream). n may be odd.
void myos_synth_normal_bf16(uint64_t seed, uint64_t stream, float mean, float std_dev,
                            uint16_t* out, size_t n, int threads) {
  parallel_for((n + 1) / 2, default_threads(threads), [&](size_t a, size_t b) {
    for (size_t p = a; p < b; ++p) {
      double z0, z1;
      normal_pair(p, stream, seed, &z0, &z1);
      size_t i = 2 * p;
      out[i] = f32_to_bf16_rne((float)((double)mean + (double)std_dev * z0));
      if (i + 1 < n) out[i + 1] = f32_to_bf16_rne((float)((double)mean + (double)std_dev * z1));
    }
  });
}

// Block [row0, row0 + nrows) x [col0, col0 + ncols) of the rows x cols
// tensor myos_synth_normal_bf16 makes, written at its place in out (a
// rows x cols buffer); the rest of out is left as it was. Same values as the
// whole tensor (element i is a pure function of seed, stream and i).
void myos_synth_normal_bf16_block(uint64_t seed, uint64_t stream, float mean, float std_dev,
                                  uint16_t* out, size_t rows, size_t cols, size_t row0,
                                  size_t nrows, size_t col0, size_t ncols, int threads) {
  if (nrows == 0 || ncols == 0 || row0 + nrows > rows || col0 + ncols > cols) return;
  parallel_for(nrows, default_threads(threads), [&](size_t a, size_t b) {
    auto value = [&](double z) { return f32_to_bf16_rne((float)((double)mean + (double)std_dev * z)); };
    for (size_t r = row0 + a; r < row0 + b; ++r) {
      const size_t first = r * cols + col0, last = first + ncols;  // elements [first, last)
      size_t p = first / 2;
      double z0, z1;
      if (first & 1) {  // the row starts with the second value of a pair
        normal_pair(p, stream, seed, &z0, &z1);
        out[first] = value(z1);
        ++p;
      }
      const size_t pend = last / 2;  // pairs wholly inside the row
      for (; p < pend; ++p) {  // the whole-tensor loop's body, without edge tests
        normal_pair(p, stream, seed, &z0, &z1);
        out[2 * p] = value(z0);
        out[2 * p + 1] = value(z1);
      }
      if ((last & 1) && 2 * pend >= first) {  // the row ends with the first value of a pair
        normal_pair(pend, stream, seed, &z0, &z1);
        out[last - 1] = value(z0);
      }
    }
  }, nrows * ncols);
}

// f32 variant (activations for the GEMV microbench).
void myos_synth_normal_f32(uint64_t seed, uint64_t stream, float mean, float std_dev, float* out,
                           size_t n, int threads) {
  parallel_for((n + 1) / 2, default_threads(threads), [&](size_t a, size_t b) {
    for (size_t p = a; p < b; ++p) {
      double z0, z1;
      normal_pair(p, stream, seed, &z0, &z1);
      size_t i = 2 * p;
      out[i] = (float)((double)mean + (double)std_dev * z0);
      if (i + 1 < n) out[i + 1] = (float)((double)mean + (double)std_dev * z1);
    }
  });
}

// Uniform ids in [0, bound): 64-bit draw reduced by multiply-shift (bias < 2^-32).
void myos_synth_uniform_u32(uint64_t seed, uint64_t stream, uint32_t bound, uint32_t* out,
                            size_t n) {
  for (size_t i = 0; i < n; ++i) {
    Block b = philox(i, stream, seed);
    uint64_t r = ((uint64_t)b.v[0] << 32) | b.v[1];
    out[i] = (uint32_t)(((unsigned __int128)r * bound) >> 64);
  }
}

}  // extern "C"
