// myos — command-line runner over the C ABI (include/myos_cuda.h), with the
// flags, exit codes, stdout lines and run artefacts of the reference's
// runtime CLI (crates/runtime/src/main.rs:58-212, fingerprint.rs,
// meter.rs:183-232):
//
//   myos [--weights PATH] [--block-fixture] [--steps N] [--threads N]
//        [--fingerprint-dir DIR] [--prompt-ids PATH] [--ref-ids PATH]
//        [--arena-s1] [--warmup N] [--repeats N] [--cost-card PATH]
//
// Exit codes: 2 usage, 1 load/decode failure, 0 success (also when the
// reference-id comparison prints CORRECT: FAIL). All model arithmetic runs
// in libmyos_cuda on the GPU; --threads is accepted and recorded (it sizes
// the reference's CPU pool) but does not change the device work.
#include <errno.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "myos_cuda.h"

namespace {

constexpr int kSmokeVocab = 4;
constexpr size_t kSmokeSteps = 4;
constexpr uint32_t kSmokePrompt = 0;
constexpr size_t kShowdownThreads = 8;
constexpr size_t kThreadsMax = 64;
const char* kUsage =
    "myos [--weights PATH] [--block-fixture] [--steps N] [--threads N] [--fingerprint-dir DIR] "
    "[--prompt-ids PATH] [--ref-ids PATH] [--arena-s1] [--warmup N] [--repeats N] "
    "[--cost-card PATH]";

struct Cli {
  std::string weights;
  bool has_weights = false;
  bool block_fixture = false;
  size_t steps = kSmokeSteps;
  size_t threads = kShowdownThreads;
  std::string fingerprint_dir, prompt_ids, ref_ids, cost_card;
  bool has_fp = false, has_prompt = false, has_ref = false, has_card = false;
  bool arena_s1 = false;
  size_t warmup = 3, repeats = 5;
};

struct UsageError {
  std::string msg;
};

const char* flag_noun(const std::string& name) {
  if (name == "--steps" || name == "--threads" || name == "--repeats") return "a positive integer";
  if (name == "--warmup") return "a non-negative integer";
  return "a path";
}

// `--name VALUE` or `--name=VALUE`; false when `arg` is another token.
bool match_flag(const std::string& arg, const std::string& name, int* i, int argc, char** argv,
                std::string* out) {
  const std::string prefix = name + "=";
  if (arg.compare(0, prefix.size(), prefix) == 0) {
    *out = arg.substr(prefix.size());
    if (out->empty()) throw UsageError{name + " needs " + flag_noun(name)};
    return true;
  }
  if (arg == name) {
    if (*i + 1 >= argc) throw UsageError{name + " needs " + flag_noun(name)};
    *out = argv[++*i];
    if (out->empty()) throw UsageError{name + " needs " + flag_noun(name)};
    return true;
  }
  return false;
}

bool parse_uint(const std::string& s, size_t* out) {
  if (s.empty() || s.size() > 19) return false;
  size_t v = 0;
  for (char c : s) {
    if (c < '0' || c > '9') return false;
    v = v * 10 + (size_t)(c - '0');
  }
  *out = v;
  return true;
}

Cli parse_cli(int argc, char** argv) {
  Cli c;
  bool steps_set = false, threads_set = false, warmup_set = false, repeats_set = false;
  for (int i = 1; i < argc; ++i) {
    const std::string arg = argv[i];
    std::string v;
    if (arg == "--block-fixture") {
      if (c.block_fixture) throw UsageError{"--block-fixture was given more than once"};
      c.block_fixture = true;
    } else if (match_flag(arg, "--weights", &i, argc, argv, &v)) {
      if (c.has_weights) throw UsageError{"--weights was given more than once"};
      c.weights = v;
      c.has_weights = true;
    } else if (match_flag(arg, "--steps", &i, argc, argv, &v)) {
      if (steps_set) throw UsageError{"--steps was given more than once"};
      size_t n;
      if (!parse_uint(v, &n) || n == 0) throw UsageError{"--steps needs a positive integer, got `" + v + "`"};
      c.steps = n;
      steps_set = true;
    } else if (match_flag(arg, "--threads", &i, argc, argv, &v)) {
      if (threads_set) throw UsageError{"--threads was given more than once"};
      size_t n;
      if (!parse_uint(v, &n) || n < 1 || n > kThreadsMax)
        throw UsageError{"--threads needs an integer from 1 to " + std::to_string(kThreadsMax) +
                         ", got `" + v + "`"};
      c.threads = n;
      threads_set = true;
    } else if (arg == "--arena-s1") {
      if (c.arena_s1) throw UsageError{"--arena-s1 was given more than once"};
      c.arena_s1 = true;
    } else if (match_flag(arg, "--warmup", &i, argc, argv, &v)) {
      if (warmup_set) throw UsageError{"--warmup was given more than once"};
      size_t n;
      if (!parse_uint(v, &n) || n > 100)
        throw UsageError{"--warmup needs an integer from 0 to 100, got `" + v + "`"};
      c.warmup = n;
      warmup_set = true;
    } else if (match_flag(arg, "--repeats", &i, argc, argv, &v)) {
      if (repeats_set) throw UsageError{"--repeats was given more than once"};
      size_t n;
      if (!parse_uint(v, &n) || n < 1 || n > 100)
        throw UsageError{"--repeats needs an integer from 1 to 100, got `" + v + "`"};
      c.repeats = n;
      repeats_set = true;
    } else if (match_flag(arg, "--cost-card", &i, argc, argv, &v)) {
      if (c.has_card) throw UsageError{"--cost-card was given more than once"};
      c.cost_card = v;
      c.has_card = true;
    } else if (match_flag(arg, "--fingerprint-dir", &i, argc, argv, &v)) {
      if (c.has_fp) throw UsageError{"--fingerprint-dir was given more than once"};
      c.fingerprint_dir = v;
      c.has_fp = true;
    } else if (match_flag(arg, "--prompt-ids", &i, argc, argv, &v)) {
      if (c.has_prompt) throw UsageError{"--prompt-ids was given more than once"};
      c.prompt_ids = v;
      c.has_prompt = true;
    } else if (match_flag(arg, "--ref-ids", &i, argc, argv, &v)) {
      if (c.has_ref) throw UsageError{"--ref-ids was given more than once"};
      c.ref_ids = v;
      c.has_ref = true;
    } else {
      throw UsageError{"unknown argument `" + arg + "`"};
    }
  }
  if (c.has_fp && !c.has_weights && !c.block_fixture)
    throw UsageError{"--fingerprint-dir needs --weights or --block-fixture"};
  if (c.has_prompt && !c.has_weights) throw UsageError{"--prompt-ids needs --weights"};
  if (c.has_prompt && c.block_fixture)
    throw UsageError{"--prompt-ids cannot be combined with --block-fixture"};
  if (c.arena_s1 && c.block_fixture)
    throw UsageError{"--arena-s1 cannot be combined with --block-fixture"};
  if (c.arena_s1 && !c.has_weights) throw UsageError{"--arena-s1 needs --weights"};
  if (c.arena_s1 && !c.has_prompt) throw UsageError{"--arena-s1 needs --prompt-ids"};
  if (c.arena_s1 && !c.has_ref) throw UsageError{"--arena-s1 needs --ref-ids"};
  if (!c.arena_s1 && (warmup_set || repeats_set || c.has_card))
    throw UsageError{"--warmup, --repeats, and --cost-card need --arena-s1"};
  if (c.arena_s1 && !steps_set) c.steps = 128;
  return c;
}

// ------------------------------------------------------------------ ids
bool read_token_ids(const std::string& path, std::vector<uint32_t>* ids, std::string* err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    *err = path + ": " + strerror(errno);
    return false;
  }
  std::stringstream ss;
  ss << f.rdbuf();
  std::string tok;
  ids->clear();
  while (ss >> tok) {
    size_t v;
    if (!parse_uint(tok, &v) || v > 0xffffffffull) {
      *err = path + ": `" + tok + "` is not a u32";
      return false;
    }
    ids->push_back((uint32_t)v);
  }
  if (ids->empty()) {
    *err = path + ": file is empty";
    return false;
  }
  return true;
}

std::string debug_ids(const std::vector<uint32_t>& ids) {
  std::string s = "[";
  for (size_t i = 0; i < ids.size(); ++i) s += (i ? ", " : "") + std::to_string(ids[i]);
  return s + "]";
}

std::string correct_line(const std::vector<uint32_t>& got, const std::vector<uint32_t>& ref) {
  if (got.size() != ref.size())
    return "CORRECT: FAIL length mismatch got=" + std::to_string(got.size()) +
           " ref=" + std::to_string(ref.size());
  for (size_t i = 0; i < got.size(); ++i)
    if (got[i] != ref[i])
      return "CORRECT: FAIL first_diff@" + std::to_string(i) + ": got=" + std::to_string(got[i]) +
             " ref=" + std::to_string(ref[i]);
  return "CORRECT: PASS";
}

// ------------------------------------------------------------------ files
bool mkdirs(const std::string& dir) {
  std::string cur;
  std::stringstream ss(dir);
  std::string part;
  if (!dir.empty() && dir[0] == '/') cur = "/";
  while (std::getline(ss, part, '/')) {
    if (part.empty()) continue;
    cur += part + "/";
    if (mkdir(cur.c_str(), 0777) != 0 && errno != EEXIST) return false;
  }
  return true;
}

bool write_file(const std::string& path, const std::string& text) {
  std::ofstream f(path, std::ios::binary);
  if (!f) return false;
  f << text;
  return (bool)f;
}

std::string json_str(const std::string& s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    if (c == '"' || c == '\\') {
      o += '\\';
      o += (char)c;
    } else if (c < 0x20) {
      char b[8];
      snprintf(b, sizeof b, "\\u%04x", c);
      o += b;
    } else {
      o += (char)c;
    }
  }
  return o + "\"";
}

std::string json_f64(double v) {
  char b[64];
  snprintf(b, sizeof b, "%.9g", v);
  return b;
}

// HEAD of the repository holding `start`, if any (fingerprint.rs:237-260).
std::string git_commit() {
  char buf[4096];
  if (!getcwd(buf, sizeof buf)) return "";
  std::string dir = buf;
  while (true) {
    struct stat st;
    const std::string git = dir + "/.git";
    if (stat(git.c_str(), &st) == 0 && S_ISDIR(st.st_mode)) {
      std::ifstream h(git + "/HEAD");
      std::string head;
      std::getline(h, head);
      if (head.compare(0, 5, "ref: ") != 0) return head;
      std::ifstream r(git + "/" + head.substr(5));
      std::string sha;
      if (std::getline(r, sha)) return sha;
      std::ifstream packed(git + "/packed-refs");
      std::string line;
      while (std::getline(packed, line))
        if (line.size() > 41 && line.substr(41) == head.substr(5)) return line.substr(0, 40);
      return "";
    }
    const size_t slash = dir.rfind('/');
    if (slash == std::string::npos || dir == "/") return "";
    dir = slash == 0 ? "/" : dir.substr(0, slash);
  }
}

long proc_status_kib(const char* key) {
  std::ifstream f("/proc/self/status");
  std::string line;
  const size_t n = strlen(key);
  while (std::getline(f, line))
    if (line.compare(0, n, key) == 0) return atol(line.c_str() + n + 1);
  return -1;
}

std::string g_cmdline;

enum class RunKind { Weights, BlockFixture };

struct FpSpec {
  RunKind kind;
  myos_shape shape;
  bool pinned;  // the 1.5B shape
  uint32_t prompt_token;
  size_t n_prompt, steps, threads;
  bool prompt_ids;
  std::string run_id;
  int device;
};

// run_fingerprint.json with the reference's fields (fingerprint.rs:146-209),
// device/gpus naming the GPU run.
std::string fingerprint_json(const FpSpec& s) {
  const bool w = s.kind == RunKind::Weights;
  const std::string commit = git_commit();
  std::vector<std::pair<std::string, std::string>> f = {
      {"model_id", w && s.pinned ? json_str("Qwen/Qwen2.5-1.5B-Instruct") : "null"},
      {"model_sha256", "null"},
      {"fmt", json_str(w ? "safetensors" : "in-process")},
      {"quant_or_dtype", json_str("bf16")},
      {"acc_path", json_str("bf16_w_fp32_acc")},
      {"n_ctx", std::to_string(s.n_prompt + s.steps)},
      {"n_prompt", std::to_string(s.n_prompt)},
      {"n_gen", std::to_string(s.steps)},
      {"batch", "1"},
      {"threads", std::to_string(s.threads)},
      {"gemv_pack", "false"},
      {"device", json_str("cuda:" + std::to_string(s.device))},
      {"deterministic", "true"},
      {"seed", "null"},
      {"commit", commit.empty() ? "null" : json_str(commit)},
      {"cmdline", json_str(g_cmdline)},
      {"scenario_id", json_str("S1")},
      {"run_id", json_str(s.run_id)},
      {"layout", json_str(w ? (s.pinned ? "qwen25_1_5b" : "not-qwen25-1.5b") : "block-fixture")},
      {"num_layers", std::to_string(s.shape.num_layers)},
      {"hidden_size", std::to_string(s.shape.hidden)},
      {"intermediate_size", std::to_string(s.shape.intermediate)},
      {"vocab_size", std::to_string(s.shape.vocab)},
      {"prompt_token", std::to_string(s.prompt_token)},
      {"gpus", "1"},
      {"notes", json_str(std::string("model_sha256 is null: this process does not hash the file. ") +
                         (s.prompt_ids ? "n_prompt is the --prompt-ids length; n_gen is --steps. "
                                       : "n_prompt is 1 (the smoke prompt id). ") +
                         "Arithmetic runs on the GPU (libmyos_cuda, sm_100a); threads is recorded "
                         "as given.")},
  };
  std::string o = "{\n";
  for (size_t i = 0; i < f.size(); ++i)
    o += "  \"" + f[i].first + "\": " + f[i].second + (i + 1 < f.size() ? ",\n" : "\n");
  return o + "}\n";
}

struct Sample {
  double t_load_s = 0, t_prefill_s = 0, t_decode_s = 0;
  size_t n_prompt = 0, n_gen = 0;
  long m_peak_kib = -1, m_rss_after_load_kib = -1;
  int correct = -1;  // -1 unknown, 0 fail, 1 pass
};

// metrics.json (meter.rs:183-232): the sample and its derived figures.
std::string metrics_json(const Sample& s, size_t threads) {
  auto opt = [](bool ok, double v) { return ok ? json_f64(v) : std::string("null"); };
  const double ttft_ms = s.t_prefill_s * 1000.0;
  const bool dec = s.t_decode_s > 0 && s.n_gen > 0;
  const double wall = s.t_prefill_s + s.t_decode_s;
  std::vector<std::pair<std::string, std::string>> f = {
      {"scenario_id", json_str("S1")},
      {"threads", std::to_string(threads)},
      {"batch", "1"},
      {"quant_or_dtype", json_str("bf16")},
      {"acc_path", json_str("bf16_w_fp32_acc")},
      {"gemv_pack", "false"},
      {"n_prompt", std::to_string(s.n_prompt)},
      {"n_gen", std::to_string(s.n_gen)},
      {"t_load_s", json_f64(s.t_load_s)},
      {"t_prefill_s", json_f64(s.t_prefill_s)},
      {"t_decode_s", json_f64(s.t_decode_s)},
      {"T_decode_tok_s", opt(dec, dec ? (double)s.n_gen / s.t_decode_s : 0)},
      {"L_TTFT_ms", json_f64(ttft_ms)},
      {"L_prefill_ms", json_f64(ttft_ms)},
      {"L_TPOT_ms", opt(s.n_gen > 0, s.n_gen ? s.t_decode_s * 1000.0 / (double)s.n_gen : 0)},
      {"T_e2e_tok_s", opt(wall > 0, wall > 0 ? (double)(s.n_prompt + s.n_gen) / wall : 0)},
      {"M_peak_KiB", s.m_peak_kib >= 0 ? std::to_string(s.m_peak_kib) : "null"},
      {"M_peak_MiB", opt(s.m_peak_kib >= 0, s.m_peak_kib / 1024.0)},
      {"M_rss_after_load_KiB",
       s.m_rss_after_load_kib >= 0 ? std::to_string(s.m_rss_after_load_kib) : "null"},
      {"M_rss_after_load_MiB", opt(s.m_rss_after_load_kib >= 0, s.m_rss_after_load_kib / 1024.0)},
      {"correct", s.correct < 0 ? "null" : (s.correct ? "true" : "false")},
      {"timing",
       json_str("t_load is SafeTensors open, parse and upload to HBM; it is outside L_prefill and "
                "T_decode. t_prefill is context creation (HBM KV cache and workspace) plus the "
                "prompt forwards, ending before the first new token. t_decode is greedy_decode of "
                "n_gen new tokens. M_peak is the host VmHWM at the end of decode.")},
  };
  std::string o = "{\n";
  for (size_t i = 0; i < f.size(); ++i)
    o += "  \"" + f[i].first + "\": " + f[i].second + (i + 1 < f.size() ? ",\n" : "\n");
  return o + "}\n";
}

int device_ordinal() {
  const char* e = getenv("MYOS_DEVICE");
  return e ? atoi(e) : 0;
}

// ------------------------------------------------------------------ decodes
struct Decoded {
  std::vector<uint32_t> ids;
  double t_load = 0, t_prefill = 0, t_decode = 0;
  long rss_after_load = -1;
};

using Clock = std::chrono::steady_clock;
double secs(Clock::time_point a, Clock::time_point b) {
  return std::chrono::duration<double>(b - a).count();
}

// Context for `shape`, prompt prefill, `steps` greedy tokens
// (main.rs:520-555). `load` fills the weights.
template <class Load>
bool run_decode(const myos_shape& shape, const std::vector<uint32_t>& prompt, size_t steps,
                Load load, Decoded* out, std::string* err) {
  myos_opts o = {};
  o.device = device_ordinal();
  o.max_seq = (uint32_t)(prompt.size() + steps);
  o.kv_dtype = MYOS_KV_F32;
  o.use_graphs = 1;
  myos_ctx* ctx = nullptr;
  const auto t0 = Clock::now();
  int st = myos_ctx_create(&shape, &o, &ctx);
  if (st) {
    *err = std::string("context: ") + (ctx ? myos_last_error(ctx) : "creation failed") +
           " (status " + std::to_string(st) + ")";
    if (ctx) myos_ctx_destroy(ctx);
    return false;
  }
  if ((st = load(ctx))) {
    *err = myos_last_error(ctx);
    myos_ctx_destroy(ctx);
    return false;
  }
  if (myos_weights_ready(ctx) != 1) {  // 1: every tensor of the layout is loaded
    *err = myos_last_error(ctx);
    myos_ctx_destroy(ctx);
    return false;
  }
  const auto t1 = Clock::now();
  out->rss_after_load = proc_status_kib("VmRSS:");
  if ((st = myos_prefill(ctx, prompt.data(), prompt.size(), nullptr))) {
    *err = myos_last_error(ctx);
    myos_ctx_destroy(ctx);
    return false;
  }
  const auto t2 = Clock::now();
  out->ids.assign(steps, 0);
  if ((st = myos_greedy_decode(ctx, steps, out->ids.data()))) {
    *err = myos_last_error(ctx);
    myos_ctx_destroy(ctx);
    return false;
  }
  const auto t3 = Clock::now();
  myos_ctx_destroy(ctx);
  out->t_load = secs(t0, t1);
  out->t_prefill = secs(t1, t2);
  out->t_decode = secs(t2, t3);
  return true;
}

// Little-endian bf16 bytes of exactly-representable values.
std::vector<uint8_t> bf16_bytes(const std::vector<float>& v) {
  std::vector<uint8_t> b(v.size() * 2);
  for (size_t i = 0; i < v.size(); ++i) {
    uint32_t u;
    memcpy(&u, &v[i], 4);
    b[2 * i] = (uint8_t)(u >> 16);
    b[2 * i + 1] = (uint8_t)(u >> 24);
  }
  return b;
}

// The reference's miniature block (crates/model_core/src/qwen25_block.rs:788-938):
// hidden 2, 2 query heads over 1 KV head, head_dim 2, vocab 4, eps 0.
myos_shape fixture_shape() {
  myos_shape s = {};
  s.hidden = 2;
  s.num_q_heads = 2;
  s.num_kv_heads = 1;
  s.head_dim = 2;
  s.rope_theta = 1e6f;
  s.intermediate = 2;
  s.vocab = 4;
  s.num_layers = 1;
  s.rms_eps = 0.0f;
  s.tied_head = 1;
  return s;
}

int load_block_fixture(myos_ctx* ctx) {
  struct T {
    const char* name;
    std::vector<int64_t> shape;
    std::vector<float> v;
  };
  const std::vector<T> ts = {
      {"model.embed_tokens.weight", {4, 2}, {1, 1, 2, 0, 0, 4, -1, 0}},
      {"model.norm.weight", {2}, {1, 0}},
      {"model.layers.0.input_layernorm.weight", {2}, {1, 1}},
      {"model.layers.0.self_attn.q_proj.weight", {4, 2}, std::vector<float>(8, 0.f)},
      {"model.layers.0.self_attn.q_proj.bias", {4}, {0.5f, 0, 0, 0.25f}},
      {"model.layers.0.self_attn.k_proj.weight", {2, 2}, std::vector<float>(4, 0.f)},
      {"model.layers.0.self_attn.k_proj.bias", {2}, {0, 0}},
      {"model.layers.0.self_attn.v_proj.weight", {2, 2}, std::vector<float>(4, 0.f)},
      {"model.layers.0.self_attn.v_proj.bias", {2}, {1, 0}},
      {"model.layers.0.self_attn.o_proj.weight", {2, 4}, {1, 0, 0, 0, 1, 0, 0, 0}},
      {"model.layers.0.post_attention_layernorm.weight", {2}, {1, 1}},
      {"model.layers.0.mlp.gate_proj.weight", {2, 2}, std::vector<float>(4, 0.f)},
      {"model.layers.0.mlp.up_proj.weight", {2, 2}, std::vector<float>(4, 0.f)},
      {"model.layers.0.mlp.down_proj.weight", {2, 2}, std::vector<float>(4, 0.f)},
  };
  for (const T& t : ts) {
    const std::vector<uint8_t> b = bf16_bytes(t.v);
    const int st = myos_load_tensor(ctx, t.name, MYOS_BF16, t.shape.data(), (int32_t)t.shape.size(),
                                    b.data(), b.size());
    if (st) return st;
  }
  return MYOS_OK;
}

// The reference's cycle smoke (crates/model_core/src/lib.rs:79-97, main.rs:818-830):
// one-hot embedding, head mapping token t to t+1 mod vocab, greedy.
bool smoke_decode(uint32_t prompt, size_t steps, std::vector<uint32_t>* out, std::string* err) {
  const int V = kSmokeVocab;
  std::vector<float> embed(V * V, 0.f), head(V * V, 0.f);
  for (int t = 0; t < V; ++t) {
    embed[t * V + t] = 1.f;
    head[((t + 1) % V) * V + t] = 1.f;
  }
  const std::vector<uint8_t> hb = bf16_bytes(head);  // 0 and 1 are exact in bf16
  uint32_t tok = prompt;
  out->clear();
  std::vector<float> logits(V);
  for (size_t pos = 0; pos < steps; ++pos) {
    int st = myos_gemv_bf16(logits.data(), V, hb.data(), hb.size(), &embed[tok * V], V, V, V);
    if (!st) st = myos_greedy_token(logits.data(), V, &tok);
    if (st) {
      *err = "device step failed (status " + std::to_string(st) + ")";
      return false;
    }
    out->push_back(tok);
  }
  return true;
}

bool write_fingerprint(const FpSpec& spec, const std::string& dir,
                       const std::vector<uint32_t>* generated, std::string* err) {
  if (!mkdirs(dir) || !write_file(dir + "/run_fingerprint.json", fingerprint_json(spec))) {
    *err = dir + ": " + strerror(errno);
    return false;
  }
  if (generated) {
    std::string t;
    for (size_t i = 0; i < generated->size(); ++i)
      t += (i ? " " : "") + std::to_string((*generated)[i]);
    if (!write_file(dir + "/token_ids.txt", t + "\n")) {
      *err = dir + ": " + strerror(errno);
      return false;
    }
  }
  return true;
}

std::string showdown_id(size_t threads) {
  return "s1-myos-bf16-t" + std::to_string(threads) + "-k9";
}

// ------------------------------------------------------------------ arena
double median(std::vector<double> v) {
  std::sort(v.begin(), v.end());
  const size_t n = v.size();
  return n % 2 ? v[n / 2] : 0.5 * (v[n / 2 - 1] + v[n / 2]);
}

bool json_number(const std::string& text, const std::string& key, double* out) {
  const std::string k = "\"" + key + "\": ";
  const size_t p = text.find(k);
  if (p == std::string::npos) return false;
  const char* s = text.c_str() + p + k.size();
  if (!strncmp(s, "null", 4)) return false;
  *out = strtod(s, nullptr);
  return true;
}

// W warm-up and R scored children of this binary (crates/runtime/src/arena.rs:41-75),
// each writing warm-i/ or score-i/; medians over the scored runs.
int run_arena(const Cli& c, const char* self) {
  const std::string out_dir = c.has_fp ? c.fingerprint_dir : "runs/" + showdown_id(c.threads);
  const std::string card = c.has_card ? c.cost_card : "arena/" + showdown_id(c.threads) + "-cost-card.md";
  if (!mkdirs(out_dir)) {
    fprintf(stderr, "MyOS arena: %s: %s\n", out_dir.c_str(), strerror(errno));
    return 1;
  }
  std::vector<uint32_t> ref;
  std::string err;
  if (!read_token_ids(c.ref_ids, &ref, &err)) {
    fprintf(stderr, "MyOS arena: %s\n", err.c_str());
    return 1;
  }
  std::vector<double> tdec, ttft, tpot;
  std::vector<std::vector<uint32_t>> ids;
  bool correct = true;
  const size_t total = c.warmup + c.repeats;
  for (size_t i = 0; i < total; ++i) {
    const bool warm = i < c.warmup;
    const std::string dir =
        out_dir + "/" + (warm ? "warm-" + std::to_string(i + 1) : "score-" + std::to_string(i + 1 - c.warmup));
    fprintf(stderr, "=== %s %zu/%zu ===\n", warm ? "WARM" : "SCORE", warm ? i + 1 : i + 1 - c.warmup,
            warm ? c.warmup : c.repeats);
    const pid_t pid = fork();
    if (pid == 0) {  // the child's stdout goes to its run directory
      const std::string log = dir + "/stdout.txt";
      FILE* f = mkdirs(dir) ? fopen(log.c_str(), "w") : nullptr;
      if (!f || dup2(fileno(f), 1) < 0) _exit(126);
      const std::string steps = std::to_string(c.steps), threads = std::to_string(c.threads);
      execl(self, self, "--weights", c.weights.c_str(), "--prompt-ids", c.prompt_ids.c_str(),
            "--ref-ids", c.ref_ids.c_str(), "--steps", steps.c_str(), "--threads", threads.c_str(),
            "--fingerprint-dir", dir.c_str(), (char*)nullptr);
      _exit(127);
    }
    int status = 0;
    if (pid < 0 || waitpid(pid, &status, 0) < 0 || !WIFEXITED(status) || WEXITSTATUS(status) != 0) {
      fprintf(stderr, "MyOS arena: child run in %s failed\n", dir.c_str());
      return 1;
    }
    if (warm) continue;
    std::ifstream m(dir + "/metrics.json");
    std::stringstream ss;
    ss << m.rdbuf();
    double d, t, p;
    if (!json_number(ss.str(), "T_decode_tok_s", &d) || !json_number(ss.str(), "L_TTFT_ms", &t) ||
        !json_number(ss.str(), "L_TPOT_ms", &p)) {
      fprintf(stderr, "MyOS arena: %s/metrics.json: missing fields\n", dir.c_str());
      return 1;
    }
    tdec.push_back(d);
    ttft.push_back(t);
    tpot.push_back(p);
    std::vector<uint32_t> got;
    if (!read_token_ids(dir + "/token_ids.txt", &got, &err)) {
      fprintf(stderr, "MyOS arena: %s\n", err.c_str());
      return 1;
    }
    correct = correct && got == ref;
    ids.push_back(got);
  }
  bool det = true;
  for (const auto& v : ids) det = det && v == ids[0];
  const double md = median(tdec), mt = median(ttft), mp = median(tpot);
  const size_t slash = card.rfind('/');
  if (slash != std::string::npos) mkdirs(card.substr(0, slash));
  char body[2048];
  snprintf(body, sizeof body,
           "# S1 cost card: myos bf16 on %s\n\n"
           "| field | value |\n|---|---|\n"
           "| warmup / repeats | %zu / %zu |\n| CORRECT | %s |\n| DET | %s |\n"
           "| T_decode (tok/s, median) | %.4f |\n| L_TTFT (ms, median) | %.3f |\n"
           "| L_TPOT (ms, median) | %.3f |\n| run dir | %s |\n",
           ("cuda:" + std::to_string(device_ordinal())).c_str(), c.warmup, c.repeats,
           correct ? "PASS" : "FAIL", det ? "PASS" : "FAIL", md, mt, mp, out_dir.c_str());
  write_file(card, body);
  printf("ARENA S1 threads=%zu W=%zu R=%zu CORRECT=%s DET=%s device=cuda T_decode=%.4f "
         "L_TTFT_ms=%.3f L_TPOT_ms=%.3f\n",
         c.threads, c.warmup, c.repeats, correct ? "PASS" : "FAIL", det ? "PASS" : "FAIL", md, mt,
         mp);
  printf("cost-card: %s\n", card.c_str());
  printf("run-dir: %s\n", out_dir.c_str());
  return correct && det ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  for (int i = 0; i < argc; ++i) g_cmdline += (i ? " " : "") + std::string(argv[i]);
  Cli cli;
  try {
    cli = parse_cli(argc, argv);
  } catch (const UsageError& e) {
    fprintf(stderr, "MyOS: %s\nusage: %s\n", e.msg.c_str(), kUsage);
    return 2;
  }
  if (cli.arena_s1) return run_arena(cli, "/proc/self/exe");

  std::vector<uint32_t> ref;
  std::string err;
  if (cli.has_ref && !read_token_ids(cli.ref_ids, &ref, &err)) {
    fprintf(stderr, "MyOS ref-ids: %s\n", err.c_str());
    return 1;
  }
  // CLI path wins; otherwise a non-empty MYOS_WEIGHTS (main.rs:416-422).
  std::string weights = cli.weights;
  bool has_weights = cli.has_weights;
  if (!has_weights) {
    const char* e = getenv("MYOS_WEIGHTS");
    if (e && *e) {
      weights = e;
      has_weights = true;
    }
  }

  if (cli.block_fixture) {
    if (has_weights) {
      size_t n = 0;
      char msg[512] = {0};
      if (myos_check_safetensors(weights.c_str(), &n, msg, sizeof msg)) {
        fprintf(stderr, "MyOS weights %s: %s\n", weights.c_str(), msg);
        return 1;
      }
    }
    Decoded d;
    const myos_shape shape = fixture_shape();
    if (!run_decode(shape, {kSmokePrompt}, cli.steps, load_block_fixture, &d, &err)) {
      fprintf(stderr, "MyOS Phase1 block fixture failed: %s\n", err.c_str());
      return 1;
    }
    FpSpec fp = {RunKind::BlockFixture, shape, false, kSmokePrompt, 1, cli.steps, cli.threads,
                 false, "s1-block-fixture", device_ordinal()};
    if (!write_fingerprint(fp, cli.has_fp ? cli.fingerprint_dir : "runs/s1-block-fixture", nullptr,
                           &err)) {
      fprintf(stderr, "MyOS fingerprint: %s\n", err.c_str());
      return 1;
    }
    printf("MyOS Phase1 block fixture (prompt=%u): %s\n", kSmokePrompt, debug_ids(d.ids).c_str());
    if (cli.has_ref) printf("%s\n", correct_line(d.ids, ref).c_str());
    return 0;
  }

  if (has_weights) {
    std::vector<uint32_t> prompt = {kSmokePrompt};
    if (cli.has_prompt && !read_token_ids(cli.prompt_ids, &prompt, &err)) {
      fprintf(stderr, "MyOS prompt-ids: %s\n", err.c_str());
      return 1;
    }
    const myos_shape shape = myos_shape_qwen25_1_5b();
    Decoded d;
    auto load = [&](myos_ctx* ctx) { return myos_load_safetensors(ctx, weights.c_str()); };
    if (!run_decode(shape, prompt, cli.steps, load, &d, &err)) {
      fprintf(stderr, "MyOS weights %s: %s\n", weights.c_str(), err.c_str());
      return 1;
    }
    const std::string dir = cli.has_fp ? cli.fingerprint_dir : "runs/s1-weights";
    FpSpec fp = {RunKind::Weights, shape, true, prompt[0], prompt.size(), cli.steps, cli.threads,
                 cli.has_prompt, "s1-weights", device_ordinal()};
    if (!write_fingerprint(fp, dir, cli.has_prompt ? &d.ids : nullptr, &err)) {
      fprintf(stderr, "MyOS fingerprint: %s\n", err.c_str());
      return 1;
    }
    Sample s;
    s.t_load_s = d.t_load;
    s.t_prefill_s = d.t_prefill;
    s.t_decode_s = d.t_decode;
    s.n_prompt = prompt.size();
    s.n_gen = cli.steps;
    s.m_peak_kib = proc_status_kib("VmHWM:");
    s.m_rss_after_load_kib = d.rss_after_load;
    if (cli.has_ref) s.correct = correct_line(d.ids, ref) == "CORRECT: PASS";
    if (!write_file(dir + "/metrics.json", metrics_json(s, cli.threads))) {
      fprintf(stderr, "MyOS metrics: %s: %s\n", dir.c_str(), strerror(errno));
      return 1;
    }
    printf("MyOS Phase1 weights decode (prompt=%u, steps=%zu): %s\n", prompt[0], cli.steps,
           debug_ids(d.ids).c_str());
    if (cli.has_ref) printf("%s\n", correct_line(d.ids, ref).c_str());
    return 0;
  }

  std::vector<uint32_t> ids;
  if (!smoke_decode(kSmokePrompt, cli.steps, &ids, &err)) {
    fprintf(stderr, "MyOS Phase1 smoke failed: %s\n", err.c_str());
    return 1;
  }
  printf("MyOS Phase1 smoke decode (prompt=%u): %s\n", kSmokePrompt, debug_ids(ids).c_str());
  if (cli.has_ref) printf("%s\n", correct_line(ids, ref).c_str());
  return 0;
}
