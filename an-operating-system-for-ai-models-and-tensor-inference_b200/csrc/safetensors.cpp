// SafeTensors header parser. The format is fixed by the safetensors project:
//   [u64 little-endian N][N bytes of JSON][data]
// with one JSON entry per tensor {"dtype", "shape", "data_offsets"} plus an
// optional "__metadata__" map of strings. Checks follow the crate the
// reference uses (crates/weight_loader/src/safe_tensors.rs:30-43 calls
// SafeTensors::deserialize): size limits, JSON shape, offsets that tile the
// data section with no gap or overlap, and per-tensor byte lengths.
#include "safetensors.h"

#include <string.h>

#include <algorithm>
#include <map>

namespace myos {

namespace {

constexpr uint64_t kMaxHeader = 100000000;  // the crate's MAX_HEADER_SIZE

struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  std::string str;
  double num = 0;
  bool is_int = false;
  uint64_t uval = 0;
  bool neg = false;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), e_(p + n) {}
  bool parse(Json* out) {
    ws();
    if (!value(out, 0)) return false;
    ws();
    return p_ == e_;
  }

 private:
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if ((size_t)(e_ - p_) < n || memcmp(p_, s, n) != 0) return false;
    p_ += n;
    return true;
  }
  bool value(Json* v, int depth) {
    if (depth > 64 || p_ >= e_) return false;
    char c = *p_;
    if (c == '{') return object(v, depth);
    if (c == '[') return array(v, depth);
    if (c == '"') {
      v->kind = Json::STR;
      return string(&v->str);
    }
    if (c == 't') {
      v->kind = Json::BOOL;
      return lit("true");
    }
    if (c == 'f') {
      v->kind = Json::BOOL;
      return lit("false");
    }
    if (c == 'n') {
      v->kind = Json::NUL;
      return lit("null");
    }
    return number(v);
  }
  bool number(Json* v) {
    const char* s = p_;
    if (p_ < e_ && *p_ == '-') ++p_;
    if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return false;
    bool integral = true;
    uint64_t u = 0;
    bool overflow = false;
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
      uint64_t d = (uint64_t)(*p_ - '0');
      if (u > (UINT64_MAX - d) / 10) overflow = true;
      u = u * 10 + d;
      ++p_;
    }
    if (p_ < e_ && *p_ == '.') {
      integral = false;
      ++p_;
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    v->kind = Json::NUM;
    v->neg = *s == '-';
    v->is_int = integral && !overflow;
    v->uval = u;
    v->num = strtod(std::string(s, p_).c_str(), nullptr);
    return true;
  }
  bool string(std::string* out) {
    ++p_;  // opening quote
    while (p_ < e_) {
      char c = *p_++;
      if (c == '"') return true;
      if ((unsigned char)c < 0x20) return false;
      if (c == '\\') {
        if (p_ >= e_) return false;
        char esc = *p_++;
        switch (esc) {
          case '"': out->push_back('"'); break;
          case '\\': out->push_back('\\'); break;
          case '/': out->push_back('/'); break;
          case 'b': out->push_back('\b'); break;
          case 'f': out->push_back('\f'); break;
          case 'n': out->push_back('\n'); break;
          case 'r': out->push_back('\r'); break;
          case 't': out->push_back('\t'); break;
          case 'u': {
            if (e_ - p_ < 4) return false;
            unsigned cp = 0;
            for (int i = 0; i < 4; ++i) {
              char h = *p_++;
              cp <<= 4;
              if (h >= '0' && h <= '9') cp |= (unsigned)(h - '0');
              else if (h >= 'a' && h <= 'f') cp |= (unsigned)(h - 'a' + 10);
              else if (h >= 'A' && h <= 'F') cp |= (unsigned)(h - 'A' + 10);
              else return false;
            }
            if (cp < 0x80) {
              out->push_back((char)cp);
            } else if (cp < 0x800) {
              out->push_back((char)(0xC0 | (cp >> 6)));
              out->push_back((char)(0x80 | (cp & 0x3F)));
            } else {
              out->push_back((char)(0xE0 | (cp >> 12)));
              out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
              out->push_back((char)(0x80 | (cp & 0x3F)));
            }
            break;
          }
          default: return false;
        }
      } else {
        out->push_back(c);
      }
    }
    return false;
  }
  bool array(Json* v, int depth) {
    v->kind = Json::ARR;
    ++p_;
    ws();
    if (p_ < e_ && *p_ == ']') {
      ++p_;
      return true;
    }
    for (;;) {
      Json item;
      ws();
      if (!value(&item, depth + 1)) return false;
      v->arr.push_back(std::move(item));
      ws();
      if (p_ >= e_) return false;
      if (*p_ == ',') {
        ++p_;
        continue;
      }
      if (*p_ == ']') {
        ++p_;
        return true;
      }
      return false;
    }
  }
  bool object(Json* v, int depth) {
    v->kind = Json::OBJ;
    ++p_;
    ws();
    if (p_ < e_ && *p_ == '}') {
      ++p_;
      return true;
    }
    for (;;) {
      ws();
      if (p_ >= e_ || *p_ != '"') return false;
      std::string key;
      if (!string(&key)) return false;
      ws();
      if (p_ >= e_ || *p_ != ':') return false;
      ++p_;
      ws();
      Json item;
      if (!value(&item, depth + 1)) return false;
      v->obj.emplace_back(std::move(key), std::move(item));
      ws();
      if (p_ >= e_) return false;
      if (*p_ == ',') {
        ++p_;
        continue;
      }
      if (*p_ == '}') {
        ++p_;
        return true;
      }
      return false;
    }
  }
  const char* p_;
  const char* e_;
};

bool valid_utf8(const uint8_t* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    uint8_t c = s[i];
    size_t len = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
    if (len == 0 || i + len > n) return false;
    for (size_t k = 1; k < len; ++k)
      if ((s[i + k] & 0xC0) != 0x80) return false;
    i += len;
  }
  return true;
}

}  // namespace

size_t st_dtype_size(const std::string& t) {
  static const std::map<std::string, size_t> sizes = {
      {"BOOL", 1}, {"U8", 1},   {"I8", 1},  {"F8_E5M2", 1}, {"F8_E4M3", 1}, {"F8_E8M0", 1},
      {"I16", 2},  {"U16", 2},  {"F16", 2}, {"BF16", 2},    {"I32", 4},     {"U32", 4},
      {"F32", 4},  {"F64", 8},  {"I64", 8}, {"U64", 8},     {"C64", 8}};
  auto it = sizes.find(t);
  return it == sizes.end() ? 0 : it->second;
}

int st_parse(const uint8_t* buf, size_t len, std::vector<StTensor>* out, size_t* data_offset,
             std::string* why) {
  out->clear();
  if (len < 8) {
    *why = "header too small";
    return 1;
  }
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | buf[i];
  if (n > kMaxHeader) {
    *why = "header too large";
    return 1;
  }
  if (n > len - 8) {
    *why = "invalid header length";
    return 1;
  }
  const uint8_t* h = buf + 8;
  if (!valid_utf8(h, (size_t)n)) {
    *why = "header is not utf-8";
    return 1;
  }
  if (n == 0 || h[0] != '{') {
    *why = "header does not start with '{'";
    return 1;
  }
  Json root;
  Parser ps((const char*)h, (size_t)n);
  if (!ps.parse(&root) || root.kind != Json::OBJ) {
    *why = "header is not a JSON object";
    return 1;
  }
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      if (kv.second.kind == Json::NUL) continue;
      if (kv.second.kind != Json::OBJ) {
        *why = "__metadata__ is not an object";
        return 1;
      }
      for (auto& m : kv.second.obj)
        if (m.second.kind != Json::STR) {
          *why = "__metadata__ values must be strings";
          return 1;
        }
      continue;
    }
    const Json& info = kv.second;
    if (info.kind != Json::OBJ) {
      *why = "tensor entry is not an object";
      return 1;
    }
    const Json *dt = nullptr, *sh = nullptr, *off = nullptr;
    for (auto& f : info.obj) {
      if (f.first == "dtype") dt = &f.second;
      else if (f.first == "shape") sh = &f.second;
      else if (f.first == "data_offsets") off = &f.second;
      else {
        *why = "unknown field in tensor entry";
        return 1;
      }
    }
    if (!dt || !sh || !off || dt->kind != Json::STR || sh->kind != Json::ARR ||
        off->kind != Json::ARR || off->arr.size() != 2) {
      *why = "malformed tensor entry";
      return 1;
    }
    if (st_dtype_size(dt->str) == 0) {
      *why = "unknown dtype";
      return 1;
    }
    StTensor t;
    t.name = kv.first;
    t.dtype = dt->str;
    for (auto& d : sh->arr) {
      if (d.kind != Json::NUM || !d.is_int || d.neg) {
        *why = "shape entries must be non-negative integers";
        return 1;
      }
      t.shape.push_back((int64_t)d.uval);
    }
    for (int i = 0; i < 2; ++i)
      if (off->arr[i].kind != Json::NUM || !off->arr[i].is_int || off->arr[i].neg) {
        *why = "data_offsets must be non-negative integers";
        return 1;
      }
    t.begin = (size_t)off->arr[0].uval;
    t.end = (size_t)off->arr[1].uval;
    out->push_back(std::move(t));
  }
  // Offsets must tile [0, data_len) in order of their start.
  std::vector<const StTensor*> order;
  for (auto& t : *out) order.push_back(&t);
  std::sort(order.begin(), order.end(), [](const StTensor* a, const StTensor* b) {
    return a->begin != b->begin ? a->begin < b->begin : a->end < b->end;
  });
  size_t cursor = 0;
  for (auto* t : order) {
    if (t->begin != cursor || t->end < t->begin) {
      *why = "invalid data_offsets for " + t->name;
      return 1;
    }
    unsigned __int128 numel = 1;
    for (int64_t d : t->shape) {
      numel *= (unsigned __int128)d;
      if (numel > ((unsigned __int128)1 << 62)) {
        *why = "shape overflows";
        return 1;
      }
    }
    unsigned __int128 bytes = numel * st_dtype_size(t->dtype);
    if (bytes != (unsigned __int128)(t->end - t->begin)) {
      *why = "byte length does not match shape for " + t->name;
      return 1;
    }
    cursor = t->end;
  }
  if (cursor != len - 8 - (size_t)n) {
    *why = "data section length does not match the offsets";
    return 1;
  }
  *data_offset = 8 + (size_t)n;
  return 0;
}

}  // namespace myos
