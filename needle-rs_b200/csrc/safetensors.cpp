// safetensors.cpp — see safetensors.h.
#include "safetensors.h"

#include <cstring>

namespace ndl {
namespace {

// Minimal JSON value for the SafeTensors header (objects, arrays, strings,
// numbers kept as their source text, literals).
struct JVal {
  enum Kind { OBJ, ARR, STR, NUM, LIT } kind = LIT;
  std::string text;                                   // STR (unescaped) / NUM / LIT
  std::vector<std::pair<std::string, JVal>> members;  // OBJ
  std::vector<JVal> items;                            // ARR
};

struct JParser {
  const char *p, *e;
  std::string err;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool str(std::string &out) {
    if (p >= e || *p != '"') return false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= e) return false;
        char c = *p++;
        switch (c) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (e - p < 4) return false;
            unsigned cp = (unsigned)std::stoul(std::string(p, 4), nullptr, 16);
            p += 4;
            if (cp < 0x80) {
              out += (char)cp;
            } else if (cp < 0x800) {
              out += (char)(0xC0 | (cp >> 6));
              out += (char)(0x80 | (cp & 0x3F));
            } else {
              out += (char)(0xE0 | (cp >> 12));
              out += (char)(0x80 | ((cp >> 6) & 0x3F));
              out += (char)(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: out += c;
        }
      } else {
        out += *p++;
      }
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool value(JVal &v, int depth) {
    if (depth > 64) return false;
    ws();
    if (p >= e) return false;
    if (*p == '{') {
      v.kind = JVal::OBJ;
      ++p;
      ws();
      if (p < e && *p == '}') { ++p; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (p >= e || *p != ':') return false;
        ++p;
        JVal c;
        if (!value(c, depth + 1)) return false;
        v.members.emplace_back(std::move(k), std::move(c));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; return true; }
        return false;
      }
    }
    if (*p == '[') {
      v.kind = JVal::ARR;
      ++p;
      ws();
      if (p < e && *p == ']') { ++p; return true; }
      for (;;) {
        JVal c;
        if (!value(c, depth + 1)) return false;
        v.items.push_back(std::move(c));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; return true; }
        return false;
      }
    }
    if (*p == '"') {
      v.kind = JVal::STR;
      return str(v.text);
    }
    const char *s = p;
    while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n' && *p != '\r' && *p != '\t') ++p;
    if (p == s) return false;
    v.text.assign(s, p);
    v.kind = (v.text == "true" || v.text == "false" || v.text == "null") ? JVal::LIT : JVal::NUM;
    return true;
  }
};

bool as_usize(const JVal &v, size_t &out) {
  if (v.kind != JVal::NUM || v.text.empty()) return false;
  for (char c : v.text)
    if (c < '0' || c > '9') return false;
  out = (size_t)std::stoull(v.text);
  return true;
}

bool usize_array(const JVal *v, std::vector<size_t> &out) {
  // safetensors.rs:323-339: each comma-separated piece must parse as usize;
  // the empty body of "[]" does not.
  if (!v || v->kind != JVal::ARR || v->items.empty()) return false;
  out.clear();
  for (const JVal &i : v->items) {
    size_t x;
    if (!as_usize(i, x)) return false;
    out.push_back(x);
  }
  return true;
}

const JVal *member(const JVal &o, const char *k) {
  for (auto &m : o.members)
    if (m.first == k) return &m.second;
  return nullptr;
}

inline int8_t sext4(uint8_t n) { return (n & 0x8) ? (int8_t)(n | 0xF0) : (int8_t)n; }

}  // namespace

float f16_to_f32(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits >> 15) << 31;
  uint32_t exp = (bits >> 10) & 0x1F, mant = bits & 0x3FF;
  if (exp == 0) {
    float val = (float)mant / (float)(1u << 24);
    return sign ? -val : val;
  }
  uint32_t o = exp == 31 ? (sign | 0x7F800000u | (mant << 13)) : (sign | ((exp + 127 - 15) << 23) | (mant << 13));
  float f;
  std::memcpy(&f, &o, 4);
  return f;
}

bool SafeTensors::parse(std::vector<uint8_t> raw, std::string &err) {
  if (raw.size() < 8) { err = "buffer too short"; return false; }
  uint64_t hl;
  std::memcpy(&hl, raw.data(), 8);
  if (hl > raw.size() - 8) { err = "truncated header"; return false; }
  const char *h = (const char *)raw.data() + 8;
  // The header must be valid UTF-8 (std::str::from_utf8 in the reference).
  for (size_t i = 0; i < hl;) {
    unsigned char c = (unsigned char)h[i];
    size_t n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
    if (!n || i + n > hl) { err = "invalid UTF-8 header"; return false; }
    for (size_t j = 1; j < n; ++j)
      if (((unsigned char)h[i + j] >> 6) != 2) { err = "invalid UTF-8 header"; return false; }
    i += n;
  }
  JParser jp{h, h + hl, {}};
  JVal root;
  jp.ws();
  if (jp.p >= jp.e || *jp.p != '{' || !jp.value(root, 0) || root.kind != JVal::OBJ) {
    err = "expected JSON object";
    return false;
  }
  for (auto &m : root.members) {
    if (m.first == "__metadata__") {
      if (m.second.kind == JVal::OBJ)
        for (auto &kv : m.second.members) meta_[kv.first] = kv.second.text;
      continue;
    }
    const JVal &v = m.second;
    if (v.kind != JVal::OBJ) { err = "missing dtype for " + m.first; return false; }
    const JVal *dt = member(v, "dtype");
    if (!dt || dt->kind != JVal::STR) { err = "missing dtype for " + m.first; return false; }
    TensorMeta tm;
    if (!usize_array(member(v, "shape"), tm.shape)) { err = "missing shape for " + m.first; return false; }
    std::vector<size_t> offs;
    if (!usize_array(member(v, "data_offsets"), offs)) { err = "missing data_offsets for " + m.first; return false; }
    if (offs.size() != 2) { err = "data_offsets must have 2 elements"; return false; }
    const std::string &d = dt->text;
    if (d == "F32") tm.dtype = DType::F32;
    else if (d == "BF16") tm.dtype = DType::BF16;
    else if (d == "F16") tm.dtype = DType::F16;
    else if (d == "I8") tm.dtype = DType::I8;
    else if (d == "I4") tm.dtype = DType::I4;
    else { err = "unknown dtype " + d; return false; }
    tm.start = offs[0];
    tm.end = offs[1];
    tensors_[m.first] = tm;
  }
  data_ = std::move(raw);
  data_off_ = 8 + hl;
  size_t dsz = data_.size() - data_off_;
  for (auto &t : tensors_)
    if (t.second.start > t.second.end || t.second.end > dsz) {
      err = "tensor " + t.first + " data_offsets out of range";
      return false;
    }
  return true;
}

const TensorMeta *SafeTensors::meta(const std::string &name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

const std::string *SafeTensors::metadata(const std::string &key) const {
  auto it = meta_.find(key);
  return it == meta_.end() ? nullptr : &it->second;
}

const uint8_t *SafeTensors::get_raw(const std::string &name, size_t *len) const {
  const TensorMeta *m = meta(name);
  if (!m) return nullptr;
  if (len) *len = m->end - m->start;
  return data_.data() + data_off_ + m->start;
}

bool SafeTensors::get_f32(const std::string &name, std::vector<float> &out) const {
  const TensorMeta *m = meta(name);
  if (!m) return false;
  const uint8_t *raw = data_.data() + data_off_ + m->start;
  size_t n = m->end - m->start;
  out.clear();
  switch (m->dtype) {
    case DType::F32:
      out.resize(n / 4);
      std::memcpy(out.data(), raw, (n / 4) * 4);
      break;
    case DType::BF16:
      out.resize(n / 2);
      for (size_t i = 0; i < n / 2; ++i) {
        uint32_t bits = (uint32_t)(raw[2 * i] | (raw[2 * i + 1] << 8)) << 16;
        std::memcpy(&out[i], &bits, 4);
      }
      break;
    case DType::F16:
      out.resize(n / 2);
      for (size_t i = 0; i < n / 2; ++i) out[i] = f16_to_f32((uint16_t)(raw[2 * i] | (raw[2 * i + 1] << 8)));
      break;
    case DType::I8:
      out.resize(n);
      for (size_t i = 0; i < n; ++i) out[i] = (float)(int8_t)raw[i];
      break;
    case DType::I4: {
      size_t vol = 1;
      for (size_t s : m->shape) vol *= s;
      if (n * 2 != vol) return false;  // safetensors.rs:99-110
      out.resize(vol);
      for (size_t i = 0; i < n; ++i) {
        out[2 * i] = (float)sext4(raw[i] & 0x0F);
        out[2 * i + 1] = (float)sext4(raw[i] >> 4);
      }
      break;
    }
  }
  return true;
}

bool SafeTensors::is_bf16_exact(const std::string &name) const {
  const TensorMeta *m = meta(name);
  if (!m) return false;
  if (m->dtype == DType::BF16) return true;
  if (m->dtype != DType::F32) return false;
  const uint8_t *raw = data_.data() + data_off_ + m->start;
  size_t n = (m->end - m->start) / 4;
  for (size_t i = 0; i < n; ++i) {
    uint32_t b;
    std::memcpy(&b, raw + 4 * i, 4);
    if (b & 0xFFFFu) return false;
  }
  return true;
}

}  // namespace ndl
