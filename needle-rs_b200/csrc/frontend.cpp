// frontend.cpp — see frontend.h.
#include "frontend.h"

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <queue>

namespace ndl {
namespace text {

namespace {

const char kSpSpace[] = "\xE2\x96\x81";  // U+2581, SentencePiece's word boundary

// Decode the code point at s[i], advancing i.  s must be valid UTF-8.
uint32_t next_cp(const std::string &s, size_t &i) {
  const unsigned char c = (unsigned char)s[i];
  int n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : 4;
  uint32_t cp = n == 1 ? c : n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
  for (int k = 1; k < n; ++k) cp = (cp << 6) | ((unsigned char)s[i + k] & 0x3F);
  i += n;
  return cp;
}

// Unicode White_Space (the set char::is_whitespace and str::trim use).
bool is_ws(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F ||
         c == 0x3000;
}

// ' ', \t, \n, \f, \r (u8::is_ascii_whitespace).
bool is_ascii_ws(unsigned char b) { return b == ' ' || b == '\t' || b == '\n' || b == '\f' || b == '\r'; }

std::string trim_unicode(const std::string &s, bool front, bool back) {
  size_t b = 0, e = s.size();
  if (front) {
    while (b < e) {
      size_t j = b;
      if (!is_ws(next_cp(s, j))) break;
      b = j;
    }
  }
  if (back) {
    while (e > b) {
      size_t j = e - 1;
      while (j > b && ((unsigned char)s[j] & 0xC0) == 0x80) --j;
      size_t k = j;
      if (!is_ws(next_cp(s, k))) break;
      e = j;
    }
  }
  return s.substr(b, e - b);
}

std::string replace_all(const std::string &s, const std::string &from, const std::string &to) {
  std::string out;
  size_t i = 0;
  while (true) {
    size_t j = s.find(from, i);
    if (j == std::string::npos) break;
    out.append(s, i, j - i);
    out += to;
    i = j + from.size();
  }
  out.append(s, i, std::string::npos);
  return out;
}

std::string byte_piece(unsigned char b) {
  static const char hex[] = "0123456789ABCDEF";
  std::string p = "<0x";
  p += hex[b >> 4];
  p += hex[b & 15];
  p += '>';
  return p;
}

// f32 parse with the forms str::parse::<f32> accepts (decimal and
// exponent notation, inf / infinity / nan in any case, optional sign); any
// other text scores 0.
float parse_score(const std::string &t) {
  if (t.empty()) return 0.0f;
  size_t i = (t[0] == '+' || t[0] == '-') ? 1 : 0;
  std::string body = t.substr(i);
  for (auto &c : body) c = (char)std::tolower((unsigned char)c);
  if (body == "inf" || body == "infinity") return t[0] == '-' ? -INFINITY : INFINITY;
  if (body == "nan") return NAN;
  bool digit = false;
  for (size_t k = 0; k < body.size(); ++k) {
    char c = body[k];
    if (c >= '0' && c <= '9') {
      digit = true;
    } else if (!(c == '.' || c == 'e' || ((c == '+' || c == '-') && k > 0 && body[k - 1] == 'e'))) {
      return 0.0f;
    }
  }
  if (!digit) return 0.0f;
  char *end = nullptr;
  errno = 0;
  float v = std::strtof(t.c_str(), &end);
  if (!end || *end != '\0') return 0.0f;
  return v;
}

}  // namespace

bool utf8_valid(const std::string &s) {
  size_t i = 0, n = s.size();
  while (i < n) {
    unsigned char c = (unsigned char)s[i];
    int len;
    uint32_t cp;
    if (c < 0x80) {
      ++i;
      continue;
    } else if ((c >> 5) == 6) {
      len = 2;
      cp = c & 0x1F;
    } else if ((c >> 4) == 14) {
      len = 3;
      cp = c & 0x0F;
    } else if ((c >> 3) == 30) {
      len = 4;
      cp = c & 0x07;
    } else {
      return false;
    }
    if (i + len > n) return false;
    for (int k = 1; k < len; ++k) {
      unsigned char d = (unsigned char)s[i + k];
      if ((d & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (d & 0x3F);
    }
    // overlong forms, surrogates, beyond U+10FFFF
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) || cp > 0x10FFFF ||
        (cp >= 0xD800 && cp <= 0xDFFF))
      return false;
    i += len;
  }
  return true;
}

// ── Vocab (tokenizer.rs:31-246) ─────────────────────────────────────────────

void Vocab::parse(const std::string &content) {
  id_to_piece_.clear();
  piece_to_id_.clear();
  scores_.clear();
  max_piece_bytes_ = 0;
  bool has_scores = false;
  size_t i = 0;
  while (i < content.size()) {  // str::lines: '\n' separators; "\r\n" counts as one
    size_t j = content.find('\n', i);
    const bool newline = j != std::string::npos;
    if (!newline) j = content.size();
    std::string line = content.substr(i, j - i);
    if (newline && !line.empty() && line.back() == '\r') line.pop_back();
    i = j + 1;
    const uint32_t id = (uint32_t)id_to_piece_.size();
    std::string piece;
    float score = 0.0f;
    size_t tab = line.find('\t');
    if (tab != std::string::npos) {
      has_scores = true;
      piece = line.substr(0, tab);
      score = parse_score(trim_unicode(line.substr(tab + 1), true, true));
    } else {
      piece = line;
    }
    max_piece_bytes_ = std::max(max_piece_bytes_, piece.size());
    piece_to_id_[piece] = id;  // a repeated piece maps to its last line
    id_to_piece_.push_back(piece);
    scores_.push_back(score);
  }
  if (!has_scores) scores_.clear();
}

bool Vocab::lookup(const std::string &piece, uint32_t &id) const {
  auto it = piece_to_id_.find(piece);
  if (it == piece_to_id_.end()) return false;
  id = it->second;
  return true;
}

std::string Vocab::piece_text(uint32_t id) const {
  if (id >= id_to_piece_.size()) return std::string();
  return replace_all(id_to_piece_[id], kSpSpace, " ");
}

std::vector<uint32_t> Vocab::encode(const std::string &raw) const {
  const std::string text = trim_unicode(raw, true, true);
  if (text.empty()) return {};
  std::string norm = kSpSpace;  // normalize_sp (tokenizer.rs:220-236)
  bool prev_space = false;
  for (size_t i = 0; i < text.size();) {
    size_t j = i;
    uint32_t cp = next_cp(text, j);
    if (is_ws(cp)) {
      if (!prev_space) norm += kSpSpace;
      prev_space = true;
    } else {
      norm.append(text, i, j - i);
      prev_space = false;
    }
    i = j;
  }
  return scores_.empty() ? encode_greedy(norm) : encode_bpe(norm);
}

// BPE merges (tokenizer.rs:97-159): repeatedly merge the adjacent pair whose
// concatenation is a piece with the highest score, the leftmost pair among
// equal scores, until no adjacent pair forms a piece.  The reference rescans
// every pair after each merge; here candidates sit in a max-heap keyed by
// (score, -position) with stale entries skipped, which picks the same pair.
std::vector<uint32_t> Vocab::encode_bpe(const std::string &norm) const {
  struct Unit {
    std::string s;
    uint32_t id;
    int prev, next;
    bool alive;
    uint32_t version;
  };
  std::vector<Unit> u;
  for (size_t i = 0; i < norm.size();) {
    size_t j = i;
    next_cp(norm, j);
    std::string ch = norm.substr(i, j - i);
    uint32_t id;
    if (lookup(ch, id)) {
      u.push_back({ch, id, 0, 0, true, 0});
    } else {  // byte fallback, one <0xXX> unit per UTF-8 byte
      for (size_t k = i; k < j; ++k) {
        std::string fb = byte_piece((unsigned char)norm[k]);
        uint32_t fid;
        if (!lookup(fb, fid)) fid = kUnkId;
        u.push_back({fb, fid, 0, 0, true, 0});
      }
    }
    i = j;
  }
  const int n = (int)u.size();
  for (int i = 0; i < n; ++i) {
    u[i].prev = i - 1;
    u[i].next = i + 1 < n ? i + 1 : -1;
  }
  struct Cand {
    float score;
    int left;  // index of the left unit (its position never changes)
    uint32_t vl, vr;
    uint32_t id;
  };
  auto worse = [](const Cand &a, const Cand &b) {
    if (a.score != b.score) return a.score < b.score;
    return a.left > b.left;  // smaller position first
  };
  std::priority_queue<Cand, std::vector<Cand>, decltype(worse)> heap(worse);
  auto push = [&](int l) {
    if (l < 0) return;
    int r = u[l].next;
    if (r < 0) return;
    uint32_t id;
    if (!lookup(u[l].s + u[r].s, id)) return;
    float sc = scores_[id];
    if (!(sc > -INFINITY)) return;  // the reference never picks -inf or NaN scores
    heap.push({sc, l, u[l].version, u[r].version, id});
  };
  for (int i = 0; i + 1 < n; ++i) push(i);
  while (!heap.empty()) {
    Cand c = heap.top();
    heap.pop();
    const int l = c.left;
    if (!u[l].alive || u[l].version != c.vl) continue;
    const int r = u[l].next;
    if (r < 0 || u[r].version != c.vr) continue;
    u[l].s += u[r].s;
    u[l].id = c.id;
    ++u[l].version;
    u[r].alive = false;
    u[l].next = u[r].next;
    if (u[r].next >= 0) u[u[r].next].prev = l;
    push(u[l].prev);
    push(l);
  }
  std::vector<uint32_t> ids;
  for (int i = n > 0 ? 0 : -1; i >= 0; i = u[i].next) ids.push_back(u[i].id);
  return ids;
}

// Greedy longest match (tokenizer.rs:162-201), for vocabularies without scores.
std::vector<uint32_t> Vocab::encode_greedy(const std::string &b) const {
  const size_t n = b.size();
  auto cont = [&](size_t k) { return ((unsigned char)b[k] & 0xC0) == 0x80; };
  std::vector<uint32_t> ids;
  size_t pos = 0;
  while (pos < n) {
    size_t end = std::min(pos + max_piece_bytes_, n);
    while (end > pos && end < n && cont(end)) --end;
    bool found = false;
    while (end > pos) {
      std::string piece = b.substr(pos, end - pos);
      uint32_t id;
      if (utf8_valid(piece) && lookup(piece, id)) {
        ids.push_back(id);
        pos = end;
        found = true;
        break;
      }
      --end;
      while (end > pos && cont(end)) --end;
    }
    if (!found) {
      uint32_t id;
      if (!lookup(byte_piece((unsigned char)b[pos]), id)) id = kUnkId;
      ids.push_back(id);
      pos += 1;
    }
  }
  return ids;
}

std::string Vocab::decode_ids(const std::vector<uint32_t> &ids) const {
  std::string out;
  for (uint32_t id : ids)
    if (id < id_to_piece_.size()) out += replace_all(id_to_piece_[id], kSpSpace, " ");
  return trim_unicode(out, true, false);
}

// tokenizer.rs:248-292.  ASCII letters, digits and '_' follow the
// reference's rules exactly; other non-ASCII characters are kept as
// alphanumeric characters with no case.
std::string to_snake_case(const std::string &name) {
  std::vector<uint32_t> ch;
  std::vector<std::string> raw;
  for (size_t i = 0; i < name.size();) {
    size_t j = i;
    ch.push_back(next_cp(name, j));
    raw.push_back(name.substr(i, j - i));
    i = j;
  }
  auto upper = [](uint32_t c) { return c >= 'A' && c <= 'Z'; };
  auto lower = [](uint32_t c) { return c >= 'a' && c <= 'z'; };
  auto digit = [](uint32_t c) { return c >= '0' && c <= '9'; };
  auto alnum = [&](uint32_t c) { return upper(c) || lower(c) || digit(c) || c >= 0x80; };
  std::string out;
  bool prev_us = false, prev_up = false;
  const size_t n = ch.size();
  for (size_t i = 0; i < n; ++i) {
    const uint32_t c = ch[i];
    if (alnum(c) || c == '_') {
      if (c == '_') {
        if (!prev_us && !out.empty()) {
          out += '_';
          prev_us = true;
        }
        prev_up = false;
      } else if (upper(c)) {
        const bool prev_lower = i > 0 && (lower(ch[i - 1]) || digit(ch[i - 1]));
        const bool next_lower = i + 1 < n && lower(ch[i + 1]);
        if (i > 0 && !prev_us && (prev_lower || (prev_up && next_lower))) out += '_';
        out += (char)(c - 'A' + 'a');
        prev_us = false;
        prev_up = true;
      } else {
        out += raw[i];
        prev_us = false;
        prev_up = false;
      }
    } else {
      if (!prev_us && !out.empty()) {
        out += '_';
        prev_us = true;
      }
      prev_up = false;
    }
  }
  while (!out.empty() && out.back() == '_') out.pop_back();
  return out;
}

// ── tool JSON (constrained.rs:378-689) ──────────────────────────────────────

namespace {

// Index of the delimiter closing the one at `start`, skipping strings; the
// last index when unbalanced.
size_t find_matching(const std::string &b, size_t start, char open, char close) {
  size_t depth = 0;
  bool in_str = false, esc = false;
  for (size_t i = start; i < b.size(); ++i) {
    char c = b[i];
    if (in_str) {
      if (esc)
        esc = false;
      else if (c == '\\')
        esc = true;
      else if (c == '"')
        in_str = false;
    } else if (c == '"') {
      in_str = true;
    } else if (c == open) {
      ++depth;
    } else if (c == close) {
      depth = depth ? depth - 1 : 0;
      if (depth == 0) return i;
    }
  }
  return b.empty() ? 0 : b.size() - 1;
}

bool extract_string(const std::string &obj, const std::string &field, std::string &out) {
  const std::string key = "\"" + field + "\":\"";
  size_t pos = obj.find(key);
  if (pos == std::string::npos) return false;
  size_t s = pos + key.size();
  bool esc = false;
  for (size_t i = s; i < obj.size(); ++i) {
    if (esc)
      esc = false;
    else if (obj[i] == '\\')
      esc = true;
    else if (obj[i] == '"') {
      out = obj.substr(s, i - s);
      return true;
    }
  }
  return false;
}

bool extract_object(const std::string &obj, const std::string &field, std::string &out) {
  const std::string key = "\"" + field + "\":";
  size_t pos = obj.find(key);
  if (pos == std::string::npos) return false;
  std::string after = trim_unicode(obj.substr(pos + key.size()), true, false);
  if (after.empty() || after[0] != '{') return false;
  size_t end = find_matching(after, 0, '{', '}');
  out = after.substr(0, end + 1);
  return true;
}

size_t skip_value(const std::string &b, size_t i) {
  if (i >= b.size()) return i;
  if (b[i] == '{') return find_matching(b, i, '{', '}') + 1;
  if (b[i] == '[') return find_matching(b, i, '[', ']') + 1;
  if (b[i] == '"') {
    ++i;
    bool esc = false;
    while (i < b.size()) {
      if (esc)
        esc = false;
      else if (b[i] == '\\')
        esc = true;
      else if (b[i] == '"')
        return i + 1;
      ++i;
    }
    return i;
  }
  while (i < b.size() && b[i] != ',' && b[i] != '}' && b[i] != ']') ++i;
  return i;
}

// Top-level keys of an object; object_values_only keeps keys whose value is
// an object.
std::vector<std::string> object_keys(const std::string &b, bool object_values_only) {
  std::vector<std::string> keys;
  size_t i = 0;
  if (i < b.size() && b[i] == '{') ++i;
  while (i < b.size()) {
    while (i < b.size() && (b[i] == ',' || is_ascii_ws((unsigned char)b[i]))) ++i;
    if (i >= b.size() || b[i] == '}') break;
    if (b[i] != '"') {
      ++i;
      continue;
    }
    ++i;
    const size_t ks = i;
    bool esc = false;
    while (i < b.size()) {
      if (esc)
        esc = false;
      else if (b[i] == '\\')
        esc = true;
      else if (b[i] == '"')
        break;
      ++i;
    }
    std::string key = b.substr(ks, std::min(i, b.size()) - ks);
    ++i;
    while (i < b.size() && b[i] != ':') ++i;
    ++i;
    while (i < b.size() && is_ascii_ws((unsigned char)b[i])) ++i;
    if (object_values_only) {
      if (i < b.size() && b[i] == '{') {
        if (!key.empty()) keys.push_back(key);
        i = find_matching(b, i, '{', '}') + 1;
      } else {
        i = skip_value(b, i);
      }
    } else {
      if (!key.empty()) keys.push_back(key);
      i = skip_value(b, i);
    }
  }
  return keys;
}

// "name" values rewritten through `map` (from -> to) by a byte scan that
// leaves every other byte as it was (engine.rs:359-426, 477-546).
std::string rename_names(const std::string &json, const std::vector<std::pair<std::string, std::string>> &map) {
  if (map.empty()) return json;
  std::string out;
  size_t i = 0, flushed = 0;
  const size_t n = json.size();
  while (i < n) {
    if (json.compare(i, 6, "\"name\"") == 0) {
      out.append(json, flushed, i - flushed);
      out += "\"name\"";
      i += 6;
      while (i < n && is_ascii_ws((unsigned char)json[i])) ++i;
      if (i < n && json[i] == ':') {
        out += ':';
        ++i;
      }
      while (i < n && is_ascii_ws((unsigned char)json[i])) ++i;
      if (i < n && json[i] == '"') {
        out += '"';
        ++i;
        const size_t vs = i;
        while (i < n) {
          if (json[i] == '\\') {
            i += 2;
            continue;
          }
          if (json[i] == '"') break;
          ++i;
        }
        if (i > n) i = n;
        const std::string val = json.substr(vs, i - vs);
        const std::string *rep = &val;
        for (auto &p : map)
          if (p.first == val) {
            rep = &p.second;
            break;
          }
        out += *rep;
        if (i < n) {
          out += '"';
          ++i;
        }
      }
      flushed = i;
    } else {
      ++i;
    }
  }
  if (flushed < n) out.append(json, flushed, std::string::npos);
  return out;
}

}  // namespace

std::vector<ToolDef> parse_tools_json(const std::string &json) {
  std::vector<ToolDef> tools;
  size_t i = 0;
  const size_t n = json.size();
  while (i < n && json[i] != '[' && json[i] != '{') ++i;
  if (i >= n) return tools;
  if (json[i] == '[') ++i;
  while (i < n) {
    while (i < n && (json[i] == ',' || is_ascii_ws((unsigned char)json[i]))) ++i;
    if (i >= n || json[i] == ']') break;
    if (json[i] != '{') {
      ++i;
      continue;
    }
    const size_t end = find_matching(json, i, '{', '}');
    const std::string obj = json.substr(i, end + 1 - i);
    ToolDef t;
    if (extract_string(obj, "name", t.name)) {  // parse_single_tool
      t.snake_name = to_snake_case(t.name);
      std::string params, props;
      if (extract_object(obj, "parameters", params)) {
        if (extract_object(params, "properties", props))
          t.param_keys = object_keys(props, false);  // JSON Schema
        else
          t.param_keys = object_keys(params, true);  // flat {"key": {...}}
      }
      tools.push_back(std::move(t));
    }
    i = end + 1;
  }
  return tools;
}

std::string normalize_tools_json(const std::string &json, const std::vector<ToolDef> &defs) {
  std::vector<std::pair<std::string, std::string>> map;
  for (auto &t : defs)
    if (t.name != t.snake_name) map.push_back({t.name, t.snake_name});
  return rename_names(json, map);
}

std::string restore_tool_names(const std::string &text, const std::vector<ToolDef> &defs) {
  std::vector<std::pair<std::string, std::string>> map;
  for (auto &t : defs)
    if (t.name != t.snake_name) map.push_back({t.snake_name, t.name});
  // longest snake name first; equal lengths keep their order
  std::stable_sort(map.begin(), map.end(),
                   [](const auto &a, const auto &b) { return a.first.size() > b.first.size(); });
  return rename_names(text, map);
}

std::string compact_json(const std::string &s) {
  std::string out;
  bool in_str = false;
  for (size_t i = 0; i < s.size();) {
    size_t j = i;
    next_cp(s, j);  // whole characters, so an escaped multi-byte character is copied intact
    const unsigned char c = (unsigned char)s[i];
    if (in_str) {
      out.append(s, i, j - i);
      if (c == '\\') {
        if (j < s.size()) {
          size_t k = j;
          next_cp(s, k);
          out.append(s, j, k - j);
          j = k;
        }
      } else if (c == '"') {
        in_str = false;
      }
    } else if (c == '"') {
      in_str = true;
      out += '"';
    } else if (!(j - i == 1 && is_ascii_ws(c))) {
      out.append(s, i, j - i);
    }
    i = j;
  }
  return out;
}

// ── Trie and JSON state machine (constrained.rs:15-292) ─────────────────────

Trie::Trie() { nodes_.emplace_back(); }

void Trie::insert(const std::string &s) {
  int cur = 0;
  for (unsigned char b : s) {
    auto it = nodes_[cur].children.find(b);
    if (it == nodes_[cur].children.end()) {
      int nn = (int)nodes_.size();
      nodes_.emplace_back();
      nodes_[cur].children[b] = nn;
      cur = nn;
    } else {
      cur = it->second;
    }
  }
  nodes_[cur].terminal = true;
}

int Trie::advance(int node, const std::string &s) const {
  int cur = node;
  for (unsigned char b : s) {
    auto it = nodes_[cur].children.find(b);
    if (it == nodes_[cur].children.end()) return -1;
    cur = it->second;
  }
  return cur;
}

bool Trie::token_valid(const std::string &bytes, int node) const {
  int cur = node;
  for (unsigned char b : bytes) {
    if (b == '"') return nodes_[cur].terminal;
    auto it = nodes_[cur].children.find(b);
    if (it == nodes_[cur].children.end()) return false;
    cur = it->second;
  }
  return true;
}

void JsonStateMachine::push_tail(uint8_t b) {
  tail_ += (char)b;
  if (tail_.size() > 13) tail_.erase(0, tail_.size() - 13);
}

bool JsonStateMachine::tail_ends_with(const char *pat, size_t n) const {
  return tail_.size() >= n && tail_.compare(tail_.size() - n, n, pat, n) == 0;
}

void JsonStateMachine::feed_byte(uint8_t b) {
  if (state == JsonState::InName || state == JsonState::InArgKey) {
    if (b == '"') {
      if (state == JsonState::InName) current_function = constrained_buf;
      constrained_buf.clear();
      state = JsonState::Free;
    } else {
      constrained_buf += (char)b;
    }
    return;
  }
  push_tail(b);
  if (in_string_) {  // inside a value string (opened by :")
    if (prev_escape_) {
      prev_escape_ = false;
    } else if (b == '\\') {
      prev_escape_ = true;
    } else if (b == '"') {
      in_string_ = false;
    }
    return;
  }
  if (b == '{' || b == '[') {
    ++nesting_depth_;
  } else if (b == '}' || b == ']') {
    nesting_depth_ = nesting_depth_ ? nesting_depth_ - 1 : 0;
    if (b == '}' && in_arguments_ && nesting_depth_ < arguments_depth_) in_arguments_ = false;
    return;
  }
  if (!in_arguments_ && tail_ends_with("\"name\":\"", 8)) {
    state = JsonState::InName;
    constrained_buf.clear();
    return;
  }
  if (tail_ends_with("\"arguments\":{", 13)) {
    in_arguments_ = true;
    arguments_depth_ = nesting_depth_;
    return;
  }
  const size_t n = tail_.size();
  if (in_arguments_ && nesting_depth_ == arguments_depth_ && n >= 2 && (tail_[n - 2] == '{' || tail_[n - 2] == ',') &&
      tail_[n - 1] == '"') {
    state = JsonState::InArgKey;
    constrained_buf.clear();
    return;
  }
  if (b == '"' && n >= 2 && tail_[n - 2] == ':') in_string_ = true;
}

// ── constrained decoder (constrained.rs:300-375) ────────────────────────────

ConstrainedDecoder::ConstrainedDecoder(const std::vector<ToolDef> &tools, const Vocab &vocab) {
  for (auto &t : tools) {
    name_trie_.insert(t.snake_name);
    Trie keys;
    for (auto &k : t.param_keys) keys.insert(k);
    param_index_[t.snake_name] = (int)param_tries_.size();  // a repeated name keeps its last tool
    param_tries_.push_back(std::move(keys));
  }
  token_texts_.resize(vocab.size());
  for (uint32_t i = 0; i < vocab.size(); ++i) token_texts_[i] = vocab.piece_text(i);
}

void ConstrainedDecoder::update(uint32_t token) {
  if (token < token_texts_.size()) sm_.feed(token_texts_[token]);
}

bool ConstrainedDecoder::trie_mask(const Trie &trie, int trie_id, int node, size_t V, std::vector<uint64_t> &bits) {
  if (V != cache_vocab_) {
    cache_.clear();
    cache_vocab_ = V;
  }
  const uint64_t key = ((uint64_t)(uint32_t)trie_id << 32) | (uint32_t)node;
  auto it = cache_.find(key);
  if (it == cache_.end()) {
    std::vector<uint64_t> b((V + 63) / 64, 0ull);
    bool any = false;
    for (size_t id = 0; id < token_texts_.size() && id < V; ++id)
      if (trie.token_valid(token_texts_[id], node)) {
        b[id >> 6] |= 1ull << (id & 63);
        any = true;
      }
    it = cache_.emplace(key, std::make_pair(any, std::move(b))).first;
  }
  if (!it->second.first) return false;  // nothing valid: unconstrained, as the reference falls back
  bits = it->second.second;
  return true;
}

bool ConstrainedDecoder::mask(size_t V, std::vector<uint64_t> &bits) {
  if (sm_.state == JsonState::InName) {
    int node = name_trie_.advance(0, sm_.constrained_buf);
    return node >= 0 && trie_mask(name_trie_, -1, node, V, bits);
  }
  if (sm_.state == JsonState::InArgKey) {
    auto it = param_index_.find(sm_.current_function);
    if (it == param_index_.end()) return false;
    const Trie &t = param_tries_[it->second];
    int node = t.advance(0, sm_.constrained_buf);
    return node >= 0 && trie_mask(t, it->second, node, V, bits);
  }
  return false;
}

}  // namespace text
}  // namespace ndl
