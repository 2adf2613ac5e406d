// capi.cpp — the extern "C" boundary: needle.h (reference ABI) and
// needle_b200.h (batched / kernel-level extensions).
//
// Mirrors crates/needle-c/src/lib.rs: thread-local last error (:21-33),
// NULL-tolerant frees (:112-127), NULL handle -> NULL without an error
// (:81-83), error strings "load error: ..." (:63, :164).
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <string>
#include <algorithm>
#include <vector>

#include "../../include/needle_b200.h"
#include "capi_internal.h"
#include "engine.h"
#include "frontend.h"

using namespace ndl;

struct NeedleVocab {
  text::Vocab v;
};

struct NeedleConstraint {
  std::unique_ptr<text::ConstrainedDecoder> d;
  std::vector<uint64_t> bits;
};

struct NeedleHandle {
  std::unique_ptr<DevModel> model;
  std::string vocab_text;
  NeedleVocab vocab;  // parsed once at load; read-only afterwards
};

struct NeedleBatch {
  NeedleHandle *h = nullptr;
  std::unique_ptr<Batch> batch;
  BatchSpec spec;
  std::vector<uint64_t> offsets;
  int timed_cls = 0;
  int next_step = -1;  // step-wise decoding: next step to run (-1 before needle_batch_begin)
};

namespace {

thread_local std::string g_err;
thread_local bool g_has_err = false;

void set_err(const std::string &s) {
  g_err = s;
  g_has_err = true;
}
void clear_err() {
  g_err.clear();
  g_has_err = false;
}

int default_device() {
  const char *e = std::getenv("NEEDLE_DEVICE");
  return e ? std::atoi(e) : 0;
}

bool read_file(const char *path, std::vector<uint8_t> &out, std::string &err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = std::string("No such file or directory (os error 2): ") + path;
    return false;
  }
  out.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  return true;
}

bool valid_utf8(const uint8_t *s, size_t n) {
  for (size_t i = 0; i < n;) {
    unsigned char c = s[i];
    size_t k = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
    if (!k || i + k > n) return false;
    for (size_t j = 1; j < k; ++j)
      if ((s[i + j] >> 6) != 2) return false;
    i += k;
  }
  return true;
}

NeedleHandle *load_impl(std::vector<uint8_t> weights, const std::string &vocab_text, int device) {
  std::string err;
  auto model = load_model(std::move(weights), device, err);
  if (!model) {
    set_err("load error: " + err);
    return nullptr;
  }
  auto *h = new NeedleHandle();
  h->model = std::move(model);
  h->vocab_text = vocab_text;
  h->vocab.v.parse(vocab_text);
  return h;
}

NeedleHandle *load_path(const char *wp, const char *vp, int device) {
  if (!wp || !vp) return nullptr;
  if (!valid_utf8((const uint8_t *)wp, std::strlen(wp)) || !valid_utf8((const uint8_t *)vp, std::strlen(vp)))
    return nullptr;
  clear_err();
  std::vector<uint8_t> w, v;
  std::string err;
  if (!read_file(wp, w, err) || !read_file(vp, v, err)) {
    set_err("load error: " + err);
    return nullptr;
  }
  return load_impl(std::move(w), std::string(v.begin(), v.end()), device);
}

NeedleHandle *load_bytes(const uint8_t *wd, size_t wl, const uint8_t *vd, size_t vl, int device) {
  if (!wd || !vd) {
    set_err("null pointer passed to needle_load_bytes");
    return nullptr;
  }
  if (!valid_utf8(vd, vl)) {
    set_err("vocab is not valid UTF-8");
    return nullptr;
  }
  clear_err();
  return load_impl(std::vector<uint8_t>(wd, wd + wl), std::string((const char *)vd, vl), device);
}

bool make_spec(NeedleHandle *h, const uint32_t *ids, const uint64_t *off, size_t n_req, uint32_t max_new,
               const uint64_t *mask, uint32_t flags, BatchSpec &s) {
  if (!h) return false;
  if (!ids || !off || n_req == 0 || n_req > (size_t)INT32_MAX) {
    set_err("invalid batch arguments");
    return false;
  }
  s.ids = ids;
  s.offsets = off;
  s.n_req = (int)n_req;
  s.max_new = (int)max_new;
  s.mask = mask;
  uint32_t f = 0;
  if (flags & NEEDLE_STOP_ON_EOS) f |= BATCH_STOP_ON_EOS;
  if (flags & NEEDLE_DEVICE_POINTERS) f |= BATCH_DEVICE_INPUTS;
  if (flags & NEEDLE_NO_GRAPH) f |= BATCH_NO_GRAPH;
  if (flags & NEEDLE_NO_PDL) f |= BATCH_NO_PDL;
  s.flags = f;
  return true;
}

int run_batch(NeedleHandle *h, const uint32_t *ids, const uint64_t *off, size_t n_req, uint32_t max_new,
              const uint64_t *mask, uint32_t flags, uint32_t *out_ids, uint32_t *out_lens, float *logits) {
  if (!h) return -1;
  clear_err();
  BatchSpec s;
  if (!make_spec(h, ids, off, n_req, max_new, mask, flags, s)) return -1;
  s.want_logits = logits != nullptr;
  Batch b(h->model.get());
  std::string err;
  if (!b.prepare(s, err) || !b.run(err) || !b.download(out_ids, out_lens, logits, nullptr, err)) {
    set_err(err);
    return -1;
  }
  return 0;
}

}  // namespace

void ndl::capi_set_last_error(const std::string &msg) { set_err(msg); }
void ndl::capi_clear_last_error() { clear_err(); }

extern "C" {

NeedleHandle *needle_load(const char *weights_path, const char *vocab_path) {
  return load_path(weights_path, vocab_path, default_device());
}

NeedleHandle *needle_load_bytes(const uint8_t *wd, size_t wl, const uint8_t *vd, size_t vl) {
  return load_bytes(wd, wl, vd, vl, default_device());
}

NeedleHandle *needle_load_on_device(const char *weights_path, const char *vocab_path, int device) {
  return load_path(weights_path, vocab_path, device);
}

NeedleHandle *needle_load_bytes_on_device(const uint8_t *wd, size_t wl, const uint8_t *vd, size_t vl, int device) {
  return load_bytes(wd, wl, vd, vl, device);
}

// NeedleEngine::run_impl (crates/needle-infer/src/engine.rs:226-322) on the
// GPU engine, for n requests at once (run_batch, engine.rs:142-144): per
// request the tools JSON is normalised and compacted, the encoder input is
// query ++ [TOOLS] ++ tools (truncated to max_enc_len as the reference
// truncates), and greedy decoding runs from EOS one step at a time so that
// each request's constrained-decoding mask for step s+1 follows its token of
// step s; a request stops at EOS (not emitted); the output has the
// <tool_call> prefix stripped and the original tool names restored.  cb (n =
// 1 only) fires per emitted token in order.
static bool run_text_batch(NeedleHandle *h, const std::vector<std::string> &queries,
                           const std::vector<std::string> &tools, NeedleStreamCallback cb, void *ud,
                           std::vector<std::string> &outs) {
  const Config &c = h->model->cfg;
  const size_t n = queries.size();
  outs.assign(n, std::string());
  std::vector<std::vector<text::ToolDef>> defs(n);
  std::vector<uint32_t> ids;
  std::vector<uint64_t> off(1, 0);
  std::vector<size_t> slot;  // request index of each batch row
  for (size_t r = 0; r < n; ++r) {
    defs[r] = text::parse_tools_json(tools[r]);
    const std::string compact = text::compact_json(text::normalize_tools_json(tools[r], defs[r]));
    const std::vector<uint32_t> q = h->vocab.v.encode(queries[r]), t = h->vocab.v.encode(compact);
    const size_t max_enc = (size_t)c.max_enc_len;
    if ((q.empty() && t.empty()) || max_enc == 0) continue;  // empty result, no decoding
    const size_t q_len = std::min(q.size(), max_enc >= 2 ? max_enc - 2 : 0);
    const size_t rem = max_enc >= q_len + 1 ? max_enc - (q_len + 1) : 0;
    const size_t t_len = std::min(t.size(), rem);
    ids.insert(ids.end(), q.begin(), q.begin() + q_len);
    ids.push_back(text::kToolsId);
    ids.insert(ids.end(), t.begin(), t.begin() + t_len);
    off.push_back(ids.size());
    slot.push_back(r);
  }
  for (uint32_t id : ids)
    if (id >= (uint32_t)c.vocab_size) {
      set_err("the vocabulary has token ids beyond the model's vocab_size");
      return false;
    }
  const int B = (int)slot.size(), steps = c.max_dec_len;
  std::vector<std::vector<uint32_t>> gen(B);
  if (B > 0 && steps > 0) {
    const size_t W = ((size_t)c.vocab_size + 63) / 64;
    std::vector<uint64_t> init((size_t)B * steps * W, ~0ull);  // every step starts unconstrained
    BatchSpec s;
    s.ids = ids.data();
    s.offsets = off.data();
    s.n_req = B;
    s.max_new = steps;
    s.mask = init.data();
    s.flags = BATCH_STOP_ON_EOS;
    Batch b(h->model.get());
    std::string err;
    std::vector<text::ConstrainedDecoder> dec;
    dec.reserve(B);
    for (int i = 0; i < B; ++i) dec.emplace_back(defs[slot[i]], h->vocab.v);
    if (!b.prepare(s, err) || !b.begin(err)) {
      set_err(err);
      return false;
    }
    std::vector<uint64_t> rows((size_t)B * W), bits;
    std::vector<uint32_t> tok(B), lens(B);
    std::vector<uint8_t> done(B), finished(B, 0);
    int active = B;
    for (int step = 0; step < steps && active > 0; ++step) {
      bool any = false;
      for (int i = 0; i < B; ++i) {
        uint64_t *row = rows.data() + (size_t)i * W;
        if (!finished[i] && dec[i].mask((size_t)c.vocab_size, bits)) {
          std::copy(bits.begin(), bits.end(), row);
          any = true;
        } else {
          std::fill(row, row + W, ~0ull);
        }
      }
      if (any && !b.set_mask_step(step, rows.data(), err)) {
        set_err(err);
        return false;
      }
      if (!b.step(err) || !b.peek_step(step, tok.data(), lens.data(), done.data(), err)) {
        set_err(err);
        return false;
      }
      for (int i = 0; i < B; ++i) {
        if (finished[i]) continue;
        if (done[i] || lens[i] <= (uint32_t)step) {  // EOS
          finished[i] = 1;
          --active;
          continue;
        }
        if (cb) {
          const std::string piece = h->vocab.v.piece_text(tok[i]);
          if (piece.find('\0') == std::string::npos) cb(tok[i], piece.c_str(), ud);
        }
        gen[i].push_back(tok[i]);
        dec[i].update(tok[i]);
      }
    }
  }
  const std::string tc = h->vocab.v.size() > text::kToolCallId ? h->vocab.v.piece_text(text::kToolCallId) : std::string();
  for (int i = 0; i < B; ++i) {
    std::string raw = h->vocab.v.decode_ids(gen[i]);
    if (!tc.empty() && raw.compare(0, tc.size(), tc) == 0) raw.erase(0, tc.size());
    outs[slot[i]] = text::restore_tool_names(raw, defs[slot[i]]);
  }
  return true;
}

static char *dup_text(const std::string &out) {
  if (out.find('\0') != std::string::npos) {
    set_err("output contained null byte");
    return nullptr;
  }
  char *r = (char *)std::malloc(out.size() + 1);
  if (!r) {
    set_err("out of host memory");
    return nullptr;
  }
  std::memcpy(r, out.c_str(), out.size() + 1);
  return r;
}

static char *run_text(NeedleHandle *h, const char *query, const char *tools_json, NeedleStreamCallback cb,
                      void *ud) {
  if (!h) return nullptr;
  if (!query || !tools_json) return nullptr;
  if (!valid_utf8((const uint8_t *)query, std::strlen(query)) ||
      !valid_utf8((const uint8_t *)tools_json, std::strlen(tools_json)))
    return nullptr;
  clear_err();
  std::vector<std::string> outs;
  if (!run_text_batch(h, {query}, {tools_json}, cb, ud, outs)) return nullptr;
  return dup_text(outs[0]);
}

NeedleVocab *needle_vocab_parse(const char *text, size_t len) {
  clear_err();
  if (!text && len) {
    set_err("null vocabulary text");
    return nullptr;
  }
  std::string s(text ? text : "", len);
  if (!text::utf8_valid(s)) {
    set_err("vocab is not valid UTF-8");
    return nullptr;
  }
  auto *v = new NeedleVocab();
  v->v.parse(s);
  return v;
}

const NeedleVocab *needle_handle_vocab(NeedleHandle *h) { return h ? &h->vocab : nullptr; }

size_t needle_vocab_size(const NeedleVocab *v) { return v ? v->v.size() : 0; }

size_t needle_vocab_encode(const NeedleVocab *v, const char *text, uint32_t *out, size_t cap) {
  if (!v || !text || !text::utf8_valid(text)) return (size_t)-1;
  const std::vector<uint32_t> ids = v->v.encode(text);
  if (out)
    for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  return ids.size();
}

char *needle_vocab_decode(const NeedleVocab *v, const uint32_t *ids, size_t n) {
  clear_err();
  if (!v || (!ids && n)) {
    set_err("invalid decode arguments");
    return nullptr;
  }
  return dup_text(v->v.decode_ids(std::vector<uint32_t>(ids, ids + n)));
}

void needle_vocab_free(NeedleVocab *v) { delete v; }

char *needle_snake_case(const char *name) {
  clear_err();
  if (!name || !text::utf8_valid(name)) {
    set_err("null or invalid UTF-8 name");
    return nullptr;
  }
  return dup_text(text::to_snake_case(name));
}

char *needle_tools_encoder_text(const char *tools_json) {
  clear_err();
  if (!tools_json || !text::utf8_valid(tools_json)) {
    set_err("null or invalid UTF-8 tools JSON");
    return nullptr;
  }
  const auto defs = text::parse_tools_json(tools_json);
  return dup_text(text::compact_json(text::normalize_tools_json(tools_json, defs)));
}

char *needle_tools_restore_names(const char *tools_json, const char *output) {
  clear_err();
  if (!tools_json || !output || !text::utf8_valid(tools_json) || !text::utf8_valid(output)) {
    set_err("null or invalid UTF-8 argument");
    return nullptr;
  }
  return dup_text(text::restore_tool_names(output, text::parse_tools_json(tools_json)));
}

NeedleConstraint *needle_constraint_new(const char *tools_json, const NeedleVocab *v) {
  clear_err();
  if (!tools_json || !v || !text::utf8_valid(tools_json)) {
    set_err("null vocabulary or null / invalid UTF-8 tools JSON");
    return nullptr;
  }
  auto *c = new NeedleConstraint();
  c->d = std::make_unique<text::ConstrainedDecoder>(text::parse_tools_json(tools_json), v->v);
  return c;
}

int needle_constraint_update(NeedleConstraint *c, uint32_t token) {
  if (!c) return -1;
  c->d->update(token);
  return 0;
}

int needle_constraint_feed(NeedleConstraint *c, const char *bytes, size_t len) {
  if (!c || (!bytes && len)) return -1;
  c->d->feed_bytes(std::string(bytes ? bytes : "", len));
  return 0;
}

int needle_constraint_mask(NeedleConstraint *c, size_t vocab_size, uint64_t *bits) {
  if (!c || !bits || vocab_size == 0) return -1;
  const size_t W = (vocab_size + 63) / 64;
  if (c->d->mask(vocab_size, c->bits)) {
    std::copy(c->bits.begin(), c->bits.begin() + W, bits);
    return 1;
  }
  std::fill(bits, bits + W, ~0ull);
  return 0;
}

int needle_constraint_state(const NeedleConstraint *c) {
  if (!c) return -1;
  switch (c->d->state_machine().state) {
    case text::JsonState::InName:
      return 1;
    case text::JsonState::InArgKey:
      return 2;
    default:
      return 0;
  }
}

void needle_constraint_free(NeedleConstraint *c) { delete c; }

int needle_run_batch(NeedleHandle *h, const char *const *queries, const char *const *tools_json, size_t n,
                     char **out_texts) {
  if (!h) return -1;
  clear_err();
  if (!queries || !tools_json || !out_texts || n > (size_t)INT32_MAX) {
    set_err("invalid batch arguments");
    return -1;
  }
  std::vector<std::string> q(n), t(n);
  for (size_t i = 0; i < n; ++i) {
    out_texts[i] = nullptr;
    if (!queries[i] || !tools_json[i] || !valid_utf8((const uint8_t *)queries[i], std::strlen(queries[i])) ||
        !valid_utf8((const uint8_t *)tools_json[i], std::strlen(tools_json[i]))) {
      set_err("request " + std::to_string(i) + ": null or invalid UTF-8 query or tools");
      return -1;
    }
    q[i] = queries[i];
    t[i] = tools_json[i];
  }
  std::vector<std::string> outs;
  if (!run_text_batch(h, q, t, nullptr, nullptr, outs)) return -1;
  for (size_t i = 0; i < n; ++i) {
    if (!(out_texts[i] = dup_text(outs[i]))) {
      for (size_t k = 0; k < i; ++k) {
        std::free(out_texts[k]);
        out_texts[k] = nullptr;
      }
      return -1;
    }
  }
  return 0;
}

char *needle_run(NeedleHandle *h, const char *query, const char *tools_json) {
  return run_text(h, query, tools_json, nullptr, nullptr);
}

char *needle_run_stream(NeedleHandle *h, const char *query, const char *tools_json, NeedleStreamCallback cb,
                        void *ud) {
  return run_text(h, query, tools_json, cb, ud);
}

static bool dev_check(cudaError_t e);

// encode_contrastive (engine.rs:153-181) for several texts in one
// prefill-only batch: emb [n][c_dim] (zeros for a text without tokens).
static bool contrastive_batch(NeedleHandle *h, const std::vector<std::string> &texts, std::vector<float> &emb) {
  const DevModel &m = *h->model;
  const int c = m.c_dim, d = m.cfg.d_model;
  emb.assign(texts.size() * (size_t)c, 0.0f);
  std::vector<uint32_t> ids;
  std::vector<uint64_t> off(1, 0);
  std::vector<size_t> slot;
  for (size_t i = 0; i < texts.size(); ++i) {
    const std::vector<uint32_t> t = h->vocab.v.encode(texts[i]);
    if (t.empty()) continue;
    if (t.size() > (size_t)m.cfg.max_enc_len) {
      set_err("text " + std::to_string(i) + " has " + std::to_string(t.size()) + " tokens, more than max_enc_len");
      return false;
    }
    for (uint32_t id : t)
      if (id >= (uint32_t)m.cfg.vocab_size) {
        set_err("the vocabulary has token ids beyond the model's vocab_size");
        return false;
      }
    ids.insert(ids.end(), t.begin(), t.end());
    off.push_back(ids.size());
    slot.push_back(i);
  }
  if (slot.empty()) return true;
  const int B = (int)slot.size();
  BatchSpec s;
  s.ids = ids.data();
  s.offsets = off.data();
  s.n_req = B;
  s.max_new = 0;
  s.want_enc_out = true;
  Batch b(h->model.get());
  std::string err;
  if (!b.prepare(s, err) || !b.run(err)) {
    set_err(err);
    return false;
  }
  cudaStream_t st = b.stream();
  float *dout = nullptr;
  std::vector<float> host((size_t)B * c);
  bool ok = dev_check(cudaMallocAsync(&dout, host.size() * sizeof(float), st)) &&
            dev_check(contrastive_embed(b.enc_out_dev(), b.seq_off_dev(), B, d, m.c_hk, m.c_hb, m.c_hidden, m.c_pk,
                                        c, dout, st)) &&
            dev_check(cudaMemcpyAsync(host.data(), dout, host.size() * sizeof(float), cudaMemcpyDeviceToHost, st));
  if (dout) cudaFreeAsync(dout, st);
  if (!ok || !dev_check(cudaStreamSynchronize(st))) return false;
  for (int i = 0; i < B; ++i) std::copy(&host[(size_t)i * c], &host[(size_t)(i + 1) * c], &emb[slot[i] * c]);
  return true;
}

size_t needle_contrastive_dim(NeedleHandle *h) { return h ? (size_t)h->model->c_dim : 0; }

bool needle_encode_contrastive(NeedleHandle *h, const char *text, float *out, size_t dim) {
  if (!h || !out || !text || !valid_utf8((const uint8_t *)text, std::strlen(text))) return false;
  if (!h->model->c_dim) return false;
  std::vector<float> emb;
  if (!contrastive_batch(h, {text}, emb) || emb.size() != dim) return false;
  std::copy(emb.begin(), emb.end(), out);
  return true;
}

// retrieve_tools (engine.rs:189-217): query and descriptions embedded in one
// batch, dot-product scores (sequential f32 sums), a stable sort by
// descending score in f32::total_cmp order, the first top_k written.
size_t needle_retrieve_tools(NeedleHandle *h, const char *query, const char **descs, size_t n, size_t k,
                             size_t *idx, float *scores) {
  if (!h || !query || !descs || !idx || !scores || n == 0 || k == 0) return 0;
  if (!valid_utf8((const uint8_t *)query, std::strlen(query))) return 0;
  std::vector<std::string> texts{query};
  for (size_t i = 0; i < n; ++i) {
    if (!descs[i] || !valid_utf8((const uint8_t *)descs[i], std::strlen(descs[i]))) return 0;
    texts.push_back(descs[i]);
  }
  const size_t c = (size_t)h->model->c_dim;
  if (!c) return 0;
  std::vector<float> emb;
  if (!contrastive_batch(h, texts, emb)) return 0;
  std::vector<std::pair<size_t, float>> res(n);
  for (size_t i = 0; i < n; ++i) {
    float sc = 0.0f;
    for (size_t j = 0; j < c; ++j) sc += emb[j] * emb[(i + 1) * c + j];
    res[i] = {i, sc};
  }
  auto key = [](float x) {  // f32::total_cmp as a signed integer order
    int32_t b;
    std::memcpy(&b, &x, 4);
    return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
  };
  std::stable_sort(res.begin(), res.end(),
                   [&](const auto &a, const auto &b) { return key(a.second) > key(b.second); });
  const size_t m = std::min(k, n);
  for (size_t i = 0; i < m; ++i) {
    idx[i] = res[i].first;
    scores[i] = res[i].second;
  }
  return m;
}

void needle_free_str(char *s) { std::free(s); }

void needle_free(NeedleHandle *h) { delete h; }

const char *needle_last_error(void) { return g_has_err ? g_err.c_str() : nullptr; }

int needle_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

int needle_model_config(NeedleHandle *h, int64_t *cfg) {
  if (!h || !cfg) return -1;
  const Config &c = h->model->cfg;
  int64_t v[12] = {c.d_model,   c.num_heads,   c.num_kv_heads, c.num_layers,     c.num_dec_layers, c.vocab_size,
                   c.max_enc_len, c.max_dec_len, c.ffn_dim,      c.no_feedforward, c.activation,     c.head_dim()};
  std::memcpy(cfg, v, sizeof(v));
  return 0;
}

int needle_handle_device(NeedleHandle *h) { return h ? h->model->device : -1; }

int needle_run_batch_ids(NeedleHandle *h, const uint32_t *ids, const uint64_t *off, size_t n_req, uint32_t max_new,
                         const uint64_t *mask, uint32_t flags, uint32_t *out_ids, uint32_t *out_lens) {
  return run_batch(h, ids, off, n_req, max_new, mask, flags, out_ids, out_lens, nullptr);
}

int needle_run_batch_ids_logits(NeedleHandle *h, const uint32_t *ids, const uint64_t *off, size_t n_req,
                                uint32_t max_new, const uint64_t *mask, uint32_t flags, uint32_t *out_ids,
                                uint32_t *out_lens, float *logits) {
  return run_batch(h, ids, off, n_req, max_new, mask, flags, out_ids, out_lens, logits);
}

NeedleBatch *needle_batch_prepare(NeedleHandle *h, const uint32_t *ids, const uint64_t *off, size_t n_req,
                                  uint32_t max_new, const uint64_t *mask, uint32_t flags) {
  if (!h) return nullptr;
  clear_err();
  auto nb = std::make_unique<NeedleBatch>();
  nb->h = h;
  if (!make_spec(h, ids, off, n_req, max_new, mask, flags, nb->spec)) return nullptr;
  nb->offsets.assign(off, off + n_req + 1);
  nb->spec.offsets = nb->offsets.data();
  nb->batch = std::make_unique<Batch>(h->model.get());
  std::string err;
  if (!nb->batch->prepare(nb->spec, err)) {
    set_err(err);
    return nullptr;
  }
  return nb.release();
}

int needle_batch_run(NeedleBatch *nb) {
  if (!nb) return -1;
  clear_err();
  std::string err;
  nb->batch->set_timed_class(nb->timed_cls);
  if (!nb->batch->run(err)) {
    set_err(err);
    return -1;
  }
  return 0;
}

int needle_batch_sync(NeedleBatch *nb) {
  if (!nb) return -1;
  cudaError_t e = cudaStreamSynchronize(nb->batch->stream());
  if (e != cudaSuccess) {
    set_err(std::string("cudaStreamSynchronize failed: ") + cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

int needle_batch_results(NeedleBatch *nb, uint32_t *out_ids, uint32_t *out_lens) {
  if (!nb) return -1;
  std::string err;
  if (!nb->batch->download(out_ids, out_lens, nullptr, nullptr, err)) {
    set_err(err);
    return -1;
  }
  return 0;
}

int needle_batch_begin(NeedleBatch *nb) {
  if (!nb) return -1;
  clear_err();
  std::string err;
  nb->batch->set_timed_class(nb->timed_cls);
  if (!nb->batch->begin(err)) {
    set_err(err);
    return -1;
  }
  nb->next_step = 0;
  return 0;
}

int needle_batch_set_step_mask(NeedleBatch *nb, uint32_t step, const uint64_t *rows) {
  if (!nb || !rows) return -1;
  clear_err();
  std::string err;
  if (!nb->batch->set_mask_step((int)step, rows, err)) {
    set_err(err);
    return -1;
  }
  return 0;
}

int needle_batch_step(NeedleBatch *nb, uint32_t *tokens, uint32_t *lens, uint8_t *done) {
  if (!nb) return -1;
  clear_err();
  if (nb->next_step < 0) {
    set_err("needle_batch_begin must run first");
    return -1;
  }
  std::string err;
  const int step = nb->next_step;
  std::vector<uint32_t> tk(tokens ? 0 : nb->spec.n_req), ln(lens ? 0 : nb->spec.n_req);
  std::vector<uint8_t> dn(done ? 0 : nb->spec.n_req);
  if (!nb->batch->step(err) ||
      !nb->batch->peek_step(step, tokens ? tokens : tk.data(), lens ? lens : ln.data(), done ? done : dn.data(),
                            err)) {
    set_err(err);
    return -1;
  }
  ++nb->next_step;
  return 0;
}

void *needle_batch_stream(NeedleBatch *nb) { return nb ? (void *)nb->batch->stream() : nullptr; }

int64_t needle_batch_kernel_launches(NeedleBatch *nb) { return nb ? nb->batch->kernels_launched() : -1; }

int needle_batch_time_kernel(NeedleBatch *nb, int kernel_class) {
  if (!nb || kernel_class < 0 || kernel_class > 7) return -1;
  nb->timed_cls = kernel_class;
  return 0;
}

int needle_batch_kernel_timing(NeedleBatch *nb, double *ms_total, int64_t *launches, double *flops,
                               double *bytes) {
  if (!nb) return -1;
  std::string err;
  if (!nb->batch->collect_timing(err)) {
    set_err(err);
    return -1;
  }
  if (ms_total) *ms_total = nb->batch->timed_ms();
  if (launches) *launches = nb->batch->timed_launches();
  if (flops) *flops = nb->batch->timed_flops();
  if (bytes) *bytes = nb->batch->timed_bytes();
  return 0;
}

void needle_batch_free(NeedleBatch *nb) { delete nb; }

int needle_shard_requests(const uint64_t *off, size_t n_req, int shards, int32_t *assignment) {
  if (!off || !assignment || shards <= 0) {
    set_err("invalid shard arguments");
    return -1;
  }
  shard_requests(off, (int)n_req, shards, assignment);
  return 0;
}

int needle_debug_forward(NeedleHandle *h, const uint32_t *enc_ids, size_t n_enc, const uint32_t *dec_ids,
                         size_t n_dec, float *enc_out, float *logits) {
  if (!h) return -1;
  clear_err();
  if (!enc_ids || n_enc == 0 || (n_dec && !dec_ids)) {
    set_err("invalid arguments");
    return -1;
  }
  uint64_t off[2] = {0, n_enc};
  BatchSpec s;
  s.ids = enc_ids;
  s.offsets = off;
  s.n_req = 1;
  s.max_new = (int)n_dec;
  s.teacher = dec_ids;
  s.want_logits = logits != nullptr;
  s.want_enc_out = enc_out != nullptr;
  s.flags = BATCH_NO_GRAPH;
  Batch b(h->model.get());
  std::string err;
  for (size_t i = 0; i < n_dec; ++i)
    if (dec_ids[i] >= (uint32_t)h->model->cfg.vocab_size) {
      set_err("decoder token id out of range");
      return -1;
    }
  if (!b.prepare(s, err) || !b.run(err) || !b.download(nullptr, nullptr, logits, enc_out, err)) {
    set_err(err);
    return -1;
  }
  return 0;
}

static bool dev_check(cudaError_t e) {
  if (e != cudaSuccess) {
    set_err(std::string("CUDA error: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

static bool ensure_kernels() {
  static std::mutex mu;
  static std::vector<bool> done;
  int dev = 0;
  if (!dev_check(cudaGetDevice(&dev))) return false;
  std::lock_guard<std::mutex> g(mu);
  if ((int)done.size() <= dev) done.resize(dev + 1, false);
  if (!done[dev]) {
    if (!dev_check(init_kernels())) return false;
    done[dev] = true;
  }
  return true;
}

static int *device_err_flag() {
  static std::mutex mu;
  static std::vector<int *> flags;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if ((int)flags.size() <= dev) flags.resize(dev + 1, nullptr);
  if (!flags[dev]) {
    if (cudaMalloc(&flags[dev], sizeof(int)) != cudaSuccess || cudaMemset(flags[dev], 0, sizeof(int)) != cudaSuccess)
      flags[dev] = nullptr;
  }
  return flags[dev];
}

// The standalone INT4 matmul takes the tensor-core GEMM from 9 rows: the
// CUDA-core kernels spread only the output columns over CTAs, so between 9
// and 127 rows a narrow W leaves most SMs idle.  x is staged in planes of at
// least one 128-row tile; the rows past M are never stored.
constexpr int kTcMinRowsOp = 9;
inline int tc_stage_rows(int M) { return M < 128 ? 128 : M; }

// Y = x @ W with the tensor-core GEMM (W and x staged as bf16 hi/lo planes in
// per-call device buffers) from kTcMinRowsOp rows, the CUDA-core kernels
// below.
static bool matmul_any(const float *x, int64_t ldx, int M, const Int4Weight &W, const MatmulOut &o, cudaStream_t st) {
  const bool aligned = ((uintptr_t)o.y % 16 == 0) && (o.ldy % 4 == 0);
  if (M < kTcMinRowsOp || !aligned) return dev_check(int4_matmul(x, ldx, M, W, o, st));
  int *flag = device_err_flag();
  if (!flag) {
    set_err("device error flag allocation failed");
    return false;
  }
  const int Kp = tc_padded_k(W.K);
  void *buf = nullptr;
  size_t wbytes = (size_t)W.N * Kp * 2, xbytes = (size_t)tc_stage_rows(M) * Kp * 2;
  wbytes = (wbytes + 255) & ~(size_t)255;
  xbytes = (xbytes + 255) & ~(size_t)255;
  if (!dev_check(cudaMallocAsync(&buf, 2 * wbytes + 2 * xbytes + tc_splitk_ws_bytes() + 1024, st))) return false;
  char *b = (char *)(((uintptr_t)buf + 255) & ~(uintptr_t)255);
  void *wh = b, *wl = b + wbytes, *xh = b + 2 * wbytes, *xl = b + 2 * wbytes + xbytes;
  MatmulOut os = o;
  os.splitk_ws = (float *)(b + 2 * wbytes + 2 * xbytes);
  TcPlanes A, B;
  bool ok = dev_check(tc_make_planes(wh, wl, W.N, Kp, 128, B)) &&
            dev_check(tc_make_planes(xh, xl, tc_stage_rows(M), Kp, 128, A)) &&
            dev_check(tc_prep_weight(W, Kp, wh, wl, st)) && dev_check(tc_split_rows(x, ldx, M, W.K, Kp, xh, xl, st)) &&
            dev_check(tc_matmul(A, M, B, W.N, os, flag, st));
  cudaFreeAsync(buf, st);
  if (!ok) return false;
  int kerr = 0;
  if (!dev_check(cudaMemcpyAsync(&kerr, flag, sizeof(int), cudaMemcpyDeviceToHost, st)) ||
      !dev_check(cudaStreamSynchronize(st)))
    return false;
  if (kerr) {
    cudaMemset(flag, 0, sizeof(int));
    set_err("a tensor-core GEMM wait timed out");
    return false;
  }
  return true;
}

int needle_int4_matmul(const float *x, size_t M, size_t K, const uint8_t *w, const float *s, size_t N, size_t G,
                       float *y, void *stream) {
  clear_err();
  if (!x || !w || !s || !y || M == 0 || K == 0 || N == 0 || G == 0 || M > INT32_MAX || K > INT32_MAX ||
      N > INT32_MAX || G > INT32_MAX) {
    set_err("invalid matmul arguments");
    return -1;
  }
  if (!ensure_kernels()) return -1;
  Int4Weight W{w, s, (int)K, (int)N, (int)G, (int)(K < 32 ? K : 32)};
  MatmulOut o;
  o.y = y;
  o.ldy = (int64_t)N;
  return matmul_any(x, (int64_t)K, (int)M, W, o, (cudaStream_t)stream) ? 0 : -1;
}

int needle_int4_matmul_ex(const float *x, size_t M, size_t K, const uint8_t *w, const float *s, size_t N, size_t G,
                          float *y, uint32_t flags, void *stream) {
  clear_err();
  if (!x || !w || !s || !y || M == 0 || K == 0 || N == 0 || G == 0 || M > INT32_MAX || K > INT32_MAX ||
      N > INT32_MAX || G > INT32_MAX || (flags & ~NEEDLE_INT4_OVERLAP)) {
    set_err("invalid matmul arguments");
    return -1;
  }
  if (!ensure_kernels()) return -1;
  Int4Weight W{w, s, (int)K, (int)N, (int)G, (int)(K < 32 ? K : 32)};
  MatmulOut o;
  o.y = y;
  o.ldy = (int64_t)N;
  if (M < (size_t)kTcMinRowsOp)
    return dev_check(int4_matmul(x, (int64_t)K, (int)M, W, o, (cudaStream_t)stream, (flags & NEEDLE_INT4_OVERLAP) != 0))
               ? 0
               : -1;
  return matmul_any(x, (int64_t)K, (int)M, W, o, (cudaStream_t)stream) ? 0 : -1;
}

}  // extern "C"

struct NeedleInt4Plan {
  int device = 0;
  ndl::Int4Weight W{};
  int Kp = 0, max_m = 0;
  void *buf = nullptr;  // weight hi/lo planes, x hi/lo planes, split-K workspace
  ndl::TcPlanes A, B;
  float *ws = nullptr;
  bool tc = false;
  int *flag = nullptr;
};

extern "C" {

NeedleInt4Plan *needle_int4_plan_create(const uint8_t *w, const float *s, size_t K, size_t N, size_t G, size_t max_m,
                                        void *stream) {
  clear_err();
  if (!w || !s || K == 0 || N == 0 || G == 0 || max_m == 0 || K > INT32_MAX || N > INT32_MAX || G > INT32_MAX ||
      max_m > INT32_MAX) {
    set_err("invalid plan arguments");
    return nullptr;
  }
  if (!ensure_kernels()) return nullptr;
  auto *p = new NeedleInt4Plan();
  cudaGetDevice(&p->device);
  p->W = Int4Weight{w, s, (int)K, (int)N, (int)G, (int)(K < 32 ? K : 32)};
  p->max_m = (int)max_m;
  p->tc = max_m >= (size_t)kTcMinRowsOp;
  if (p->tc) {
    cudaStream_t st = (cudaStream_t)stream;
    p->Kp = tc_padded_k((int)K);
    size_t wbytes = N * (size_t)p->Kp * 2, xbytes = (size_t)tc_stage_rows((int)max_m) * p->Kp * 2;
    wbytes = (wbytes + 255) & ~(size_t)255;
    xbytes = (xbytes + 255) & ~(size_t)255;
    p->flag = device_err_flag();
    if (!p->flag || !dev_check(cudaMalloc(&p->buf, 2 * wbytes + 2 * xbytes + tc_splitk_ws_bytes() + 1024))) {
      if (!p->flag) set_err("device error flag allocation failed");
      delete p;
      return nullptr;
    }
    char *b = (char *)(((uintptr_t)p->buf + 255) & ~(uintptr_t)255);
    void *wh = b, *wl = b + wbytes, *xh = b + 2 * wbytes, *xl = b + 2 * wbytes + xbytes;
    p->ws = (float *)(b + 2 * wbytes + 2 * xbytes);
    if (!dev_check(tc_make_planes(wh, wl, (int)N, p->Kp, 128, p->B)) ||
        !dev_check(tc_make_planes(xh, xl, tc_stage_rows((int)max_m), p->Kp, 128, p->A)) ||
        !dev_check(tc_prep_weight(p->W, p->Kp, wh, wl, st)) || !dev_check(cudaStreamSynchronize(st))) {
      cudaFree(p->buf);
      delete p;
      return nullptr;
    }
  }
  return p;
}

int needle_int4_plan_matmul(NeedleInt4Plan *p, const float *x, size_t M, float *y, uint32_t flags, void *stream) {
  clear_err();
  if (!p || !x || !y || M == 0 || M > (size_t)p->max_m || (flags & ~NEEDLE_INT4_OVERLAP)) {
    set_err("invalid plan matmul arguments");
    return -1;
  }
  cudaStream_t st = (cudaStream_t)stream;
  MatmulOut o;
  o.y = y;
  o.ldy = (int64_t)p->W.N;
  o.splitk_ws = p->ws;
  if (!p->tc || M < (size_t)kTcMinRowsOp || ((uintptr_t)y % 16) != 0 || (p->W.N % 4) != 0)
    return dev_check(int4_matmul(x, (int64_t)p->W.K, (int)M, p->W, o, st, (flags & NEEDLE_INT4_OVERLAP) != 0)) ? 0
                                                                                                              : -1;
  if (!dev_check(tc_split_rows(x, (int64_t)p->W.K, (int)M, p->W.K, p->Kp, const_cast<void *>(p->A.hi_ptr), const_cast<void *>(p->A.lo_ptr), st)) ||
      !dev_check(tc_matmul(p->A, (int)M, p->B, p->W.N, o, p->flag, st)))
    return -1;
  return 0;
}

int needle_int4_plan_status(NeedleInt4Plan *p) {
  clear_err();
  if (!p) {
    set_err("null plan");
    return -1;
  }
  if (!p->flag) return dev_check(cudaDeviceSynchronize()) ? 0 : -1;
  int kerr = 0;
  if (!dev_check(cudaDeviceSynchronize()) || !dev_check(cudaMemcpy(&kerr, p->flag, sizeof(int), cudaMemcpyDeviceToHost)))
    return -1;
  if (kerr) {
    cudaMemset(p->flag, 0, sizeof(int));
    set_err("a tensor-core GEMM wait timed out");
    return -1;
  }
  return 0;
}

void needle_int4_plan_free(NeedleInt4Plan *p) {
  if (!p) return;
  if (p->buf) {
    cudaDeviceSynchronize();
    cudaFree(p->buf);
  }
  delete p;
}

}  // extern "C"

// A prepared MLP block (ffn_forward, crates/needle-core/src/ffn.rs:19-56):
// gate and up interleaved into one weight, its bf16 hi/lo staging and the
// down projection's, plus the per-call workspace (x planes, hidden planes,
// f32 hidden for the CUDA-core path), all allocated at creation.
struct NeedleFfnPlan {
  int device = 0;
  int d = 0, ff = 0, max_t = 0, Kd = 0, Kf = 0;
  ndl::Int4Weight gu{}, dn{};
  bool tc = false;
  void *buf = nullptr;
  float *hidden = nullptr;  // [max_t][ff] for the CUDA-core path
  ndl::TcPlanes Wgu, Wdn, X, H;
  float *ws = nullptr;  // split-K workspace
  int *flag = nullptr;
};

extern "C" {

NeedleFfnPlan *needle_ffn_plan_create(size_t d, size_t ff, const uint8_t *gd, const float *gs, const uint8_t *ud,
                                      const float *us, const uint8_t *dd, const float *ds, size_t max_t,
                                      void *stream) {
  clear_err();
  if (!gd || !gs || !ud || !us || !dd || !ds || d == 0 || ff == 0 || max_t == 0 || d > (1u << 20) ||
      ff > (1u << 20) || max_t > INT32_MAX || max_t * ff > ((size_t)1 << 34)) {
    set_err("invalid ffn plan arguments");
    return nullptr;
  }
  if (!ensure_kernels()) return nullptr;
  auto *p = new NeedleFfnPlan();
  cudaGetDevice(&p->device);
  p->d = (int)d;
  p->ff = (int)ff;
  p->max_t = (int)max_t;
  const int gs1 = (int)(d < 32 ? d : 32), gs2 = (int)(ff < 32 ? ff : 32);
  p->gu = Int4Weight{gd, gs, (int)d, (int)(2 * ff), (int)((d + gs1 - 1) / gs1), gs1};
  p->gu.w2 = ud;
  p->gu.s2 = us;
  p->dn = Int4Weight{dd, ds, (int)ff, (int)d, (int)((ff + gs2 - 1) / gs2), gs2};
  p->tc = max_t >= (size_t)kTcMinRowsOp && d % 4 == 0;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t hbytes = max_t * ff * sizeof(float);
  size_t total = hbytes + 256;
  size_t wgu = 0, wdn = 0, xb = 0, hb = 0;
  if (p->tc) {
    p->Kd = tc_padded_k((int)d);
    p->Kf = tc_padded_k((int)ff);
    const size_t rows = (size_t)tc_stage_rows((int)max_t);
    wgu = 2 * ff * (size_t)p->Kd * 2;
    wdn = d * (size_t)p->Kf * 2;
    xb = rows * p->Kd * 2;
    hb = rows * p->Kf * 2;
    total += 2 * (wgu + wdn + xb + hb) + tc_splitk_ws_bytes() + 9 * 256;
    p->flag = device_err_flag();
    if (!p->flag) {
      set_err("device error flag allocation failed");
      delete p;
      return nullptr;
    }
  }
  if (!dev_check(cudaMalloc(&p->buf, total))) {
    delete p;
    return nullptr;
  }
  char *b = (char *)(((uintptr_t)p->buf + 255) & ~(uintptr_t)255);
  auto take = [&](size_t n) {
    char *r = b;
    b += (n + 255) & ~(size_t)255;
    return (void *)r;
  };
  p->hidden = (float *)take(hbytes);
  bool ok = true;
  if (p->tc) {
    void *guh = take(wgu), *gul = take(wgu), *dnh = take(wdn), *dnl = take(wdn);
    void *xh = take(xb), *xl = take(xb), *hh = take(hb), *hl = take(hb);
    p->ws = (float *)take(tc_splitk_ws_bytes());
    const int rows = tc_stage_rows((int)max_t);
    // the hidden planes' pad columns (ff .. Kf) are never written: zero them once
    ok = dev_check(cudaMemsetAsync(hh, 0, hb, st)) && dev_check(cudaMemsetAsync(hl, 0, hb, st)) &&
         dev_check(tc_make_planes(guh, gul, (int)(2 * ff), p->Kd, 128, p->Wgu)) &&
         dev_check(tc_make_planes(dnh, dnl, (int)d, p->Kf, 128, p->Wdn)) &&
         dev_check(tc_make_planes(xh, xl, rows, p->Kd, 128, p->X)) &&
         dev_check(tc_make_planes(hh, hl, rows, p->Kf, 128, p->H)) &&
         dev_check(tc_prep_weight(p->gu, p->Kd, guh, gul, st)) && dev_check(tc_prep_weight(p->dn, p->Kf, dnh, dnl, st));
  }
  if (!ok || !dev_check(cudaStreamSynchronize(st))) {
    cudaFree(p->buf);
    delete p;
    return nullptr;
  }
  return p;
}

int needle_ffn_plan_forward(NeedleFfnPlan *p, const float *x, size_t T, int act, float *out, void *stream) {
  clear_err();
  if (!p || !x || !out || T == 0 || T > (size_t)p->max_t || act < 0 || act > 2) {
    set_err("invalid ffn plan arguments");
    return -1;
  }
  cudaStream_t st = (cudaStream_t)stream;
  MatmulOut o;
  o.y = out;
  o.ldy = p->d;
  o.splitk_ws = p->ws;
  if (!p->tc || T < (size_t)kTcMinRowsOp || ((uintptr_t)out % 16) || (p->d % 4)) {
    MatmulOut a;
    a.y = p->hidden;
    a.ldy = p->ff;
    a.epi = EPI_ACT;
    a.act = act;
    return dev_check(int4_matmul(x, p->d, (int)T, p->gu, a, st)) &&
                   dev_check(int4_matmul(p->hidden, p->ff, (int)T, p->dn, o, st))
               ? 0
               : -1;
  }
  // x -> bf16 planes; gate|up GEMM whose epilogue writes act(gate) * up as the
  // down projection's operand planes; down GEMM into out
  MatmulOut a;
  a.epi = EPI_ACT;
  a.act = act;
  a.planes[0] = const_cast<void *>(p->H.hi_ptr);
  a.planes[1] = const_cast<void *>(p->H.lo_ptr);
  a.ldy = p->Kf;
  a.splitk_ws = p->ws;
  return dev_check(tc_split_rows(x, p->d, (int)T, p->d, p->Kd, const_cast<void *>(p->X.hi_ptr),
                                 const_cast<void *>(p->X.lo_ptr), st)) &&
                 dev_check(tc_matmul(p->X, (int)T, p->Wgu, 2 * p->ff, a, p->flag, st)) &&
                 dev_check(tc_matmul(p->H, (int)T, p->Wdn, p->d, o, p->flag, st))
             ? 0
             : -1;
}

int needle_ffn_plan_status(NeedleFfnPlan *p) {
  clear_err();
  if (!p) {
    set_err("null plan");
    return -1;
  }
  if (!dev_check(cudaDeviceSynchronize())) return -1;
  if (!p->flag) return 0;
  int kerr = 0;
  if (!dev_check(cudaMemcpy(&kerr, p->flag, sizeof(int), cudaMemcpyDeviceToHost))) return -1;
  if (kerr) {
    cudaMemset(p->flag, 0, sizeof(int));
    set_err("a tensor-core GEMM wait timed out");
    return -1;
  }
  return 0;
}

void needle_ffn_plan_free(NeedleFfnPlan *p) {
  if (!p) return;
  if (p->buf) {
    cudaDeviceSynchronize();
    cudaFree(p->buf);
  }
  delete p;
}

int needle_int4_quantize(const float *w, size_t K, size_t N, uint8_t *data, float *scales, void *stream) {
  clear_err();
  if (!w || !data || !scales || K == 0 || N == 0 || K > INT32_MAX || N > INT32_MAX) {
    set_err("invalid quantize arguments");
    return -1;
  }
  if (!ensure_kernels()) return -1;
  return dev_check(int4_quantize(w, (int)K, (int)N, data, scales, (cudaStream_t)stream)) ? 0 : -1;
}

int needle_int4_dequantize(const uint8_t *data, const float *scales, size_t K, size_t N, size_t G, float *out,
                           void *stream) {
  clear_err();
  if (!data || !scales || !out || K == 0 || N == 0 || G == 0 || K > INT32_MAX || N > INT32_MAX) {
    set_err("invalid dequantize arguments");
    return -1;
  }
  if (!ensure_kernels()) return -1;
  return dev_check(int4_dequantize(data, scales, (int)K, (int)N, (int)G, out, (cudaStream_t)stream)) ? 0 : -1;
}

int needle_ffn_forward(const float *x, size_t T, size_t d, size_t ff, const uint8_t *gd, const float *gs,
                       const uint8_t *ud, const float *us, const uint8_t *dd, const float *ds, int act, float *out,
                       void *stream) {
  clear_err();
  if (!x || !gd || !gs || !ud || !us || !dd || !ds || !out || T == 0 || d == 0 || ff == 0 || act < 0 || act > 2 ||
      T > INT32_MAX || d > INT32_MAX || ff > INT32_MAX) {
    set_err("invalid ffn arguments");
    return -1;
  }
  if (!ensure_kernels()) return -1;
  cudaStream_t st = (cudaStream_t)stream;
  int gsz = (int)(d < 32 ? d : 32), gsd = (int)(ff < 32 ? ff : 32);
  int G1 = (int)((d + gsz - 1) / gsz), G2 = (int)((ff + gsd - 1) / gsd);
  float *hid = nullptr;
  if (!dev_check(cudaMallocAsync((void **)&hid, T * ff * sizeof(float), st))) return -1;
  Int4Weight gu{gd, gs, (int)d, (int)(2 * ff), G1, gsz};
  gu.w2 = ud;
  gu.s2 = us;
  MatmulOut a;
  a.y = hid;
  a.ldy = (int64_t)ff;
  a.epi = EPI_ACT;
  a.act = act;
  bool ok = matmul_any(x, (int64_t)d, (int)T, gu, a, st);
  if (ok) {
    Int4Weight dn{dd, ds, (int)ff, (int)d, G2, gsd};
    MatmulOut o;
    o.y = out;
    o.ldy = (int64_t)d;
    ok = matmul_any(hid, (int64_t)ff, (int)T, dn, o, st);
  }
  cudaFreeAsync(hid, st);
  return ok ? 0 : -1;
}

}  // extern "C"

// ── SafeTensors reader (crates/needle-infer/src/safetensors.rs) ──

struct NeedleSafeTensors {
  ndl::SafeTensors st;
};

extern "C" {

NeedleSafeTensors *needle_safetensors_parse(const uint8_t *data, size_t len) {
  clear_err();
  if (!data && len) {
    set_err("null pointer passed to needle_safetensors_parse");
    return nullptr;
  }
  auto *p = new NeedleSafeTensors();
  std::string err;
  if (!p->st.parse(std::vector<uint8_t>(data, data + len), err)) {
    set_err("SafeTensors error: " + err);
    delete p;
    return nullptr;
  }
  return p;
}

const char *needle_safetensors_metadata(const NeedleSafeTensors *p, const char *key) {
  if (!p || !key) return nullptr;
  const std::string *v = p->st.metadata(key);
  return v ? v->c_str() : nullptr;
}

size_t needle_safetensors_get_f32(const NeedleSafeTensors *p, const char *name, float *out, size_t cap) {
  if (!p || !name) return (size_t)-1;
  std::vector<float> v;
  if (!p->st.get_f32(name, v)) return (size_t)-1;
  if (out) std::memcpy(out, v.data(), std::min(cap, v.size()) * sizeof(float));
  return v.size();
}

void needle_safetensors_free(NeedleSafeTensors *p) { delete p; }

}  // extern "C"
