// engine.cpp — see engine.h.
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <numeric>

#include <cuda_bf16.h>

namespace ndl {

#define NDL_CK(call)                                                                 \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    if (e_ != cudaSuccess) {                                                         \
      err = std::string(#call) + " failed: " + cudaGetErrorString(e_);               \
      return false;                                                                  \
    }                                                                                \
  } while (0)

const char *Config::validate() const {  // config.rs:83-103
  if (num_heads <= 0) return "num_heads must be > 0";
  if (num_kv_heads <= 0) return "num_kv_heads must be > 0";
  if (d_model <= 0) return "d_model must be > 0";
  if (d_model % num_heads) return "d_model must be divisible by num_heads";
  if (num_heads % num_kv_heads) return "num_heads must be divisible by num_kv_heads";
  if (vocab_size <= 0) return "vocab_size must be > 0";
  return nullptr;
}

DevModel::~DevModel() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  for (void *p : allocs) cudaFree(p);
  if (stream) cudaStreamDestroy(stream);
  cudaSetDevice(prev);
}

namespace {

struct HostQW {
  std::vector<uint8_t> data;
  std::vector<float> scales;
  int K = 0, N = 0, G = 0, gs = 0;
};

bool parse_usize(const std::string &s, long long &out) {
  size_t i = (!s.empty() && s[0] == '+') ? 1 : 0;
  if (i >= s.size() || s.size() - i > 18) return false;
  for (size_t j = i; j < s.size(); ++j)
    if (s[j] < '0' || s[j] > '9') return false;
  out = std::stoll(s.substr(i));
  return true;
}

// engine.rs:578-624
Config load_config(const SafeTensors &st) {
  Config d, c;
  auto uf = [&](const char *k, int fb) {
    const std::string *v = st.metadata(k);
    long long x;
    return (v && parse_usize(*v, x) && x <= (1LL << 30)) ? (int)x : fb;
  };
  auto ff = [&](const char *k, float fb) {
    const std::string *v = st.metadata(k);
    if (!v || v->empty()) return fb;
    char *e = nullptr;
    float x = std::strtof(v->c_str(), &e);
    return (e && *e == 0) ? x : fb;
  };
  auto bf = [&](const char *k, bool fb) {
    const std::string *v = st.metadata(k);
    return v ? (*v == "True" || *v == "true" || *v == "1") : fb;
  };
  long long me;
  const std::string *v;
  if ((v = st.metadata("max_enc_len")) && parse_usize(*v, me) && me <= (1LL << 30))
    c.max_enc_len = (int)me;
  else if ((v = st.metadata("max_seq_len")) && parse_usize(*v, me) && me <= (1LL << 30))
    c.max_enc_len = (int)me;
  else
    c.max_enc_len = d.max_enc_len;
  c.activation = ACT_DRELU;
  if ((v = st.metadata("activation"))) c.activation = *v == "swiglu" ? ACT_SWIGLU : *v == "geglu" ? ACT_GELU : ACT_DRELU;
  c.d_model = uf("d_model", d.d_model);
  c.num_heads = uf("num_heads", d.num_heads);
  c.num_kv_heads = uf("num_kv_heads", d.num_kv_heads);
  c.num_layers = uf("num_encoder_layers", d.num_layers);
  c.num_dec_layers = uf("num_decoder_layers", d.num_dec_layers);
  c.vocab_size = uf("vocab_size", d.vocab_size);
  c.max_dec_len = uf("max_dec_len", d.max_dec_len);
  c.ffn_dim = uf("ffn_dim", d.ffn_dim);
  c.no_feedforward = bf("no_feedforward", d.no_feedforward);
  c.rope_theta = ff("rope_theta", d.rope_theta);
  return c;
}

struct Loader {
  const SafeTensors &st;
  DevModel &m;
  std::string &err;

  template <class T>
  bool dalloc(T *&p, size_t n) {
    void *q = nullptr;
    NDL_CK(cudaMalloc(&q, std::max<size_t>(n, 1) * sizeof(T)));
    m.allocs.push_back(q);
    m.weight_bytes += n * sizeof(T);
    p = (T *)q;
    return true;
  }
  template <class T>
  bool upload(T *&p, const T *src, size_t n) {
    if (!dalloc(p, n)) return false;
    NDL_CK(cudaMemcpy(p, src, n * sizeof(T), cudaMemcpyHostToDevice));
    return true;
  }
  bool vec(const std::string &name, size_t len, float *&p) {  // engine.rs:784-786
    std::vector<float> v;
    if (!st.get_f32(name, v)) v.assign(len, 0.0f);
    if (v.size() < len) {  // the reference would index past the end
      err = name + ": expected " + std::to_string(len) + " values, found " + std::to_string(v.size());
      return false;
    }
    v.resize(len);
    return upload(p, v.data(), len);
  }
  bool vec_host(const std::string &name, size_t len, std::vector<float> &v) {
    if (!st.get_f32(name, v)) v.assign(len, 0.0f);
    if (v.size() < len) {
      err = name + ": expected " + std::to_string(len) + " values, found " + std::to_string(v.size());
      return false;
    }
    v.resize(len);
    return true;
  }
  float gate(const std::string &name) {  // engine.rs:788-792, then ops.rs:40-42 sigmoid
    std::vector<float> v;
    float g = (st.get_f32(name, v) && !v.empty()) ? v[0] : 0.0f;
    return 1.0f / (1.0f + std::exp(-g));
  }
  bool quantize_dev(const std::vector<float> &w, int K, int N, HostQW &q) {
    int gs = K < 32 ? K : 32;
    if (gs <= 0 || (gs & 1)) {
      err = "in_feat " + std::to_string(K) + " below 32 must be even to pack pairs";
      return false;
    }
    int Kp = K + (gs - K % gs) % gs, G = Kp / gs;
    q.K = K;
    q.N = N;
    q.G = G;
    q.gs = gs;
    q.data.assign((size_t)Kp / 2 * N, 0);
    q.scales.assign((size_t)G * N, 0.0f);
    float *dw = nullptr, *ds = nullptr;
    uint8_t *dd = nullptr;
    NDL_CK(cudaMalloc(&dw, w.size() * sizeof(float) + 16));
    NDL_CK(cudaMalloc(&dd, q.data.size() + 16));
    NDL_CK(cudaMalloc(&ds, q.scales.size() * sizeof(float) + 16));
    bool ok = cudaMemcpy(dw, w.data(), w.size() * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess &&
              int4_quantize(dw, K, N, dd, ds, m.stream) == cudaSuccess &&
              cudaMemcpyAsync(q.data.data(), dd, q.data.size(), cudaMemcpyDeviceToHost, m.stream) == cudaSuccess &&
              cudaMemcpyAsync(q.scales.data(), ds, q.scales.size() * sizeof(float), cudaMemcpyDeviceToHost,
                              m.stream) == cudaSuccess &&
              cudaStreamSynchronize(m.stream) == cudaSuccess;
    cudaFree(dw);
    cudaFree(dd);
    cudaFree(ds);
    if (!ok) err = "device quantization failed";
    return ok;
  }
  // engine.rs:752-782
  bool quant(const std::string &name, int K, int N, HostQW &q) {
    size_t rawlen = 0;
    const uint8_t *raw = st.get_raw(name, &rawlen);
    std::vector<float> scales;
    if (raw && st.get_f32(name + ".scale", scales)) {
      if (N == 0 || scales.size() % (size_t)N != 0) {
        std::fprintf(stderr, "Warning: %s.scale length %zu is not divisible by out_feat %d; re-quantizing\n",
                     name.c_str(), scales.size(), N);
        std::vector<float> w;
        if (!st.get_f32(name, w)) w.assign((size_t)K * N, 0.0f);
        if (w.size() != (size_t)K * N) {
          err = name + ": cannot re-quantize a tensor of " + std::to_string(w.size()) + " values";
          return false;
        }
        return quantize_dev(w, K, N, q);
      }
      q.K = K;
      q.N = N;
      q.G = (int)(scales.size() / N);
      q.gs = K < 32 ? K : 32;
      if (q.gs & 1) {
        err = name + ": odd group size";
        return false;
      }
      size_t need = (size_t)q.G * q.gs / 2 * N;
      if (rawlen < need) {
        err = name + ": packed data holds " + std::to_string(rawlen) + " bytes, its scales need " +
              std::to_string(need);
        return false;
      }
      q.data.assign(raw, raw + need);
      q.scales = std::move(scales);
      return true;
    }
    std::vector<float> w;
    if (!st.get_f32(name, w)) {
      std::fprintf(stderr, "Warning: missing tensor %s, using zeros\n", name.c_str());
      w.assign((size_t)K * N, 0.0f);
    }
    if (w.size() != (size_t)K * N) {
      err = name + ": expected " + std::to_string((size_t)K * N) + " values, found " + std::to_string(w.size());
      return false;
    }
    return quantize_dev(w, K, N, q);
  }
  bool put(const HostQW &q, Lin &l) {
    l.K = q.K;
    l.N = q.N;
    l.G = q.G;
    l.gs = q.gs;
    if (!upload(l.w, q.data.data(), q.data.size()) || !upload(l.s, q.scales.data(), q.scales.size())) return false;
    // bf16 hi/lo staging planes for the tensor-core GEMM
    const int Kp = tc_padded_k(l.K);
    __nv_bfloat16 *hi = nullptr, *lo = nullptr;
    if (!dalloc(hi, (size_t)l.N * Kp) || !dalloc(lo, (size_t)l.N * Kp)) return false;
    NDL_CK(tc_prep_weight(l.view(), Kp, hi, lo, m.stream));
    NDL_CK(cudaStreamSynchronize(m.stream));
    l.tc_hi = hi;
    l.tc_lo = lo;
    l.tc_ready = tc_make_planes(hi, lo, l.N, Kp, 128, l.tc) == cudaSuccess;
    return true;
  }
};

// Concatenate along N (the reference layout keeps each pair-row contiguous
// over N, so this is a per-row splice).  Groups are padded to the largest G
// with zero codes and scales, which contribute exactly 0.
HostQW concat_cols(const std::vector<const HostQW *> &parts) {
  HostQW o;
  o.K = parts[0]->K;
  o.gs = parts[0]->gs;
  for (auto *p : parts) {
    o.N += p->N;
    o.G = std::max(o.G, p->G);
  }
  size_t npairs = (size_t)o.G * o.gs / 2;
  o.data.assign(npairs * o.N, 0);
  o.scales.assign((size_t)o.G * o.N, 0.0f);
  int c = 0;
  for (auto *p : parts) {
    size_t pp = (size_t)p->G * p->gs / 2;
    for (size_t r = 0; r < pp; ++r) std::memcpy(&o.data[r * o.N + c], &p->data[r * p->N], p->N);
    for (int g = 0; g < p->G; ++g) std::memcpy(&o.scales[(size_t)g * o.N + c], &p->scales[(size_t)g * p->N], p->N * 4);
    c += p->N;
  }
  return o;
}

// Interleave columns of two same-shape weights: (a_0, b_0, a_1, b_1, ...).
HostQW interleave_cols(const HostQW &a, const HostQW &b) {
  HostQW o;
  o.K = a.K;
  o.gs = a.gs;
  o.G = std::max(a.G, b.G);
  o.N = a.N * 2;
  size_t npairs = (size_t)o.G * o.gs / 2;
  o.data.assign(npairs * o.N, 0);
  o.scales.assign((size_t)o.G * o.N, 0.0f);
  for (int s = 0; s < 2; ++s) {
    const HostQW &p = s ? b : a;
    size_t pp = (size_t)p.G * p.gs / 2;
    for (size_t r = 0; r < pp; ++r)
      for (int n = 0; n < p.N; ++n) o.data[r * o.N + 2 * n + s] = p.data[r * p.N + n];
    for (int g = 0; g < p.G; ++g)
      for (int n = 0; n < p.N; ++n) o.scales[(size_t)g * o.N + 2 * n + s] = p.scales[(size_t)g * p.N + n];
  }
  return o;
}

}  // namespace

std::unique_ptr<DevModel> load_model(std::vector<uint8_t> raw, int device, std::string &err) {
  SafeTensors st;
  if (!st.parse(std::move(raw), err)) return nullptr;
  Config c = load_config(st);
  if (const char *e = c.validate()) {
    err = e;
    return nullptr;
  }
  const int d = c.d_model, H = c.num_heads, KVH = c.num_kv_heads, hd = c.head_dim(), V = c.vocab_size;
  // Shapes the sm_100a kernels support (the shipped config is d=512, hd=64).
  if ((d % 4) || (hd % 4) || hd > 64) {
    err = "unsupported dims for the GPU path: d_model % 4 == 0, head_dim % 4 == 0 and head_dim <= 64 required";
    return nullptr;
  }
  if (std::max(c.max_enc_len, c.max_dec_len) > 8192 || c.ffn_dim <= 0 && !c.no_feedforward) {
    err = "unsupported max_enc_len / max_dec_len / ffn_dim";
    return nullptr;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    err = "no CUDA device available";
    return nullptr;
  }
  if (device < 0 || device >= ndev) {
    err = "device index " + std::to_string(device) + " out of range (" + std::to_string(ndev) + " devices)";
    return nullptr;
  }
  auto m = std::make_unique<DevModel>();
  m->device = device;
  m->cfg = c;
  if (cudaSetDevice(device) != cudaSuccess || init_kernels() != cudaSuccess ||
      cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
    err = "CUDA initialisation failed on device " + std::to_string(device);
    return nullptr;
  }
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  Loader L{st, *m, err};
  if (!L.dalloc(m->kerr, 1)) return nullptr;
  if (cudaMemset(m->kerr, 0, sizeof(int)) != cudaSuccess) {
    err = "cudaMemset failed";
    return nullptr;
  }
  std::vector<float> emb;
  if (!st.get_f32("embedding", emb)) {
    err = "missing embedding tensor";
    return nullptr;
  }
  if (emb.size() != (size_t)V * d) {
    err = "embedding size mismatch: got " + std::to_string(emb.size()) + ", expected " + std::to_string((size_t)V * d);
    return nullptr;
  }
  m->emb_bf16_exact = st.is_bf16_exact("embedding");
  if (!L.upload(m->emb, emb.data(), emb.size())) return nullptr;
  {
    const int Kp = tc_padded_k(d);
    __nv_bfloat16 *hi = nullptr, *lo = nullptr;
    if (!L.dalloc(hi, (size_t)V * Kp) || !L.dalloc(lo, (size_t)V * Kp)) return nullptr;
    if (tc_split_rows(m->emb, d, V, d, Kp, hi, lo, m->stream) != cudaSuccess ||
        cudaStreamSynchronize(m->stream) != cudaSuccess) {
      err = "embedding staging failed";
      return nullptr;
    }
    m->emb_hi = hi;
    m->emb_lo = lo;
    m->emb_tc_ready = tc_make_planes(hi, lo, V, Kp, 128, m->emb_tc) == cudaSuccess;
  }

  auto load_ffn = [&](const std::string &p, Lin &gu, Lin &down, float *&norm, float &gate) {
    HostQW g, u, dn;
    if (!L.quant(p + ".ffn.gate_proj", d, c.ffn_dim, g) || !L.quant(p + ".ffn.up_proj", d, c.ffn_dim, u) ||
        !L.quant(p + ".ffn.down_proj", c.ffn_dim, d, dn))
      return false;
    gate = L.gate(p + ".ffn_gate");
    return L.put(interleave_cols(g, u), gu) && L.put(dn, down) && L.vec(p + ".ffn_norm", d, norm);
  };

  m->enc.resize(c.num_layers);
  for (int i = 0; i < c.num_layers; ++i) {  // engine.rs:677-696
    std::string p = "encoder." + std::to_string(i);
    EncLayerDev &E = m->enc[i];
    if (!c.no_feedforward) {
      E.ffn = true;
      if (!load_ffn(p, E.gate_up, E.down, E.ffn_norm, E.ffn_gate)) return nullptr;
    }
    HostQW wq, wk, wv, wo;
    std::string a = p + ".self_attn";
    if (!L.quant(a + ".wq", d, H * hd, wq) || !L.quant(a + ".wk", d, KVH * hd, wk) ||
        !L.quant(a + ".wv", d, KVH * hd, wv) || !L.quant(a + ".wo", H * hd, d, wo))
      return nullptr;
    if (!L.put(concat_cols({&wq, &wk, &wv}), E.qkv) || !L.put(wo, E.o) || !L.vec(a + ".q_norm", hd, E.q_norm) ||
        !L.vec(a + ".k_norm", hd, E.k_norm) || !L.vec(p + ".norm", d, E.norm))
      return nullptr;
    E.gate = L.gate(p + ".self_attn_gate");
  }
  m->dec.resize(c.num_dec_layers);
  std::vector<HostQW> cross_parts(2 * c.num_dec_layers);
  std::vector<float> knorm_all;
  for (int i = 0; i < c.num_dec_layers; ++i) {  // engine.rs:698-720
    std::string p = "decoder." + std::to_string(i);
    DecLayerDev &D = m->dec[i];
    if (!c.no_feedforward) {
      D.ffn = true;
      if (!load_ffn(p, D.gate_up, D.down, D.ffn_norm, D.ffn_gate)) return nullptr;
    }
    HostQW wq, wk, wv, wo, cq, co;
    std::string a = p + ".self_attn", x = p + ".cross_attn";
    if (!L.quant(a + ".wq", d, H * hd, wq) || !L.quant(a + ".wk", d, KVH * hd, wk) ||
        !L.quant(a + ".wv", d, KVH * hd, wv) || !L.quant(a + ".wo", H * hd, d, wo) ||
        !L.quant(x + ".wq", d, H * hd, cq) || !L.quant(x + ".wk", d, KVH * hd, cross_parts[2 * i]) ||
        !L.quant(x + ".wv", d, KVH * hd, cross_parts[2 * i + 1]) || !L.quant(x + ".wo", H * hd, d, co))
      return nullptr;
    std::vector<float> kn;
    if (!L.put(concat_cols({&wq, &wk, &wv}), D.sa_qkv) || !L.put(wo, D.sa_o) || !L.put(cq, D.ca_q) ||
        !L.put(co, D.ca_o) || !L.vec(a + ".q_norm", hd, D.sa_qn) || !L.vec(a + ".k_norm", hd, D.sa_kn) ||
        !L.vec(x + ".q_norm", hd, D.ca_qn) || !L.vec_host(x + ".k_norm", hd, kn) ||
        !L.vec(p + ".self_attn_norm", d, D.sa_norm) || !L.vec(p + ".cross_attn_norm", d, D.ca_norm))
      return nullptr;
    knorm_all.insert(knorm_all.end(), kn.begin(), kn.end());
    D.sa_gate = L.gate(p + ".self_attn_gate");
    D.ca_gate = L.gate(p + ".cross_attn_gate");
  }
  if (c.num_dec_layers > 0) {
    std::vector<const HostQW *> parts;
    for (auto &q : cross_parts) parts.push_back(&q);
    if (!L.put(concat_cols(parts), m->cross_kv) || !L.upload(m->cross_knorm, knorm_all.data(), knorm_all.size()))
      return nullptr;
  }
  if (!L.vec("encoder_final_norm", d, m->enc_final_norm) || !L.vec("decoder_final_norm", d, m->dec_final_norm))
    return nullptr;
  {  // load_contrastive_head (engine.rs:548-573): all three tensors with
     // consistent shapes, else no head
    std::vector<float> pk, hk, hb;
    if (st.get_f32("contrastive_proj_kernel", pk) && st.get_f32("contrastive_hidden_kernel", hk) &&
        st.get_f32("contrastive_hidden_bias", hb)) {
      const size_t h = hb.size();
      if (h != 0 && hk.size() == (size_t)d * h && pk.size() % h == 0 && h <= (size_t)INT32_MAX &&
          pk.size() / h <= (size_t)INT32_MAX) {
        if (!L.upload(m->c_hk, hk.data(), hk.size()) || !L.upload(m->c_hb, hb.data(), hb.size()) ||
            !L.upload(m->c_pk, pk.data(), pk.size()))
          return nullptr;
        m->c_hidden = (int)h;
        m->c_dim = (int)(pk.size() / h);
      }
    }
  }
  // RoPE table (rope.rs:20-41, model.rs:52-56), computed on the host with the
  // reference's formula and uploaded.
  m->rope_len = std::max(c.max_enc_len, c.max_dec_len);
  int half = hd / 2;
  std::vector<float> rc((size_t)m->rope_len * half), rs((size_t)m->rope_len * half);
  for (int pos = 0; pos < m->rope_len; ++pos)
    for (int i = 0; i < half; ++i) {
      float e = 2.0f * (float)i;
      e = e / (float)hd;
      float theta = (float)pos / std::pow(c.rope_theta, e);
      rc[(size_t)pos * half + i] = std::cos(theta);
      rs[(size_t)pos * half + i] = std::sin(theta);
    }
  if (!L.upload(m->rope_cos, rc.data(), rc.size()) || !L.upload(m->rope_sin, rs.data(), rs.size())) return nullptr;
  m->embed_scale = std::sqrt((float)d);  // model.rs:63
  m->ad.H = H;
  m->ad.KVH = KVH;
  m->ad.HD = hd;
  m->ad.scale = std::pow((float)hd, -0.5f);  // attn.rs:142
  return m;
}

// ── Batch ──────────────────────────────────────────────────────────────────
Batch::Batch(DevModel *m) : m_(m) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m_->device);
  if (cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking) != cudaSuccess) st_ = nullptr;
  if (cudaStreamCreateWithFlags(&cst_, cudaStreamNonBlocking) != cudaSuccess) cst_ = nullptr;
  cudaSetDevice(prev);
}

template <class T>
T *Batch::alloc(size_t n, std::string &err) {
  void *p = nullptr;
  if (!st_) {
    err = "stream creation failed";
    return nullptr;
  }
  cudaError_t e = cudaMallocAsync(&p, std::max<size_t>(n, 1) * sizeof(T), st_);
  if (e != cudaSuccess) {
    err = std::string("device allocation of ") + std::to_string(n * sizeof(T)) + " bytes failed: " +
          cudaGetErrorString(e);
    return nullptr;
  }
  bufs_.push_back(p);
  return (T *)p;
}

Batch::~Batch() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m_->device);
  for (auto &g : graphs_)
    if (g) cudaGraphExecDestroy(g);
  if (st_) cudaStreamSynchronize(st_);
  if (cst_) {
    cudaStreamSynchronize(cst_);
    cudaStreamDestroy(cst_);
  }
  if (mask_ev_) cudaEventDestroy(mask_ev_);
  for (auto &e : timed_) {
    cudaEventDestroy(e.a);
    cudaEventDestroy(e.b);
  }
  if (st_) {
    for (void *p : bufs_) cudaFreeAsync(p, st_);
    cudaStreamSynchronize(st_);
    cudaStreamDestroy(st_);
  }
  cudaSetDevice(prev);
}

bool Batch::prepare(const BatchSpec &spec, std::string &err) {
  const Config &c = m_->cfg;
  NDL_CK(cudaSetDevice(m_->device));
  spec_ = spec;
  const int B = spec.n_req;
  if (B <= 0) {
    err = "empty batch";
    return false;
  }
  if (spec.max_new < 0 || spec.max_new > c.max_dec_len) {
    // engine.rs:290 bounds generation by max_dec_len.
    err = "max_new must be in [0, max_dec_len=" + std::to_string(c.max_dec_len) + "]";
    return false;
  }
  if (!spec.offsets || (!spec.ids)) {
    err = "null prompt pointer";
    return false;
  }
  off_h_.assign(spec.offsets, spec.offsets + B + 1);
  const uint64_t base = off_h_[0];
  for (auto &o : off_h_) o -= base;
  tmax_ = 0;
  for (int r = 0; r < B; ++r) {
    if (spec.offsets[r + 1] < spec.offsets[r]) {
      err = "prompt offsets must be non-decreasing";
      return false;
    }
    int64_t T = (int64_t)(off_h_[r + 1] - off_h_[r]);
    if (T < 1 || T > c.max_enc_len) {
      err = "request " + std::to_string(r) + " has " + std::to_string(T) + " prompt tokens; 1.." +
            std::to_string(c.max_enc_len) + " allowed";
      return false;
    }
    tmax_ = std::max<int>(tmax_, (int)T);
  }
  ttot_ = (int64_t)off_h_[B];
  const bool dev_in = spec.flags & BATCH_DEVICE_INPUTS;
  const int d = c.d_model, V = c.vocab_size, hd = c.head_dim();
  const int kvd = c.num_kv_heads * hd, qd = c.num_heads * hd, qkvd = qd + 2 * kvd, L = c.num_dec_layers;
  W_ = (V + 63) / 64;
  cap_ = std::max(1, spec.max_new);
  cudaStream_t st = st_;

  // prompt ids: validated (an out-of-range id would index past the embedding)
  std::vector<uint32_t> ids_h;
  if (dev_in) {
    ids_h.resize(ttot_);
    NDL_CK(cudaMemcpy(ids_h.data(), spec.ids + base, ttot_ * sizeof(uint32_t), cudaMemcpyDeviceToHost));
  }
  const uint32_t *idp = dev_in ? ids_h.data() : spec.ids + base;
  for (int64_t i = 0; i < ttot_; ++i)
    if (idp[i] >= (uint32_t)V) {
      err = "token id " + std::to_string(idp[i]) + " out of range (vocab " + std::to_string(V) + ")";
      return false;
    }
  if (spec.teacher)
    for (int64_t i = 0; i < (int64_t)B * spec.max_new; ++i)
      if (spec.teacher[i] >= (uint32_t)V) {
        err = "teacher token id out of range";
        return false;
      }
  if (dev_in) {
    ids_ = const_cast<uint32_t *>(spec.ids + base);
  } else {
    if (!(ids_ = alloc<uint32_t>(ttot_, err))) return false;
    NDL_CK(cudaMemcpyAsync(ids_, spec.ids + base, ttot_ * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  }
  std::vector<int64_t> so(off_h_.begin(), off_h_.end());
  std::vector<int32_t> tp(ttot_);
  for (int r = 0; r < B; ++r)
    for (uint64_t t = off_h_[r]; t < off_h_[r + 1]; ++t) tp[t] = (int32_t)(t - off_h_[r]);
  if (!(seq_off_ = alloc<int64_t>(B + 1, err)) || !(tok_pos_ = alloc<int32_t>(ttot_, err))) return false;
  NDL_CK(cudaMemcpyAsync(seq_off_, so.data(), so.size() * sizeof(int64_t), cudaMemcpyHostToDevice, st));
  NDL_CK(cudaMemcpyAsync(tok_pos_, tp.data(), tp.size() * sizeof(int32_t), cudaMemcpyHostToDevice, st));
  if (spec.mask && spec.max_new > 0) {
    size_t n = (size_t)B * spec.max_new * W_;
    if (dev_in) {
      mask_ = const_cast<uint64_t *>(spec.mask);
    } else {
      if (!(mask_ = alloc<uint64_t>(n, err))) return false;
      if (cst_ && (mask_ev_ || cudaEventCreateWithFlags(&mask_ev_, cudaEventDisableTiming) == cudaSuccess)) {
        NDL_CK(cudaEventRecord(mask_ev_, st));  // the allocation, ordered on st, precedes the copy
        NDL_CK(cudaStreamWaitEvent(cst_, mask_ev_, 0));
        NDL_CK(cudaMemcpyAsync(mask_, spec.mask, n * sizeof(uint64_t), cudaMemcpyHostToDevice, cst_));
        NDL_CK(cudaEventRecord(mask_ev_, cst_));
        mask_async_ = true;
      } else {
        NDL_CK(cudaMemcpyAsync(mask_, spec.mask, n * sizeof(uint64_t), cudaMemcpyHostToDevice, st));
      }
    }
  }
  std::vector<uint32_t> first(B, kEosId);  // decoding starts from EOS (engine.rs:287)
  if (spec.teacher && spec.max_new > 0) {
    if (!(teacher_ = alloc<uint32_t>((size_t)B * spec.max_new, err))) return false;
    NDL_CK(cudaMemcpyAsync(teacher_, spec.teacher, (size_t)B * spec.max_new * 4, cudaMemcpyHostToDevice, st));
    for (int b = 0; b < B; ++b) first[b] = spec.teacher[(size_t)b * spec.max_new];
  }
  uint32_t *first_d = alloc<uint32_t>(B, err);
  if (!first_d) return false;
  NDL_CK(cudaMemcpyAsync(first_d, first.data(), B * 4, cudaMemcpyHostToDevice, st));

  // prefill chunks bounded by a token budget
  const int64_t budget = std::max<int64_t>(524288, tmax_);
  chunks_.clear();
  chunk_tok_max_ = 0;
  std::vector<int64_t> rel_all;
  for (int r = 0; r < B;) {
    Chunk ch{r, r, (int64_t)off_h_[r], 0, 0, nullptr};
    while (ch.r1 < B && (ch.ntok + (int64_t)(off_h_[ch.r1 + 1] - off_h_[ch.r1]) <= budget || ch.r1 == r)) {
      ch.ntok += (int64_t)(off_h_[ch.r1 + 1] - off_h_[ch.r1]);
      ch.tmax = std::max<int>(ch.tmax, (int)(off_h_[ch.r1 + 1] - off_h_[ch.r1]));
      ++ch.r1;
    }
    chunk_tok_max_ = std::max(chunk_tok_max_, ch.ntok);
    chunks_.push_back(ch);
    r = ch.r1;
  }
  // tensor-core encoder attention: head dim 64.  A work item pairs two
  // (Q head, 128-row query tile) slots of one request that read the same KV
  // head (the GQA heads of a KV head at one tile; an odd slot left over runs
  // alone): {request, qtile_a | qtile_b << 16, head_a | head_b << 16, kv head},
  // head_b = 0xFFFF for an empty slot b.
  tc_attn_ = hd == 64 && (c.num_heads % c.num_kv_heads) == 0;
  if (tc_attn_) {
    const int rep = c.num_heads / c.num_kv_heads;
    std::vector<int32_t> it;
    std::vector<size_t> start;
    std::vector<std::pair<int, int>> slots;  // (qtile, head)
    for (auto &ch : chunks_) {
      start.push_back(it.size() / 4);
      for (int r = ch.r0; r < ch.r1; ++r) {
        int T = (int)(off_h_[r + 1] - off_h_[r]);
        for (int g = 0; g < c.num_kv_heads; ++g) {
          slots.clear();
          for (int qt = 0; qt < (T + 127) / 128; ++qt)
            for (int h = g * rep; h < (g + 1) * rep; ++h) slots.push_back({qt, h});
          for (size_t i = 0; i < slots.size(); i += 2) {
            const bool two = i + 1 < slots.size();
            const int qb = two ? slots[i + 1].first : 0, hb = two ? slots[i + 1].second : 0xFFFF;
            it.insert(it.end(), {r - ch.r0, slots[i].first | (qb << 16), slots[i].second | (hb << 16), g});
          }
        }
      }
    }
    int32_t *dit = alloc<int32_t>(it.size(), err);
    if (!dit) return false;
    NDL_CK(cudaMemcpyAsync(dit, it.data(), it.size() * 4, cudaMemcpyHostToDevice, st));
    for (size_t i = 0; i < chunks_.size(); ++i) {
      size_t end = i + 1 < chunks_.size() ? start[i + 1] : it.size() / 4;
      chunks_[i].items = dit + 4 * start[i];
      chunks_[i].n_items = (int)(end - start[i]);
    }
  }
  int64_t nrel = 0;
  for (auto &ch : chunks_) nrel += ch.r1 - ch.r0 + 1;
  int64_t *rel = alloc<int64_t>(nrel, err);
  if (!rel) return false;
  {
    std::vector<int64_t> rh;
    for (auto &ch : chunks_) {
      ch.rel_off = rel + rh.size();
      for (int r = ch.r0; r <= ch.r1; ++r) rh.push_back((int64_t)off_h_[r] - ch.tok0);
    }
    NDL_CK(cudaMemcpyAsync(rel, rh.data(), rh.size() * sizeof(int64_t), cudaMemcpyHostToDevice, st));
  }
  const int64_t ct = chunk_tok_max_;
  if (!(px_ = alloc<float>(ct * d, err)) || !(pxn_ = alloc<float>(ct * d, err)) ||
      !(pqkv_ = alloc<float>(ct * qkvd, err)) || !(patt_ = alloc<float>(ct * qd, err)))
    return false;
  if (!c.no_feedforward && !(pffn_ = alloc<float>(ct * c.ffn_dim, err))) return false;
  if (tc_attn_) {
    void *pb[6];
    const int64_t slab = ct;
    for (int i = 0; i < 6; ++i) {
      size_t n = (size_t)(i < 2 ? c.num_heads : c.num_kv_heads) * slab * 64;
      if (!(pb[i] = alloc<__nv_bfloat16>(n, err))) return false;
      // rows past a chunk's last request are read (and given zero weight)
      // by the last query tile: keep them finite
      NDL_CK(cudaMemsetAsync(pb[i], 0, n * 2, st));
    }
    if (attn_planes_make(pb, c.num_heads, c.num_kv_heads, (int)slab, attn_planes_) != cudaSuccess) tc_attn_ = false;
  }
  if (L > 0 && !(kv_planes_ = alloc<float>((size_t)2 * L * ttot_ * kvd, err))) return false;
  kv_map_ok_ = false;
  if (L > 0 && hd == 64 && c.num_heads == 2 * c.num_kv_heads) {  // the cross-attention kernel's tile loads
    const int64_t rows = (int64_t)2 * L * c.num_kv_heads * ttot_;
    if (rows > INT32_MAX) {
      err = "batch too large for the cross-attention tile map";
      return false;
    }
    NDL_CK(tma_map_f32(kv_planes_, rows, 64, 64, 64, kv_map_));
    kv_map_ok_ = true;
  }
  {  // tensor-core staging planes, shared by every batched GEMM of the call
    const int64_t rows = std::max<int64_t>(ct, B);
    std::vector<int> kps = {tc_padded_k(d), tc_padded_k(qd)};
    if (!c.no_feedforward) kps.push_back(tc_padded_k(c.ffn_dim));
    int kmax = *std::max_element(kps.begin(), kps.end());
    if (rows >= kTcMinRows) {
      if (!(tc_hi_ = alloc<__nv_bfloat16>((size_t)rows * kmax, err)) ||
          !(tc_lo_ = alloc<__nv_bfloat16>((size_t)rows * kmax, err)) ||
          !(splitk_ws_ = alloc<float>(tc_splitk_ws_bytes() / sizeof(float), err)))
        return false;
      tc_maps_.clear();
      for (int kp : kps) {
        bool have = false;
        for (auto &t : tc_maps_) have |= t.Kp == kp;
        if (have) continue;
        TcPlanes t;
        if (tc_make_planes(tc_hi_, tc_lo_, (int)rows, kp, 128, t) == cudaSuccess) tc_maps_.push_back(t);
      }
    }
  }
  if (spec.want_enc_out && !(enc_out_ = alloc<float>((size_t)ttot_ * d, err))) return false;

  // decoder state
  if (spec.max_new > 0) {
    size_t cache = (size_t)L * B * cap_ * kvd;
    if (!(self_k_ = alloc<float>(cache, err)) || !(self_v_ = alloc<float>(cache, err)) ||
        !(x_ = alloc<float>((size_t)B * d, err)) || !(xn_ = alloc<float>((size_t)B * d, err)) ||
        !(h_ = alloc<float>((size_t)B * d, err)) || !(qkv_ = alloc<float>((size_t)B * qkvd, err)) ||
        !(att_ = alloc<float>((size_t)B * qd, err)) || !(q_ = alloc<float>((size_t)B * qd, err)) ||
        !(keys_ = alloc<unsigned long long>(B, err)) || !(pos_ = alloc<int32_t>(B, err)) ||
        !(out_ids_ = alloc<uint32_t>((size_t)B * spec.max_new, err)) || !(lens_ = alloc<uint32_t>(B, err)) ||
        !(done_ = alloc<uint8_t>(B, err)) || !(n_done_ = alloc<unsigned int>(1, err)))
      return false;
    if (!c.no_feedforward && !(ffn_ = alloc<float>((size_t)B * c.ffn_dim, err))) return false;
    if (spec.want_logits && !(logits_ = alloc<float>((size_t)B * spec.max_new * V, err))) return false;
  }
  first_ids_ = first_d;
  return true;
}

bool Batch::reset_decoder(std::string &err) {
  // Fresh decoder state for a (re-)run; inputs and the encoder buffers are
  // reused as uploaded by prepare().
  if (spec_.max_new == 0) return true;
  const int B = spec_.n_req, d = m_->cfg.d_model;
  cudaStream_t st = st_;
  NDL_CK(cudaMemsetAsync(keys_, 0, B * sizeof(unsigned long long), st));
  NDL_CK(cudaMemsetAsync(pos_, 0, B * sizeof(int32_t), st));
  NDL_CK(cudaMemsetAsync(lens_, 0, B * sizeof(uint32_t), st));
  NDL_CK(cudaMemsetAsync(done_, 0, B, st));
  NDL_CK(cudaMemsetAsync(n_done_, 0, sizeof(unsigned int), st));
  NDL_CK(cudaMemsetAsync(out_ids_, 0, (size_t)B * spec_.max_new * 4, st));
  NDL_CK(embed_rows(first_ids_, m_->emb, x_, B, d, m_->embed_scale, st));
  ++launches_;
  return true;
}

// Launch of a timed class with no algorithmic work accounting.
#define NDL_TK(cls, capture, call)                                                   \
  do {                                                                               \
    cudaEvent_t ev_;                                                                 \
    if (!tbegin(cls, capture, ev_, err)) return false;                               \
    NDL_LK(call);                                                                    \
    if (!tend(ev_, 0.0, 0.0, err)) return false;                                     \
  } while (0)

#define NDL_LK(call)                                                                 \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    ++launches_;                                                                     \
    if (e_ != cudaSuccess) {                                                         \
      err = std::string(#call) + " failed: " + cudaGetErrorString(e_);               \
      return false;                                                                  \
    }                                                                                \
  } while (0)

bool Batch::tbegin(int cls, bool capture, cudaEvent_t &a, std::string &err) {
  a = nullptr;
  if (capture || cls != timed_cls_) return true;
  NDL_CK(cudaEventCreate(&a));
  NDL_CK(cudaEventRecord(a, st_));
  return true;
}

bool Batch::tend(cudaEvent_t a, double flops, double bytes, std::string &err) {
  if (!a) return true;
  cudaEvent_t b;
  NDL_CK(cudaEventCreate(&b));
  NDL_CK(cudaEventRecord(b, st_));
  timed_.push_back({a, b, flops, bytes});
  return true;
}

namespace {
// Algorithmic work of Y[M,N] = X[M,K] @ W (INT4 + f32 scales, f32 in/out).
inline double mm_flops(int M, const Lin &w) { return 2.0 * M * w.N * (double)w.K; }
inline double mm_bytes(int M, const Lin &w) {
  return (double)w.G * w.gs / 2 * w.N + (double)w.G * w.N * 4 + 4.0 * M * w.K + 4.0 * M * w.N;
}
// The tensor-core path reads the weight's bf16 hi/lo planes (4 bytes per
// element of [N][Kp]) and the activation's planes, not the INT4 codes.
inline double mm_tc_bytes(int M, const Lin &w) {
  return 4.0 * w.N * w.tc.Kp + 4.0 * M * w.tc.Kp + 4.0 * M * w.N;
}
}  // namespace

bool Batch::mm(int cls, bool capture, const float *x, int64_t ldx, int M, const Lin &w, const MatmulOut &o,
               std::string &err) {
  cudaEvent_t a;
  if (!tbegin(cls, capture, a, err)) return false;
  const TcPlanes *ap = nullptr;
  if (M >= kTcMinRows && w.tc_ready && (!o.col_block || o.col_block % 64 == 0))
    for (auto &t : tc_maps_)
      if (t.Kp == w.tc.Kp && M <= t.rows) ap = &t;
  if (ap) {
    MatmulOut os = o;
    os.splitk_ws = splitk_ws_;
    NDL_LK(tc_split_rows(x, ldx, M, w.K, ap->Kp, tc_hi_, tc_lo_, st_));
    NDL_LK(tc_matmul(*ap, M, w.tc, w.N, os, m_->kerr, st_));
  } else {
    NDL_LK(int4_matmul(x, ldx, M, w.view(), o, st_, pdl_on()));
  }
  return tend(a, mm_flops(M, w), mm_bytes(M, w), err);
}

const TcPlanes *Batch::tc_map(int Kp, int rows) const {
  for (auto &t : tc_maps_)
    if (t.Kp == Kp && rows <= t.rows) return &t;
  return nullptr;
}

// Matmul whose input is either already staged as bf16 hi/lo planes (`planes`,
// written by the producing kernel) or f32 rows (x, ldx).
bool Batch::mm_in(int cls, bool capture, const TcPlanes *planes, const float *x, int64_t ldx, int M, const Lin &w,
                  const MatmulOut &o, std::string &err) {
  if (!planes) return mm(cls, capture, x, ldx, M, w, o, err);
  if (!w.tc_ready || planes->Kp != w.tc.Kp || (o.col_block && o.col_block % 64)) {
    err = "internal: staged matmul input without a tensor-core weight";
    return false;
  }
  cudaEvent_t a;
  if (!tbegin(cls, capture, a, err)) return false;
  MatmulOut os = o;
  os.splitk_ws = splitk_ws_;
  NDL_LK(tc_matmul(*planes, M, w.tc, w.N, os, m_->kerr, st_));
  return tend(a, mm_flops(M, w), mm_tc_bytes(M, w), err);
}

bool Batch::prefill(std::string &err) {
  const DevModel &m = *m_;
  const Config &c = m.cfg;
  const int d = c.d_model, hd = c.head_dim(), qd = c.num_heads * hd, kvd = c.num_kv_heads * hd;
  const int qkvd = qd + 2 * kvd, L = c.num_dec_layers;
  cudaStream_t st = st_;
  for (const Chunk &ch : chunks_) {
    const int rows = (int)ch.ntok, nr = ch.r1 - ch.r0;
    // inputs of the tensor-core matmuls staged straight by their producers
    const TcPlanes *pd = (rows >= kTcMinRows && d == 512) ? tc_map(tc_padded_k(d), rows) : nullptr;
    const TcPlanes *pq = (rows >= kTcMinRows && tc_attn_) ? tc_map(tc_padded_k(qd), rows) : nullptr;
    auto norm = [&](const float *scale, float *f32_out) -> bool {
      if (pd) {
        NDL_TK(TIME_ELEMENTWISE, false,
               rms_norm_planes(px_, d, tc_hi_, tc_lo_, pd->Kp, f32_out, d, scale, rows, d, st));
      } else {
        NDL_TK(TIME_ELEMENTWISE, false, rms_norm_rows(px_, d, pxn_, d, scale, rows, d, st));
      }
      return true;
    };
    NDL_TK(TIME_ELEMENTWISE, false, embed_rows(ids_ + ch.tok0, m.emb, px_, rows, d, m.embed_scale, st));
    for (const EncLayerDev &E : m.enc) {  // layers.rs:46-93
      if (!norm(E.norm, nullptr)) return false;
      MatmulOut o;
      o.y = pqkv_;
      o.ldy = qkvd;
      const bool fused_post = tc_attn_ && pd != nullptr;
      if (fused_post) {  // norm + RoPE + bf16 split of Q/K/V in the matmul epilogue
        o.epi = EPI_QKV;
        o.pos = tok_pos_ + ch.tok0;
        o.q_norm = E.q_norm;
        o.k_norm = E.k_norm;
        o.rope_cos = m.rope_cos;
        o.rope_sin = m.rope_sin;
        for (int i = 0; i < 6; ++i) o.planes[i] = attn_planes_.buf[i];
        o.slab = attn_planes_.slab;
        o.heads_q = c.num_heads;
        o.heads_kv = c.num_kv_heads;
      }
      if (!mm_in(TIME_PREFILL_MATMUL, false, pd, pxn_, d, rows, E.qkv, o, err)) return false;
      if (fused_post) {
      } else if (!tc_attn_)
        NDL_TK(TIME_ELEMENTWISE, false, qk_norm_rope_rows(pqkv_, rows, tok_pos_ + ch.tok0, E.q_norm, E.k_norm, m.rope_cos, m.rope_sin, m.ad,
                                 st));
      else
        NDL_TK(TIME_ELEMENTWISE, false, qkv_post(pqkv_, rows, tok_pos_ + ch.tok0, E.q_norm, E.k_norm, m.rope_cos, m.rope_sin, m.ad,
                        attn_planes_, st));
      {
        cudaEvent_t ev;
        if (!tbegin(TIME_ENCODER_ATTENTION, false, ev, err)) return false;
        if (tc_attn_)
          NDL_LK(encoder_attention_tc(attn_planes_, ch.rel_off, ch.items, ch.n_items, pq ? nullptr : patt_,
                                      pq ? tc_hi_ : nullptr, pq ? tc_lo_ : nullptr, pq ? pq->Kp : 0, rows,
                                      m.ad, m_->kerr, st));
        else
          NDL_LK(encoder_attention(pqkv_, ch.rel_off, nr, ch.tmax, patt_, m.ad, st));
        double Tq = 0.0;  // sum of T^2 over the chunk's requests
        for (int r = ch.r0; r < ch.r1; ++r) Tq += std::pow((double)(off_h_[r + 1] - off_h_[r]), 2.0);
        if (!tend(ev, 4.0 * Tq * c.num_heads * hd, (double)rows * (qkvd + qd) * 4, err)) return false;
      }
      MatmulOut r;
      r.y = px_;
      r.ldy = d;
      r.epi = EPI_RESID;
      r.gate = E.gate;
      if (!mm_in(TIME_PREFILL_MATMUL, false, tc_attn_ ? pq : nullptr, patt_, qd, rows, E.o, r, err)) return false;
      if (E.ffn) {
        if (!norm(E.ffn_norm, nullptr)) return false;
        MatmulOut a;
        a.y = pffn_;
        a.ldy = c.ffn_dim;
        a.epi = EPI_ACT;
        a.act = c.activation;
        if (!mm_in(TIME_PREFILL_MATMUL, false, pd, pxn_, d, rows, E.gate_up, a, err)) return false;
        MatmulOut f;
        f.y = px_;
        f.ldy = d;
        f.epi = EPI_RESID;
        f.gate = E.ffn_gate;
        if (!mm(TIME_PREFILL_MATMUL, false, pffn_, c.ffn_dim, rows, E.down, f, err)) return false;
      }
    }
    if (!norm(m.enc_final_norm, enc_out_ ? pxn_ : nullptr)) return false;  // model.rs:184-186
    if (enc_out_)
      NDL_CK(cudaMemcpyAsync(enc_out_ + ch.tok0 * d, pxn_, (size_t)rows * d * 4, cudaMemcpyDeviceToDevice, st));
    if (L > 0) {  // fill_cross_kv (model.rs:196-231): all layers' K|V in one matmul
      MatmulOut o;
      if (kv_map_ok_) {  // head-major: one 64-column block per (layer, K|V, head)
        o.y = kv_planes_ + ch.tok0 * 64;
        o.ldy = 64;
        o.col_block = 64;
        o.block_stride = ttot_ * 64;
        o.kv_block = kvd;
      } else {
        o.y = kv_planes_ + ch.tok0 * kvd;
        o.ldy = kvd;
        o.col_block = kvd;
        o.block_stride = ttot_ * kvd;
      }
      const bool fused_norm = (hd == 64) && (kvd % 64 == 0);
      o.epi = fused_norm ? EPI_KNORM : EPI_STORE;
      o.vec = m.cross_knorm;
      if (!mm_in(TIME_PREFILL_MATMUL, false, pd, pxn_, d, rows, m.cross_kv, o, err)) return false;
      if (!fused_norm)
        for (int l = 0; l < L; ++l)
          NDL_TK(TIME_ELEMENTWISE, false, head_norm_rows(kv_planes_ + (size_t)2 * l * ttot_ * kvd + ch.tok0 * kvd, rows, kvd,
                                c.num_kv_heads, hd, m.cross_knorm + (size_t)l * hd, st));
    }
  }
  return true;
}

bool Batch::decode_step(std::string &err, bool capture, int att_rows) {
  // the step's kernels start during their predecessor's tail (each waits for
  // it before touching global memory)
  struct PdlScope {
    explicit PdlScope(bool on) { set_pdl(on); }
    ~PdlScope() { set_pdl(false); }
  } pdl_scope(!(spec_.flags & BATCH_NO_PDL));
  const DevModel &m = *m_;
  const Config &c = m.cfg;
  const int B = spec_.n_req, d = c.d_model, hd = c.head_dim(), qd = c.num_heads * hd, kvd = c.num_kv_heads * hd;
  const int qkvd = qd + 2 * kvd;
  cudaStream_t st = st_;
  const TcPlanes *pd = (B >= kTcMinRows && d == 512) ? tc_map(tc_padded_k(d), B) : nullptr;
  // attention outputs written straight as the output projections' operand planes
  const TcPlanes *pa = (B >= kTcMinRows && hd == 64 && c.num_heads == 2 * c.num_kv_heads && qd == tc_padded_k(qd))
                           ? tc_map(tc_padded_k(qd), B)
                           : nullptr;
  auto norm = [&](const float *scale, float *f32_out) -> bool {
    if (pd) {
      NDL_TK(TIME_ELEMENTWISE, capture, rms_norm_planes(x_, d, tc_hi_, tc_lo_, pd->Kp, f32_out, d, scale, B, d, st));
    } else {
      NDL_TK(TIME_ELEMENTWISE, capture, rms_norm_rows(x_, d, f32_out ? f32_out : xn_, d, scale, B, d, st));
    }
    return true;
  };
  for (size_t l = 0; l < m.dec.size(); ++l) {  // layers.rs:100-149
    const DecLayerDev &D = m.dec[l];
    const TcPlanes *pal = (pa && D.sa_o.tc_ready && D.ca_o.tc_ready && D.sa_o.tc.Kp == pa->Kp && D.ca_o.tc.Kp == pa->Kp)
                              ? pa
                              : nullptr;
    void *ahi = pal ? tc_hi_ : nullptr, *alo = pal ? tc_lo_ : nullptr;
    const int64_t aldp = pal ? pal->Kp : 0;
    const size_t coff = l * (size_t)B * cap_ * kvd;
    // tensor-core path: q/k norm, RoPE and the cache append run in the QKV
    // projection's epilogue
    const bool prep = pd && D.sa_qkv.tc_ready && hd == 64 && c.num_heads == 2 * c.num_kv_heads;
    MatmulOut o;
    o.y = qkv_;
    o.ldy = qkvd;
    if (prep) {
      o.epi = EPI_QKV_DEC;
      o.pos = pos_;
      o.q_norm = D.sa_qn;
      o.k_norm = D.sa_kn;
      o.rope_cos = m.rope_cos;
      o.rope_sin = m.rope_sin;
      o.heads_q = c.num_heads;
      o.heads_kv = c.num_kv_heads;
      o.kcache = self_k_ + coff;
      o.vcache = self_v_ + coff;
      o.cache_cap = cap_;
    }
    // CUDA-core path: the matvec norms its input rows as it loads them
    const bool sa_in = !pd && int4_matmul_norms_input(B, D.sa_qkv.view(), o);
    if (sa_in)
      o.in_norm = D.sa_norm;
    else if (!norm(D.sa_norm, nullptr))
      return false;
    if (!mm_in(TIME_DECODE_MATMUL, capture, pd, sa_in ? x_ : xn_, d, B, D.sa_qkv, o, err)) return false;
    NDL_TK(TIME_SELF_ATTENTION, capture, decoder_self_attention(qkv_, pos_, D.sa_qn, D.sa_kn, m.rope_cos, m.rope_sin, self_k_ + coff,
                                  self_v_ + coff, cap_, B, att_, m.ad, st, ahi, alo, aldp, prep, att_rows));
    MatmulOut r;
    r.y = x_;
    r.ldy = d;
    r.epi = EPI_RESID;
    r.gate = D.sa_gate;
    if (!mm_in(TIME_DECODE_MATMUL, capture, pal, att_, qd, B, D.sa_o, r, err)) return false;
    MatmulOut qo;
    qo.y = q_;
    qo.ldy = qd;
    const bool ca_in = !pd && int4_matmul_norms_input(B, D.ca_q.view(), qo);
    if (ca_in)
      qo.in_norm = D.ca_norm;
    else if (!norm(D.ca_norm, nullptr))
      return false;
    if (!mm_in(TIME_DECODE_MATMUL, capture, pd, ca_in ? x_ : xn_, d, B, D.ca_q, qo, err)) return false;
    const float *kp = kv_planes_ + (size_t)2 * l * ttot_ * kvd, *vp = kp + (size_t)ttot_ * kvd;
    cudaEvent_t ev;
    if (!tbegin(TIME_CROSS_ATTENTION, capture, ev, err)) return false;
    NDL_LK(decoder_cross_attention(q_, D.ca_qn, kp, vp, seq_off_, B, att_, m.ad, st, tmax_, ahi, alo, aldp, m.kerr,
                                   kv_map_ok_ ? kv_map_ : nullptr, (int64_t)2 * l * c.num_kv_heads * ttot_,
                                   (int64_t)(2 * l + 1) * c.num_kv_heads * ttot_, ttot_));
    // algorithmic bytes: the encoder K and V rows once, q in, attention out
    if (!tend(ev, 4.0 * (double)ttot_ * kvd * c.num_heads / c.num_kv_heads,
              (double)ttot_ * kvd * 8 + (double)B * qd * 8, err))
      return false;
    MatmulOut r2;
    r2.y = x_;
    r2.ldy = d;
    r2.epi = EPI_RESID;
    r2.gate = D.ca_gate;
    if (!mm_in(TIME_DECODE_MATMUL, capture, pal, att_, qd, B, D.ca_o, r2, err)) return false;
    if (D.ffn) {
      if (!norm(D.ffn_norm, nullptr)) return false;
      MatmulOut a;
      a.y = ffn_;
      a.ldy = c.ffn_dim;
      a.epi = EPI_ACT;
      a.act = c.activation;
      if (!mm_in(TIME_DECODE_MATMUL, capture, pd, xn_, d, B, D.gate_up, a, err)) return false;
      MatmulOut f;
      f.y = x_;
      f.ldy = d;
      f.epi = EPI_RESID;
      f.gate = D.ffn_gate;
      if (!mm(TIME_DECODE_MATMUL, capture, ffn_, c.ffn_dim, B, D.down, f, err)) return false;
    }
  }
  if (!norm(m.dec_final_norm, h_)) return false;  // model.rs:263
  cudaEvent_t ev;
  if (!tbegin(TIME_HEAD, capture, ev, err)) return false;
  const TcPlanes *hp = nullptr;
  if (B >= kTcMinRows && m.emb_tc_ready)
    for (auto &t : tc_maps_)
      if (t.Kp == m.emb_tc.Kp && B <= t.rows) hp = &t;
  if (hp) {  // logits on the tensor cores, mask + argmax in the epilogue
    if (!pd) NDL_LK(tc_split_rows(h_, d, B, d, hp->Kp, tc_hi_, tc_lo_, st));
    MatmulOut o;
    o.epi = EPI_ARGMAX;
    o.mask = mask_;
    o.mask_words = W_;
    o.max_new = spec_.max_new;
    o.pos = pos_;
    o.keys = keys_;
    o.logits = logits_;
    o.splitk_ws = splitk_ws_;
    NDL_LK(tc_matmul(*hp, B, m.emb_tc, c.vocab_size, o, m.kerr, st, m.emb_bf16_exact));
  } else {
    NDL_LK(head_argmax(h_, B, m.emb, c.vocab_size, d, mask_, W_, logits_, spec_.max_new, pos_, keys_, st,
                       m.emb_bf16_exact && m.emb_tc_ready ? m.emb_hi : nullptr, m.emb_tc.Kp));
  }
  if (!tend(ev, 2.0 * B * c.vocab_size * (double)d,
            (double)c.vocab_size * d * 4 + (double)B * d * 4 + (mask_ ? (double)B * W_ * 8 : 0.0), err))
    return false;
  NDL_TK(TIME_ELEMENTWISE, capture, finish_step(keys_, B, spec_.max_new, (spec_.flags & BATCH_STOP_ON_EOS) ? 1 : 0, out_ids_, lens_, done_,
                     pos_, n_done_, teacher_, m.emb, x_, d, m.embed_scale, st));
  return true;
}

bool Batch::begin(std::string &err) {
  NDL_CK(cudaSetDevice(m_->device));
  launches_ = 0;
  steps_done_ = 0;
  for (auto &e : timed_) {
    cudaEventDestroy(e.a);
    cudaEventDestroy(e.b);
  }
  timed_.clear();
  if (!reset_decoder(err) || !prefill(err)) return false;
  if (mask_async_) NDL_CK(cudaStreamWaitEvent(st_, mask_ev_, 0));  // masks in place before the first step
  use_graph_ = !(spec_.flags & BATCH_NO_GRAPH) && !timed_cls_ && spec_.max_new > 0;
  // one graph per self-attention row bound the steps of this batch reach
  for (int s = 0; use_graph_ && s < spec_.max_new; ++s) {
    const int rows = att_rows(s);
    cudaGraphExec_t &ge = graphs_[att_slot(rows)];
    if (ge) continue;
    cudaStream_t st = st_;
    int64_t before = launches_;
    NDL_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    std::string cerr;
    bool ok = decode_step(cerr, true, rows);
    cudaGraph_t g = nullptr;
    cudaError_t ce = cudaStreamEndCapture(st, &g);
    if (!ok || ce != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      err = ok ? std::string("graph capture failed: ") + cudaGetErrorString(ce) : cerr;
      return false;
    }
    cudaError_t ie = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
      ge = nullptr;
      err = std::string("graph instantiate failed: ") + cudaGetErrorString(ie);
      return false;
    }
    step_launches_ = launches_ - before;
    launches_ = before;
  }
  return true;
}

bool Batch::step(std::string &err) {
  if (steps_done_ >= spec_.max_new) {
    err = "all decode steps already run";
    return false;
  }
  if (use_graph_) {
    NDL_CK(cudaGraphLaunch(graphs_[att_slot(att_rows(steps_done_))], st_));
    launches_ += step_launches_;
  } else if (!decode_step(err, false, att_rows(steps_done_))) {
    return false;
  }
  ++steps_done_;
  return true;
}

bool Batch::peek(uint32_t *lens, uint8_t *done, uint32_t *ids, std::string &err) {
  cudaStream_t st = st_;
  const int B = spec_.n_req;
  if (lens) NDL_CK(cudaMemcpyAsync(lens, lens_, (size_t)B * 4, cudaMemcpyDeviceToHost, st));
  if (done) NDL_CK(cudaMemcpyAsync(done, done_, (size_t)B, cudaMemcpyDeviceToHost, st));
  if (ids) NDL_CK(cudaMemcpyAsync(ids, out_ids_, (size_t)B * spec_.max_new * 4, cudaMemcpyDeviceToHost, st));
  NDL_CK(cudaStreamSynchronize(st));
  return true;
}

bool Batch::set_mask_row(int req, int step, const uint64_t *bits, std::string &err) {
  if (!mask_ || req < 0 || req >= spec_.n_req || step < 0 || step >= spec_.max_new) {
    err = "set_mask_row: no such mask row";
    return false;
  }
  if (mask_async_) NDL_CK(cudaStreamWaitEvent(st_, mask_ev_, 0));
  uint64_t *dst = mask_ + ((size_t)req * spec_.max_new + step) * W_;
  NDL_CK(cudaMemcpyAsync(dst, bits, (size_t)W_ * sizeof(uint64_t), cudaMemcpyHostToDevice, st_));
  return true;
}

bool Batch::set_mask_step(int step, const uint64_t *rows, std::string &err) {
  if (!mask_ || step < 0 || step >= spec_.max_new) {
    err = "set_mask_step: no such mask step";
    return false;
  }
  if (mask_async_) NDL_CK(cudaStreamWaitEvent(st_, mask_ev_, 0));
  const size_t row = (size_t)W_ * sizeof(uint64_t);
  NDL_CK(cudaMemcpy2DAsync(mask_ + (size_t)step * W_, (size_t)spec_.max_new * row, rows, row, row,
                           (size_t)spec_.n_req, cudaMemcpyHostToDevice, st_));
  return true;
}

bool Batch::peek_step(int step, uint32_t *tokens, uint32_t *lens, uint8_t *done, std::string &err) {
  if (step < 0 || step >= spec_.max_new) {
    err = "peek_step: no such step";
    return false;
  }
  cudaStream_t st = st_;
  const int B = spec_.n_req;
  if (tokens)
    NDL_CK(cudaMemcpy2DAsync(tokens, sizeof(uint32_t), out_ids_ + step, (size_t)spec_.max_new * sizeof(uint32_t),
                             sizeof(uint32_t), (size_t)B, cudaMemcpyDeviceToHost, st));
  if (lens) NDL_CK(cudaMemcpyAsync(lens, lens_, (size_t)B * 4, cudaMemcpyDeviceToHost, st));
  if (done) NDL_CK(cudaMemcpyAsync(done, done_, (size_t)B, cudaMemcpyDeviceToHost, st));
  NDL_CK(cudaStreamSynchronize(st));
  return true;
}

bool Batch::run(std::string &err) {
  if (!begin(err)) return false;
  const int steps = spec_.max_new;
  const bool stop = spec_.flags & BATCH_STOP_ON_EOS;
  unsigned int ndone = 0;
  for (int s = 0; s < steps; ++s) {
    if (!step(err)) return false;
    if (stop && ((s & 7) == 7) && s + 1 < steps) {
      NDL_CK(cudaMemcpyAsync(&ndone, n_done_, sizeof(ndone), cudaMemcpyDeviceToHost, st_));
      NDL_CK(cudaStreamSynchronize(st_));
      if ((int)ndone >= spec_.n_req) break;
    }
  }
  return true;
}

bool Batch::download(uint32_t *out_ids, uint32_t *out_lens, float *logits, float *enc_out, std::string &err) {
  NDL_CK(cudaSetDevice(m_->device));
  cudaStream_t st = st_;
  const int B = spec_.n_req;
  const bool dev_out = spec_.flags & BATCH_DEVICE_INPUTS;
  const cudaMemcpyKind k = dev_out ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
  if (spec_.max_new > 0) {
    if (out_ids) NDL_CK(cudaMemcpyAsync(out_ids, out_ids_, (size_t)B * spec_.max_new * 4, k, st));
    if (out_lens) NDL_CK(cudaMemcpyAsync(out_lens, lens_, (size_t)B * 4, k, st));
    if (logits && logits_)
      NDL_CK(cudaMemcpyAsync(logits, logits_, (size_t)B * spec_.max_new * m_->cfg.vocab_size * 4, k, st));
  } else if (out_lens) {
    if (dev_out)
      NDL_CK(cudaMemsetAsync(out_lens, 0, (size_t)B * 4, st));
    else
      std::memset(out_lens, 0, (size_t)B * 4);
  }
  if (enc_out && enc_out_) NDL_CK(cudaMemcpyAsync(enc_out, enc_out_, (size_t)ttot_ * m_->cfg.d_model * 4, k, st));
  int kerr = 0;
  NDL_CK(cudaMemcpyAsync(&kerr, m_->kerr, sizeof(int), cudaMemcpyDeviceToHost, st));
  NDL_CK(cudaStreamSynchronize(st));
  if (kerr) {
    cudaMemsetAsync(m_->kerr, 0, sizeof(int), st);
    err = "a tensor-core GEMM wait timed out; results are invalid";
    return false;
  }
  if (!spec_.max_new || !out_lens || dev_out) return true;
  for (int b = 0; b < B; ++b) out_lens[b] = std::min<uint32_t>(out_lens[b], (uint32_t)spec_.max_new);
  return true;
}

bool Batch::collect_timing(std::string &err) {
  NDL_CK(cudaStreamSynchronize(st_));
  timed_ms_ = timed_flops_ = timed_bytes_ = 0.0;
  timed_n_ = 0;
  for (auto &e : timed_) {
    float ms = 0.0f;
    NDL_CK(cudaEventElapsedTime(&ms, e.a, e.b));
    timed_ms_ += ms;
    timed_flops_ += e.flops;
    timed_bytes_ += e.bytes;
    ++timed_n_;
  }
  return true;
}

void shard_requests(const uint64_t *offsets, int n_req, int shards, int32_t *assignment) {
  // Longest-processing-time-first: cost of a request ~ prefill (T^2 attention
  // + T projections) plus its decode share (proportional to T for the
  // cross-attention reads).
  std::vector<int> order(n_req);
  std::iota(order.begin(), order.end(), 0);
  auto cost = [&](int r) {
    double T = (double)(offsets[r + 1] - offsets[r]);
    return T * T + 2048.0 * T;
  };
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost(a) > cost(b); });
  std::vector<double> load(std::max(shards, 1), 0.0);
  for (int r : order) {
    int s = (int)(std::min_element(load.begin(), load.end()) - load.begin());
    assignment[r] = s;
    load[s] += cost(r);
  }
}

}  // namespace ndl
