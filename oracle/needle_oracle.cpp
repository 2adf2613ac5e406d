// needle_oracle.cpp — CPU restatement of the needle-rs reference path.
//
// TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA product and the
// timed CPU baseline of bench.py.  The product never links or calls this.
//
// Each function follows the reference file:line cited beside it, keeping the
// reference's f32 evaluation order.  Built with -ffp-contract=off so that no
// multiply-add is fused unless the reference itself uses an FMA
// (_mm256_fmadd_ps in quant.rs:273 and model.rs:131).
#include "needle_oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr size_t GROUP_SIZE = 32;      // quant.rs:17
constexpr float SCALE_MIN = 1e-8f;     // quant.rs:18
constexpr float NORM_EPS = 1e-6f;      // norm.rs:6
constexpr uint32_t EOS_ID = 1;         // tokenizer.rs:23
constexpr float MASK_BLOCKED = -1e9f;  // constrained.rs:93-116 (additive bias)

bool cpu_has_avx2() {
  static int cached = -1;
  if (cached < 0) {
    __builtin_cpu_init();
    cached = (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) ? 1 : 0;
  }
  return cached == 1;
}

// quant.rs:413-419
inline int8_t sign_extend4(uint8_t nibble) {
  return (nibble & 0x8) ? (int8_t)(nibble | 0xF0) : (int8_t)nibble;
}

// ── QuantizedWeight (quant.rs:52-58) ─────────────────────────────────────────
struct QW {
  std::vector<uint8_t> data;
  std::vector<float> scales;
  size_t in_feat = 0, out_feat = 0, num_groups = 0;
};

void quantize(const float *w, size_t in_feat, size_t out_feat, uint8_t *data,
              float *scales) {
  // quant.rs:63-128
  size_t gs = std::min(GROUP_SIZE, in_feat);
  size_t pad = (gs - in_feat % gs) % gs;
  size_t in_padded = in_feat + pad;
  size_t num_groups = in_padded / gs;
  size_t num_pairs = in_padded / 2;
  for (size_t g = 0; g < num_groups; ++g) {
    size_t row_start = g * gs;
    for (size_t o = 0; o < out_feat; ++o) {
      float max_abs = 0.0f;
      for (size_t r = 0; r < gs; ++r) {
        size_t gr = row_start + r;
        float val = gr < in_feat ? std::fabs(w[gr * out_feat + o]) : 0.0f;
        if (val > max_abs) max_abs = val;
      }
      // (max_abs / 7.0).max(SCALE_MIN): f32::max returns the non-NaN operand.
      float s = max_abs / 7.0f;
      scales[g * out_feat + o] = std::isnan(s) ? SCALE_MIN : std::max(s, SCALE_MIN);
    }
  }
  for (size_t pair = 0; pair < num_pairs; ++pair) {
    size_t r0 = pair * 2, r1 = pair * 2 + 1;
    size_t g = r0 / gs;
    for (size_t o = 0; o < out_feat; ++o) {
      float scale = scales[g * out_feat + o];
      float v0 = r0 < in_feat ? w[r0 * out_feat + o] : 0.0f;
      float v1 = r1 < in_feat ? w[r1 * out_feat + o] : 0.0f;
      // math::round = libm roundf (half away from zero); f32::clamp; `as i8`
      // saturates and maps NaN to 0.
      float f0 = std::roundf(v0 / scale), f1 = std::roundf(v1 / scale);
      f0 = std::isnan(f0) ? 0.0f : std::min(std::max(f0, -8.0f), 7.0f);
      f1 = std::isnan(f1) ? 0.0f : std::min(std::max(f1, -8.0f), 7.0f);
      int8_t q0 = (int8_t)f0, q1 = (int8_t)f1;
      uint8_t lo = (uint8_t)q0 & 0x0F;
      uint8_t hi = (uint8_t)(((uint8_t)q1 & 0x0F) << 4);
      data[pair * out_feat + o] = lo | hi;
    }
  }
}

QW quantize_qw(const float *w, size_t in_feat, size_t out_feat) {
  QW q;
  size_t gs = std::min(GROUP_SIZE, in_feat);
  size_t in_padded = in_feat + (gs - in_feat % gs) % gs;
  q.in_feat = in_feat;
  q.out_feat = out_feat;
  q.num_groups = in_padded / gs;
  q.data.assign(in_padded / 2 * out_feat, 0);
  q.scales.assign(q.num_groups * out_feat, 0.0f);
  quantize(w, in_feat, out_feat, q.data.data(), q.scales.data());
  return q;
}

void matvec_scalar(const uint8_t *data, const float *scales, size_t in_feat,
                   size_t out_feat, size_t num_groups, const float *x, float *y) {
  // quant.rs:184-206 — no FMA: Rust does not contract a*b+c.
  size_t gs = std::min(GROUP_SIZE, in_feat);
  size_t num_pairs = num_groups * gs / 2;
  for (size_t pair = 0; pair < num_pairs; ++pair) {
    size_t r0 = pair * 2, r1 = pair * 2 + 1;
    size_t g = r0 / gs;
    float x0 = r0 < in_feat ? x[r0] : 0.0f;
    float x1 = r1 < in_feat ? x[r1] : 0.0f;
    size_t base = pair * out_feat, sbase = g * out_feat;
    for (size_t o = 0; o < out_feat; ++o) {
      uint8_t byte = data[base + o];
      float lo = (float)sign_extend4(byte & 0x0F);
      float hi = (float)sign_extend4((byte >> 4) & 0x0F);
      float scale = scales[sbase + o];
      float t0 = lo * x0;
      float t1 = hi * x1;
      float t = t0 + t1;
      y[o] += t * scale;
    }
  }
}

__attribute__((target("avx2,fma"))) void matvec_avx2(
    const uint8_t *data, const float *scales, size_t in_feat, size_t out_feat,
    size_t num_groups, const float *x, float *y) {
  // quant.rs:209-297, same intrinsics in the same order.
  size_t gs = std::min(GROUP_SIZE, in_feat);
  size_t num_pairs = num_groups * gs / 2;
  const __m256i mask_lo = _mm256_set1_epi32(0x0F0F0F0F);
  for (size_t pair = 0; pair < num_pairs; ++pair) {
    size_t r0 = pair * 2, r1 = pair * 2 + 1;
    size_t g = r0 / gs;
    float x0 = r0 < in_feat ? x[r0] : 0.0f;
    float x1 = r1 < in_feat ? x[r1] : 0.0f;
    __m256 x0v = _mm256_set1_ps(x0);
    __m256 x1v = _mm256_set1_ps(x1);
    size_t data_base = pair * out_feat, scale_base = g * out_feat;
    size_t full_blocks = out_feat / 8, remainder = out_feat % 8;
    for (size_t blk = 0; blk < full_blocks; ++blk) {
      size_t o = blk * 8;
      __m128i b128 = _mm_loadl_epi64((const __m128i *)(data + data_base + o));
      __m256i b256 = _mm256_cvtepu8_epi32(b128);
      __m256i lo256 = _mm256_and_si256(b256, mask_lo);
      __m256i hi256 = _mm256_and_si256(_mm256_srli_epi32(b256, 4), mask_lo);
      __m256i lo_sign = _mm256_and_si256(lo256, _mm256_set1_epi32(8));
      __m256i lo_neg = _mm256_cmpeq_epi32(lo_sign, _mm256_set1_epi32(8));
      __m256i lo_ext = _mm256_and_si256(lo_neg, _mm256_set1_epi32(~0x0F));
      __m256i lo_i32 = _mm256_or_si256(lo256, lo_ext);
      __m256i hi_sign = _mm256_and_si256(hi256, _mm256_set1_epi32(8));
      __m256i hi_neg = _mm256_cmpeq_epi32(hi_sign, _mm256_set1_epi32(8));
      __m256i hi_ext = _mm256_and_si256(hi_neg, _mm256_set1_epi32(~0x0F));
      __m256i hi_i32 = _mm256_or_si256(hi256, hi_ext);
      __m256 lo_f = _mm256_cvtepi32_ps(lo_i32);
      __m256 hi_f = _mm256_cvtepi32_ps(hi_i32);
      __m256 scale_v = _mm256_loadu_ps(scales + scale_base + o);
      __m256 contrib_lo = _mm256_mul_ps(lo_f, x0v);
      __m256 contrib = _mm256_fmadd_ps(hi_f, x1v, contrib_lo);
      __m256 scaled = _mm256_mul_ps(contrib, scale_v);
      __m256 yv = _mm256_loadu_ps(y + o);
      _mm256_storeu_ps(y + o, _mm256_add_ps(yv, scaled));
    }
    if (remainder > 0) {
      size_t ob = full_blocks * 8;
      for (size_t o = 0; o < remainder; ++o) {
        uint8_t byte = data[data_base + ob + o];
        float lo = (float)sign_extend4(byte & 0x0F);
        float hi = (float)sign_extend4((byte >> 4) & 0x0F);
        float scale = scales[scale_base + ob + o];
        float t0 = lo * x0;
        float t1 = hi * x1;
        float t = t0 + t1;
        y[ob + o] += t * scale;
      }
    }
  }
}

void matvec(const QW &w, const float *x, float *y, int path = -1) {
  // quant.rs:160-181 — zero y, then dispatch (AVX2 when CPUID has it).
  std::fill(y, y + w.out_feat, 0.0f);
  bool avx = path < 0 ? cpu_has_avx2() : (path == 1 && cpu_has_avx2());
  if (avx)
    matvec_avx2(w.data.data(), w.scales.data(), w.in_feat, w.out_feat, w.num_groups, x, y);
  else
    matvec_scalar(w.data.data(), w.scales.data(), w.in_feat, w.out_feat, w.num_groups, x, y);
}

void matmul(const QW &w, const float *x, size_t batch, float *y) {
  // quant.rs:400-410
  for (size_t b = 0; b < batch; ++b) matvec(w, x + b * w.in_feat, y + b * w.out_feat);
}

// norm.rs:23-30
void zc_rms_norm_vec(float *x, const float *scale, size_t n) {
  float sum = 0.0f;  // Iterator::sum over f32 is a sequential fold
  for (size_t i = 0; i < n; ++i) {
    float sq = x[i] * x[i];
    sum += sq;
  }
  float mean_sq = sum / (float)n;
  float inv = 1.0f / std::sqrt(mean_sq + NORM_EPS);
  for (size_t i = 0; i < n; ++i) {
    float a = (1.0f + scale[i]) * x[i];
    x[i] = a * inv;
  }
}

// ops.rs:5-36
void softmax_inplace(float *x, size_t n) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, x[i]);  // f32::max ignores NaN
  if (mx == -INFINITY) {
    float u = 1.0f / (float)n;
    for (size_t i = 0; i < n; ++i) x[i] = u;
    return;
  }
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    x[i] = std::exp(x[i] - mx);
    sum += x[i];
  }
  if (sum == 0.0f) {
    float u = 1.0f / (float)n;
    for (size_t i = 0; i < n; ++i) x[i] = u;
    return;
  }
  float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

inline float sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }  // ops.rs:40-42

inline float gelu(float x) {  // ops.rs:47-52
  const float C = 0.79788456f, A = 0.044715f;
  float ax = A * x;
  float axx = ax * x;
  float axxx = axx * x;
  float inner = C * (x + axxx);
  float t = 1.0f + std::tanh(inner);
  float hx = 0.5f * x;
  return hx * t;
}

// ops.rs:56-63 — sequential, no FMA.
inline float dot(const float *a, const float *b, size_t n) {
  float acc = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float p = a[i] * b[i];
    acc += p;
  }
  return acc;
}

// ── RoPE (rope.rs) ────────────────────────────────────────────────────────────
struct Rope {
  std::vector<float> cos, sin;
  size_t max_len = 0, half_dim = 0;
};

void rope_table(size_t max_len, size_t head_dim, float base, float *cos_t, float *sin_t) {
  // rope.rs:20-41
  size_t half = head_dim / 2;
  for (size_t pos = 0; pos < max_len; ++pos)
    for (size_t i = 0; i < half; ++i) {
      float e = 2.0f * (float)i;
      e = e / (float)head_dim;
      float theta = (float)pos / std::pow(base, e);
      cos_t[pos * half + i] = std::cos(theta);
      sin_t[pos * half + i] = std::sin(theta);
    }
}

void rope_apply(const float *cos_t, const float *sin_t, size_t half, float *x,
                size_t seq_len, size_t num_heads, size_t head_dim, size_t offset) {
  // rope.rs:44-77
  for (size_t t = 0; t < seq_len; ++t) {
    size_t pos = t + offset;
    const float *cr = cos_t + pos * half;
    const float *sr = sin_t + pos * half;
    for (size_t h = 0; h < num_heads; ++h) {
      float *left = x + (t * num_heads + h) * head_dim;
      float *right = left + half;
      for (size_t i = 0; i < half; ++i) {
        float x0 = left[i], x1 = right[i];
        float a = x0 * cr[i], b = x1 * sr[i];
        float c = x1 * cr[i], d = x0 * sr[i];
        left[i] = a - b;
        right[i] = c + d;
      }
    }
  }
}

// ── KvCache (attn.rs:22-68) ───────────────────────────────────────────────────
struct KvCache {
  std::vector<float> k, v;
  size_t len = 0, max_len = 0, kv_heads = 0, head_dim = 0;
  KvCache(size_t ml, size_t kh, size_t hd)
      : k(ml * kh * hd, 0.0f), v(ml * kh * hd, 0.0f), max_len(ml), kv_heads(kh), head_dim(hd) {}
  void push_kv(const float *kv, const float *vv) {
    if (len >= max_len) return;  // saturates silently (attn.rs:54-61)
    size_t stride = kv_heads * head_dim, base = len * stride;
    std::memcpy(&k[base], kv, stride * sizeof(float));
    std::memcpy(&v[base], vv, stride * sizeof(float));
    ++len;
  }
};

// ── Config (config.rs:22-103) ─────────────────────────────────────────────────
struct Config {
  size_t d_model = 512, num_heads = 8, num_kv_heads = 4, num_layers = 12,
         num_dec_layers = 8, vocab_size = 8192, max_enc_len = 1024,
         max_dec_len = 512, ffn_dim = 2048;
  bool no_feedforward = true;
  int activation = 0;  // 0 drelu, 1 swiglu, 2 geglu
  float rope_theta = 10000.0f;
  size_t head_dim() const { return d_model / num_heads; }
  size_t kv_repeat() const { return num_heads / num_kv_heads; }
  const char *validate() const {
    if (num_heads == 0) return "num_heads must be > 0";
    if (num_kv_heads == 0) return "num_kv_heads must be > 0";
    if (d_model == 0) return "d_model must be > 0";
    if (d_model % num_heads) return "d_model must be divisible by num_heads";
    if (num_heads % num_kv_heads) return "num_heads must be divisible by num_kv_heads";
    if (vocab_size == 0) return "vocab_size must be > 0";
    return nullptr;
  }
};

struct Attn {
  QW wq, wk, wv, wo;
  std::vector<float> q_norm, k_norm;
};
struct Ffn {
  QW gate, up, down;
};
struct EncLayer {
  Attn sa;
  float sa_gate = 0;
  std::vector<float> norm;
  bool has_ffn = false;
  Ffn ffn;
  float ffn_gate = 0;
  std::vector<float> ffn_norm;
};
struct DecLayer {
  Attn sa, ca;
  float sa_gate = 0, ca_gate = 0;
  std::vector<float> sa_norm, ca_norm;
  bool has_ffn = false;
  Ffn ffn;
  float ffn_gate = 0;
  std::vector<float> ffn_norm;
};

struct Model {
  Config cfg;
  std::vector<float> emb;
  std::vector<EncLayer> enc;
  std::vector<DecLayer> dec;
  std::vector<float> enc_final_norm, dec_final_norm;
  Rope rope;
  float embed_scale = 0;
  // contrastive head (engine.rs:28-34), present when the file has its tensors
  std::vector<float> c_hk, c_hb, c_pk;  // [d][h], [h], [h][c]
  size_t c_hidden = 0, c_dim = 0;
};

// ffn.rs:19-56
void ffn_forward(const Ffn &w, size_t d_ff, const float *x, float *out, int act) {
  std::vector<float> gate(d_ff), up(d_ff);
  matvec(w.gate, x, gate.data());
  matvec(w.up, x, up.data());
  for (size_t i = 0; i < d_ff; ++i) {
    float g = gate[i], u = up[i];
    if (act == 1) {
      float sg = g * sigmoid(g);
      gate[i] = sg * u;
    } else if (act == 2) {
      gate[i] = gelu(g) * u;
    } else {
      float rg = g > 0.0f ? g : 0.0f, ru = u > 0.0f ? u : 0.0f;
      gate[i] = rg * ru;
    }
  }
  matvec(w.down, gate.data(), out);
}

// attn.rs:100-183
void self_attn_incremental(const Model &m, const float *x, float *out, const Attn &w,
                           KvCache &cache) {
  const Config &c = m.cfg;
  size_t d = c.d_model, h = c.num_heads, kvh = c.num_kv_heads, hd = c.head_dim();
  std::vector<float> q(h * hd), k(kvh * hd), v(kvh * hd);
  matvec(w.wq, x, q.data());
  matvec(w.wk, x, k.data());
  matvec(w.wv, x, v.data());
  for (size_t i = 0; i < h; ++i) zc_rms_norm_vec(&q[i * hd], w.q_norm.data(), hd);
  for (size_t i = 0; i < kvh; ++i) zc_rms_norm_vec(&k[i * hd], w.k_norm.data(), hd);
  rope_apply(m.rope.cos.data(), m.rope.sin.data(), m.rope.half_dim, q.data(), 1, h, hd, cache.len);
  rope_apply(m.rope.cos.data(), m.rope.sin.data(), m.rope.half_dim, k.data(), 1, kvh, hd, cache.len);
  cache.push_kv(k.data(), v.data());
  size_t ctx = cache.len;
  float scale = std::pow((float)hd, -0.5f);
  std::vector<float> scores(ctx), head_out(d, 0.0f);
  size_t kvs = kvh * hd;
  for (size_t hi = 0; hi < h; ++hi) {
    size_t kvi = hi / c.kv_repeat();
    const float *qh = &q[hi * hd];
    for (size_t t = 0; t < ctx; ++t) scores[t] = dot(qh, &cache.k[t * kvs + kvi * hd], hd) * scale;
    softmax_inplace(scores.data(), ctx);
    float *oh = &head_out[hi * hd];
    for (size_t e = 0; e < hd; ++e) oh[e] = 0.0f;
    for (size_t t = 0; t < ctx; ++t) {
      const float *vh = &cache.v[t * kvs + kvi * hd];
      float a = scores[t];
      for (size_t e = 0; e < hd; ++e) {
        float p = a * vh[e];
        oh[e] += p;
      }
    }
  }
  matvec(w.wo, head_out.data(), out);
}

// attn.rs:189-273 (mask = None: the encoder is bidirectional)
void self_attn_full(const Model &m, const float *x, float *out, const Attn &w, size_t T) {
  const Config &c = m.cfg;
  size_t h = c.num_heads, kvh = c.num_kv_heads, hd = c.head_dim();
  size_t qd = h * hd, kvd = kvh * hd;
  std::vector<float> q(T * qd), k(T * kvd), v(T * kvd);
  matmul(w.wq, x, T, q.data());
  matmul(w.wk, x, T, k.data());
  matmul(w.wv, x, T, v.data());
  for (size_t t = 0; t < T; ++t) {
    for (size_t i = 0; i < h; ++i) zc_rms_norm_vec(&q[(t * h + i) * hd], w.q_norm.data(), hd);
    for (size_t i = 0; i < kvh; ++i) zc_rms_norm_vec(&k[(t * kvh + i) * hd], w.k_norm.data(), hd);
  }
  rope_apply(m.rope.cos.data(), m.rope.sin.data(), m.rope.half_dim, q.data(), T, h, hd, 0);
  rope_apply(m.rope.cos.data(), m.rope.sin.data(), m.rope.half_dim, k.data(), T, kvh, hd, 0);
  float scale = std::pow((float)hd, -0.5f);
  std::vector<float> head_out(T * qd, 0.0f), scores(T);
  for (size_t t = 0; t < T; ++t)
    for (size_t hi = 0; hi < h; ++hi) {
      size_t kvi = hi / c.kv_repeat();
      const float *qh = &q[(t * h + hi) * hd];
      for (size_t s = 0; s < T; ++s) scores[s] = dot(qh, &k[(s * kvh + kvi) * hd], hd) * scale;
      softmax_inplace(scores.data(), T);
      float *oh = &head_out[(t * h + hi) * hd];
      for (size_t e = 0; e < hd; ++e) oh[e] = 0.0f;
      for (size_t s = 0; s < T; ++s) {
        const float *vh = &v[(s * kvh + kvi) * hd];
        float a = scores[s];
        for (size_t e = 0; e < hd; ++e) {
          float p = a * vh[e];
          oh[e] += p;
        }
      }
    }
  matmul(w.wo, head_out.data(), T, out);
}

// attn.rs:281-337
void cross_attn_incremental(const Model &m, const float *x, float *out, const Attn &w,
                            const KvCache &enc_kv) {
  const Config &c = m.cfg;
  size_t h = c.num_heads, kvh = c.num_kv_heads, hd = c.head_dim();
  size_t qd = h * hd, ctx = enc_kv.len;
  std::vector<float> q(qd);
  matvec(w.wq, x, q.data());
  for (size_t i = 0; i < h; ++i) zc_rms_norm_vec(&q[i * hd], w.q_norm.data(), hd);
  float scale = std::pow((float)hd, -0.5f);
  size_t kvs = kvh * hd;
  std::vector<float> scores(ctx), head_out(qd, 0.0f);
  for (size_t hi = 0; hi < h; ++hi) {
    size_t kvi = hi / c.kv_repeat();
    const float *qh = &q[hi * hd];
    for (size_t t = 0; t < ctx; ++t) scores[t] = dot(qh, &enc_kv.k[t * kvs + kvi * hd], hd) * scale;
    softmax_inplace(scores.data(), ctx);
    float *oh = &head_out[hi * hd];
    for (size_t e = 0; e < hd; ++e) oh[e] = 0.0f;
    for (size_t t = 0; t < ctx; ++t) {
      const float *vh = &enc_kv.v[t * kvs + kvi * hd];
      float a = scores[t];
      for (size_t e = 0; e < hd; ++e) {
        float p = a * vh[e];
        oh[e] += p;
      }
    }
  }
  matvec(w.wo, head_out.data(), out);
}

// layers.rs:46-93
void encoder_layer_forward(const Model &m, float *x, const EncLayer &L, size_t T) {
  size_t d = m.cfg.d_model;
  std::vector<float> normed(x, x + T * d), tmp(T * d);
  for (size_t t = 0; t < T; ++t) zc_rms_norm_vec(&normed[t * d], L.norm.data(), d);
  self_attn_full(m, normed.data(), tmp.data(), L.sa, T);
  float gate = sigmoid(L.sa_gate);
  for (size_t i = 0; i < T * d; ++i) {
    float p = gate * tmp[i];
    x[i] += p;
  }
  if (L.has_ffn) {
    float fg = sigmoid(L.ffn_gate);
    std::vector<float> row(d), o(d);
    for (size_t t = 0; t < T; ++t) {
      std::copy(x + t * d, x + (t + 1) * d, row.begin());
      zc_rms_norm_vec(row.data(), L.ffn_norm.data(), d);
      ffn_forward(L.ffn, m.cfg.ffn_dim, row.data(), o.data(), m.cfg.activation);
      for (size_t i = 0; i < d; ++i) {
        float p = fg * o[i];
        x[t * d + i] += p;
      }
    }
  }
}

// layers.rs:100-149
void decoder_layer_forward(const Model &m, float *x, const DecLayer &L, const KvCache &enc_kv,
                           KvCache &self_kv) {
  size_t d = m.cfg.d_model;
  std::vector<float> normed(x, x + d), tmp(d);
  zc_rms_norm_vec(normed.data(), L.sa_norm.data(), d);
  self_attn_incremental(m, normed.data(), tmp.data(), L.sa, self_kv);
  float g = sigmoid(L.sa_gate);
  for (size_t i = 0; i < d; ++i) {
    float p = g * tmp[i];
    x[i] += p;
  }
  std::copy(x, x + d, normed.begin());
  zc_rms_norm_vec(normed.data(), L.ca_norm.data(), d);
  cross_attn_incremental(m, normed.data(), tmp.data(), L.ca, enc_kv);
  float cg = sigmoid(L.ca_gate);
  for (size_t i = 0; i < d; ++i) {
    float p = cg * tmp[i];
    x[i] += p;
  }
  if (L.has_ffn) {
    std::copy(x, x + d, normed.begin());
    zc_rms_norm_vec(normed.data(), L.ffn_norm.data(), d);
    ffn_forward(L.ffn, m.cfg.ffn_dim, normed.data(), tmp.data(), m.cfg.activation);
    float fg = sigmoid(L.ffn_gate);
    for (size_t i = 0; i < d; ++i) {
      float p = fg * tmp[i];
      x[i] += p;
    }
  }
}

// model.rs:103-115
void lm_head_scalar(const Model &m, const float *hidden, float *logits) {
  size_t d = m.cfg.d_model, V = m.cfg.vocab_size;
  for (size_t tok = 0; tok < V; ++tok) {
    const float *e = &m.emb[tok * d];
    float acc = 0.0f;
    for (size_t i = 0; i < d; ++i) {
      float p = hidden[i] * e[i];
      acc += p;
    }
    logits[tok] = acc;
  }
}

// model.rs:119-149, same intrinsics and horizontal-sum order.
__attribute__((target("avx2,fma"))) void lm_head_avx2(const Model &m, const float *hidden,
                                                      float *logits) {
  size_t d = m.cfg.d_model, V = m.cfg.vocab_size, chunks = d / 8;
  for (size_t tok = 0; tok < V; ++tok) {
    const float *ep = m.emb.data() + tok * d;
    __m256 acc = _mm256_setzero_ps();
    for (size_t c = 0; c < chunks; ++c) {
      __m256 h = _mm256_loadu_ps(hidden + c * 8);
      __m256 e = _mm256_loadu_ps(ep + c * 8);
      acc = _mm256_fmadd_ps(h, e, acc);
    }
    __m128 hi128 = _mm256_extractf128_ps(acc, 1);
    __m128 lo128 = _mm256_castps256_ps128(acc);
    __m128 sum128 = _mm_add_ps(hi128, lo128);
    __m128 shuf = _mm_shuffle_ps(sum128, sum128, 0x4E);
    __m128 sum64 = _mm_add_ps(sum128, shuf);
    __m128 shuf2 = _mm_shuffle_ps(sum64, sum64, 0xB1);
    __m128 sum32 = _mm_add_ss(sum64, shuf2);
    float result = _mm_cvtss_f32(sum32);
    for (size_t i = chunks * 8; i < d; ++i) {
      float p = hidden[i] * ep[i];
      result += p;
    }
    logits[tok] = result;
  }
}

void lm_head(const Model &m, const float *hidden, float *logits) {  // model.rs:89-100
  if (cpu_has_avx2())
    lm_head_avx2(m, hidden, logits);
  else
    lm_head_scalar(m, hidden, logits);
}

// model.rs:196-231
void fill_cross_kv(const Model &m, const float *enc, size_t T, std::vector<KvCache> &caches) {
  size_t kvh = m.cfg.num_kv_heads, hd = m.cfg.head_dim(), kvd = kvh * hd;
  for (size_t li = 0; li < m.dec.size(); ++li) {
    KvCache &kv = caches[li];
    kv.len = 0;
    std::vector<float> ka(T * kvd), va(T * kvd);
    matmul(m.dec[li].ca.wk, enc, T, ka.data());
    matmul(m.dec[li].ca.wv, enc, T, va.data());
    for (size_t t = 0; t < T; ++t)
      for (size_t i = 0; i < kvh; ++i)
        zc_rms_norm_vec(&ka[(t * kvh + i) * hd], m.dec[li].ca.k_norm.data(), hd);
    for (size_t t = 0; t < T; ++t) kv.push_kv(&ka[t * kvd], &va[t * kvd]);
  }
}

// model.rs:153-192
std::vector<float> encode(const Model &m, const uint32_t *ids, size_t T,
                          std::vector<KvCache> &enc_kv) {
  size_t d = m.cfg.d_model;
  std::vector<float> x(T * d);
  for (size_t t = 0; t < T; ++t) {
    const float *row = &m.emb[(size_t)ids[t] * d];
    for (size_t i = 0; i < d; ++i) x[t * d + i] = row[i] * m.embed_scale;
  }
  for (const auto &L : m.enc) encoder_layer_forward(m, x.data(), L, T);
  for (size_t t = 0; t < T; ++t) zc_rms_norm_vec(&x[t * d], m.enc_final_norm.data(), d);
  fill_cross_kv(m, x.data(), T, enc_kv);
  return x;
}

// model.rs:235-265
void decode_step(const Model &m, uint32_t tok, const std::vector<KvCache> &enc_kv,
                 std::vector<KvCache> &dec_kv, float *logits) {
  size_t d = m.cfg.d_model;
  std::vector<float> x(d);
  const float *row = &m.emb[(size_t)tok * d];
  for (size_t i = 0; i < d; ++i) x[i] = row[i] * m.embed_scale;
  for (size_t li = 0; li < m.dec.size(); ++li)
    decoder_layer_forward(m, x.data(), m.dec[li], enc_kv[li], dec_kv[li]);
  zc_rms_norm_vec(x.data(), m.dec_final_norm.data(), d);
  lm_head(m, x.data(), logits);
}

std::vector<KvCache> make_enc_kv(const Model &m, size_t T) {  // model.rs:268-272
  return std::vector<KvCache>(m.cfg.num_dec_layers, KvCache(T, m.cfg.num_kv_heads, m.cfg.head_dim()));
}
std::vector<KvCache> make_dec_kv(const Model &m) {  // model.rs:275-285
  return std::vector<KvCache>(m.cfg.num_dec_layers,
                              KvCache(m.cfg.max_dec_len, m.cfg.num_kv_heads, m.cfg.head_dim()));
}

// Total order of f32::total_cmp (IEEE 754 totalOrder) as an unsigned key.
inline uint32_t total_order_key(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// engine.rs:286-322 on token IDs.
size_t generate(const Model &m, const uint32_t *ids, size_t T, size_t max_new,
                const uint64_t *mask_bits, int stop_on_eos, uint32_t *out_ids, float *margins,
                float *logits_out, float *tops = nullptr) {
  size_t V = m.cfg.vocab_size, words = (V + 63) / 64;
  auto enc_kv = make_enc_kv(m, T);
  auto dec_kv = make_dec_kv(m);
  encode(m, ids, T, enc_kv);
  std::vector<float> logits(V);
  uint32_t cur = EOS_ID;
  size_t n = 0;
  for (size_t step = 0; step < max_new; ++step) {
    decode_step(m, cur, enc_kv, dec_kv, logits.data());
    if (mask_bits) {
      const uint64_t *mb = mask_bits + step * words;
      for (size_t v = 0; v < V; ++v)
        logits[v] += ((mb[v >> 6] >> (v & 63)) & 1) ? 0.0f : MASK_BLOCKED;
    }
    // max_by(total_cmp): the last of equal maxima wins.
    size_t best = 0;
    for (size_t v = 1; v < V; ++v)
      if (total_order_key(logits[v]) >= total_order_key(logits[best])) best = v;
    if (margins) {
      float second = -INFINITY;
      for (size_t v = 0; v < V; ++v)
        if (v != best) second = std::max(second, logits[v]);
      margins[step] = logits[best] - second;
    }
    if (tops) tops[step] = logits[best];
    if (logits_out) std::memcpy(logits_out + step * V, logits.data(), V * sizeof(float));
    uint32_t next = (uint32_t)best;
    if (stop_on_eos && next == EOS_ID) break;
    out_ids[n++] = next;
    cur = next;
  }
  return n;
}

// ── SafeTensors (crates/needle-infer/src/safetensors.rs) ───────────────────────
enum class DType { F32, BF16, F16, I8, I4 };
struct TensorMeta {
  DType dtype;
  std::vector<size_t> shape;
  size_t start, end;
};

struct SafeTensors {
  std::vector<uint8_t> data;
  std::map<std::string, TensorMeta> tensors;
  std::map<std::string, std::string> metadata;

  bool get_f32(const std::string &name, std::vector<float> &out) const {  // :72-122
    auto it = tensors.find(name);
    if (it == tensors.end()) return false;
    const TensorMeta &mt = it->second;
    const uint8_t *raw = data.data() + mt.start;
    size_t n = mt.end - mt.start;
    out.clear();
    switch (mt.dtype) {
      case DType::F32:
        out.resize(n / 4);
        for (size_t i = 0; i < n / 4; ++i) std::memcpy(&out[i], raw + 4 * i, 4);
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
        size_t expected = 1;
        for (size_t s : mt.shape) expected *= s;
        if (n * 2 != expected) return false;
        out.resize(expected);
        for (size_t i = 0; i < n; ++i) {
          out[2 * i] = (float)sign_extend4(raw[i] & 0x0F);
          out[2 * i + 1] = (float)sign_extend4(raw[i] >> 4);
        }
        break;
      }
    }
    return true;
  }
  const TensorMeta *meta(const std::string &name) const {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : &it->second;
  }
  static float f16_to_f32(uint16_t bits) {  // safetensors.rs:376-398
    uint32_t sign = (uint32_t)(bits >> 15) << 31;
    uint32_t exp = (bits >> 10) & 0x1F, mant = bits & 0x3FF;
    if (exp == 0) {
      float val = (float)mant / (float)(1u << 24);
      return sign ? -val : val;
    }
    uint32_t out;
    if (exp == 31)
      out = sign | 0x7F800000u | (mant << 13);
    else
      out = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    float f;
    std::memcpy(&f, &out, 4);
    return f;
  }
};

// Minimal header parsing in the manner of safetensors.rs:140-339.
size_t find_matching_brace(const std::string &s, size_t start) {
  size_t depth = 0;
  for (size_t i = start; i < s.size(); ++i) {
    char c = s[i];
    if (c == '{' || c == '[')
      ++depth;
    else if (c == '}' || c == ']') {
      depth = depth ? depth - 1 : 0;
      if (depth == 0) return i;
    }
  }
  return s.size() - 1;
}

std::vector<std::pair<std::string, std::string>> split_entries(const std::string &s) {
  std::vector<std::pair<std::string, std::string>> res;
  size_t i = 0, n = s.size();
  auto ws = [](char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f'; };
  while (i < n) {
    while (i < n && (s[i] == ',' || ws(s[i]))) ++i;
    if (i >= n || s[i] != '"') break;
    ++i;
    size_t ks = i;
    while (i < n) {
      if (s[i] == '\\') { i += 2; continue; }
      if (s[i] == '"') break;
      ++i;
    }
    std::string key = s.substr(ks, std::min(i, n) - ks);
    ++i;
    while (i < n && s[i] != ':') ++i;
    if (i >= n) break;
    ++i;
    while (i < n && ws(s[i])) ++i;
    if (i >= n) break;
    size_t vs = i;
    std::string val;
    if (s[i] == '{') {
      size_t e = find_matching_brace(s, i);
      i = e + 1;
      val = s.substr(vs, e + 1 - vs);
    } else if (s[i] == '"') {
      ++i;
      while (i < n) {
        if (s[i] == '\\') { i += 2; continue; }
        if (s[i] == '"') break;
        ++i;
      }
      ++i;
      val = s.substr(vs, std::min(i, n) - vs);
    } else {
      while (i < n && s[i] != ',' && s[i] != '}') ++i;
      val = s.substr(vs, i - vs);
    }
    res.emplace_back(key, val);
  }
  return res;
}

bool extract_str(const std::string &obj, const std::string &field, std::string &out) {
  std::string nd = "\"" + field + "\"";
  size_t p = obj.find(nd);
  if (p == std::string::npos) return false;
  size_t c = obj.find(':', p + nd.size());
  if (c == std::string::npos) return false;
  size_t q = c + 1;
  while (q < obj.size() && isspace((unsigned char)obj[q])) ++q;
  if (q >= obj.size() || obj[q] != '"') return false;
  size_t e = obj.find('"', q + 1);
  if (e == std::string::npos) return false;
  out = obj.substr(q + 1, e - q - 1);
  return true;
}

bool extract_usize_array(const std::string &obj, const std::string &field, std::vector<size_t> &out) {
  // safetensors.rs:323-339: split the bracket body on ',' and parse each
  // trimmed piece; any piece that fails (including the empty body of "[]")
  // fails the whole array.
  std::string nd = "\"" + field + "\"";
  size_t p = obj.find(nd);
  if (p == std::string::npos) return false;
  size_t b = obj.find('[', p + nd.size());
  if (b == std::string::npos) return false;
  size_t e = obj.find(']', b + 1);
  if (e == std::string::npos) return false;
  std::string inner = obj.substr(b + 1, e - b - 1);
  out.clear();
  size_t i = 0;
  for (;;) {
    size_t comma = inner.find(',', i);
    std::string tok = inner.substr(i, comma == std::string::npos ? std::string::npos : comma - i);
    size_t a = tok.find_first_not_of(" \t\n\r"), z = tok.find_last_not_of(" \t\n\r");
    if (a == std::string::npos) return false;
    tok = tok.substr(a, z - a + 1);
    if (tok[0] == '+') tok = tok.substr(1);
    if (tok.empty()) return false;
    for (char ch : tok)
      if (ch < '0' || ch > '9') return false;
    out.push_back(std::stoull(tok));
    if (comma == std::string::npos) break;
    i = comma + 1;
  }
  return true;
}

bool parse_safetensors(std::vector<uint8_t> raw, SafeTensors &st, std::string &err) {
  // safetensors.rs:43-69, 140-214
  if (raw.size() < 8) { err = "buffer too short"; return false; }
  uint64_t hl = 0;
  std::memcpy(&hl, raw.data(), 8);
  if (hl > raw.size() - 8) { err = "truncated header"; return false; }
  std::string header((const char *)raw.data() + 8, hl);
  size_t a = header.find_first_not_of(" \t\n\r"), z = header.find_last_not_of(" \t\n\r");
  if (a == std::string::npos || header[a] != '{' || header[z] != '}') { err = "expected JSON object"; return false; }
  std::string inner = header.substr(a + 1, z - a - 1);
  for (auto &kv : split_entries(inner)) {
    if (kv.first == "__metadata__") {
      std::string o = kv.second;
      size_t oa = o.find_first_not_of(" \t\n\r"), oz = o.find_last_not_of(" \t\n\r");
      if (oa != std::string::npos && o[oa] == '{' && o[oz] == '}') {
        for (auto &mv : split_entries(o.substr(oa + 1, oz - oa - 1))) {
          std::string v = mv.second;
          if (v.size() >= 2 && v.front() == '"' && v.back() == '"') v = v.substr(1, v.size() - 2);
          st.metadata[mv.first] = v;
        }
      }
      continue;
    }
    std::string dt;
    std::vector<size_t> shape, offs;
    if (!extract_str(kv.second, "dtype", dt)) { err = "missing dtype for " + kv.first; return false; }
    if (!extract_usize_array(kv.second, "shape", shape)) {
      // "[]" (a scalar) splits into one empty token that fails to parse.
      err = "missing shape for " + kv.first;
      return false;
    }
    if (!extract_usize_array(kv.second, "data_offsets", offs)) { err = "missing data_offsets for " + kv.first; return false; }
    if (offs.size() != 2) { err = "data_offsets must have 2 elements"; return false; }
    DType d;
    if (dt == "F32") d = DType::F32;
    else if (dt == "BF16") d = DType::BF16;
    else if (dt == "F16") d = DType::F16;
    else if (dt == "I8") d = DType::I8;
    else if (dt == "I4") d = DType::I4;
    else { err = "unknown dtype " + dt; return false; }
    st.tensors[kv.first] = TensorMeta{d, shape, offs[0], offs[1]};
  }
  st.data.assign(raw.begin() + 8 + hl, raw.end());
  for (auto &kv : st.tensors)
    if (kv.second.start > kv.second.end || kv.second.end > st.data.size()) {
      err = "tensor " + kv.first + " data_offsets out of range";  // a slice panic in the reference
      return false;
    }
  return true;
}

// engine.rs:578-624
bool parse_usize(const std::string &s, size_t &out) {
  if (s.empty()) return false;
  size_t i = s[0] == '+' ? 1 : 0;
  if (i >= s.size()) return false;
  for (size_t j = i; j < s.size(); ++j)
    if (s[j] < '0' || s[j] > '9') return false;
  out = std::stoull(s.substr(i));
  return true;
}

Config load_config(const SafeTensors &st) {
  Config c;
  auto uf = [&](const char *k, size_t fb) {
    auto it = st.metadata.find(k);
    size_t v;
    return (it != st.metadata.end() && parse_usize(it->second, v)) ? v : fb;
  };
  auto ff = [&](const char *k, float fb) {
    auto it = st.metadata.find(k);
    if (it == st.metadata.end()) return fb;
    char *e = nullptr;
    float v = std::strtof(it->second.c_str(), &e);
    return (e && *e == 0 && !it->second.empty()) ? v : fb;
  };
  auto bf = [&](const char *k, bool fb) {
    auto it = st.metadata.find(k);
    if (it == st.metadata.end()) return fb;
    return it->second == "True" || it->second == "true" || it->second == "1";
  };
  Config d;
  size_t me;
  auto it = st.metadata.find("max_enc_len");
  if (it != st.metadata.end() && parse_usize(it->second, me))
    c.max_enc_len = me;
  else if ((it = st.metadata.find("max_seq_len")) != st.metadata.end() && parse_usize(it->second, me))
    c.max_enc_len = me;
  else
    c.max_enc_len = d.max_enc_len;
  auto ai = st.metadata.find("activation");
  c.activation = 0;
  if (ai != st.metadata.end()) c.activation = ai->second == "swiglu" ? 1 : ai->second == "geglu" ? 2 : 0;
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

std::vector<float> load_vec(const SafeTensors &st, const std::string &n, size_t len) {  // :784-786
  std::vector<float> v;
  if (!st.get_f32(n, v)) v.assign(len, 0.0f);
  return v;
}
float load_scalar(const SafeTensors &st, const std::string &n) {  // :788-792
  std::vector<float> v;
  if (!st.get_f32(n, v) || v.empty()) return 0.0f;
  return v[0];
}

bool load_quant(const SafeTensors &st, const std::string &name, size_t in, size_t out, QW &q,
                std::string &err) {
  // engine.rs:752-782
  const TensorMeta *raw = st.meta(name);
  std::vector<float> scales;
  if (raw && st.get_f32(name + ".scale", scales)) {
    if (out == 0 || scales.size() % out != 0) {
      std::vector<float> w;
      if (!st.get_f32(name, w)) w.assign(in * out, 0.0f);
      if (w.size() != in * out) { err = name + ": re-quantize size mismatch"; return false; }
      q = quantize_qw(w.data(), in, out);
      return true;
    }
    q.in_feat = in;
    q.out_feat = out;
    q.num_groups = scales.size() / out;
    q.scales = std::move(scales);
    q.data.assign(st.data.begin() + raw->start, st.data.begin() + raw->end);
    size_t gs = std::min(GROUP_SIZE, in);
    if (q.num_groups * gs < in || q.data.size() < q.num_groups * gs / 2 * out) {
      // The reference would index out of bounds inside matvec (a panic).
      err = name + ": packed data smaller than its scales imply";
      return false;
    }
    return true;
  }
  std::vector<float> w;
  if (!st.get_f32(name, w)) w.assign(in * out, 0.0f);
  if (w.size() != in * out) { err = name + ": tensor size mismatch"; return false; }
  q = quantize_qw(w.data(), in, out);
  return true;
}

bool load_attn(const SafeTensors &st, const Config &c, const std::string &p, Attn &a, std::string &err) {
  // engine.rs:732-750
  size_t d = c.d_model, h = c.num_heads, kvh = c.num_kv_heads, hd = c.head_dim();
  if (!load_quant(st, p + ".wq", d, h * hd, a.wq, err) || !load_quant(st, p + ".wk", d, kvh * hd, a.wk, err) ||
      !load_quant(st, p + ".wv", d, kvh * hd, a.wv, err) || !load_quant(st, p + ".wo", h * hd, d, a.wo, err))
    return false;
  a.q_norm = load_vec(st, p + ".q_norm", hd);
  a.k_norm = load_vec(st, p + ".k_norm", hd);
  return true;
}

bool load_ffn(const SafeTensors &st, const Config &c, const std::string &p, Ffn &f, std::string &err) {
  // engine.rs:722-730
  return load_quant(st, p + ".gate_proj", c.d_model, c.ffn_dim, f.gate, err) &&
         load_quant(st, p + ".up_proj", c.d_model, c.ffn_dim, f.up, err) &&
         load_quant(st, p + ".down_proj", c.ffn_dim, c.d_model, f.down, err);
}

Model *load_model(std::vector<uint8_t> raw, std::string &err) {
  SafeTensors st;
  if (!parse_safetensors(std::move(raw), st, err)) return nullptr;
  Config c = load_config(st);
  if (const char *e = c.validate()) { err = e; return nullptr; }
  auto *m = new Model();
  m->cfg = c;
  size_t d = c.d_model, V = c.vocab_size;
  if (!st.get_f32("embedding", m->emb)) { err = "missing embedding tensor"; delete m; return nullptr; }
  if (m->emb.size() != V * d) {
    err = "embedding size mismatch: got " + std::to_string(m->emb.size()) + ", expected " + std::to_string(V * d);
    delete m;
    return nullptr;
  }
  m->enc.resize(c.num_layers);
  for (size_t i = 0; i < c.num_layers; ++i) {  // engine.rs:677-696
    std::string p = "encoder." + std::to_string(i);
    EncLayer &L = m->enc[i];
    if (!c.no_feedforward) {
      L.has_ffn = true;
      if (!load_ffn(st, c, p + ".ffn", L.ffn, err)) { delete m; return nullptr; }
      L.ffn_gate = load_scalar(st, p + ".ffn_gate");
      L.ffn_norm = load_vec(st, p + ".ffn_norm", d);
    }
    if (!load_attn(st, c, p + ".self_attn", L.sa, err)) { delete m; return nullptr; }
    L.sa_gate = load_scalar(st, p + ".self_attn_gate");
    L.norm = load_vec(st, p + ".norm", d);
  }
  m->dec.resize(c.num_dec_layers);
  for (size_t i = 0; i < c.num_dec_layers; ++i) {  // engine.rs:698-720
    std::string p = "decoder." + std::to_string(i);
    DecLayer &L = m->dec[i];
    if (!c.no_feedforward) {
      L.has_ffn = true;
      if (!load_ffn(st, c, p + ".ffn", L.ffn, err)) { delete m; return nullptr; }
      L.ffn_gate = load_scalar(st, p + ".ffn_gate");
      L.ffn_norm = load_vec(st, p + ".ffn_norm", d);
    }
    if (!load_attn(st, c, p + ".self_attn", L.sa, err) || !load_attn(st, c, p + ".cross_attn", L.ca, err)) {
      delete m;
      return nullptr;
    }
    L.sa_gate = load_scalar(st, p + ".self_attn_gate");
    L.sa_norm = load_vec(st, p + ".self_attn_norm", d);
    L.ca_gate = load_scalar(st, p + ".cross_attn_gate");
    L.ca_norm = load_vec(st, p + ".cross_attn_norm", d);
  }
  m->enc_final_norm = load_vec(st, "encoder_final_norm", d);
  m->dec_final_norm = load_vec(st, "decoder_final_norm", d);
  // Norm vectors of the wrong length would be indexed past their end by the
  // reference (a panic there); reject them here.
  auto badlen = [&](const std::vector<float> &v, size_t n) { return v.size() < n; };
  size_t hd = c.head_dim();
  bool bad = badlen(m->enc_final_norm, d) || badlen(m->dec_final_norm, d);
  for (auto &L : m->enc) bad |= badlen(L.norm, d) || badlen(L.sa.q_norm, hd) || badlen(L.sa.k_norm, hd);
  for (auto &L : m->dec)
    bad |= badlen(L.sa_norm, d) || badlen(L.ca_norm, d) || badlen(L.sa.q_norm, hd) || badlen(L.sa.k_norm, hd) ||
           badlen(L.ca.q_norm, hd) || badlen(L.ca.k_norm, hd);
  if (bad) { err = "norm vector shorter than its dimension"; delete m; return nullptr; }
  // model.rs:44-75
  m->rope.max_len = std::max(c.max_enc_len, c.max_dec_len);
  m->rope.half_dim = hd / 2;
  m->rope.cos.assign(m->rope.max_len * m->rope.half_dim, 0.0f);
  m->rope.sin.assign(m->rope.max_len * m->rope.half_dim, 0.0f);
  rope_table(m->rope.max_len, hd, c.rope_theta, m->rope.cos.data(), m->rope.sin.data());
  m->embed_scale = std::sqrt((float)d);
  // load_contrastive_head (engine.rs:548-573): all three tensors, shapes
  // consistent with d_model, else no head
  {
    std::vector<float> pk, hk, hb;
    if (st.get_f32("contrastive_proj_kernel", pk) && st.get_f32("contrastive_hidden_kernel", hk) &&
        st.get_f32("contrastive_hidden_bias", hb)) {
      size_t h = hb.size();
      if (h != 0 && hk.size() == d * h && pk.size() % h == 0) {
        m->c_hk = std::move(hk);
        m->c_hb = std::move(hb);
        m->c_pk = std::move(pk);
        m->c_hidden = h;
        m->c_dim = m->c_pk.size() / h;
      }
    }
  }
  return m;
}

void set_err(char *err, size_t errlen, const std::string &s) {
  if (err && errlen) {
    std::snprintf(err, errlen, "%s", s.c_str());
  }
}

bool ids_valid(const Model &m, const uint32_t *ids, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (ids[i] >= m.cfg.vocab_size) return false;
  return true;
}

}  // namespace

// ── C API ─────────────────────────────────────────────────────────────────────
extern "C" {

void orc_quant_sizes(size_t in_feat, size_t out_feat, size_t *data_bytes, size_t *num_groups) {
  size_t gs = std::min(GROUP_SIZE, in_feat);
  size_t in_padded = gs ? in_feat + (gs - in_feat % gs) % gs : 0;
  if (data_bytes) *data_bytes = in_padded / 2 * out_feat;
  if (num_groups) *num_groups = gs ? in_padded / gs : 0;
}

void orc_quantize(const float *w, size_t in_feat, size_t out_feat, uint8_t *data, float *scales) {
  quantize(w, in_feat, out_feat, data, scales);
}

void orc_dequantize(const uint8_t *data, const float *scales, size_t in_feat, size_t out_feat,
                    size_t num_groups, float *out) {
  // quant.rs:131-155
  size_t gs = std::min(GROUP_SIZE, in_feat);
  size_t num_pairs = num_groups * gs / 2;
  for (size_t pair = 0; pair < num_pairs; ++pair) {
    size_t r0 = pair * 2, r1 = r0 + 1, g = r0 / gs, base = pair * out_feat;
    for (size_t o = 0; o < out_feat; ++o) {
      uint8_t byte = data[base + o];
      float scale = scales[g * out_feat + o];
      if (r0 < in_feat) out[r0 * out_feat + o] = (float)sign_extend4(byte & 0x0F) * scale;
      if (r1 < in_feat) out[r1 * out_feat + o] = (float)sign_extend4((byte >> 4) & 0x0F) * scale;
    }
  }
}

void orc_matvec(const uint8_t *data, const float *scales, size_t in_feat, size_t out_feat,
                size_t num_groups, const float *x, float *y, int path) {
  std::fill(y, y + out_feat, 0.0f);
  if (path == 1 && cpu_has_avx2())
    matvec_avx2(data, scales, in_feat, out_feat, num_groups, x, y);
  else
    matvec_scalar(data, scales, in_feat, out_feat, num_groups, x, y);
}

void orc_matmul(const uint8_t *data, const float *scales, size_t in_feat, size_t out_feat,
                size_t num_groups, const float *x, size_t batch, float *y, int path) {
  for (size_t b = 0; b < batch; ++b)
    orc_matvec(data, scales, in_feat, out_feat, num_groups, x + b * in_feat, y + b * out_feat, path);
}

int orc_sign_extend4(uint8_t nibble) { return sign_extend4(nibble); }

void orc_zc_rms_norm(float *x, const float *scale, size_t n) { zc_rms_norm_vec(x, scale, n); }
void orc_rope_table(size_t max_len, size_t head_dim, float base, float *c, float *s) {
  rope_table(max_len, head_dim, base, c, s);
}
void orc_rope_apply(const float *c, const float *s, size_t half, float *x, size_t seq_len,
                    size_t num_heads, size_t head_dim, size_t offset) {
  rope_apply(c, s, half, x, seq_len, num_heads, head_dim, offset);
}
void orc_softmax(float *x, size_t n) { softmax_inplace(x, n); }
float orc_sigmoid(float x) { return sigmoid(x); }
float orc_gelu(float x) { return gelu(x); }

void orc_ffn_forward(const uint8_t *gd, const float *gs, const uint8_t *ud, const float *us,
                     const uint8_t *dd, const float *ds, size_t d_model, size_t d_ff,
                     const float *x, float *out, int act) {
  Ffn f;
  size_t db, ng;
  orc_quant_sizes(d_model, d_ff, &db, &ng);
  f.gate.data.assign(gd, gd + db);
  f.gate.scales.assign(gs, gs + ng * d_ff);
  f.gate.in_feat = d_model; f.gate.out_feat = d_ff; f.gate.num_groups = ng;
  f.up.data.assign(ud, ud + db);
  f.up.scales.assign(us, us + ng * d_ff);
  f.up.in_feat = d_model; f.up.out_feat = d_ff; f.up.num_groups = ng;
  orc_quant_sizes(d_ff, d_model, &db, &ng);
  f.down.data.assign(dd, dd + db);
  f.down.scales.assign(ds, ds + ng * d_model);
  f.down.in_feat = d_ff; f.down.out_feat = d_model; f.down.num_groups = ng;
  ffn_forward(f, d_ff, x, out, act);
}

void *orc_model_load_file(const char *path, char *err, size_t errlen) {
  std::ifstream f(path, std::ios::binary);
  if (!f) { set_err(err, errlen, std::string("cannot open ") + path); return nullptr; }
  std::vector<uint8_t> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  std::string e;
  Model *m = load_model(std::move(raw), e);
  if (!m) set_err(err, errlen, e);
  return m;
}

void *orc_model_load_bytes(const uint8_t *bytes, size_t len, char *err, size_t errlen) {
  if (!bytes) { set_err(err, errlen, "null pointer"); return nullptr; }
  std::string e;
  Model *m = load_model(std::vector<uint8_t>(bytes, bytes + len), e);
  if (!m) set_err(err, errlen, e);
  return m;
}

void orc_model_free(void *m) { delete (Model *)m; }

void orc_model_config(const void *mp, int64_t *cfg) {
  const Config &c = ((const Model *)mp)->cfg;
  int64_t v[12] = {(int64_t)c.d_model, (int64_t)c.num_heads, (int64_t)c.num_kv_heads,
                   (int64_t)c.num_layers, (int64_t)c.num_dec_layers, (int64_t)c.vocab_size,
                   (int64_t)c.max_enc_len, (int64_t)c.max_dec_len, (int64_t)c.ffn_dim,
                   (int64_t)c.no_feedforward, (int64_t)c.activation, (int64_t)c.head_dim()};
  std::memcpy(cfg, v, sizeof(v));
}

int orc_forward(const void *mp, const uint32_t *enc_ids, size_t n_enc, const uint32_t *dec_ids,
                size_t n_dec, float *enc_out, float *logits) {
  const Model &m = *(const Model *)mp;
  if (n_enc == 0 || !ids_valid(m, enc_ids, n_enc) || !ids_valid(m, dec_ids, n_dec)) return -1;
  auto enc_kv = make_enc_kv(m, n_enc);
  auto dec_kv = make_dec_kv(m);
  auto x = encode(m, enc_ids, n_enc, enc_kv);
  if (enc_out) std::memcpy(enc_out, x.data(), x.size() * sizeof(float));
  std::vector<float> lg(m.cfg.vocab_size);
  for (size_t i = 0; i < n_dec; ++i) {
    decode_step(m, dec_ids[i], enc_kv, dec_kv, lg.data());
    if (logits) std::memcpy(logits + i * m.cfg.vocab_size, lg.data(), lg.size() * sizeof(float));
  }
  return 0;
}

// encode_contrastive (engine.rs:153-181) + ContrastiveHead::encode
// (engine.rs:37-69): encoder output mean-pooled over positions (sequential
// sums, then * 1/T), relu(pooled @ hidden_kernel + bias) @ proj_kernel, L2
// normalised with eps 1e-12.  Returns the embedding length (0: no head);
// an empty id list gives the zero vector.
size_t orc_encode_contrastive(const void *mp, const uint32_t *ids, size_t n, float *out) {
  const Model &m = *(const Model *)mp;
  if (!m.c_dim) return 0;
  const size_t d = m.cfg.d_model, h = m.c_hidden, c = m.c_dim;
  if (n == 0) {
    std::fill(out, out + c, 0.0f);
    return c;
  }
  if (!ids_valid(m, ids, n)) return 0;
  auto enc_kv = make_enc_kv(m, n);
  auto x = encode(m, ids, n, enc_kv);
  std::vector<float> pooled(d, 0.0f), hidden(h), proj(c);
  for (size_t t = 0; t < n; ++t)
    for (size_t j = 0; j < d; ++j) pooled[j] += x[t * d + j];
  const float inv_n = 1.0f / (float)n;
  for (auto &v : pooled) v *= inv_n;
  for (size_t j = 0; j < h; ++j) {
    float acc = m.c_hb[j];
    for (size_t i = 0; i < d; ++i) acc += pooled[i] * m.c_hk[i * h + j];
    hidden[j] = std::max(acc, 0.0f);
  }
  for (size_t j = 0; j < c; ++j) {
    float acc = 0.0f;
    for (size_t i = 0; i < h; ++i) acc += hidden[i] * m.c_pk[i * c + j];
    proj[j] = acc;
  }
  float sq = 0.0f;
  for (float v : proj) sq += v * v;
  const float norm = std::sqrt(sq + 1e-12f);
  for (size_t j = 0; j < c; ++j) out[j] = proj[j] / norm;
  return c;
}

size_t orc_contrastive_dim(const void *mp) { return ((const Model *)mp)->c_dim; }

size_t orc_generate(const void *mp, const uint32_t *enc_ids, size_t n_enc, size_t max_new,
                    const uint64_t *mask_bits, int stop_on_eos, uint32_t *out_ids, float *margins,
                    float *logits) {
  const Model &m = *(const Model *)mp;
  if (n_enc == 0 || !ids_valid(m, enc_ids, n_enc)) return 0;
  return generate(m, enc_ids, n_enc, max_new, mask_bits, stop_on_eos, out_ids, margins, logits);
}

int orc_run_batch(const void *mp, const uint32_t *ids, const uint64_t *offsets, size_t n_req,
                  size_t max_new, const uint64_t *mask_bits, int stop_on_eos, uint32_t *out_ids,
                  uint32_t *out_lens, float *margins, int n_threads, float *tops) {
  const Model &m = *(const Model *)mp;
  size_t words = (m.cfg.vocab_size + 63) / 64;
  std::atomic<size_t> next{0};
  std::atomic<int> bad{0};
  auto worker = [&]() {
    for (;;) {
      size_t r = next.fetch_add(1);
      if (r >= n_req) return;
      size_t a = offsets[r], b = offsets[r + 1];
      if (b <= a || !ids_valid(m, ids + a, b - a)) {
        out_lens[r] = 0;
        bad = 1;
        continue;
      }
      out_lens[r] = (uint32_t)generate(m, ids + a, b - a, max_new,
                                       mask_bits ? mask_bits + r * max_new * words : nullptr,
                                       stop_on_eos, out_ids + r * max_new,
                                       margins ? margins + r * max_new : nullptr, nullptr,
                                       tops ? tops + r * max_new : nullptr);
    }
  };
  int nt = std::max(1, n_threads);
  std::vector<std::thread> th;
  for (int i = 0; i < nt; ++i) th.emplace_back(worker);
  for (auto &t : th) t.join();
  return bad ? -1 : 0;
}

size_t orc_kv_cache_push_count(size_t max_len, size_t n_push) {
  KvCache c(max_len, 1, 1);
  float z = 0;
  for (size_t i = 0; i < n_push; ++i) c.push_kv(&z, &z);
  return c.len;
}

}  // extern "C"
