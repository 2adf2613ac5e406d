// attention.cu — norms, embedding, RoPE and the three attention variants.
//
// Reference: crates/needle-core/src/{attn.rs,norm.rs,rope.rs,ops.rs,model.rs}.
// All arithmetic is f32; expf/sqrtf/division are the IEEE-accurate device
// versions (no fast-math), so results differ from the reference only by
// summation order.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace ndl {

namespace {
thread_local bool g_pdl = false;
}
void set_pdl(bool on) { g_pdl = on; }
bool pdl_on() { return g_pdl; }

namespace {

// ── ZCRMSNorm rows (norm.rs:23-30) ─────────────────────────────────────────
__global__ void rms_norm_kernel(const float *__restrict__ x, int64_t ldx, float *out, int64_t ldo,
                                const float *__restrict__ scale, int rows, int d) {
  pdl_trigger();
  pdl_wait();
  int row = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *xr = x + (int64_t)row * ldx;
  float *orow = out + (int64_t)row * ldo;
  if (d == 512) {
    float v[16];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float4 t = *reinterpret_cast<const float4 *>(xr + i * 128 + lane * 4);
      v[i * 4 + 0] = t.x;
      v[i * 4 + 1] = t.y;
      v[i * 4 + 2] = t.z;
      v[i * 4 + 3] = t.w;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) ss += v[i] * v[i];
    ss = warp_sum(ss);
    float inv = 1.0f / sqrtf(ss / 512.0f + 1e-6f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float4 s = __ldg(reinterpret_cast<const float4 *>(scale + i * 128 + lane * 4));
      float4 r;
      r.x = ((1.0f + s.x) * v[i * 4 + 0]) * inv;
      r.y = ((1.0f + s.y) * v[i * 4 + 1]) * inv;
      r.z = ((1.0f + s.z) * v[i * 4 + 2]) * inv;
      r.w = ((1.0f + s.w) * v[i * 4 + 3]) * inv;
      *reinterpret_cast<float4 *>(orow + i * 128 + lane * 4) = r;
    }
    return;
  }
  float ss = 0.0f;
  for (int i = lane; i < d; i += 32) ss += xr[i] * xr[i];
  ss = warp_sum(ss);
  float inv = 1.0f / sqrtf(ss / (float)d + 1e-6f);
  for (int i = lane; i < d; i += 32) orow[i] = ((1.0f + __ldg(scale + i)) * xr[i]) * inv;
}

// ZCRMSNorm of 512-wide rows written straight as the bf16 hi/lo planes the
// tensor-core GEMM consumes (row stride ldp), optionally also as f32.
__global__ void rms_norm_planes_kernel(const float *__restrict__ x, int64_t ldx, __nv_bfloat16 *hi, __nv_bfloat16 *lo,
                                       int64_t ldp, float *out, int64_t ldo, const float *__restrict__ scale,
                                       int rows) {
  pdl_trigger();
  pdl_wait();
  int row = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *xr = x + (int64_t)row * ldx;
  float v[16];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 t = *reinterpret_cast<const float4 *>(xr + i * 128 + lane * 4);
    v[i * 4 + 0] = t.x;
    v[i * 4 + 1] = t.y;
    v[i * 4 + 2] = t.z;
    v[i * 4 + 3] = t.w;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) ss += v[i] * v[i];
  ss = warp_sum(ss);
  float inv = 1.0f / sqrtf(ss / 512.0f + 1e-6f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 s4 = __ldg(reinterpret_cast<const float4 *>(scale + i * 128 + lane * 4));
    float r0 = ((1.0f + s4.x) * v[i * 4 + 0]) * inv;
    float r1 = ((1.0f + s4.y) * v[i * 4 + 1]) * inv;
    float r2 = ((1.0f + s4.z) * v[i * 4 + 2]) * inv;
    float r3 = ((1.0f + s4.w) * v[i * 4 + 3]) * inv;
    if (out) *reinterpret_cast<float4 *>(out + (int64_t)row * ldo + i * 128 + lane * 4) = make_float4(r0, r1, r2, r3);
    __nv_bfloat162 h01 = __floats2bfloat162_rn(r0, r1), h23 = __floats2bfloat162_rn(r2, r3);
    float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    __nv_bfloat162 l01 = __floats2bfloat162_rn(r0 - f01.x, r1 - f01.y), l23 = __floats2bfloat162_rn(r2 - f23.x, r3 - f23.y);
    const int64_t o = (int64_t)row * ldp + i * 128 + lane * 4;
    *reinterpret_cast<uint2 *>(hi + o) = make_uint2(*reinterpret_cast<uint32_t *>(&h01), *reinterpret_cast<uint32_t *>(&h23));
    *reinterpret_cast<uint2 *>(lo + o) = make_uint2(*reinterpret_cast<uint32_t *>(&l01), *reinterpret_cast<uint32_t *>(&l23));
  }
}

__global__ void embed_kernel(const uint32_t *__restrict__ ids, const float *__restrict__ emb, float *x, int rows,
                             int d, float es) {
  int row = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *e = emb + (int64_t)ids[row] * d;
  float *xr = x + (int64_t)row * d;
  for (int i = lane; i < d; i += 32) xr[i] = e[i] * es;
}

// Per-head ZCRMSNorm then split-half RoPE for one head of HD values held as
// pairs (i, i + HD/2) by lane i (HD <= 128: two pairs per lane).
__device__ __forceinline__ void norm_rope_head(float *v, int HD, const float *__restrict__ nscale,
                                               const float *__restrict__ cr, const float *__restrict__ sr,
                                               bool rope, int lane) {
  const int half = HD >> 1;
  float a[2], b[2];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    int i = lane + 32 * u;
    a[u] = i < half ? v[i] : 0.0f;
    b[u] = i < half ? v[i + half] : 0.0f;
    ss += a[u] * a[u] + b[u] * b[u];
  }
  ss = warp_sum(ss);
  float inv = 1.0f / sqrtf(ss / (float)HD + 1e-6f);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    int i = lane + 32 * u;
    if (i < half) {
      float x0 = ((1.0f + __ldg(nscale + i)) * a[u]) * inv;
      float x1 = ((1.0f + __ldg(nscale + i + half)) * b[u]) * inv;
      if (rope) {  // rope.rs:63-75
        float c = __ldg(cr + i), s = __ldg(sr + i);
        float l = x0 * c - x1 * s;
        float r = x1 * c + x0 * s;
        x0 = l;
        x1 = r;
      }
      v[i] = x0;
      v[i + half] = x1;
    }
  }
}

// One warp per (row, Q-or-K head).
__global__ void qk_norm_rope_kernel(float *qkv, int rows, const int32_t *__restrict__ pos,
                                    const float *__restrict__ qn, const float *__restrict__ kn,
                                    const float *__restrict__ rc, const float *__restrict__ rs, AttnDims a) {
  int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  int heads = a.H + a.KVH;
  if (w >= (int64_t)rows * heads) return;
  int row = (int)(w / heads), h = (int)(w % heads);
  int ld = (a.H + 2 * a.KVH) * a.HD;
  float *v = qkv + (int64_t)row * ld + h * a.HD;
  int p = pos[row], half = a.HD >> 1;
  norm_rope_head(v, a.HD, h < a.H ? qn : kn, rc + (int64_t)p * half, rs + (int64_t)p * half, true, lane);
}

// One warp per (row, head): per-head ZCRMSNorm without RoPE.
__global__ void head_norm_kernel(float *x, int rows, int64_t ld, int heads, int HD, const float *__restrict__ sc) {
  int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= (int64_t)rows * heads) return;
  int row = (int)(w / heads), h = (int)(w % heads);
  norm_rope_head(x + (int64_t)row * ld + h * HD, HD, sc, nullptr, nullptr, false, threadIdx.x & 31);
}

// ── encoder attention (attn.rs:189-273), flash-style online softmax ────────
// CTA = (64 query rows, one Q head, one request); K/V tiles of 64 keys.
constexpr int EQ = 64, EK = 64, EP = 68;  // padded row stride

__global__ void __launch_bounds__(256) encoder_attn_kernel(const float *__restrict__ qkv,
                                                           const int64_t *__restrict__ seq_off, float *out,
                                                           AttnDims a) {
  extern __shared__ __align__(16) float sm[];
  float *Qs = sm;               // [HD][EP]   Qs[d][r]
  float *Ks = Qs + 64 * EP;     // [HD][EP]   Ks[d][k]
  float *Vs = Ks + 64 * EP;     // [EK][EP]   Vs[k][d]
  float *Ps = Vs + EK * EP;     // [EK][EP]   Ps[k][r]
  const int r_req = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * EQ;
  const int64_t off = seq_off[r_req];
  const int T = (int)(seq_off[r_req + 1] - off);
  if (q0 >= T) return;
  const int HD = a.HD, g = h / (a.H / a.KVH);
  const int ld = (a.H + 2 * a.KVH) * HD;
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const float scale = a.scale;
  const int hd4 = HD >> 2;

  // Q tile -> Qs (transposed)
  for (int i = tid; i < EQ * hd4; i += 256) {
    int r = i / hd4, d4 = i - r * hd4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < T) v = *reinterpret_cast<const float4 *>(qkv + (off + q0 + r) * ld + h * HD + d4 * 4);
    Qs[(d4 * 4 + 0) * EP + r] = v.x;
    Qs[(d4 * 4 + 1) * EP + r] = v.y;
    Qs[(d4 * 4 + 2) * EP + r] = v.z;
    Qs[(d4 * 4 + 3) * EP + r] = v.w;
  }

  float o[4][4];
  float mrow[4], lrow[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.0f;
  }

  for (int k0 = 0; k0 < T; k0 += EK) {
    __syncthreads();
    for (int i = tid; i < EK * hd4; i += 256) {
      int k = i / hd4, d4 = i - k * hd4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (k0 + k < T) {
        const float *row = qkv + (off + k0 + k) * ld;
        kv = *reinterpret_cast<const float4 *>(row + (a.H + g) * HD + d4 * 4);
        vv = *reinterpret_cast<const float4 *>(row + (a.H + a.KVH + g) * HD + d4 * 4);
      }
      Ks[(d4 * 4 + 0) * EP + k] = kv.x;
      Ks[(d4 * 4 + 1) * EP + k] = kv.y;
      Ks[(d4 * 4 + 2) * EP + k] = kv.z;
      Ks[(d4 * 4 + 3) * EP + k] = kv.w;
      *reinterpret_cast<float4 *>(Vs + k * EP + d4 * 4) = vv;
    }
    __syncthreads();
    // S = Q K^T for rows tr*4.., keys tc*4..
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
    for (int d = 0; d < HD; ++d) {
      float4 q = *reinterpret_cast<const float4 *>(Qs + d * EP + tr * 4);
      float4 k = *reinterpret_cast<const float4 *>(Ks + d * EP + tc * 4);
      float qa[4] = {q.x, q.y, q.z, q.w}, ka[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qa[i], ka[j], s[i][j]);
    }
    // online softmax per row; a row's 64 keys live in the 16 lanes sharing tr
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = (k0 + tc * 4 + j < T) ? s[i][j] * scale : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int o2 = 8; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
      float mnew = fmaxf(mrow[i], mx);
      float corr = expf(mrow[i] - mnew);  // exp(-inf) = 0 on the first tile
      float ps = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float p = expf(s[i][j] - mnew);
        s[i][j] = p;
        ps += p;
      }
#pragma unroll
      for (int o2 = 8; o2 > 0; o2 >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o2);
      lrow[i] = lrow[i] * corr + ps;
      mrow[i] = mnew;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[i][j] *= corr;
    }
    // P -> smem (transposed: Ps[k][r])
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4 *>(Ps + (tc * 4 + j) * EP + tr * 4) = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
    __syncthreads();
    // O += P V   rows tr*4.., dims tc*4..
    if (tc * 4 < HD) {
      const int kmax = min(EK, T - k0);
      for (int k = 0; k < kmax; ++k) {
        float4 p = *reinterpret_cast<const float4 *>(Ps + k * EP + tr * 4);
        float4 v = *reinterpret_cast<const float4 *>(Vs + k * EP + tc * 4);
        float pa[4] = {p.x, p.y, p.z, p.w}, va[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) o[i][j] = fmaf(pa[i], va[j], o[i][j]);
      }
    }
  }
  if (tc * 4 < HD) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int r = q0 + tr * 4 + i;
      if (r < T) {
        float inv = 1.0f / lrow[i];
        float4 v = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
        *reinterpret_cast<float4 *>(out + (off + r) * (int64_t)(a.H * HD) + h * HD + tc * 4) = v;
      }
    }
  }
}

// ── decoder self-attention, one new token per request (attn.rs:100-183) ───
// CTA = one request.  Warp w handles heads w, w+8, ...
__global__ void __launch_bounds__(256) dec_self_attn_kernel(const float *__restrict__ qkv,
                                                            const int32_t *__restrict__ step,
                                                            const float *__restrict__ qn,
                                                            const float *__restrict__ kn,
                                                            const float *__restrict__ rc,
                                                            const float *__restrict__ rs, float *kc, float *vc,
                                                            int cap, float *out, AttnDims a) {
  extern __shared__ __align__(16) float sm[];
  const int b = blockIdx.x, HD = a.HD, half = HD >> 1;
  const int qd = a.H * HD, kvd = a.KVH * HD, ld = qd + 2 * kvd;
  float *qs = sm;                 // [H*HD]
  float *sc = sm + qd;            // [H][cap]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = step[b];
  const float *row = qkv + (int64_t)b * ld;
  float *kcb = kc + (int64_t)b * cap * kvd;
  float *vcb = vc + (int64_t)b * cap * kvd;
  const float *cr = rc + (int64_t)pos * half, *sr = rs + (int64_t)pos * half;
  const bool append = pos < cap;  // push_kv saturates silently (attn.rs:53-61)

  for (int h = warp; h < a.H + a.KVH; h += 8) {
    float v[128];
    const float *src = row + h * HD;  // q heads then k heads are contiguous
    for (int i = lane; i < half; i += 32) {
      v[i] = src[i];
      v[i + half] = src[i + half];
    }
    norm_rope_head(v, HD, h < a.H ? qn : kn, cr, sr, true, lane);
    if (h < a.H) {
      for (int i = lane; i < half; i += 32) {
        qs[h * HD + i] = v[i];
        qs[h * HD + i + half] = v[i + half];
      }
    } else if (append) {
      int g = h - a.H;
      float *kd = kcb + (int64_t)pos * kvd + g * HD;
      float *vd = vcb + (int64_t)pos * kvd + g * HD;
      const float *vs = row + qd + kvd + g * HD;
      for (int i = lane; i < half; i += 32) {
        kd[i] = v[i];
        kd[i + half] = v[i + half];
        vd[i] = vs[i];
        vd[i + half] = vs[i + half];
      }
    }
  }
  __syncthreads();
  const int ctx = append ? pos + 1 : cap;
  const int rep = a.H / a.KVH;
  const float scale = a.scale;
  for (int h = warp; h < a.H; h += 8) {
    const int g = h / rep;
    float *s = sc + h * cap;
    float mx = -INFINITY;
    for (int t = lane; t < ctx; t += 32) {
      const float *k = kcb + (int64_t)t * kvd + g * HD;
      float acc = 0.0f;
      for (int d = 0; d < HD; ++d) acc = fmaf(qs[h * HD + d], k[d], acc);
      acc *= scale;
      s[t] = acc;
      mx = fmaxf(mx, acc);
    }
    mx = warp_max(mx);
    float sum = 0.0f;
    for (int t = lane; t < ctx; t += 32) {
      float p = expf(s[t] - mx);
      s[t] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    float inv = 1.0f / sum;
    __syncwarp();
    for (int d = lane; d < HD; d += 32) {
      float acc = 0.0f;
      for (int t = 0; t < ctx; ++t) acc = fmaf(s[t] * inv, vcb[(int64_t)t * kvd + g * HD + d], acc);
      out[(int64_t)b * qd + h * HD + d] = acc;
    }
  }
}

// ── decoder attention over a K/V row range, head dim 64 ────────────────────
// One value as the bf16 pair (hi, lo) of a tensor-core operand plane:
// hi = bf16(v), lo = bf16(v - hi).
__device__ __forceinline__ void store_split(__nv_bfloat16 *hi, __nv_bfloat16 *lo, float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  *hi = h;
  *lo = __float2bfloat16_rn(v - __bfloat162float(h));
}

constexpr int CA_TILE = 64, CA_STAGES = 3, CA_HD = 64, CA_REP = 2;

// Dynamic shared memory of cross_attn_kernel for prompts of up to max_len:
// 128 bytes of alignment slack, the ring, q, statistics, scores, barriers.
inline int ca_pad(int n) { return (n + CA_TILE - 1) / CA_TILE * CA_TILE; }
inline size_t cross_attn_smem(int max_len) {
  return 128 +
         ((size_t)CA_STAGES * CA_TILE * CA_HD + CA_REP * CA_HD + CA_REP * 8 + (size_t)CA_REP * ca_pad(max_len)) *
             sizeof(float) +
         CA_STAGES * sizeof(uint64_t) + 8;
}

// Decoder cross-attention (attn.rs:281-337), head dim 64, two query heads
// per KV head.  CTA = (request, KV head), 256 threads = 16 half-warps.  The
// dominant HBM reader of batched decode: each CTA streams its request's
// encoder K rows, then its V rows, exactly once, through a ring of CA_STAGES
// shared-memory tiles of 64 rows x 64 dimensions: one TMA load per tile
// (thread 0; the head-major K/V planes as one [rows][64] tensor, in which
// this head's rows of the request are contiguous),
// completing on the stage's mbarrier, CA_STAGES - 1 tiles ahead of the tile
// being read, so the V tiles are in flight while the softmax runs and no
// register holds data in flight.  Rows past the request belong to the next
// request (or read as zeros past the planes) and are masked.
// Exact softmax as ops.rs:5-36: scores of all rows, maximum, exponentials
// and their sum, then P V.  A half-warp reads one row (lane l: dimensions
// 4l..4l+3) and the two query heads share every read.
__global__ void __launch_bounds__(256) cross_attn_kernel(const __grid_constant__ CUtensorMap kvmap,
                                                         const float *__restrict__ q, const float *__restrict__ qn,
                                                         int64_t k_row0, int64_t v_row0, int64_t head_rows,
                                                         const int64_t *__restrict__ seq_off, float *out,
                                                         __nv_bfloat16 *hi, __nv_bfloat16 *lo, int64_t ldp,
                                                         AttnDims a, int max_len, int *err) {
  constexpr int HD = CA_HD, REP = CA_REP, NHW = 16, NW = 8, NT = 256;
  extern __shared__ __align__(16) unsigned char ca_smem[];
  float *sm = reinterpret_cast<float *>(((uintptr_t)ca_smem + 127) & ~(uintptr_t)127);
  float(*ring)[CA_TILE][HD] = reinterpret_cast<float(*)[CA_TILE][HD]>(sm);
  float *qs = sm + CA_STAGES * CA_TILE * HD;  // [REP][64]
  float *stat = qs + REP * HD;                // [REP][NW]
  float *sc = stat + REP * NW;                // [REP][Tp] scores, then weights (0 past T)
  float *red = sm;                            // [16][REP][64], over the ring once it is drained
  uint64_t *full =
      reinterpret_cast<uint64_t *>(((uintptr_t)(sc + REP * ((max_len + CA_TILE - 1) / CA_TILE * CA_TILE)) + 7) &
                                   ~(uintptr_t)7);
  const int b = blockIdx.y, g = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, hw = tid >> 4, hl = tid & 15;
  pdl_trigger();
  if (tid == 0) {
    for (int s = 0; s < CA_STAGES; ++s) tc::mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();
  const int64_t off = seq_off[b];
  const int T = (int)(seq_off[b + 1] - off);
  const int qd = a.H * HD;
  const int nt = (T + CA_TILE - 1) / CA_TILE, ntot = 2 * nt;  // K tiles, then V tiles
  const int Tp = nt * CA_TILE;                                 // score rows, padded to whole tiles
  auto issue = [&](int k) {  // thread 0
    const int s = k % CA_STAGES;
    const bool isv = k >= nt;
    const int64_t y = (isv ? v_row0 : k_row0) + g * head_rows + off + (int64_t)(isv ? k - nt : k) * CA_TILE;
    tc::mbar_expect_tx(&full[s], (uint32_t)(CA_TILE * HD * 4));
    tc::tma_load_2d(&ring[s][0][0], &kvmap, &full[s], 0, (int)y);
  };
  if (tid == 0)
    for (int k = 0; k < CA_STAGES - 1 && k < ntot; ++k) issue(k);
  if (warp < REP) {  // q heads of this group, q_norm (attn.rs:296-300); no RoPE
    float *v = qs + warp * HD;
    const float *src = q + (int64_t)b * qd + (g * REP + warp) * HD;
    v[lane] = src[lane];
    v[lane + 32] = src[lane + 32];
    __syncwarp();
    norm_rope_head(v, HD, qn, nullptr, nullptr, false, lane);
  }
  __syncthreads();
  float qr[REP][4];
#pragma unroll
  for (int j = 0; j < REP; ++j) {
    const float4 t = *reinterpret_cast<const float4 *>(qs + j * HD + hl * 4);
    qr[j][0] = t.x;
    qr[j][1] = t.y;
    qr[j][2] = t.z;
    qr[j][3] = t.w;
  }
  float acc[REP][4];
#pragma unroll
  for (int j = 0; j < REP; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  int k = 0;
  bool ok = true;  // the same in every thread
  const bool b3 = hl & 8, b2 = hl & 4, b1 = hl & 2;
  for (; k < ntot; ++k) {
    // the stage of tile k + CA_STAGES - 1 was freed by the barrier ending tile k - 1
    if (tid == 0 && k + CA_STAGES - 1 < ntot) issue(k + CA_STAGES - 1);
    const int s = k % CA_STAGES;
    // warp 0 waits for the tile; the others block in the barrier
    const bool got = warp != 0 || tc::warp_wait(&full[s], (uint32_t)(k / CA_STAGES) & 1u, err);
    ok = __syncthreads_and(got) != 0;
    if (!ok) break;
    if (k < nt) {  // scores of K tile k
      const int t0 = k * CA_TILE;
      // partial dots of this lane's 4 dimensions, value i = 2u + j for row
      // hw + 16u and query head j
      float v[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 kv = *reinterpret_cast<const float4 *>(&ring[s][hw + NHW * u][hl * 4]);
#pragma unroll
        for (int j = 0; j < REP; ++j)
          v[2 * u + j] = qr[j][0] * kv.x + qr[j][1] * kv.y + qr[j][2] * kv.z + qr[j][3] * kv.w;
      }
      // transposed reduction over the half-warp: at each level a lane keeps
      // half of its values and adds its partner's copies of them, so lane hl
      // ends with the full dot of value hl >> 1
      float w[4], x[2];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float send = b3 ? v[e] : v[e + 4], keep = b3 ? v[e + 4] : v[e];
        w[e] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float send = b2 ? w[e] : w[e + 2], keep = b2 ? w[e + 2] : w[e];
        x[e] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      float y = (b1 ? x[1] : x[0]) + __shfl_xor_sync(0xffffffffu, b1 ? x[0] : x[1], 2);
      y += __shfl_xor_sync(0xffffffffu, y, 1);
      if ((hl & 1) == 0) {
        const int t = t0 + hw + NHW * (hl >> 2), j = (hl >> 1) & 1;
        sc[j * Tp + t] = t < T ? y * a.scale : -INFINITY;
      }
    } else {
      if (k == nt) {  // every score is in: maximum, exponentials, sum, weights
#pragma unroll
        for (int j = 0; j < REP; ++j) {
          float m = -INFINITY;
          for (int t = tid; t < T; t += NT) m = fmaxf(m, sc[j * Tp + t]);
          m = warp_max(m);
          if (lane == 0) stat[j * NW + warp] = m;
        }
        __syncthreads();
        float mx[REP];
#pragma unroll
        for (int j = 0; j < REP; ++j) {
          float m = stat[j * NW];
          for (int w = 1; w < NW; ++w) m = fmaxf(m, stat[j * NW + w]);
          mx[j] = m;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < REP; ++j) {
          float sum = 0.0f;
          for (int t = tid; t < Tp; t += NT) {
            const float p = expf(sc[j * Tp + t] - mx[j]);  // 0 past T
            sc[j * Tp + t] = p;
            sum += p;
          }
          sum = warp_sum(sum);
          if (lane == 0) stat[j * NW + warp] = sum;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < REP; ++j) {
          float sum = 0.0f;
          for (int w = 0; w < NW; ++w) sum += stat[j * NW + w];
          const float inv = 1.0f / sum;
          for (int t = tid; t < Tp; t += NT) sc[j * Tp + t] *= inv;
        }
        __syncthreads();
      }
      const int t0 = (k - nt) * CA_TILE;
#pragma unroll
      for (int u = 0; u < CA_TILE / NHW; ++u) {
        const int r = hw + NHW * u;
        const float4 vv = *reinterpret_cast<const float4 *>(&ring[s][r][hl * 4]);
#pragma unroll
        for (int j = 0; j < REP; ++j) {
          const float p = sc[j * Tp + t0 + r];  // 0 past T
          acc[j][0] = fmaf(p, vv.x, acc[j][0]);
          acc[j][1] = fmaf(p, vv.y, acc[j][1]);
          acc[j][2] = fmaf(p, vv.z, acc[j][2]);
          acc[j][3] = fmaf(p, vv.w, acc[j][3]);
        }
      }
    }
    __syncthreads();  // stage s free
  }
  if (!ok) {
    // a wait gave up: let the copies already started land before the
    // shared memory is released (each wait bounded), and write nothing
    for (int kk = k; kk < ntot && kk < k + CA_STAGES; ++kk)
      if (tid == 0) tc::mbar_drain(&full[kk % CA_STAGES], (uint32_t)(kk / CA_STAGES) & 1u);
    __syncthreads();
    return;
  }
#pragma unroll
  for (int j = 0; j < REP; ++j)
    *reinterpret_cast<float4 *>(red + (hw * REP + j) * HD + hl * 4) =
        make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
  __syncthreads();
  for (int i = tid; i < REP * HD; i += NT) {
    const int j = i / HD, d = i - j * HD;
    float sum = 0.0f;
    for (int w = 0; w < NHW; ++w) sum += red[(w * REP + j) * HD + d];
    const int64_t col = (int64_t)(g * REP + j) * HD + d;
    if (hi)
      store_split(hi + (int64_t)b * ldp + col, lo + (int64_t)b * ldp + col, sum);
    else
      out[(int64_t)b * qd + col] = sum;
  }
}

// 16-byte global -> shared copy that completes asynchronously (no register
// holds the data in flight); cp_async_wait makes the executing thread's own
// copies visible to it.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }


// Decoder self-attention for one new token per request, head dim 64, two
// query heads per KV head (attn.rs:100-183).  CTA = (request, KV head), 128
// threads, the context in passes of CH (16, 32 or 64) cache rows; the host
// picks the smallest CH that holds the step's context, so the shared memory
// a CTA holds, and with it the CTAs resident per SM, follows the context:
//   * every thread first starts asynchronous 16-byte copies of the pass's
//     K and V rows into shared memory (K rows padded to 68 floats, so a
//     thread reading a whole row meets no bank conflict);
//   * PREP: while they are in flight, warps 0-1 apply ZCRMSNorm + RoPE
//     (position pos) to the two query heads and warp 2 does the same to the
//     new key and appends k, v at row pos (push_kv saturates at cap,
//     attn.rs:53-61; the appended row is then read from shared memory).
//     Without PREP the QKV projection's epilogue has done all of that
//     already: q is read normed from qkv and row pos is in the cache;
//   * scores: thread (head tid/64, row tid%64) forms one full 64-term dot;
//   * softmax across passes with a running maximum and sum (ops.rs:5-36 up
//     to the order of the sums);
//   * P·V: thread (row group tid/16, dimensions 4·(tid%16)..+3) accumulates
//     both heads over the rows of its group; the eight groups are summed at
//     the end.
// The result goes to out [B, H*64] f32, or, when hi is set, straight to the
// bf16 hi/lo operand planes (row stride ldp) of the output projection.
template <bool PREP, int CH>
__global__ void __launch_bounds__(128, CH == 16 ? 12 : CH == 32 ? 10 : 6) self_attn_step_kernel(
    const float *__restrict__ qkv, const int32_t *__restrict__ step, const float *__restrict__ qn,
    const float *__restrict__ kn, const float *__restrict__ rc, const float *__restrict__ rs, float *kc, float *vc,
    int cap, float *out, __nv_bfloat16 *hi, __nv_bfloat16 *lo, int64_t ldp, AttnDims a) {
  constexpr int HD = 64, REP = 2, KP = HD + 4;
  static_assert(CH == 16 || CH == 32 || CH == 64, "pass size");
  __shared__ __align__(16) float ks[CH][KP];
  __shared__ __align__(16) float vs[CH][HD];
  __shared__ __align__(16) float qs[REP][HD];
  __shared__ __align__(16) float knew[HD], vnew[HD];
  __shared__ __align__(8) float2 ps[CH];  // (head 0, head 1) weights of a row
  __shared__ float wmax[4], wsum[4];
  float(*part)[REP][HD] = reinterpret_cast<float(*)[REP][HD]>(&vs[0][0]);  // after the last pass
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y, g = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = a.H * HD, kvd = a.KVH * HD, ld = qd + 2 * kvd;
  const int pos = step[b];
  const bool append = pos < cap;
  // rows copied from the cache: with PREP the new row is not there yet
  const int cached = PREP ? (append ? pos : cap) : (append ? pos + 1 : cap);
  const int total = append ? pos + 1 : cap;  // rows attended over
  const float *kcb = kc + (int64_t)b * cap * kvd + g * HD;
  const float *vcb = vc + (int64_t)b * cap * kvd + g * HD;
  const float *row = qkv + (int64_t)b * ld;
  auto fetch = [&](int c0) {
    const int c = tid & 15;
#pragma unroll
    for (int u = 0; u < CH / 8; ++u) {
      const int r = (tid >> 4) + 8 * u, t = c0 + r;
      if (t < cached) {
        cp_async16(&ks[r][4 * c], kcb + (int64_t)t * kvd + 4 * c);
        cp_async16(&vs[r][4 * c], vcb + (int64_t)t * kvd + 4 * c);
      }
    }
  };
  fetch(0);
  if constexpr (PREP) {
    const float *cr = rc + (int64_t)pos * (HD / 2), *sr = rs + (int64_t)pos * (HD / 2);
    if (warp < REP) {
      float *v = qs[warp];
      const float *src = row + (g * REP + warp) * HD;
      v[lane] = src[lane];
      v[lane + 32] = src[lane + 32];
      __syncwarp();
      norm_rope_head(v, HD, qn, cr, sr, true, lane);
    } else if (warp == REP) {
      const float *kr = row + qd + g * HD, *vr = row + qd + kvd + g * HD;
      knew[lane] = kr[lane];
      knew[lane + 32] = kr[lane + 32];
      vnew[lane] = vr[lane];
      vnew[lane + 32] = vr[lane + 32];
      __syncwarp();
      norm_rope_head(knew, HD, kn, cr, sr, true, lane);
      __syncwarp();
      if (append) {
        float *kd = kc + ((int64_t)b * cap + pos) * kvd + g * HD;
        float *vd = vc + ((int64_t)b * cap + pos) * kvd + g * HD;
        kd[lane] = knew[lane];
        kd[lane + 32] = knew[lane + 32];
        vd[lane] = vnew[lane];
        vd[lane + 32] = vnew[lane + 32];
      }
    }
  } else {
    if (tid < 2 * 16) cp_async16(&qs[tid >> 4][4 * (tid & 15)], row + (g * REP + (tid >> 4)) * HD + 4 * (tid & 15));
  }
  const int sj = tid >> 6, sr_ = tid & 63;  // scores: (head, row)
  const int rg = tid >> 4, dq = tid & 15;   // P·V: (row group, 4 dimensions)
  float m[REP], l[REP], acc[REP][4];
#pragma unroll
  for (int j = 0; j < REP; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.0f;
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  }
  for (int c0 = 0; c0 < total; c0 += CH) {
    if (c0 > 0) fetch(c0);
    cp_async_wait();
    __syncthreads();  // every thread's copies (and q, the new row) visible
    float sc = -INFINITY;
    {
      const int t = c0 + sr_;
      if (sr_ < CH && t < total) {
        const float *kp = (PREP && append && t == pos) ? knew : ks[sr_];
        const float *q = qs[sj];
        float d = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float4 k4 = *reinterpret_cast<const float4 *>(kp + 4 * c);
          const float4 q4 = *reinterpret_cast<const float4 *>(q + 4 * c);
          d = fmaf(q4.x, k4.x, d);
          d = fmaf(q4.y, k4.y, d);
          d = fmaf(q4.z, k4.z, d);
          d = fmaf(q4.w, k4.w, d);
        }
        sc = d * a.scale;
      }
    }
    const float wm = warp_max(sc);
    if (lane == 0) wmax[warp] = wm;
    __syncthreads();
    float corr[REP];
#pragma unroll
    for (int j = 0; j < REP; ++j) {
      const float mn = fmaxf(m[j], fmaxf(wmax[2 * j], wmax[2 * j + 1]));
      corr[j] = expf(m[j] - mn);  // 0 on the first pass (m = -inf)
      m[j] = mn;
    }
    const float p = sr_ < CH && c0 + sr_ < total ? expf(sc - (sj ? m[1] : m[0])) : 0.0f;
    if (sr_ < CH) reinterpret_cast<float *>(&ps[sr_])[sj] = p;
    const float wsm = warp_sum(p);
    if (lane == 0) wsum[warp] = wsm;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < REP; ++j) {
      l[j] = l[j] * corr[j] + (wsum[2 * j] + wsum[2 * j + 1]);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] *= corr[j];
    }
#pragma unroll
    for (int u = 0; u < CH / 8; ++u) {
      const int r = rg + 8 * u, t = c0 + r;
      if (t >= total) break;
      const float4 v4 = (PREP && append && t == pos) ? *reinterpret_cast<const float4 *>(&vnew[4 * dq])
                                                     : *reinterpret_cast<const float4 *>(&vs[r][4 * dq]);
      const float2 pj = ps[r];
      acc[0][0] = fmaf(pj.x, v4.x, acc[0][0]);
      acc[0][1] = fmaf(pj.x, v4.y, acc[0][1]);
      acc[0][2] = fmaf(pj.x, v4.z, acc[0][2]);
      acc[0][3] = fmaf(pj.x, v4.w, acc[0][3]);
      acc[1][0] = fmaf(pj.y, v4.x, acc[1][0]);
      acc[1][1] = fmaf(pj.y, v4.y, acc[1][1]);
      acc[1][2] = fmaf(pj.y, v4.z, acc[1][2]);
      acc[1][3] = fmaf(pj.y, v4.w, acc[1][3]);
    }
    __syncthreads();  // shared tiles free for the next pass
  }
  // the two row groups of a warp, then the four warps
#pragma unroll
  for (int j = 0; j < REP; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] += __shfl_xor_sync(0xffffffffu, acc[j][e], 16);
  if (lane < 16)
#pragma unroll
    for (int j = 0; j < REP; ++j)
      *reinterpret_cast<float4 *>(&part[warp][j][4 * dq]) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
  __syncthreads();
  {
    const int j = tid >> 6, d = tid & 63;
    const float o = (part[0][j][d] + part[1][j][d] + part[2][j][d] + part[3][j][d]) * (1.0f / (j ? l[1] : l[0]));
    const int64_t col = (int64_t)(g * REP + j) * HD + d;
    if (hi)
      store_split(hi + (int64_t)b * ldp + col, lo + (int64_t)b * ldp + col, o);
    else
      out[(int64_t)b * qd + col] = o;
  }
}

// Generic cross-attention for head dims other than 64 (small test models).
__global__ void cross_attn_generic_kernel(const float *__restrict__ q, const float *__restrict__ qn,
                                          const float *__restrict__ kplane, const float *__restrict__ vplane,
                                          const int64_t *__restrict__ seq_off, float *out, AttnDims a) {
  extern __shared__ __align__(16) float sm[];
  const int b = blockIdx.x, HD = a.HD;
  const int64_t off = seq_off[b];
  const int T = (int)(seq_off[b + 1] - off);
  const int kvd = a.KVH * HD, qd = a.H * HD, rep = a.H / a.KVH;
  float *qs = sm;         // [H*HD]
  float *sc = sm + qd;    // [H][T]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int h = warp; h < a.H; h += blockDim.x / 32) {
    float v[128];
    for (int i = lane; i < HD / 2; i += 32) {
      v[i] = q[(int64_t)b * qd + h * HD + i];
      v[i + HD / 2] = q[(int64_t)b * qd + h * HD + i + HD / 2];
    }
    norm_rope_head(v, HD, qn, nullptr, nullptr, false, lane);
    for (int i = lane; i < HD / 2; i += 32) {
      qs[h * HD + i] = v[i];
      qs[h * HD + i + HD / 2] = v[i + HD / 2];
    }
  }
  __syncthreads();
  const float scale = a.scale;
  for (int h = warp; h < a.H; h += blockDim.x / 32) {
    int g = h / rep;
    float *s = sc + h * T;
    float mx = -INFINITY;
    for (int t = lane; t < T; t += 32) {
      const float *k = kplane + (off + t) * kvd + g * HD;
      float acc = 0.0f;
      for (int d = 0; d < HD; ++d) acc = fmaf(qs[h * HD + d], k[d], acc);
      s[t] = acc * scale;
      mx = fmaxf(mx, s[t]);
    }
    mx = warp_max(mx);
    float sum = 0.0f;
    for (int t = lane; t < T; t += 32) {
      float p = expf(s[t] - mx);
      s[t] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    __syncwarp();
    float inv = 1.0f / sum;
    for (int d = lane; d < HD; d += 32) {
      float acc = 0.0f;
      for (int t = 0; t < T; ++t) acc = fmaf(s[t] * inv, vplane[(off + t) * kvd + g * HD + d], acc);
      out[(int64_t)b * qd + h * HD + d] = acc;
    }
  }
}

}  // namespace

cudaError_t init_attention_kernels() {
  cudaError_t e = cudaSuccess;
  auto set = [&](const void *f) {
    cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    if (r != cudaSuccess) e = r;
  };
  set((const void *)encoder_attn_kernel);
  set((const void *)dec_self_attn_kernel);
  set((const void *)cross_attn_kernel);
  set((const void *)cross_attn_generic_kernel);
  return e;
}

cudaError_t rms_norm_rows(const float *x, int64_t ldx, float *out, int64_t ldo, const float *scale, int rows,
                          int d, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (d == 512 && ((ldx | ldo) & 3)) return cudaErrorInvalidValue;
  int64_t threads = (int64_t)rows * 32;
  return launch(rms_norm_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, x, ldx, out, ldo, scale,
                rows, d);
}

cudaError_t head_norm_rows(float *x, int rows, int64_t ld, int heads, int HD, const float *scale, cudaStream_t st) {
  if (rows <= 0 || heads <= 0) return cudaSuccess;
  if (HD > 128 || (HD & 1)) return cudaErrorInvalidValue;
  int64_t threads = (int64_t)rows * heads * 32;
  head_norm_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(x, rows, ld, heads, HD, scale);
  return cudaGetLastError();
}

cudaError_t rms_norm_planes(const float *x, int64_t ldx, void *hi, void *lo, int64_t ldp, float *out, int64_t ldo,
                            const float *scale, int rows, int d, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (d != 512 || (ldx & 3) || (ldp & 3) || (out && (ldo & 3))) return cudaErrorInvalidValue;
  int64_t threads = (int64_t)rows * 32;
  return launch(rms_norm_planes_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, x, ldx,
                (__nv_bfloat16 *)hi, (__nv_bfloat16 *)lo, ldp, out, ldo, scale, rows);
}

cudaError_t embed_rows(const uint32_t *ids, const float *emb, float *x, int rows, int d, float es,
                       cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  int64_t threads = (int64_t)rows * 32;
  embed_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(ids, emb, x, rows, d, es);
  return cudaGetLastError();
}

cudaError_t qk_norm_rope_rows(float *qkv, int rows, const int32_t *pos, const float *q_norm, const float *k_norm,
                              const float *rope_cos, const float *rope_sin, AttnDims a, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (a.HD > 128 || (a.HD & 1)) return cudaErrorInvalidValue;
  int64_t threads = (int64_t)rows * (a.H + a.KVH) * 32;
  qk_norm_rope_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(qkv, rows, pos, q_norm, k_norm, rope_cos,
                                                                           rope_sin, a);
  return cudaGetLastError();
}

cudaError_t encoder_attention(const float *qkv, const int64_t *seq_off, int n_req, int max_len, float *out,
                              AttnDims a, cudaStream_t st) {
  if (n_req <= 0 || max_len <= 0) return cudaSuccess;
  if (a.HD > 64 || (a.HD & 3)) return cudaErrorInvalidValue;
  size_t sm = (size_t)4 * 64 * EP * sizeof(float);
  dim3 grid((max_len + EQ - 1) / EQ, a.H, n_req);
  encoder_attn_kernel<<<grid, 256, sm, st>>>(qkv, seq_off, out, a);
  return cudaGetLastError();
}

cudaError_t decoder_self_attention(const float *qkv, const int32_t *step, const float *q_norm,
                                   const float *k_norm, const float *rope_cos, const float *rope_sin, float *kc,
                                   float *vc, int cap, int B, float *out, AttnDims a, cudaStream_t st, void *hi_,
                                   void *lo_, int64_t ldp, bool prepared, int max_rows) {
  __nv_bfloat16 *hi = static_cast<__nv_bfloat16 *>(hi_), *lo = static_cast<__nv_bfloat16 *>(lo_);
  if (B <= 0) return cudaSuccess;
  if (a.HD > 128 || (a.HD & 1) || cap <= 0) return cudaErrorInvalidValue;
  if (a.HD == 64 && a.H == 2 * a.KVH) {
    const dim3 grid(a.KVH, B);
    const int rows = max_rows > 0 && max_rows < cap ? max_rows : cap;
    auto k = prepared ? (rows <= 16   ? self_attn_step_kernel<false, 16>
                         : rows <= 32 ? self_attn_step_kernel<false, 32>
                                      : self_attn_step_kernel<false, 64>)
                      : self_attn_step_kernel<true, 64>;
    return launch(k, grid, dim3(128), 0, st, qkv, step, q_norm, k_norm, rope_cos, rope_sin, kc, vc, cap, out, hi, lo,
                  ldp, a);
  }
  if (hi || prepared) return cudaErrorInvalidValue;
  size_t sm = ((size_t)a.H * a.HD + (size_t)a.H * cap) * sizeof(float);
  if (sm > kMaxDynSmem) return cudaErrorInvalidValue;
  dec_self_attn_kernel<<<B, 256, sm, st>>>(qkv, step, q_norm, k_norm, rope_cos, rope_sin, kc, vc, cap, out, a);
  return cudaGetLastError();
}

cudaError_t decoder_cross_attention(const float *q, const float *q_norm, const float *kplane,
                                    const float *vplane, const int64_t *seq_off, int B, float *out, AttnDims a,
                                    cudaStream_t st, int max_len, void *hi_, void *lo_, int64_t ldp, int *err,
                                    const void *kv_map, int64_t k_row0, int64_t v_row0, int64_t head_rows) {
  __nv_bfloat16 *hi = static_cast<__nv_bfloat16 *>(hi_), *lo = static_cast<__nv_bfloat16 *>(lo_);
  if (B <= 0) return cudaSuccess;
  int rep = a.H / a.KVH;
  if (a.HD == 64 && rep == 2) {
    if (!err || !kv_map || head_rows <= 0 || v_row0 + a.KVH * head_rows > INT32_MAX) return cudaErrorInvalidValue;
    const size_t sm = cross_attn_smem(max_len);
    if (sm > kMaxDynSmem) return cudaErrorInvalidValue;
    return launch(cross_attn_kernel, dim3(a.KVH, B), dim3(256), sm, st, *static_cast<const CUtensorMap *>(kv_map), q,
                  q_norm, k_row0, v_row0, head_rows, seq_off, out, hi, lo, ldp, a, max_len, err);
  }
  if (hi) return cudaErrorInvalidValue;
  if (a.HD > 128 || (a.HD & 1)) return cudaErrorInvalidValue;
  size_t sm = ((size_t)a.H * a.HD + (size_t)a.H * max_len) * sizeof(float);
  if (sm > kMaxDynSmem) return cudaErrorInvalidValue;
  cross_attn_generic_kernel<<<B, 256, sm, st>>>(q, q_norm, kplane, vplane, seq_off, out, a);
  return cudaGetLastError();
}

}  // namespace ndl
