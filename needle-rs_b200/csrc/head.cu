// head.cu — fused output head: logits + constrained-decoding mask + argmax.
//
// Reference: NeedleModel::lm_head (crates/needle-core/src/model.rs:89-149), the
// engine's additive mask and argmax (crates/needle-infer/src/engine.rs:294-304)
// and ConstrainedDecoder::logit_mask (constrained.rs:369-387: 0.0 allowed,
// -1e9 blocked).  The mask arrives as a vocabulary bitmap (bit v of word v/64
// set = allowed).  Logits are reduced to one packed (total-order key, index)
// u64 per request with atomicMax, which returns the last index among equal
// maxima exactly like Iterator::max_by(total_cmp).  Logits only reach HBM
// when the caller asks for them (parity checks).
#include "common.cuh"
#include "kernels.h"

namespace ndl {
namespace {

__device__ __forceinline__ float masked(float logit, const uint64_t *mrow, int v) {
  // The engine always adds the mask vector (all 0.0 when unconstrained), so
  // even an unmasked logit goes through `+ 0.0f` (turning -0.0 into +0.0).
  float add = 0.0f;
  if (mrow) add = ((mrow[v >> 6] >> (v & 63)) & 1ull) ? 0.0f : kMaskBlocked;
  return logit + add;
}

// Small batch: one warp per vocabulary row, h rows in shared memory.
constexpr int HB_MAX = 8, H_ROWS_PER_WARP = 4;

struct HeadIO {
  const uint64_t *mask;  // [B][max_new][W] or NULL
  int W;                 // mask words per (request, step)
  float *logits;         // [B][max_new][V] or NULL
  int max_new;
  const int32_t *pos;    // current step of each request
  __device__ __forceinline__ const uint64_t *mrow(int b) const {
    return mask ? mask + ((int64_t)b * max_new + pos[b]) * W : nullptr;
  }
  __device__ __forceinline__ float *lrow(int b, int V) const {
    return logits ? logits + ((int64_t)b * max_new + pos[b]) * V : nullptr;
  }
};

__global__ void __launch_bounds__(256) head_gemv_kernel(const float *__restrict__ h, int B,
                                                        const float *__restrict__ emb, int V, int d, HeadIO io,
                                                        unsigned long long *keys) {
  extern __shared__ __align__(16) float hs[];  // [B][d]
  __shared__ unsigned long long best_s[8][HB_MAX];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < B * d; i += 256) hs[i] = h[i];
  __syncthreads();
  unsigned long long best[HB_MAX];
#pragma unroll
  for (int b = 0; b < HB_MAX; ++b) best[b] = 0ull;
  const int d4 = d >> 2;
  const int v0 = (blockIdx.x * 8 + warp) * H_ROWS_PER_WARP;
#pragma unroll
  for (int r = 0; r < H_ROWS_PER_WARP; ++r) {
    int v = v0 + r;
    if (v >= V) break;
    const float4 *e = reinterpret_cast<const float4 *>(emb + (int64_t)v * d);
    float part[HB_MAX];
#pragma unroll
    for (int b = 0; b < HB_MAX; ++b) part[b] = 0.0f;
    for (int i = lane; i < d4; i += 32) {
      float4 ev = __ldg(e + i);
#pragma unroll
      for (int b = 0; b < HB_MAX; ++b) {
        if (b < B) {
          float4 hv = reinterpret_cast<const float4 *>(hs + b * d)[i];
          part[b] = fmaf(hv.x, ev.x, part[b]);
          part[b] = fmaf(hv.y, ev.y, part[b]);
          part[b] = fmaf(hv.z, ev.z, part[b]);
          part[b] = fmaf(hv.w, ev.w, part[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < HB_MAX; ++b) {
      if (b < B) {
        float lg = warp_sum(part[b]);
        float mv = masked(lg, io.mrow(b), v);
        float *lr = io.lrow(b, V);
        if (lr && lane == 0) lr[v] = mv;
        unsigned long long k = argmax_key(mv, (uint32_t)v);
        best[b] = k > best[b] ? k : best[b];
      }
    }
  }
  if (lane == 0)
#pragma unroll
    for (int b = 0; b < HB_MAX; ++b) best_s[warp][b] = best[b];
  __syncthreads();
  if (tid < B) {
    unsigned long long k = 0ull;
    for (int w = 0; w < 8; ++w) k = best_s[w][tid] > k ? best_s[w][tid] : k;
    atomicMax(keys + tid, k);
  }
}

// Small batch over the bf16 copy of the embedding, used when every value of
// the embedding is exactly a bf16 (as the shipped checkpoints store it):
// the same products as over the f32 copy, from half the bytes.  One warp
// per 4 vocabulary rows; each lane loads CPL 16-byte chunks (8 values) of
// every row, all of the warp's loads issued before the first is used.  Under
// programmatic dependent launch the embedding loads (weights, written by no
// kernel of the step) go out before the wait for the previous kernel; h,
// the masks and the positions are read after it.
template <int CPL>
__global__ void __launch_bounds__(256) head_gemv_bf16_kernel(const float *__restrict__ h, int B,
                                                             const uint16_t *__restrict__ emb, int64_t ld, int V,
                                                             int d, HeadIO io, unsigned long long *keys) {
  extern __shared__ __align__(16) float hs[];  // [B][d]
  __shared__ unsigned long long best_s[8][HB_MAX];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int v0 = (blockIdx.x * 8 + warp) * H_ROWS_PER_WARP;
  pdl_trigger();
  uint4 ev[H_ROWS_PER_WARP][CPL];
#pragma unroll
  for (int r = 0; r < H_ROWS_PER_WARP; ++r)
#pragma unroll
    for (int j = 0; j < CPL; ++j)
      ev[r][j] = v0 + r < V ? __ldg(reinterpret_cast<const uint4 *>(emb + (int64_t)(v0 + r) * ld) + lane + 32 * j)
                            : make_uint4(0u, 0u, 0u, 0u);
  pdl_wait();
  for (int i = tid; i < B * d; i += 256) hs[i] = h[i];
  __syncthreads();
  unsigned long long best[HB_MAX];
#pragma unroll
  for (int b = 0; b < HB_MAX; ++b) best[b] = 0ull;
#pragma unroll
  for (int r = 0; r < H_ROWS_PER_WARP; ++r) {
    const int v = v0 + r;
    if (v >= V) break;
    float part[HB_MAX];
#pragma unroll
    for (int b = 0; b < HB_MAX; ++b) part[b] = 0.0f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const uint32_t w[4] = {ev[r][j].x, ev[r][j].y, ev[r][j].z, ev[r][j].w};
      float e[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // bf16 -> f32 is exact: the bits move up
        e[2 * q] = __uint_as_float(w[q] << 16);
        e[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
      }
      const int c = 8 * (lane + 32 * j);
#pragma unroll
      for (int b = 0; b < HB_MAX; ++b) {
        if (b < B) {
          const float4 h0 = *reinterpret_cast<const float4 *>(hs + b * d + c);
          const float4 h1 = *reinterpret_cast<const float4 *>(hs + b * d + c + 4);
          part[b] = fmaf(h0.x, e[0], part[b]);
          part[b] = fmaf(h0.y, e[1], part[b]);
          part[b] = fmaf(h0.z, e[2], part[b]);
          part[b] = fmaf(h0.w, e[3], part[b]);
          part[b] = fmaf(h1.x, e[4], part[b]);
          part[b] = fmaf(h1.y, e[5], part[b]);
          part[b] = fmaf(h1.z, e[6], part[b]);
          part[b] = fmaf(h1.w, e[7], part[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < HB_MAX; ++b) {
      if (b < B) {
        const float lg = warp_sum(part[b]);
        const float mv = masked(lg, io.mrow(b), v);
        float *lr = io.lrow(b, V);
        if (lr && lane == 0) lr[v] = mv;
        const unsigned long long k = argmax_key(mv, (uint32_t)v);
        best[b] = k > best[b] ? k : best[b];
      }
    }
  }
  if (lane == 0)
#pragma unroll
    for (int b = 0; b < HB_MAX; ++b) best_s[warp][b] = best[b];
  __syncthreads();
  if (tid < B) {
    unsigned long long k = 0ull;
    for (int w = 0; w < 8; ++w) k = best_s[w][tid] > k ? best_s[w][tid] : k;
    atomicMax(keys + tid, k);
  }
}

// Large batch: 128 (requests) x 128 (vocab) tile, BK = 32, 8x8 per thread.
constexpr int HBM_ = 128, HBN = 128, HBK = 32, HXS = 132;

__global__ void __launch_bounds__(256) head_tile_kernel(const float *__restrict__ h, int B,
                                                        const float *__restrict__ emb, int V, int d, HeadIO io,
                                                        unsigned long long *keys) {
  extern __shared__ __align__(16) float smem[];
  float *Hs = smem;                    // [2][HBK][HXS]  Hs[k][m]
  float *Es = smem + 2 * HBK * HXS;    // [2][HBK][HXS]  Es[k][n]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tx = lane & 15, ty = warp * 2 + (lane >> 4);
  const int m0 = blockIdx.y * HBM_, n0 = blockIdx.x * HBN;
  const int nk = (d + HBK - 1) / HBK;
  float4 hr[4], er[4];

  auto gload = [&](int kt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = i * 256 + tid, r = idx >> 3, c4 = idx & 7, k = kt * HBK + c4 * 4;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (k < d) {  // d % 4 == 0
        if (m0 + r < B) a = __ldg(reinterpret_cast<const float4 *>(h + (int64_t)(m0 + r) * d + k));
        if (n0 + r < V) b = __ldg(reinterpret_cast<const float4 *>(emb + (int64_t)(n0 + r) * d + k));
      }
      hr[i] = a;
      er[i] = b;
    }
  };
  auto sstore = [&](int buf) {
    float *hs = Hs + buf * HBK * HXS, *es = Es + buf * HBK * HXS;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = i * 256 + tid, r = idx >> 3, c4 = idx & 7;
      hs[(c4 * 4 + 0) * HXS + r] = hr[i].x;
      hs[(c4 * 4 + 1) * HXS + r] = hr[i].y;
      hs[(c4 * 4 + 2) * HXS + r] = hr[i].z;
      hs[(c4 * 4 + 3) * HXS + r] = hr[i].w;
      es[(c4 * 4 + 0) * HXS + r] = er[i].x;
      es[(c4 * 4 + 1) * HXS + r] = er[i].y;
      es[(c4 * 4 + 2) * HXS + r] = er[i].z;
      es[(c4 * 4 + 3) * HXS + r] = er[i].w;
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  gload(0);
  sstore(0);
  __syncthreads();
  for (int kt = 0; kt < nk; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nk) gload(kt + 1);
    const float *hs = Hs + buf * HBK * HXS, *es = Es + buf * HBK * HXS;
#pragma unroll 8
    for (int k = 0; k < HBK; ++k) {
      float4 a0 = *reinterpret_cast<const float4 *>(hs + k * HXS + ty * 4);
      float4 a1 = *reinterpret_cast<const float4 *>(hs + k * HXS + 64 + ty * 4);
      float4 b0 = *reinterpret_cast<const float4 *>(es + k * HXS + tx * 4);
      float4 b1 = *reinterpret_cast<const float4 *>(es + k * HXS + 64 + tx * 4);
      float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) sstore(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    const uint64_t *mrow = m < B ? io.mrow(m) : nullptr;
    float *lrow = m < B ? io.lrow(m, V) : nullptr;
    unsigned long long best = 0ull;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int v = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (m < B && v < V) {
        float mv = masked(acc[i][j], mrow, v);
        if (lrow) lrow[v] = mv;
        unsigned long long k = argmax_key(mv, (uint32_t)v);
        best = k > best ? k : best;
      }
    }
    // reduce over the 16 lanes (tx) that share this row
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (tx == 0 && m < B) atomicMax(keys + m, best);
  }
}

__global__ void finish_step_kernel(unsigned long long *keys, int B, int max_new, int stop_on_eos,
                                   uint32_t *out_ids, uint32_t *lens, uint8_t *done, int32_t *pos,
                                   unsigned int *n_done, const uint32_t *__restrict__ teacher,
                                   const float *__restrict__ emb, float *x, int d, float es) {
  pdl_trigger();
  pdl_wait();
  int b = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (b >= B) return;
  unsigned long long k = keys[b];
  uint32_t next = (uint32_t)(k & 0xffffffffull);
  const int step = pos[b];
  __syncwarp();
  if (lane == 0) {
    keys[b] = 0ull;
    if (!done[b]) {
      // engine.rs:306-308: EOS ends the request and is not emitted.
      if (stop_on_eos && next == kEosId) {
        done[b] = 1;
        atomicAdd(n_done, 1u);
      } else {
        uint32_t n = lens[b];
        if ((int)n < max_new) out_ids[(int64_t)b * max_new + n] = next;
        lens[b] = n + 1;
      }
    }
    pos[b] = step + 1;
  }
  uint32_t in_tok = next;
  if (teacher) in_tok = step + 1 < max_new ? teacher[(int64_t)b * max_new + step + 1] : next;
  const float *e = emb + (int64_t)in_tok * d;
  float *xr = x + (int64_t)b * d;
  for (int i = lane; i < d; i += 32) xr[i] = e[i] * es;
}

}  // namespace

cudaError_t init_head_kernels() {
  cudaError_t e = cudaSuccess;
  for (const void *f : {(const void *)head_gemv_kernel, (const void *)head_tile_kernel}) {
    cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    if (r != cudaSuccess) e = r;
  }
  return e;
}

cudaError_t init_kernels() {
  cudaError_t e = init_matmul_kernels();
  if (e == cudaSuccess) e = init_attention_kernels();
  if (e == cudaSuccess) e = init_head_kernels();
  if (e == cudaSuccess) e = init_tc_kernels();
  if (e == cudaSuccess) e = init_tc_attn_kernels();
  return e;
}

cudaError_t head_argmax(const float *h, int B, const float *emb, int V, int d, const uint64_t *mask, int mask_words,
                        float *logits, int max_new, const int32_t *pos, unsigned long long *keys, cudaStream_t st,
                        const void *emb_bf16, int64_t ld_bf16) {
  HeadIO io{mask, mask_words, logits, max_new, pos};
  if (B <= 0) return cudaSuccess;
  if (d & 3) return cudaErrorInvalidValue;
  if (B <= HB_MAX) {
    size_t sm = (size_t)B * d * sizeof(float);
    if (sm > (size_t)kMaxDynSmem) return cudaErrorInvalidValue;
    int rows_per_cta = 8 * H_ROWS_PER_WARP;
    const int cpl = d / 256;
    if (emb_bf16 && d % 256 == 0 && cpl >= 1 && cpl <= 4 && ld_bf16 % 8 == 0 && ((uintptr_t)emb_bf16 % 16) == 0) {
      const uint16_t *e = (const uint16_t *)emb_bf16;
      const dim3 grid((V + rows_per_cta - 1) / rows_per_cta);
      auto k = cpl == 1   ? head_gemv_bf16_kernel<1>
               : cpl == 2 ? head_gemv_bf16_kernel<2>
               : cpl == 3 ? head_gemv_bf16_kernel<3>
                          : head_gemv_bf16_kernel<4>;
      return launch(k, grid, dim3(256), sm, st, h, B, e, ld_bf16, V, d, io, keys);
    }
    head_gemv_kernel<<<(V + rows_per_cta - 1) / rows_per_cta, 256, sm, st>>>(h, B, emb, V, d, io, keys);
    return cudaGetLastError();
  }
  size_t sm = (size_t)2 * 2 * HBK * HXS * sizeof(float);
  dim3 grid((V + HBN - 1) / HBN, (B + HBM_ - 1) / HBM_);
  head_tile_kernel<<<grid, 256, sm, st>>>(h, B, emb, V, d, io, keys);
  return cudaGetLastError();
}

cudaError_t finish_step(unsigned long long *keys, int B, int max_new, int stop_on_eos, uint32_t *out_ids,
                        uint32_t *lens, uint8_t *done, int32_t *pos, unsigned int *n_done, const uint32_t *teacher,
                        const float *emb, float *x, int d, float embed_scale, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  int64_t threads = (int64_t)B * 32;
  return launch(finish_step_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, keys, B, max_new,
                stop_on_eos, out_ids, lens, done, pos, n_done, teacher, emb, x, d, embed_scale);
}


namespace {
// Sequential f32 sums with separate multiply and add roundings, as the
// reference computes them.
__global__ void contrastive_kernel(const float *__restrict__ enc, const int64_t *__restrict__ off, int d,
                                   const float *__restrict__ hk, const float *__restrict__ hb, int h,
                                   const float *__restrict__ pk, int c, float *out) {
  extern __shared__ float cs[];
  float *pooled = cs, *hidden = cs + d, *proj = hidden + h;
  const int r = blockIdx.x;
  const int64_t o = off[r];
  const int T = (int)(off[r + 1] - o);
  const float inv_n = __fdiv_rn(1.0f, (float)T);
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float acc = 0.0f;
    for (int t = 0; t < T; ++t) acc = __fadd_rn(acc, enc[(o + t) * d + j]);
    pooled[j] = __fmul_rn(acc, inv_n);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < h; j += blockDim.x) {
    float acc = hb[j];
    for (int i = 0; i < d; ++i) acc = __fadd_rn(acc, __fmul_rn(pooled[i], hk[(int64_t)i * h + j]));
    hidden[j] = fmaxf(acc, 0.0f);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < c; j += blockDim.x) {
    float acc = 0.0f;
    for (int i = 0; i < h; ++i) acc = __fadd_rn(acc, __fmul_rn(hidden[i], pk[(int64_t)i * c + j]));
    proj[j] = acc;
  }
  __syncthreads();
  __shared__ float norm;
  if (threadIdx.x == 0) {
    float sq = 0.0f;
    for (int j = 0; j < c; ++j) sq = __fadd_rn(sq, __fmul_rn(proj[j], proj[j]));
    norm = __fsqrt_rn(__fadd_rn(sq, 1e-12f));
  }
  __syncthreads();
  for (int j = threadIdx.x; j < c; j += blockDim.x) out[(int64_t)r * c + j] = __fdiv_rn(proj[j], norm);
}
}  // namespace

cudaError_t contrastive_embed(const float *enc, const int64_t *off, int n_req, int d, const float *hk,
                              const float *hb, int h, const float *pk, int c, float *out, cudaStream_t st) {
  if (n_req <= 0) return cudaSuccess;
  const size_t sm = ((size_t)d + h + c) * sizeof(float);
  if (sm > (size_t)kMaxDynSmem) return cudaErrorInvalidValue;
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(contrastive_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
  }
  contrastive_kernel<<<n_req, 256, sm, st>>>(enc, off, d, hk, hb, h, pk, c, out);
  return cudaGetLastError();
}

}  // namespace ndl
