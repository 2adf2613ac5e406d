// int4_matmul.cu — INT4 group-quantized matmul on CUDA cores (f32 FMA).
//
// Reference: QuantizedWeight::matvec / matmul (crates/needle-core/src/quant.rs
// :160-297, :400-410).  The weight stays in the reference's packed layout in
// HBM (w[pair*N + n], two rows per byte; f32 scale per (group, n)) and is
// dequantized in registers on its way into shared memory; nothing is ever
// materialised as a full f32 matrix.
//
// Two kernels:
//   gemv_kernel  M <= 8 rows (batch-1 decode): each CTA owns 32 or 64 output
//                columns and all of K, split over 8 or 16 K-slices whose
//                partials are reduced in shared memory.
//   tile_kernel  M > 8: 128x128 output tile, BK = 32 (one scale group),
//                256 threads each holding an 8x8 accumulator, double-buffered
//                shared memory.
// Both accumulate in f32 like the reference; only the summation order
// differs (a few ulp, far inside the 1e-3 rel / 1e-4 abs logit tolerance).
#include "common.cuh"
#include "kernels.h"

namespace ndl {
namespace {

struct EpiCtx {
  MatmulOut o;
  int N;
};

__device__ __forceinline__ float act_apply(int act, float g, float u) {
  if (act == ACT_SWIGLU) {  // ffn.rs:22-27: g * sigmoid(g) * u
    float sg = g * (1.0f / (1.0f + expf(-g)));
    return sg * u;
  }
  if (act == ACT_GELU) {  // ops.rs:47-52
    const float C = 0.79788456f, A = 0.044715f;
    float ax = A * g;
    float axx = ax * g;
    float axxx = axx * g;
    float inner = C * (g + axxx);
    float t = 1.0f + tanhf(inner);
    return (0.5f * g) * t * u;
  }
  float rg = g > 0.0f ? g : 0.0f, ru = u > 0.0f ? u : 0.0f;  // drelu
  return rg * ru;
}

// Address of output element (m, n) honouring the column-block remap.
__device__ __forceinline__ float *out_ptr(const MatmulOut &o, int m, int n) {
  if (o.col_block) {
    int b = n / o.col_block, nn = n - b * o.col_block;
    return o.y + (int64_t)b * o.block_stride + (int64_t)m * o.ldy + nn;
  }
  return o.y + (int64_t)m * o.ldy + n;
}

// Store 4 consecutive outputs (n .. n+3) of row m.  n % 4 == 0.
__device__ __forceinline__ void store4(const EpiCtx &e, int m, int n, float v0, float v1, float v2, float v3,
                                       bool vec_ok) {
  const MatmulOut &o = e.o;
  float v[4] = {v0, v1, v2, v3};
  if (o.epi == EPI_ACT) {
    // (gate, up) interleaved: columns (n, n+1) -> out n/2, (n+2, n+3) -> n/2+1
    float *p = o.y + (int64_t)m * o.ldy + (n >> 1);
    if (n + 1 < e.N) p[0] = act_apply(o.act, v[0], v[1]);
    if (n + 3 < e.N) p[1] = act_apply(o.act, v[2], v[3]);
    return;
  }
  float *p = out_ptr(o, m, n);
  if (vec_ok && n + 3 < e.N) {
    float4 *p4 = reinterpret_cast<float4 *>(p);
    if (o.epi == EPI_RESID) {
      float4 r = *p4;
      r.x += o.gate * v[0];
      r.y += o.gate * v[1];
      r.z += o.gate * v[2];
      r.w += o.gate * v[3];
      *p4 = r;
    } else {
      *p4 = make_float4(v[0], v[1], v[2], v[3]);
    }
    return;
  }
  for (int j = 0; j < 4 && n + j < e.N; ++j) {
    float *q = out_ptr(o, m, n + j);
    if (o.epi == EPI_RESID)
      *q = *q + o.gate * v[j];
    else
      *q = v[j];
  }
}

// ZCRMSNorm over 64 values spread as 4 per lane across 16 lanes (norm.rs:23-30).
__device__ __forceinline__ void knorm16(float *v, const float *scale64, int sub) {
  float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = ((1.0f + __ldg(scale64 + sub * 4 + j)) * v[j]) * inv;
}

constexpr int TBM = 128, TBN = 128, TBK = 32, XS = TBM + 4;

__global__ void __launch_bounds__(256) tile_kernel(const float *__restrict__ x, int64_t ldx, int M, int K,
                                                   Int4Weight W, EpiCtx e, bool xvec, bool yvec) {
  extern __shared__ __align__(16) float smem[];
  float *Xs = smem;                   // [2][TBK][XS]   Xs[k][m]
  float *Ws = smem + 2 * TBK * XS;    // [2][TBK][TBN]  Ws[k][n]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tx = lane & 15, ty = warp * 2 + (lane >> 4);
  const int m0 = blockIdx.y * TBM, n0 = blockIdx.x * TBN;
  const int N = W.N, Kp = W.G * W.gs, npairs = Kp >> 1;
  const int nk = (Kp + TBK - 1) / TBK;

  float4 xr[4];
  uint8_t wb[8];
  float sc[8];
  const int wpr = tid >> 4, wc8 = tid & 15;

  auto gload = [&](int kt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = i * 256 + tid, r = idx >> 3, c4 = idx & 7;
      int m = m0 + r, k = kt * TBK + c4 * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < M) {
        const float *p = x + (int64_t)m * ldx + k;
        if (xvec && k + 3 < K) {
          v = __ldg(reinterpret_cast<const float4 *>(p));
        } else {
          if (k < K) v.x = __ldg(p);
          if (k + 1 < K) v.y = __ldg(p + 1);
          if (k + 2 < K) v.z = __ldg(p + 2);
          if (k + 3 < K) v.w = __ldg(p + 3);
        }
      }
      xr[i] = v;
    }
    int p = kt * (TBK / 2) + wpr;
    int n = n0 + wc8 * 8;
    if (p < npairs) {
      int g = (2 * p) / W.gs;
      if (W.w2) {
        const int Nh = N >> 1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int col = n + j;
          bool ok = col < N;
          const uint8_t *wsrc = (col & 1) ? W.w2 : W.w;
          const float *ssrc = (col & 1) ? W.s2 : W.s;
          wb[j] = ok ? __ldg(wsrc + (int64_t)p * Nh + (col >> 1)) : 0;
          sc[j] = ok ? __ldg(ssrc + (int64_t)g * Nh + (col >> 1)) : 0.0f;
        }
      } else {
        const uint8_t *wp = W.w + (int64_t)p * N + n;
        const float *sp = W.s + (int64_t)g * N + n;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          bool ok = n + j < N;
          wb[j] = ok ? __ldg(wp + j) : 0;
          sc[j] = ok ? __ldg(sp + j) : 0.0f;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        wb[j] = 0;
        sc[j] = 0.0f;
      }
    }
  };
  auto sstore = [&](int buf) {
    float *xs = Xs + buf * TBK * XS;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = i * 256 + tid, r = idx >> 3, c4 = idx & 7;
      xs[(c4 * 4 + 0) * XS + r] = xr[i].x;
      xs[(c4 * 4 + 1) * XS + r] = xr[i].y;
      xs[(c4 * 4 + 2) * XS + r] = xr[i].z;
      xs[(c4 * 4 + 3) * XS + r] = xr[i].w;
    }
    float *ws = Ws + buf * TBK * TBN;
    float lo[8], hi[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      lo[j] = (float)sign_extend4(wb[j] & 0xF) * sc[j];
      hi[j] = (float)sign_extend4(wb[j] >> 4) * sc[j];
    }
    float4 *r0 = reinterpret_cast<float4 *>(ws + (2 * wpr) * TBN + wc8 * 8);
    float4 *r1 = reinterpret_cast<float4 *>(ws + (2 * wpr + 1) * TBN + wc8 * 8);
    r0[0] = make_float4(lo[0], lo[1], lo[2], lo[3]);
    r0[1] = make_float4(lo[4], lo[5], lo[6], lo[7]);
    r1[0] = make_float4(hi[0], hi[1], hi[2], hi[3]);
    r1[1] = make_float4(hi[4], hi[5], hi[6], hi[7]);
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
    const float *xs = Xs + buf * TBK * XS;
    const float *ws = Ws + buf * TBK * TBN;
#pragma unroll 8
    for (int k = 0; k < TBK; ++k) {
      float4 a0 = *reinterpret_cast<const float4 *>(xs + k * XS + ty * 4);
      float4 a1 = *reinterpret_cast<const float4 *>(xs + k * XS + 64 + ty * 4);
      float4 b0 = *reinterpret_cast<const float4 *>(ws + k * TBN + tx * 4);
      float4 b1 = *reinterpret_cast<const float4 *>(ws + k * TBN + 64 + tx * 4);
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

  // Epilogue.
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int n = n0 + h * 64 + tx * 4;
      float v[4] = {acc[i][h * 4 + 0], acc[i][h * 4 + 1], acc[i][h * 4 + 2], acc[i][h * 4 + 3]};
      if (e.o.epi == EPI_KNORM) {
        // 64-column head = this half (h) of the tile across the 16 lanes of
        // the half-warp.  Only K blocks (even column-block index) are normed.
        // (clamped so a column past N never indexes past the scale table;
        // such columns are not stored)
        int blk = min(n, e.N - 1) / (e.o.kv_block ? e.o.kv_block : e.o.col_block);
        if ((blk & 1) == 0) knorm16(v, e.o.vec + (int64_t)(blk >> 1) * 64, tx);
      }
      if (m < M && n < e.N) store4(e, m, n, v[0], v[1], v[2], v[3], yvec);
    }
  }
}

// ── small-M path ───────────────────────────────────────────────────────────
template <int CW>
__global__ void __launch_bounds__(256) gemv_kernel(const float *__restrict__ x, int64_t ldx, int M, int K,
                                                   Int4Weight W, EpiCtx e) {
  constexpr int KS = 256 / CW;   // K-slices
  constexpr int NC = CW * 4;     // columns per CTA
  extern __shared__ __align__(16) float sm[];
  const int Kp = W.G * W.gs, npairs = Kp >> 1, N = W.N;
  float *xs = sm;                              // [M][Kp]
  float *red = sm + (size_t)M * Kp;            // [KS][M][NC]
  const int tid = threadIdx.x, c = tid % CW, ks = tid / CW;
  const int n0 = blockIdx.x * NC, n = n0 + c * 4;

  for (int i = tid; i < M * Kp; i += 256) {
    int m = i / Kp, k = i - m * Kp;
    xs[i] = k < K ? __ldg(x + (int64_t)m * ldx + k) : 0.0f;
  }
  __syncthreads();

  float acc[8][4];
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[m][j] = 0.0f;

  const int per = (npairs + KS - 1) / KS;
  const int p_beg = ks * per, p_end = min(npairs, p_beg + per);
  for (int p = p_beg; p < p_end; ++p) {
    int g = (2 * p) / W.gs;
    uint8_t b[4];
    float s[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int col = n + j;
      bool ok = col < N;
      if (W.w2) {
        const int Nh = N >> 1;
        b[j] = ok ? __ldg(((col & 1) ? W.w2 : W.w) + (int64_t)p * Nh + (col >> 1)) : 0;
        s[j] = ok ? __ldg(((col & 1) ? W.s2 : W.s) + (int64_t)g * Nh + (col >> 1)) : 0.0f;
      } else {
        b[j] = ok ? __ldg(W.w + (int64_t)p * N + col) : 0;
        s[j] = ok ? __ldg(W.s + (int64_t)g * N + col) : 0.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo = (float)sign_extend4(b[j] & 0xF), hi = (float)sign_extend4(b[j] >> 4);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        if (m < M) {
          float x0 = xs[m * Kp + 2 * p], x1 = xs[m * Kp + 2 * p + 1];
          // per-pair term in the order of matvec_avx2: (lo*x0 + hi*x1) * scale
          float t = fmaf(hi, x1, lo * x0);
          acc[m][j] += t * s[j];
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m)
    if (m < M)
#pragma unroll
      for (int j = 0; j < 4; ++j) red[(ks * M + m) * NC + c * 4 + j] = acc[m][j];
  __syncthreads();
  // Reduce the K-slices: thread -> (m, column).
  for (int i = tid; i < M * NC; i += 256) {
    int m = i / NC, cc = i - m * NC;
    float s = 0.0f;
    for (int k2 = 0; k2 < KS; ++k2) s += red[(k2 * M + m) * NC + cc];
    red[(0 * M + m) * NC + cc] = s;  // slice 0 is only read by this thread
  }
  __syncthreads();
  if (e.o.epi == EPI_KNORM) {
    // NC == 64 == one head; normalise row m if this block is a K block.
    for (int m = tid; m < M; m += 256) {
      int blk = n0 / (e.o.kv_block ? e.o.kv_block : e.o.col_block);
      if ((blk & 1) == 0) {
        float *r = red + m * NC;
        float ss = 0.0f;
        for (int j = 0; j < 64; ++j) ss += r[j] * r[j];
        float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
        const float *sv = e.o.vec + (int64_t)(blk >> 1) * 64;
        for (int j = 0; j < 64; ++j) r[j] = ((1.0f + sv[j]) * r[j]) * inv;
      }
    }
    __syncthreads();
  }
  for (int i = tid; i < M * (NC / 4); i += 256) {
    int m = i / (NC / 4), c4 = i - m * (NC / 4);
    int nn = n0 + c4 * 4;
    if (nn < N) {
      const float *r = red + m * NC + c4 * 4;
      store4(e, m, nn, r[0], r[1], r[2], r[3], false);
    }
  }
}

// Decode matvec for M <= 8 rows on 16-byte weight loads.  CTA = 256
// threads: CX column threads x (256 / CX) pair slices.  Each thread owns 16
// consecutive output columns (one 16-byte load per pair row: 16 packed
// bytes) and a contiguous run of pair rows; nibbles are unpacked in
// registers, slices are reduced with warp shuffles and then across the 8
// warps in shared memory.  The first batch of weight and scale loads is
// issued before griddepcontrol.wait, so under programmatic dependent launch
// it overlaps the previous kernel in the stream; x is read (and y written)
// only after the wait.  Requires N % 16 == 0 and 16-byte aligned weights and
// scales.
template <int MR, int CX>
__global__ void __launch_bounds__(256) gemv16_kernel(const float *__restrict__ x, int64_t ldx, int M, int K,
                                                     Int4Weight W, EpiCtx e) {
  constexpr int PY = 256 / CX;  // pair slices per CTA
  constexpr int NC = 16 * CX;   // columns per CTA
  constexpr int PF = MR >= 4 ? 4 : 8;  // pair rows loaded per batch
  extern __shared__ __align__(16) float sm[];
  asm volatile("griddepcontrol.launch_dependents;");
  const int N = W.N, Kp = W.G * W.gs, npairs = Kp >> 1;
  const int tid = threadIdx.x, tx = tid % CX, ty = tid / CX;
  const int n0 = blockIdx.x * NC, n = n0 + 16 * tx;
  const bool col_ok = n < N;
  const int pp = (npairs + PY - 1) / PY;
  const int p_beg = min(npairs, ty * pp), p_end = min(npairs, p_beg + pp);
  float *xs = sm;                                   // [M][Kp]
  float *red = sm + (((size_t)M * Kp + 3) & ~(size_t)3);  // [8 warps][MR][NC], 16-byte aligned

  uint4 wb[PF];
  auto load_batch = [&](int pb) {
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const int pi = pb + i;
      wb[i] = (col_ok && pi < p_end) ? __ldg(reinterpret_cast<const uint4 *>(W.w + (int64_t)pi * N + n))
                                     : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  float sc[16];
  int gcur = -1;
  auto load_scales = [&](int g) {
    if (col_ok) {
      const float4 *sp = reinterpret_cast<const float4 *>(W.s + (int64_t)g * N + n);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 v = __ldg(sp + q);
        sc[4 * q] = v.x;
        sc[4 * q + 1] = v.y;
        sc[4 * q + 2] = v.z;
        sc[4 * q + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) sc[j] = 0.0f;
    }
    gcur = g;
  };
  load_batch(p_beg);
  if (p_beg < p_end) load_scales((2 * p_beg) / W.gs);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = tid; i < M * Kp; i += 256) {
    int m = i / Kp, k = i - m * Kp;
    xs[i] = k < K ? x[(int64_t)m * ldx + k] : 0.0f;
  }
  __syncthreads();

  float acc[MR][16];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[m][j] = 0.0f;

  for (int p = p_beg; p < p_end; p += PF) {
    if (p != p_beg) load_batch(p);
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const int pi = p + i;
      if (pi < p_end) {
        const int g = (2 * pi) / W.gs;
        if (g != gcur) load_scales(g);
        const uint32_t wd[4] = {wb[i].x, wb[i].y, wb[i].z, wb[i].w};
        float lo[16], hi[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const uint32_t b = (wd[j >> 2] >> (8 * (j & 3))) & 0xFFu;
          lo[j] = (float)sign_extend4(b & 0xFu);
          hi[j] = (float)sign_extend4(b >> 4);
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m < M) {
            const float x0 = xs[m * Kp + 2 * pi], x1 = xs[m * Kp + 2 * pi + 1];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // per-pair term in the order of matvec_avx2: (lo*x0 + hi*x1) * scale
              const float t = fmaf(hi[j], x1, lo[j] * x0);
              acc[m][j] += t * sc[j];
            }
          }
        }
      }
    }
  }
  // Reduce the slices of this warp (lanes with equal tx), then across warps.
#pragma unroll
  for (int off = CX; off < 32; off <<= 1)
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], off);
  const int warp = tid >> 5, lane = tid & 31;
  if (lane < CX) {
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4 *>(red + (warp * MR + m) * NC + 16 * lane + j) =
            make_float4(acc[m][j], acc[m][j + 1], acc[m][j + 2], acc[m][j + 3]);
  }
  __syncthreads();
  for (int i = tid; i < M * (NC / 4); i += 256) {
    const int m = i / (NC / 4), c4 = i - m * (NC / 4);
    const int nn = n0 + 4 * c4;
    if (nn < N) {
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float4 r = *reinterpret_cast<const float4 *>(red + (w * MR + m) * NC + 4 * c4);
        v[0] += r.x;
        v[1] += r.y;
        v[2] += r.z;
        v[3] += r.w;
      }
      store4(e, m, nn, v[0], v[1], v[2], v[3], false);
    }
  }
}

template <int MR, int CX>
cudaError_t launch_gemv16(const float *x, int64_t ldx, int M, const Int4Weight &W, const EpiCtx &e, bool pdl,
                          cudaStream_t stream) {
  constexpr int NC = 16 * CX;
  const int Kp = W.G * W.gs;
  const size_t sm = ((((size_t)M * Kp + 3) & ~(size_t)3) + (size_t)8 * MR * NC) * sizeof(float);
  if (sm > (size_t)kMaxDynSmem) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((W.N + NC - 1) / NC);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = sm;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv16_kernel<MR, CX>, x, ldx, M, W.K, W, e);
}

template <int CX>
cudaError_t dispatch_gemv16(const float *x, int64_t ldx, int M, const Int4Weight &W, const EpiCtx &e, bool pdl,
                            cudaStream_t stream) {
  if (M <= 1) return launch_gemv16<1, CX>(x, ldx, M, W, e, pdl, stream);
  if (M <= 2) return launch_gemv16<2, CX>(x, ldx, M, W, e, pdl, stream);
  if (M <= 4) return launch_gemv16<4, CX>(x, ldx, M, W, e, pdl, stream);
  return launch_gemv16<8, CX>(x, ldx, M, W, e, pdl, stream);
}

__global__ void quantize_kernel(const float *__restrict__ w, int K, int N, int gs, int G, uint8_t *data,
                                float *scales) {
  // quant.rs:63-128.  One thread per (group, column): computes the scale
  // then packs the group's pairs.  IEEE division and roundf (half away from
  // zero) match the reference bit for bit.
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)G * N) return;
  int g = (int)(idx / N), o = (int)(idx % N);
  float max_abs = 0.0f;
  for (int r = 0; r < gs; ++r) {
    int gr = g * gs + r;
    float v = gr < K ? fabsf(w[(int64_t)gr * N + o]) : 0.0f;
    if (v > max_abs) max_abs = v;
  }
  float s = __fdiv_rn(max_abs, 7.0f);
  s = isnan(s) ? 1e-8f : fmaxf(s, 1e-8f);
  scales[(int64_t)g * N + o] = s;
  for (int r = 0; r < gs; r += 2) {
    int r0 = g * gs + r, r1 = r0 + 1;
    float v0 = r0 < K ? w[(int64_t)r0 * N + o] : 0.0f;
    float v1 = r1 < K ? w[(int64_t)r1 * N + o] : 0.0f;
    float f0 = roundf(__fdiv_rn(v0, s)), f1 = roundf(__fdiv_rn(v1, s));
    f0 = isnan(f0) ? 0.0f : fminf(fmaxf(f0, -8.0f), 7.0f);
    f1 = isnan(f1) ? 0.0f : fminf(fmaxf(f1, -8.0f), 7.0f);
    int q0 = (int)f0, q1 = (int)f1;
    data[(int64_t)(r0 >> 1) * N + o] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
  }
}

__global__ void dequantize_kernel(const uint8_t *__restrict__ data, const float *__restrict__ scales, int K,
                                  int N, int gs, int G, float *out) {
  // quant.rs:131-155
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t npairs = (int64_t)G * gs / 2;
  if (idx >= npairs * N) return;
  int64_t pair = idx / N;
  int o = (int)(idx % N);
  int r0 = (int)(pair * 2), r1 = r0 + 1, g = r0 / gs;
  uint8_t b = data[idx];
  float s = scales[(int64_t)g * N + o];
  if (r0 < K) out[(int64_t)r0 * N + o] = (float)sign_extend4(b & 0xF) * s;
  if (r1 < K) out[(int64_t)r1 * N + o] = (float)sign_extend4(b >> 4) * s;
}

}  // namespace

cudaError_t init_matmul_kernels() {
  cudaError_t e = cudaSuccess;
  for (const void *f : {(const void *)tile_kernel, (const void *)gemv_kernel<8>, (const void *)gemv_kernel<16>,
                        (const void *)gemv16_kernel<1, 2>, (const void *)gemv16_kernel<2, 2>,
                        (const void *)gemv16_kernel<4, 2>, (const void *)gemv16_kernel<8, 2>,
                        (const void *)gemv16_kernel<1, 4>, (const void *)gemv16_kernel<2, 4>,
                        (const void *)gemv16_kernel<4, 4>, (const void *)gemv16_kernel<8, 4>}) {
    cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    if (r != cudaSuccess) e = r;
  }
  return e;
}

cudaError_t int4_matmul(const float *x, int64_t ldx, int M, const Int4Weight &W, const MatmulOut &o,
                        cudaStream_t stream, bool pdl) {
  if (M <= 0 || W.N <= 0) return cudaSuccess;
  if (W.gs <= 0 || W.G <= 0 || (W.gs & 1)) return cudaErrorInvalidValue;
  if (W.w2 && ((W.N & 1) || !W.s2)) return cudaErrorInvalidValue;
  // Output groups of 4 columns never straddle a column block; the fused
  // k-norm needs whole 64-column heads.
  if (o.col_block && (o.col_block % 4)) return cudaErrorInvalidValue;
  if (o.epi == EPI_QKV || o.epi == EPI_QKV_DEC || o.epi == EPI_ARGMAX) return cudaErrorInvalidValue;  // tensor-core only
  if (o.epi == EPI_KNORM &&
      (!o.col_block || (o.col_block % 64) || !o.vec || (o.kv_block && (o.kv_block % o.col_block))))
    return cudaErrorInvalidValue;
  if (o.epi == EPI_ACT && ((W.N & 1) || o.planes[0])) return cudaErrorInvalidValue;  // planes: tensor-core only
  EpiCtx e{o, W.N};
  const int Kp = W.G * W.gs;
  if (M <= 8 && !W.w2 && o.epi != EPI_KNORM && (W.N % 16) == 0 && ((uintptr_t)W.w % 16) == 0 &&
      ((uintptr_t)W.s % 16) == 0) {
    // 128 or more CTAs where the width allows, else 32-column CTAs
    if (W.N / 64 >= 96) return dispatch_gemv16<4>(x, ldx, M, W, e, pdl, stream);
    return dispatch_gemv16<2>(x, ldx, M, W, e, pdl, stream);
  }
  if (M <= 8) {
    if (o.epi == EPI_KNORM || W.N > 1024) {
      size_t sm = ((size_t)M * Kp + (size_t)16 * M * 64) * sizeof(float);
      if (sm > (size_t)kMaxDynSmem) return cudaErrorInvalidValue;
      gemv_kernel<16><<<(W.N + 63) / 64, 256, sm, stream>>>(x, ldx, M, W.K, W, e);
    } else {
      size_t sm = ((size_t)M * Kp + (size_t)32 * M * 32) * sizeof(float);
      if (sm > (size_t)kMaxDynSmem) return cudaErrorInvalidValue;
      gemv_kernel<8><<<(W.N + 31) / 32, 256, sm, stream>>>(x, ldx, M, W.K, W, e);
    }
    return cudaGetLastError();
  }
  bool xvec = (ldx % 4 == 0) && ((uintptr_t)x % 16 == 0);
  bool yvec = (o.ldy % 4 == 0) && ((uintptr_t)o.y % 16 == 0) &&
              (!o.col_block || (o.block_stride % 4 == 0));
  size_t sm = (size_t)2 * TBK * (XS + TBN) * sizeof(float);
  dim3 grid((W.N + TBN - 1) / TBN, (M + TBM - 1) / TBM);
  if (grid.y > 65535) return cudaErrorInvalidConfiguration;
  tile_kernel<<<grid, 256, sm, stream>>>(x, ldx, M, W.K, W, e, xvec, yvec);
  return cudaGetLastError();
}

cudaError_t int4_quantize(const float *w, int K, int N, uint8_t *data, float *scales, cudaStream_t st) {
  if (K <= 0 || N <= 0) return cudaErrorInvalidValue;
  int gs = K < 32 ? K : 32;
  if (gs & 1) return cudaErrorInvalidValue;  // an odd group would split a packed pair
  int Kp = K + (gs - K % gs) % gs, G = Kp / gs;
  int64_t n = (int64_t)G * N;
  quantize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, K, N, gs, G, data, scales);
  return cudaGetLastError();
}

cudaError_t int4_dequantize(const uint8_t *data, const float *scales, int K, int N, int G, float *out,
                            cudaStream_t st) {
  if (K <= 0 || N <= 0 || G <= 0) return cudaErrorInvalidValue;
  int gs = K < 32 ? K : 32;
  int64_t n = (int64_t)G * gs / 2 * N;
  dequantize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(data, scales, K, N, gs, G, out);
  return cudaGetLastError();
}

}  // namespace ndl
