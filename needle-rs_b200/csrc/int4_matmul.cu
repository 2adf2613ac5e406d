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

// Matvec for M <= 8 rows on 16-byte weight loads (decode with few requests,
// and the standalone INT4 matmul).  CTA = 256 threads = CX column threads x
// KS = 256 / CX pair-row slices.  Each thread owns 16 consecutive output
// columns (one 16-byte load per pair row) over a contiguous run of pair
// rows, fetched with cp.async into its own slots of a shared-memory ring 8
// pair rows ahead, so that loads stay in flight without holding registers.
//
// Unpack: the nibbles of a 32-bit word (4 columns, low nibble = row 2p, high
// = row 2p+1) are XORed with 8 once, so nibble u' = q + 8 in [0, 15].  One
// LOP3 then turns the nibble at bit s (s <= 12) into the float
// 2^23 + u' * 2^s ((w & (0xF << s)) | 0x4B000000); one packed subtract of
// (2^23 + 8 * 2^s) leaves q * 2^s exactly, and packed multiplies by x * 2^-s
// (an exact power-of-two scaling) give the products q * x.  The upper
// half-word takes one shift.  The terms are those of matvec_avx2
// (quant.rs:209-297): (lo * x0 + hi * x1) * scale per pair row and column,
// in f32; for a single row the pair terms of a 32-row scale group are
// summed first and scaled once (another summation order, same terms).
// About 4.5 instructions per weight byte with packed f32x2 arithmetic.
//
// Under programmatic dependent launch the first weight and scale loads are
// issued before griddepcontrol.wait (no kernel of the stream writes
// weights); x is read, and y written, after it.  Requires N % 16 == 0 and
// 16-byte aligned weights and scales.
// q * 2^s of the nibble (XORed with 8) at bit s of w, exactly: bias = 2^23 + 8 * 2^s.
// Nibble under `mask` (bits 0-15) of w as an exact float.  The reference
// packs two's-complement nibbles; XOR 8 makes them offset binary q + 8, and
// OR 0x4B000000 places that in a float's mantissa: 2^23 + (q + 8) * 2^s for
// the nibble at bit s.  The magic bits and the mask are disjoint, so both
// steps are one XOR with g = (0x88888888 & mask) | 0x4B000000: a single
// LOP3 when g sits in a register (a kernel argument, not an immediate,
// since the mask already takes the instruction's one immediate).
// Subtracting `bias` = 2^23 + 8 * 2^s leaves q * 2^s exactly.
__device__ __forceinline__ float q4_at(uint32_t w, uint32_t mask, uint32_t g, float bias) {
  return __uint_as_float((w & mask) ^ g) - bias;
}

// One 16-byte pair-row load of a thread (pair row p of its 16 columns) into
// the per-group sums of one row of x: lo * x0 + hi * x1 per column, with x
// pre-scaled per nibble position (x0, x0 / 256, x1 / 16, x1 / 4096), on
// packed f32 pairs: in2[2 * wq + h] holds columns 4wq + 2h, 4wq + 2h + 1 of
// 32-bit word wq.  Per lane the subtract and the two FMAs round as the
// scalar form would.
__device__ __forceinline__ void q4_row1x2(const uint4 cw, const float4 xv, uint64_t (&in2)[8], const uint4 gq) {
  const uint64_t XL = f2pack(xv.x, xv.y), XH = f2pack(xv.z, xv.w);
  const uint64_t BL = f2pack(8388616.0f, 8390656.0f), BH = f2pack(8388736.0f, 8421376.0f);
  const uint32_t wds[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
  for (int wq = 0; wq < 4; ++wq) {
    const uint32_t wl = wds[wq], wu = wds[wq] >> 16;
    const uint64_t lo01 = fsub2(f2pack(__uint_as_float((wl & 0xFu) ^ gq.x), __uint_as_float((wl & 0xF00u) ^ gq.z)), BL);
    const uint64_t lo23 = fsub2(f2pack(__uint_as_float((wu & 0xFu) ^ gq.x), __uint_as_float((wu & 0xF00u) ^ gq.z)), BL);
    const uint64_t hi01 =
        fsub2(f2pack(__uint_as_float((wl & 0xF0u) ^ gq.y), __uint_as_float((wl & 0xF000u) ^ gq.w)), BH);
    const uint64_t hi23 =
        fsub2(f2pack(__uint_as_float((wu & 0xF0u) ^ gq.y), __uint_as_float((wu & 0xF000u) ^ gq.w)), BH);
    in2[2 * wq] = ffma2(hi01, XH, ffma2(lo01, XL, in2[2 * wq]));
    in2[2 * wq + 1] = ffma2(hi23, XH, ffma2(lo23, XL, in2[2 * wq + 1]));
  }
}

template <int MR, int CX>
__global__ void __launch_bounds__(256, MR <= 2 ? 2 : 1) gemv_q4_kernel(const float *__restrict__ x, int64_t ldx,
                                                                        int M, int K, Int4Weight W, EpiCtx e,
                                                                        uint4 gq) {
  constexpr int KS = 256 / CX;  // pair-row slices per CTA
  constexpr int NC = 16 * CX;   // columns per CTA
  constexpr int D = 8;          // pair rows in flight per thread (shared-memory ring)
  extern __shared__ __align__(16) float sm[];
  asm volatile("griddepcontrol.launch_dependents;");
  const int N = W.N, Kp = W.G * W.gs, npairs = Kp >> 1, gp = W.gs >> 1;  // gp: pair rows per scale group
  const int tid = threadIdx.x, tx = tid % CX, ks = tid / CX;
  const int n0 = blockIdx.x * NC, n = n0 + 16 * tx;
  const bool col_ok = n < N;
  const int pp = (npairs + KS - 1) / KS;
  const int p_beg = min(npairs, ks * pp), p_end = min(npairs, p_beg + pp);
  uint4 *ring = reinterpret_cast<uint4 *>(sm);               // [D][256]: this thread's 16 bytes at [slot][tid]
  float4 *xq = reinterpret_cast<float4 *>(sm) + D * 256;      // [MR][npairs]: (x0, x0 / 256, x1 / 16, x1 / 4096)
  float *red = reinterpret_cast<float *>(xq + MR * npairs);  // reduction buffer

  // cp.async of pair row pi into slot (pi - p_beg) % D; one commit group per
  // call (empty past the slice), so group counts stay uniform.
  const uint32_t ring0 = (uint32_t)__cvta_generic_to_shared(ring + tid);
  const uint8_t *wcol = W.w + n;
  auto issue = [&](int pi, int slot) {
    if (col_ok && pi < p_end)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ring0 + slot * 4096u), "l"(wcol + (int64_t)pi * N)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float sc[16], scn[16];  // this and the next scale group
  auto load_scales = [&](int g, float *dst) {
    const float4 *sp = reinterpret_cast<const float4 *>(W.s + (int64_t)g * N + n);
    const bool ok = col_ok && g * gp < p_end;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = ok ? __ldg(sp + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      dst[4 * q] = v.x;
      dst[4 * q + 1] = v.y;
      dst[4 * q + 2] = v.z;
      dst[4 * q + 3] = v.w;
    }
  };
  int g = p_beg < p_end ? p_beg / gp : 0;
#pragma unroll
  for (int d = 0; d < D - 1; ++d) issue(p_beg + d, d);
  load_scales(g, sc);
  load_scales(g + 1, scn);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Stage x: row m goes to the 8 / MR warps m * WPR .. m * WPR + WPR - 1,
  // whose threads take 16-byte chunks 4q..4q+3 for q = r, r + 32 WPR, ...
  // (r the thread's rank in the group; a thread's loads are in flight
  // together), or single elements when the rows are not 16-byte aligned.
  // The rows' ZCRMSNorm folds in: the same pass sums the squares, and once
  // the group's sum is in each thread rescales the pairs it wrote.
  const float *nsc = e.o.in_norm;
  {
    constexpr int WPR = 8 / MR, GT = 32 * WPR;  // warps and threads per row
    __shared__ float ssq[8];
    const int warp = tid >> 5, lane = tid & 31, m = warp / WPR, r = tid - m * GT;
    const bool vec = ((ldx & 3) == 0) && (((uintptr_t)x & 15) == 0) && (K & 3) == 0;
    float4 *xr = xq + m * npairs;
    const float *xm = x + (int64_t)m * ldx;
    auto put = [&](float4 *dst, float x0, float x1) {
      *dst = nsc ? make_float4(x0, 0.0f, x1, 0.0f)  // rescaled below
                 : make_float4(x0, x0 * 0.00390625f, x1 * 0.0625f, x1 * 0.000244140625f);
    };
    float ss = 0.0f;
    if (vec) {
#pragma unroll 4
      for (int q = r; 2 * q < npairs; q += GT) {
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (m < M && 4 * q < K) v = *reinterpret_cast<const float4 *>(xm + 4 * q);
        ss += v.x * v.x;
        ss += v.y * v.y;
        ss += v.z * v.z;
        ss += v.w * v.w;
        put(xr + 2 * q, v.x, v.y);
        put(xr + 2 * q + 1, v.z, v.w);
      }
    } else {
#pragma unroll 4
      for (int p = r; p < npairs; p += GT) {
        const float x0 = m < M && 2 * p < K ? xm[2 * p] : 0.0f, x1 = m < M && 2 * p + 1 < K ? xm[2 * p + 1] : 0.0f;
        ss += x0 * x0;
        ss += x1 * x1;
        put(xr + p, x0, x1);
      }
    }
    if (nsc) {
      ss = warp_sum(ss);
      if (lane == 0) ssq[warp] = ss;
      __syncthreads();
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < WPR; ++w) tot += ssq[m * WPR + w];
      const float ri = 1.0f / sqrtf(tot / (float)K + 1e-6f);
      // the pairs this thread wrote: 2q, 2q + 1 (chunks) or p (elements)
      const int step = vec ? 2 * GT : GT, first = vec ? 2 * r : r, span = vec ? 2 : 1;
      for (int p0 = first; p0 < npairs; p0 += step)
        for (int p = p0; p < p0 + span; ++p) {
          const float4 v = xr[p];
          float x0 = 0.0f, x1 = 0.0f;
          if (2 * p < K) x0 = ((1.0f + __ldg(nsc + 2 * p)) * v.x) * ri;
          if (2 * p + 1 < K) x1 = ((1.0f + __ldg(nsc + 2 * p + 1)) * v.z) * ri;
          xr[p] = make_float4(x0, x0 * 0.00390625f, x1 * 0.0625f, x1 * 0.000244140625f);
        }
    }
  }
  __syncthreads();

  // one row: per-group sums of (lo * x0 + hi * x1), times the group's scale
  // when the group ends (one scale FMA per 16 pair rows); more rows: scale
  // per pair row (fewer registers)
  constexpr bool kGroupSums = MR == 1;
  float acc[MR][16], inner[kGroupSums ? MR : 1][16];
  uint64_t acc2[kGroupSums ? 1 : MR][8];  // more rows: packed column pairs
#pragma unroll
  for (int m = 0; m < (kGroupSums ? 1 : MR); ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc2[m][j] = 0ull;
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[m][j] = 0.0f;
#pragma unroll
  for (int m = 0; m < (kGroupSums ? MR : 1); ++m)
#pragma unroll
    for (int j = 0; j < 16; ++j) inner[m][j] = 0.0f;
  auto flush = [&]() {
    if constexpr (kGroupSums) {
#pragma unroll
      for (int m = 0; m < MR; ++m)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[m][j] = fmaf(inner[m][j], sc[j], acc[m][j]);
          inner[m][j] = 0.0f;
        }
    }
  };

  int slot = 0, gend = (g + 1) * gp;
  bool fast = false;
  if constexpr (kGroupSums) fast = gp == 16 && (p_beg & 15) == 0 && ((p_end - p_beg) & 15) == 0;
  if constexpr (kGroupSums) {
    // One row, whole 16-pair-row scale groups: a group per iteration, its
    // rows unrolled, so ring slots and waits are constants and the scale
    // switch falls on the iteration boundary.
    const uint8_t *src = wcol + (int64_t)(p_beg + D - 1) * N;  // the next pair row to request
    const int64_t stride = N;
    for (int pg = p_beg; fast && pg < p_end; pg += 16) {
      uint64_t in2[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) in2[j] = 0ull;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        asm volatile("cp.async.wait_group %0;" ::"n"(D - 2) : "memory");  // row pg + d has landed
        const uint4 cw = ring[(d & (D - 1)) * 256 + tid];
        if (col_ok && pg + d + D - 1 < p_end)  // into the slot row pg + d - 1 left
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ring0 + ((d + D - 1) & (D - 1)) * 4096u),
                       "l"(src)
                       : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
        src += stride;
        q4_row1x2(cw, xq[pg + d], in2, gq);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) f2unpack(in2[j], inner[0][2 * j], inner[0][2 * j + 1]);
      flush();
      ++g;
#pragma unroll
      for (int j = 0; j < 16; ++j) sc[j] = scn[j];
      load_scales(g + 1, scn);
    }
  }
#pragma unroll(kGroupSums ? 2 : 1)
  for (int pi = p_beg; !fast && pi < p_end; ++pi) {
    asm volatile("cp.async.wait_group %0;" ::"n"(D - 2) : "memory");  // row pi has landed
    const uint4 cw = ring[slot * 256 + tid];
    issue(pi + D - 1, slot == 0 ? D - 1 : slot - 1);  // into the slot row pi - 1 left
    slot = slot == D - 1 ? 0 : slot + 1;
    {
      if (pi >= gend) {  // next scale group
        flush();
        ++g;
        gend += gp;
#pragma unroll
        for (int j = 0; j < 16; ++j) sc[j] = scn[j];
        load_scales(g + 1, scn);
      }
      float4 xv[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) xv[m] = xq[m * npairs + pi];
      const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
      for (int wq = 0; wq < 4; ++wq) {
        const uint32_t wl = wd[wq], wu = wd[wq] >> 16;
        // columns 4wq .. 4wq+3: low nibbles at bits 0 / 8, high at 4 / 12 of each half-word
        if constexpr (kGroupSums) {
          const float lo[4] = {q4_at(wl, 0xFu, gq.x, 8388616.0f), q4_at(wl, 0xF00u, gq.z, 8390656.0f),
                               q4_at(wu, 0xFu, gq.x, 8388616.0f), q4_at(wu, 0xF00u, gq.z, 8390656.0f)};
          const float hi[4] = {q4_at(wl, 0xF0u, gq.y, 8388736.0f), q4_at(wl, 0xF000u, gq.w, 8421376.0f),
                               q4_at(wu, 0xF0u, gq.y, 8388736.0f), q4_at(wu, 0xF000u, gq.w, 8421376.0f)};
          // x pre-scaled per nibble position: (x0, x0 / 256, x1 / 16, x1 / 4096)
          const float xl[4] = {xv[0].x, xv[0].y, xv[0].x, xv[0].y}, xh[4] = {xv[0].z, xv[0].w, xv[0].z, xv[0].w};
#pragma unroll
          for (int c = 0; c < 4; ++c)
            inner[0][4 * wq + c] = fmaf(hi[c], xh[c], fmaf(lo[c], xl[c], inner[0][4 * wq + c]));
        } else {
          // (lo * x0 + hi * x1) * scale per column, as matvec_avx2 orders it,
          // on packed column pairs (each lane rounds as the scalar form)
          const uint64_t BL = f2pack(8388616.0f, 8390656.0f), BH = f2pack(8388736.0f, 8421376.0f);
          const uint64_t lo01 =
              fsub2(f2pack(__uint_as_float((wl & 0xFu) ^ gq.x), __uint_as_float((wl & 0xF00u) ^ gq.z)), BL);
          const uint64_t lo23 =
              fsub2(f2pack(__uint_as_float((wu & 0xFu) ^ gq.x), __uint_as_float((wu & 0xF00u) ^ gq.z)), BL);
          const uint64_t hi01 =
              fsub2(f2pack(__uint_as_float((wl & 0xF0u) ^ gq.y), __uint_as_float((wl & 0xF000u) ^ gq.w)), BH);
          const uint64_t hi23 =
              fsub2(f2pack(__uint_as_float((wu & 0xF0u) ^ gq.y), __uint_as_float((wu & 0xF000u) ^ gq.w)), BH);
          const uint64_t s01 = f2pack(sc[4 * wq], sc[4 * wq + 1]), s23 = f2pack(sc[4 * wq + 2], sc[4 * wq + 3]);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            const uint64_t XL = f2pack(xv[m].x, xv[m].y), XH = f2pack(xv[m].z, xv[m].w);
            acc2[m][2 * wq] = ffma2(ffma2(hi01, XH, fmul2(lo01, XL)), s01, acc2[m][2 * wq]);
            acc2[m][2 * wq + 1] = ffma2(ffma2(hi23, XH, fmul2(lo23, XL)), s23, acc2[m][2 * wq + 1]);
          }
        }
      }
    }
  }
  if constexpr (!kGroupSums) {
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) f2unpack(acc2[m][j], acc[m][2 * j], acc[m][2 * j + 1]);
  }
  flush();
  asm volatile("cp.async.wait_group 0;" ::: "memory");

  // Reduce the pair-row slices: lanes of one warp that share columns (CX <
  // 32) by shuffles, then the R partial rows in shared memory in a fixed order.
  constexpr int R = CX >= 32 ? KS : 8;
  const int warp = tid >> 5, lane = tid & 31;
  if constexpr (CX < 32) {
    // Transposed butterfly, row by row: at each level a lane keeps the half
    // of a row's 16 values that its offset bit selects and adds its
    // partner's copies of them.  The pairs and their order are the plain
    // butterfly's, so the sums are the same bits, with 16 - 16 / 2^L
    // shuffles a row instead of 16 L.
    constexpr int L = CX == 2 ? 4 : CX == 4 ? 3 : CX == 8 ? 2 : 1, LEN = 16 >> L;
    int base = 0;  // the lane ends with the sums of columns 16 tx + base .. + LEN - 1
#pragma unroll
    for (int l = 0; l < L; ++l) {
      const int off = CX << l, h = 8 >> l;
      const bool up = lane & off;
#pragma unroll
      for (int m = 0; m < MR; ++m)
#pragma unroll
        for (int i = 0; i < h; ++i) {
          const float send = up ? acc[m][i] : acc[m][i + h], keep = up ? acc[m][i + h] : acc[m][i];
          acc[m][i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      if (up) base += h;
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float *dst = red + (warp * MR + m) * NC + 16 * tx + base;
      if constexpr (LEN >= 4) {
#pragma unroll
        for (int i = 0; i < LEN; i += 4)
          *reinterpret_cast<float4 *>(dst + i) = make_float4(acc[m][i], acc[m][i + 1], acc[m][i + 2], acc[m][i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < LEN; ++i) dst[i] = acc[m][i];
      }
    }
  } else {
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4 *>(red + (ks * MR + m) * NC + 16 * tx + j) =
            make_float4(acc[m][j], acc[m][j + 1], acc[m][j + 2], acc[m][j + 3]);
  }
  __syncthreads();
  for (int i = tid; i < M * (NC / 4); i += 256) {
    const int m = i / (NC / 4), c4 = i - m * (NC / 4);
    const int nn = n0 + 4 * c4;
    if (nn < N) {
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float4 t = *reinterpret_cast<const float4 *>(red + (r * MR + m) * NC + 4 * c4);
        v[0] += t.x;
        v[1] += t.y;
        v[2] += t.z;
        v[3] += t.w;
      }
      store4(e, m, nn, v[0], v[1], v[2], v[3], false);
    }
  }
}

template <int MR, int CX>
size_t gemv_q4_smem(int Kp) {
  constexpr int KS = 256 / CX, R = CX >= 32 ? KS : 8;
  return (size_t)8 * 256 * 16 + (size_t)MR * (Kp / 2) * 16 + (size_t)R * MR * 16 * CX * 4;
}

template <int MR, int CX>
cudaError_t launch_gemv_q4(const float *x, int64_t ldx, int M, const Int4Weight &W, const EpiCtx &e, bool pdl,
                           cudaStream_t stream) {
  constexpr int NC = 16 * CX;
  const size_t sm = gemv_q4_smem<MR, CX>(W.G * W.gs);
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
  // (0x88888888 & mask) | 0x4B000000 for the nibble masks 0xF, 0xF0, 0xF00, 0xF000
  const uint4 gq = make_uint4(0x4B000008u, 0x4B000080u, 0x4B000800u, 0x4B008000u);
  return cudaLaunchKernelEx(&cfg, gemv_q4_kernel<MR, CX>, x, ldx, M, W.K, W, e, gq);
}

// Column threads per CTA: 1024 columns a CTA for wide matrices (long runs of
// pair rows per thread, few reductions), narrower CTAs (more pair-row
// slices, down to 32 columns) while the grid would not cover the SMs.
int gemv_q4_cx(int MR, int N) {
  const int cols16 = N / 16;
  if (MR <= 2 && cols16 >= 64 * 296) return 64;
  if (MR <= 2 && cols16 >= 32 * 296) return 32;
  if (cols16 >= 16 * 148) return 16;
  if (cols16 >= 8 * 148) return 8;
  if (cols16 >= 4 * 148) return 4;
  return 2;
}

template <int MR>
cudaError_t dispatch_gemv_q4(const float *x, int64_t ldx, int M, const Int4Weight &W, const EpiCtx &e, bool pdl,
                             cudaStream_t stream) {
  switch (gemv_q4_cx(MR, W.N)) {
    case 64:
      if constexpr (MR <= 2) return launch_gemv_q4<MR, 64>(x, ldx, M, W, e, pdl, stream);
      break;
    case 32:
      if constexpr (MR <= 2) return launch_gemv_q4<MR, 32>(x, ldx, M, W, e, pdl, stream);
      break;
    case 16:
      return launch_gemv_q4<MR, 16>(x, ldx, M, W, e, pdl, stream);
    case 8:
      return launch_gemv_q4<MR, 8>(x, ldx, M, W, e, pdl, stream);
    case 4:
      return launch_gemv_q4<MR, 4>(x, ldx, M, W, e, pdl, stream);
    default:
      break;
  }
  return launch_gemv_q4<MR, 2>(x, ldx, M, W, e, pdl, stream);
}

// The 16-byte-load matvec serves M <= 8 rows of a plain (unpaired) weight
// whose columns come in 16s, with 16-byte aligned data and scales.
bool gemv_q4_fits(int M, const Int4Weight &W, const MatmulOut &o) {
  return M <= 8 && !W.w2 && o.epi != EPI_KNORM && (W.N % 16) == 0 && ((uintptr_t)W.w % 16) == 0 &&
         ((uintptr_t)W.s % 16) == 0;
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
                        (const void *)gemv_q4_kernel<1, 8>, (const void *)gemv_q4_kernel<1, 16>,
                        (const void *)gemv_q4_kernel<1, 32>, (const void *)gemv_q4_kernel<1, 64>,
                        (const void *)gemv_q4_kernel<2, 8>, (const void *)gemv_q4_kernel<2, 16>,
                        (const void *)gemv_q4_kernel<2, 32>, (const void *)gemv_q4_kernel<2, 64>,
                        (const void *)gemv_q4_kernel<4, 8>, (const void *)gemv_q4_kernel<4, 16>,
                        (const void *)gemv_q4_kernel<8, 8>, (const void *)gemv_q4_kernel<8, 16>,
                        (const void *)gemv_q4_kernel<1, 2>, (const void *)gemv_q4_kernel<1, 4>,
                        (const void *)gemv_q4_kernel<2, 2>, (const void *)gemv_q4_kernel<2, 4>,
                        (const void *)gemv_q4_kernel<4, 2>, (const void *)gemv_q4_kernel<4, 4>,
                        (const void *)gemv_q4_kernel<8, 2>, (const void *)gemv_q4_kernel<8, 4>}) {
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
  if (o.in_norm && !gemv_q4_fits(M, W, o)) return cudaErrorInvalidValue;  // input norm: the matvec only
  EpiCtx e{o, W.N};
  const int Kp = W.G * W.gs;
  if (gemv_q4_fits(M, W, o)) {
    if (M <= 1) return dispatch_gemv_q4<1>(x, ldx, M, W, e, pdl, stream);
    if (M <= 2) return dispatch_gemv_q4<2>(x, ldx, M, W, e, pdl, stream);
    if (M <= 4) return dispatch_gemv_q4<4>(x, ldx, M, W, e, pdl, stream);
    return dispatch_gemv_q4<8>(x, ldx, M, W, e, pdl, stream);
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

bool int4_matmul_norms_input(int M, const Int4Weight &W, const MatmulOut &o) { return gemv_q4_fits(M, W, o); }

size_t int4_matmul_smem(int M, const Int4Weight &W, const MatmulOut &o) {
  if (M <= 0 || W.N <= 0 || W.G <= 0 || W.gs <= 0) return 0;
  const int Kp = W.G * W.gs;
  if (gemv_q4_fits(M, W, o)) {
    const int MR = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8, CX = gemv_q4_cx(MR, W.N);
    const int R = CX >= 32 ? 256 / CX : 8;
    return (size_t)8 * 256 * 16 + (size_t)MR * (Kp / 2) * 16 + (size_t)R * MR * 16 * CX * 4;
  }
  if (M <= 8)
    return (o.epi == EPI_KNORM || W.N > 1024) ? ((size_t)M * Kp + (size_t)16 * M * 64) * sizeof(float)
                                               : ((size_t)M * Kp + (size_t)32 * M * 32) * sizeof(float);
  return (size_t)2 * TBK * (XS + TBN) * sizeof(float);
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
