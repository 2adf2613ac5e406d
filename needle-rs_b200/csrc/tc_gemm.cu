// tc_gemm.cu — INT4-weight matmul on the 5th-generation tensor cores (tcgen05).
//
// Y[M, N] (epilogue) X[M, K] @ W for the batched paths (encoder prefill, the
// cross-attention K/V fill, batched decode), replacing the M-fold matvec loop
// of QuantizedWeight::matmul (crates/needle-core/src/quant.rs:400-410).
//
// Precision.  The reference is f32 end to end.  A single bf16 MMA would cost
// ~2^-9 relative per product, too much for 1e-3 / 1e-4 logit parity after 20
// layers, so both operands are split into bf16 pairs, hi = bf16(v) and
// lo = bf16(v - hi) (|v - hi - lo| <= 2^-18 |v|), and each K-step issues three
// MMAs, hi*hi + hi*lo + lo*hi, into one f32 accumulator in TMEM (the dropped
// lo*lo term is <= 2^-18 relative).  Net error ~1e-6 relative per GEMM.
//
// Operands.  W's dequantized values q * scale (quant.rs:131-155) are written
// once per weight, at load, as two bf16 planes [N][Kp] (K contiguous, Kp =
// K rounded up to 64): the packed INT4 weight stays the stored format and the
// planes are its tensor-core staging copy (4 bytes per weight; the whole model
// is ~100 MB).  Activations arrive as bf16 planes [M][Kp] written by the
// producing kernel (norm, attention) or by split_rows().
//
// Kernel.  Persistent, one CTA per SM, 384 threads, warp-specialised:
//   warp 0      TMA producer: 128x64 A tiles and BNx64 B tiles (hi and lo),
//               128-byte swizzle, into a shared-memory ring (3 stages at
//               BN = 128, 2 at BN = 256; B arrives as 128-row boxes)
//   warp 1      TMEM allocation + MMA issue (one elected lane):
//               tcgen05.mma.cta_group::1.kind::f16, M=128, N=BN, K=16
//   warps 2-3   idle (they complete the producer warpgroup)
//   warps 4-11  epilogue in two warpgroups, one per half of the tile's
//               columns: tcgen05.ld of the f32 accumulator (warp w owns TMEM
//               lanes 32(w%4).. = output rows), fused epilogue (store / gated
//               residual / activation / per-head k-norm / q-k norm + RoPE to
//               attention planes / masked argmax).  The producer warpgroup
//               hands registers to them with setmaxnreg.
// TMEM holds two accumulators so the epilogue of tile i overlaps the MMAs
// of tile i+1.  BN = 256 (tall matrices) halves the shared-memory operand
// bytes each MMA reads per output; BN = 128 keeps more tiles than SMs for
// the decode-sized ones.  Every TMA load fills only its own CTA's shared memory.  Every mbarrier wait
// is bounded: on expiry the kernel records an error flag and unwinds.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace ndl {
namespace {

using namespace tc;

constexpr int TC_BM = 128, TC_BK = 64, TC_THREADS = 384;
// The split-K kernel: warps 0-3 producer / MMA, warps 4-7 one epilogue
// warpgroup; 256 threads leave every thread up to 255 registers.
constexpr int TC_SPLITK_THREADS = 256;
// Registers a thread: launched at 168 (65,536 / 384, rounded down to 8); the
// producer warpgroup drops to 56 and the two epilogue warpgroups rise to 224:
// 128 x 56 + 256 x 224 = 384 x 168.
constexpr int TC_REG_LAUNCH = 168, TC_REG_PRODUCER = 56, TC_REG_EPILOGUE = 224;
static_assert(128 * TC_REG_PRODUCER + 256 * TC_REG_EPILOGUE == TC_THREADS * TC_REG_LAUNCH,
              "the register split must add up to the launch's registers");
struct TcEpi {
  MatmulOut o;
  int N;
};

__device__ __forceinline__ float act_apply_tc(int act, float g, float u) {
  if (act == ACT_SWIGLU) {
    float sg = g * (1.0f / (1.0f + expf(-g)));
    return sg * u;
  }
  if (act == ACT_GELU) {
    const float C = 0.79788456f, A = 0.044715f;
    float ax = A * g;
    float axx = ax * g;
    float axxx = axx * g;
    float inner = C * (g + axxx);
    float t = 1.0f + tanhf(inner);
    return (0.5f * g) * t * u;
  }
  float rg = g > 0.0f ? g : 0.0f, ru = u > 0.0f ? u : 0.0f;
  return rg * ru;
}

// Epilogue of `cnt` (32 or 64) consecutive columns n0.. of row m (cnt is a
// template parameter so the row stays in registers).
template <int cnt>
__device__ __forceinline__ void epi_row(const TcEpi &e, int m, int n0, float *v) {
  const MatmulOut &o = e.o;
  if (o.epi == EPI_ACT) {
    if (o.planes[0]) {  // bf16 hi/lo operand planes of the next matmul (row stride ldy elements)
      static_assert(cnt % 16 == 0, "whole 8-output groups");
      const int64_t off = (int64_t)m * o.ldy + (n0 >> 1);
      uint4 *dh = reinterpret_cast<uint4 *>((__nv_bfloat16 *)o.planes[0] + off);
      uint4 *dl = reinterpret_cast<uint4 *>((__nv_bfloat16 *)o.planes[1] + off);
#pragma unroll
      for (int q = 0; q < cnt / 16; ++q) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = 16 * q + 4 * i;
          const float a0 = (n0 + j + 1 < e.N) ? act_apply_tc(o.act, v[j], v[j + 1]) : 0.0f;
          const float a1 = (n0 + j + 3 < e.N) ? act_apply_tc(o.act, v[j + 2], v[j + 3]) : 0.0f;
          __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
          float2 hf = __bfloat1622float2(h);
          __nv_bfloat162 lo = __floats2bfloat162_rn(a0 - hf.x, a1 - hf.y);
          hw[i] = *reinterpret_cast<uint32_t *>(&h);
          lw[i] = *reinterpret_cast<uint32_t *>(&lo);
        }
        if (n0 + 16 * q < e.N) {
          dh[q] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          dl[q] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
      return;
    }
    float *p = o.y + (int64_t)m * o.ldy + (n0 >> 1);
#pragma unroll
    for (int j = 0; j + 1 < cnt; j += 2)
      if (n0 + j + 1 < e.N) p[j >> 1] = act_apply_tc(o.act, v[j], v[j + 1]);
    return;
  }
  if (o.epi == EPI_KNORM) {
    int blk = n0 / (o.kv_block ? o.kv_block : o.col_block);
    if ((blk & 1) == 0) {  // K block: ZCRMSNorm each 64-column head (norm.rs:23-30)
      const float4 *sc = reinterpret_cast<const float4 *>(o.vec + (int64_t)(blk >> 1) * 64);
#pragma unroll
      for (int h = 0; h + 64 <= cnt; h += 64) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 64; ++j) ss += v[h + j] * v[h + j];
        float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float4 s4 = __ldg(sc + j);
          v[h + 4 * j + 0] = ((1.0f + s4.x) * v[h + 4 * j + 0]) * inv;
          v[h + 4 * j + 1] = ((1.0f + s4.y) * v[h + 4 * j + 1]) * inv;
          v[h + 4 * j + 2] = ((1.0f + s4.z) * v[h + 4 * j + 2]) * inv;
          v[h + 4 * j + 3] = ((1.0f + s4.w) * v[h + 4 * j + 3]) * inv;
        }
      }
    }
  }
  // cnt columns never straddle a column block (col_block % 64 == 0)
  float *p;
  if (o.col_block) {
    int b = n0 / o.col_block;
    p = o.y + (int64_t)b * o.block_stride + (int64_t)m * o.ldy + (n0 - b * o.col_block);
  } else {
    p = o.y + (int64_t)m * o.ldy + n0;
  }
  if (n0 + cnt <= e.N) {
    float4 *p4 = reinterpret_cast<float4 *>(p);
    if (o.epi == EPI_RESID) {
#pragma unroll
      for (int j = 0; j < cnt / 4; ++j) {
        float4 r = p4[j];
        r.x += o.gate * v[4 * j + 0];
        r.y += o.gate * v[4 * j + 1];
        r.z += o.gate * v[4 * j + 2];
        r.w += o.gate * v[4 * j + 3];
        p4[j] = r;
      }
    } else {
#pragma unroll
      for (int j = 0; j < cnt / 4; ++j) p4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
  } else {
    for (int j = 0; j < cnt && n0 + j < e.N; ++j) p[j] = (o.epi == EPI_RESID) ? p[j] + o.gate * v[j] : v[j];
  }
}

// EPI_QKV / EPI_QKV_DEC on the 64 columns (one head) n0.. of row m:
// ZCRMSNorm + RoPE for Q and K heads (attn.rs:218-235, 120-140), then either
// bf16 hi/lo into the encoder attention planes or, for a decoder step, Q as
// f32 and K, V appended to the self-attention caches.
// ZCRMSNorm + RoPE (attn.rs:218-235, 120-140) of the Q or K head in the 64
// columns n0.. of row m, in place; V heads pass unchanged.  Returns the
// plane pair (0 Q, 2 K, 4 V) and writes the head's index within it.
__device__ __forceinline__ int qkv64_transform(const TcEpi &e, int m, int n0, float *v, int &head) {
  const MatmulOut &o = e.o;
  const int hh = n0 >> 6, H = o.heads_q, KVH = o.heads_kv;
  if (hh >= H + KVH) {
    head = hh - H - KVH;
    return 4;
  }
  {
    const float4 *sc = reinterpret_cast<const float4 *>(hh < H ? o.q_norm : o.k_norm);
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 64; ++j) ss += v[j] * v[j];
    float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float4 s4 = __ldg(sc + j);
      v[4 * j + 0] = ((1.0f + s4.x) * v[4 * j + 0]) * inv;
      v[4 * j + 1] = ((1.0f + s4.y) * v[4 * j + 1]) * inv;
      v[4 * j + 2] = ((1.0f + s4.z) * v[4 * j + 2]) * inv;
      v[4 * j + 3] = ((1.0f + s4.w) * v[4 * j + 3]) * inv;
    }
    const int p = o.pos[m];
    const float4 *cr = reinterpret_cast<const float4 *>(o.rope_cos + (int64_t)p * 32);
    const float4 *sr = reinterpret_cast<const float4 *>(o.rope_sin + (int64_t)p * 32);
#pragma unroll
    for (int i4 = 0; i4 < 8; ++i4) {
      float4 c4 = __ldg(cr + i4), s4 = __ldg(sr + i4);
      const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ssn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = 4 * i4 + u;
        float x0 = v[i], x1 = v[i + 32];
        float l = x0 * cc[u] - x1 * ssn[u];
        float r = x1 * cc[u] + x0 * ssn[u];
        v[i] = l;
        v[i + 32] = r;
      }
    }
  }
  head = hh < H ? hh : hh - H;
  return hh < H ? 0 : 2;
}

__device__ __forceinline__ void epi_qkv64(const TcEpi &e, int m, int n0, float *v) {
  const MatmulOut &o = e.o;
  const int hh = n0 >> 6, H = o.heads_q, KVH = o.heads_kv;
  int head;
  const int plane = qkv64_transform(e, m, n0, v, head);
  const int64_t base = ((int64_t)head * o.slab + m) * 64;
  if (o.epi == EPI_QKV_DEC) {
    float *dst;
    if (hh < H) {
      dst = o.y + (int64_t)m * o.ldy + hh * 64;
    } else {
      const int p = o.pos[m];
      if (p >= o.cache_cap) return;  // cache full: nothing appended
      dst = (hh < H + KVH ? o.kcache : o.vcache) + ((int64_t)m * o.cache_cap + p) * (KVH * 64) +
            (hh < H + KVH ? hh - H : hh - H - KVH) * 64;
    }
    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int j = 0; j < 16; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    return;
  }
  uint4 *dh = reinterpret_cast<uint4 *>((__nv_bfloat16 *)o.planes[plane] + base);
  uint4 *dl = reinterpret_cast<uint4 *>((__nv_bfloat16 *)o.planes[plane + 1] + base);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float x0 = v[8 * q + 2 * i], x1 = v[8 * q + 2 * i + 1];
      __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
      float2 hf = __bfloat1622float2(h);
      __nv_bfloat162 lo = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
      hw[i] = *reinterpret_cast<uint32_t *>(&h);
      lw[i] = *reinterpret_cast<uint32_t *>(&lo);
    }
    dh[q] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    dl[q] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

// EPI_ARGMAX over 32 columns n0.. of row m: masked logits -> best key.
__device__ __forceinline__ unsigned long long epi_argmax32(const TcEpi &e, int m, int n0, const float *v) {
  const MatmulOut &o = e.o;
  const int step = o.pos[m];
  const uint64_t *mrow = o.mask ? o.mask + ((int64_t)m * o.max_new + step) * o.mask_words : nullptr;
  float *lrow = o.logits ? o.logits + ((int64_t)m * o.max_new + step) * e.N : nullptr;
  uint64_t bits = ~0ull;
  if (mrow) {  // the 32 columns lie in one or two 64-bit words
    uint64_t w0 = mrow[n0 >> 6];
    uint64_t w1 = ((n0 & 63) + 32 > 64) ? mrow[(n0 >> 6) + 1] : 0ull;
    int sh = n0 & 63;
    bits = sh ? ((w0 >> sh) | (w1 << (64 - sh))) : w0;
  }
  unsigned long long best = 0ull;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    int n = n0 + j;
    if (n < e.N) {
      // the engine always adds the mask vector (0.0 when allowed), so -0.0 -> +0.0
      float mv = v[j] + (((bits >> j) & 1ull) ? 0.0f : kMaskBlocked);
      if (lrow) lrow[n] = mv;
      unsigned long long k = argmax_key(mv, (uint32_t)n);
      best = k > best ? k : best;
    }
  }
  return best;
}

// Epilogue of accumulator columns [c0, c1) for this thread's output row m
// (TMEM lane quarter at `base`); output column = n_base + accumulator column.
__device__ __forceinline__ void epi_tile(const TcEpi &e, int M, int N, int m, uint32_t base, int c0, int c1,
                                         int n_base) {
  const bool amax = e.o.epi == EPI_ARGMAX;
  const bool qkv = e.o.epi == EPI_QKV || e.o.epi == EPI_QKV_DEC;
  const bool wide = e.o.epi == EPI_KNORM || qkv;  // whole 64-column heads
  unsigned long long best = 0ull;
  for (int c = c0; c < c1; c += (wide ? 64 : 32)) {
    float v[64];
    tmem_ld32(base + c, v);
    if (wide) tmem_ld32(base + c + 32, v + 32);
    const int n0 = n_base + c;
    if (m < M && n0 < N) {
      if (amax) {
        unsigned long long k = epi_argmax32(e, m, n0, v);
        best = k > best ? k : best;
      } else if (qkv) {
        epi_qkv64(e, m, n0, v);
      } else if (wide) {
        epi_row<64>(e, m, n0, v);
      } else {
        epi_row<32>(e, m, n0, v);
      }
    }
  }
  if (amax && m < M) atomicMax(e.o.keys + m, best);
}

// TMA maps of the six bf16 attention planes the encoder QKV epilogue writes
// (Q hi, Q lo, K hi, K lo, V hi, V lo): each {64, rows, heads} with 32 x 64
// boxes, 128-byte swizzle.
struct QkvMaps {
  CUtensorMap m[6];
};

// Plane pair (0 Q, 2 K, 4 V) and head within it of the 64 QKV columns n0..
__device__ __forceinline__ int qkv64_plane(const MatmulOut &o, int n0, int &head) {
  const int hh = n0 >> 6;
  if (hh < o.heads_q) {
    head = hh;
    return 0;
  }
  if (hh < o.heads_q + o.heads_kv) {
    head = hh - o.heads_q;
    return 2;
  }
  head = hh - o.heads_q - o.heads_kv;
  return 4;
}

// TMA output path of the encoder QKV epilogue for one warp's 32 rows (tile
// rows m0.., TMEM lane quarter at `base`): per 64-column head, the per-row
// norm + RoPE, then the head's 32 rows go to its bf16 hi and lo attention
// planes as two 32 x 64 boxes, staged in the warp's 4 KB buffer with the
// same swizzle as epi_tile_tma (one 128-byte row per lane).  Rows past M
// are zero and clipped by the maps (their row extent is M).
__device__ __forceinline__ void epi_tile_qkv_tma(const TcEpi &e, const QkvMaps &qm, int M, int N, int m0, int lane,
                                                 uint32_t base, int c0, int c1, int n_base, uint8_t *stg) {
  for (int c = c0; c < c1; c += 64) {
    float v[64];
    tmem_ld32(base + c, v);
    tmem_ld32(base + c + 32, v + 32);
    const int n0 = n_base + c;
    if (n0 >= N) continue;  // warp-uniform
    int head;
    const int plane = qkv64_plane(e.o, n0, head);
    if (m0 + lane < M) {
      int h2;
      qkv64_transform(e, m0 + lane, n0, v, h2);
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] = 0.0f;
    }
    uint32_t hw[32], lw[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      const float2 hf = __bfloat1622float2(h);
      const __nv_bfloat162 lo = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
      hw[i] = *reinterpret_cast<const uint32_t *>(&h);
      lw[i] = *reinterpret_cast<const uint32_t *>(&lo);
    }
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      if (lane == 0) bulk_wait_read_all();  // the previous box has left `stg`
      __syncwarp();
      uint8_t *row = stg + lane * 128;
      const uint32_t *w = part ? lw : hw;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4 *>(row + ((j ^ (lane & 7)) << 4)) =
            make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&qm.m[plane + part], stg, 0, m0, head);
        bulk_commit();
      }
    }
  }
}

// Whether the epilogue `epi` writes through the TMA output map when one is
// given: the f32 outputs of the plain store, the gated residual (as a
// reduce-add of gate * acc) and the k-norm.
__device__ __forceinline__ bool epi_uses_tma(int epi) {
  return epi == EPI_STORE || epi == EPI_RESID || epi == EPI_KNORM;
}

// TMA output path of the store / gated-residual / k-norm epilogues for one
// warp's 32 rows (tile rows m0.., TMEM lane quarter at `base`), accumulator
// columns [c0, c1), output column = n_base + accumulator column.  Every
// 32 x 32 f32 box is staged in the warp's 4 KB buffer `stg` in the 128-byte
// swizzled layout of the map (row r's 16-byte chunk j at r * 128 + ((j ^
// (r & 7)) << 4): one row per lane touches every bank once) and written by
// one TMA store issued by lane 0; the residual adds gate * acc to y with a
// TMA reduce-add (each element once, so the result is deterministic).  A
// thread storing its own row directly scatters each warp instruction over
// 32 rows and reaches a fraction of the SM's store bandwidth.  Rows past M
// and columns past the map's extent are not written.  The bulk group is
// drained (read) before `stg` is reused, and completely before the CTA
// exits (tma_epi_drain).
__device__ __forceinline__ void epi_tile_tma(const TcEpi &e, const CUtensorMap *map, int N, int m0, int lane,
                                             uint32_t base, int c0, int c1, int n_base, uint8_t *stg) {
  const MatmulOut &o = e.o;
  const bool knorm = o.epi == EPI_KNORM, resid = o.epi == EPI_RESID;
  const int cnt = knorm ? 64 : 32;
  for (int c = c0; c < c1; c += cnt) {
    float v[64];
    tmem_ld32(base + c, v);
    if (knorm) tmem_ld32(base + c + 32, v + 32);
    const int n0 = n_base + c;
    if (n0 >= N) continue;  // warp-uniform
    if (knorm) {
      const int blk = n0 / (o.kv_block ? o.kv_block : o.col_block);
      if ((blk & 1) == 0) {  // K block: ZCRMSNorm of the 64-column head (norm.rs:23-30)
        const float4 *sc = reinterpret_cast<const float4 *>(o.vec + (int64_t)(blk >> 1) * 64);
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 64; ++j) ss += v[j] * v[j];
        const float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float4 s4 = __ldg(sc + j);
          v[4 * j + 0] = ((1.0f + s4.x) * v[4 * j + 0]) * inv;
          v[4 * j + 1] = ((1.0f + s4.y) * v[4 * j + 1]) * inv;
          v[4 * j + 2] = ((1.0f + s4.z) * v[4 * j + 2]) * inv;
          v[4 * j + 3] = ((1.0f + s4.w) * v[4 * j + 3]) * inv;
        }
      }
    } else if (resid) {  // layers.rs:70-74: x += gate * out
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = o.gate * v[j];
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h * 32 >= cnt) break;
      if (lane == 0) bulk_wait_read_all();  // the previous box has left `stg`
      __syncwarp();
      uint8_t *row = stg + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4 *>(row + ((j ^ (lane & 7)) << 4)) =
            make_float4(v[32 * h + 4 * j], v[32 * h + 4 * j + 1], v[32 * h + 4 * j + 2], v[32 * h + 4 * j + 3]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int n = n0 + 32 * h;
        if (o.col_block) {
          if (resid)
            tma_reduce_add_3d(map, stg, n % o.col_block, m0, n / o.col_block);
          else
            tma_store_3d(map, stg, n % o.col_block, m0, n / o.col_block);
        } else if (resid) {
          tma_reduce_add_2d(map, stg, n, m0);
        } else {
          tma_store_2d(map, stg, n, m0);
        }
        bulk_commit();
      }
    }
  }
}

// Before the CTA leaves: every TMA output store of this warp has completed.
__device__ __forceinline__ void tma_epi_drain(int lane) {
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

template <int BN, int TC_STAGES>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                   const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                   const __grid_constant__ CUtensorMap tmY, const __grid_constant__ QkvMaps tmQ, int M, int N, int Kp,
                   TcEpi e, int *err, int b_lo_zero, int y_tma, int qkv_tma) {
  constexpr int A_BYTES = TC_BM * TC_BK * 2, B_BYTES = BN * TC_BK * 2;
  constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  constexpr uint32_t IDESC = umma_idesc(TC_BM, BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment of every operand tile (128-byte swizzle atoms).
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + TC_STAGES * STAGE_BYTES);
  uint64_t *empty = full + TC_STAGES;
  uint64_t *tfull = empty + TC_STAGES;
  uint64_t *tempty = tfull + 2;
  uint32_t *tmem_slot = (uint32_t *)(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + TC_BM - 1) / TC_BM, num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n, nkb = Kp / TC_BK;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 256);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // two BN-column f32 accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *(volatile uint32_t *)tmem_slot;
  // under programmatic dependent launch the setup above overlaps the previous
  // kernel's tail; global memory is touched only after it has completed
  pdl_wait();

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(TC_REG_PRODUCER));
    if (warp == 0) {
      // ── TMA producer ──
      if (lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmAh) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmAl) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmBh) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmBl) : "memory");
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
          const int mt = t / num_n, nt = t - mt * num_n;
          for (int kb = 0; kb < nkb; ++kb) {
            if (!(ok = mbar_wait(&empty[stage], phase ^ 1, err))) break;
            uint8_t *st = smem + stage * STAGE_BYTES;
            mbar_expect_tx(&full[stage], b_lo_zero ? STAGE_BYTES - B_BYTES : STAGE_BYTES);
            tma_load_2d(st, &tmAh, &full[stage], kb * TC_BK, mt * TC_BM);
            tma_load_2d(st + A_BYTES, &tmAl, &full[stage], kb * TC_BK, mt * TC_BM);
  #pragma unroll
            for (int h = 0; h < BN / 128; ++h) {  // 128-row boxes, contiguous in shared memory
              tma_load_2d(st + 2 * A_BYTES + h * (B_BYTES * 128 / BN), &tmBh, &full[stage], kb * TC_BK,
                          nt * BN + 128 * h);
              if (!b_lo_zero)  // an all-zero lo plane is neither loaded nor multiplied
                tma_load_2d(st + 2 * A_BYTES + B_BYTES + h * (B_BYTES * 128 / BN), &tmBl, &full[stage],
                            kb * TC_BK, nt * BN + 128 * h);
            }
            if (++stage == TC_STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        // Drain: wait until the MMAs consumed every issued stage, so no TMA
        // write is still in flight when the CTA exits.
        for (int s = 0; s < TC_STAGES && ok; ++s) {
          ok = mbar_wait(&empty[stage], phase ^ 1, err);
          if (++stage == TC_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    } else if (warp == 1) {
      // ── MMA issuer ──
      if (lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        int i = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
          const int buf = i & 1;
          if (!(ok = mbar_wait(&tempty[buf], ((i >> 1) & 1) ^ 1, err))) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t d = tmem + (uint32_t)(buf * BN);
          for (int kb = 0; kb < nkb; ++kb) {
            if (!(ok = mbar_wait(&full[stage], phase, err))) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint8_t *st = smem + stage * STAGE_BYTES;
            const uint64_t ah = umma_desc(st), al = umma_desc(st + A_BYTES);
            const uint64_t bh = umma_desc(st + 2 * A_BYTES), bl = umma_desc(st + 2 * A_BYTES + B_BYTES);
  #pragma unroll
            for (int k = 0; k < TC_BK / 16; ++k) {
              const uint64_t adv = (uint64_t)((k * 32) >> 4);  // 16 bf16 = 32 bytes along K
              umma_bf16(d, ah + adv, bh + adv, IDESC, (kb | k) ? 1u : 0u);
              if (!b_lo_zero) umma_bf16(d, ah + adv, bl + adv, IDESC, 1u);
              umma_bf16(d, al + adv, bh + adv, IDESC, 1u);
            }
            umma_commit(&empty[stage]);  // frees the stage once these MMAs complete
            if (++stage == TC_STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (ok) umma_commit(&tfull[buf]);
        }
      }
    }
  } else {
    // ── epilogue: warpgroup `half` takes columns [half * BN/2, (half + 1) * BN/2) ──
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(TC_REG_EPILOGUE));
    const int q = warp & 3, half = (warp - 4) >> 2;
    const bool tma_out = y_tma && epi_uses_tma(e.o.epi), qkv_out = qkv_tma && e.o.epi == EPI_QKV;
    uint8_t *stg = smem + TC_STAGES * STAGE_BYTES + 1024 + (warp - 4) * 4096;  // 1024-byte aligned
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      if (!warp_wait(&tfull[buf], (i >> 1) & 1, err)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int mt = t / num_n, nt = t - mt * num_n;
      const int m = mt * TC_BM + q * 32 + lane;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      if (tma_out)
        epi_tile_tma(e, &tmY, N, m - lane, lane, base, half * (BN / 2), (half + 1) * (BN / 2), nt * BN, stg);
      else if (qkv_out)
        epi_tile_qkv_tma(e, tmQ, M, N, m - lane, lane, base, half * (BN / 2), (half + 1) * (BN / 2), nt * BN, stg);
      else
        epi_tile(e, M, N, m, base, half * (BN / 2), (half + 1) * (BN / 2), nt * BN);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&tempty[buf]);
    }
    if (tma_out || qkv_out) tma_epi_drain(lane);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  }
}

// CTA-pair GEMM for tall matrices: a cluster of two CTAs computes 256 x 256
// output tiles with tcgen05.mma.cta_group::2 M256 N256 K16.  Each CTA loads
// its own 128 rows of A and its own 128 rows (output columns) of B into its
// shared memory (64 KB per K block of 64, 3 stages); the leader CTA issues
// the MMAs, which read both CTAs' tiles at the same offsets and leave each
// CTA's 128 output rows in its own TMEM.  Per MMA a CTA's shared memory
// supplies half the operand bytes of the single-CTA M128 N256 form.
// Synchronisation: both CTAs' loads complete on the leader's `full`
// barrier (the leader expects both CTAs' bytes); MMA completion is
// signalled to both CTAs' `empty` and `tfull` barriers; both CTAs'
// epilogue warps arrive on the leader's `tempty`.  Every wait is bounded.
template <int STAGES>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                        const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                        const __grid_constant__ CUtensorMap tmY, const __grid_constant__ QkvMaps tmQ, int M, int N,
                        int Kp, TcEpi e, int *err, int b_lo_zero, int y_tma, int qkv_tma) {
  constexpr int HALF = 128, BN = 256;
  constexpr int A_BYTES = HALF * TC_BK * 2, B_BYTES = HALF * TC_BK * 2;
  constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  constexpr uint32_t IDESC = umma_idesc(2 * HALF, BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + STAGES * STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint32_t *tmem_slot = (uint32_t *)(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (M + 2 * HALF - 1) / (2 * HALF), num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n, nkb = Kp / TC_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 16);  // 8 epilogue warps in each CTA
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // two 256-column f32 accumulators in each CTA's TMEM
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *(volatile uint32_t *)tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(TC_REG_PRODUCER));
    if (warp == 0 && lane == 0) {
      // ── TMA producer (both CTAs) ──
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmAh) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmAl) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmBh) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmBl) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int mt = t / num_n, nt = t - mt * num_n;
        const int arow = mt * 2 * HALF + (int)rank * HALF, brow = nt * BN + (int)rank * HALF;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!(ok = mbar_wait(&empty[stage], phase ^ 1, err))) break;
          if (rank == 0)  // both CTAs' bytes
            mbar_expect_tx(&full[stage], 2 * (b_lo_zero ? STAGE_BYTES - B_BYTES : STAGE_BYTES));
          const uint32_t fb = pair_leader_addr(&full[stage]);
          uint8_t *st = smem + stage * STAGE_BYTES;
          tma_load_2d_pair(st, &tmAh, fb, kb * TC_BK, arow);
          tma_load_2d_pair(st + A_BYTES, &tmAl, fb, kb * TC_BK, arow);
          tma_load_2d_pair(st + 2 * A_BYTES, &tmBh, fb, kb * TC_BK, brow);
          if (!b_lo_zero) tma_load_2d_pair(st + 2 * A_BYTES + B_BYTES, &tmBl, fb, kb * TC_BK, brow);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every issued stage consumed before the CTA exits.
      for (int s = 0; s < STAGES && ok; ++s) {
        ok = mbar_wait(&empty[stage], phase ^ 1, err);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    } else if (warp == 1 && lane == 0 && rank == 0) {
      // ── MMA issuer (leader CTA) ──
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs, ++i) {
        const int buf = i & 1;
        if (!(ok = mbar_wait(&tempty[buf], ((i >> 1) & 1) ^ 1, err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!(ok = mbar_wait(&full[stage], phase, err))) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          uint8_t *st = smem + stage * STAGE_BYTES;
          const uint64_t ah = umma_desc(st), al = umma_desc(st + A_BYTES);
          const uint64_t bh = umma_desc(st + 2 * A_BYTES), bl = umma_desc(st + 2 * A_BYTES + B_BYTES);
#pragma unroll
          for (int k = 0; k < TC_BK / 16; ++k) {
            const uint64_t adv = (uint64_t)((k * 32) >> 4);  // 16 bf16 = 32 bytes along K
            umma_bf16_pair(d, ah + adv, bh + adv, IDESC, (kb | k) ? 1u : 0u);
            if (!b_lo_zero) umma_bf16_pair(d, ah + adv, bl + adv, IDESC, 1u);
            umma_bf16_pair(d, al + adv, bh + adv, IDESC, 1u);
          }
          umma_commit_pair(&empty[stage]);  // both CTAs' stage is free once these MMAs complete
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit_pair(&tfull[buf]);
      }
    }
  } else {
    // ── epilogue (both CTAs): warpgroup `half` takes 128 of the 256 columns ──
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(TC_REG_EPILOGUE));
    const int q = warp & 3, half = (warp - 4) >> 2;
    const bool tma_out = y_tma && epi_uses_tma(e.o.epi), qkv_out = qkv_tma && e.o.epi == EPI_QKV;
    uint8_t *stg = smem + STAGES * STAGE_BYTES + 1024 + (warp - 4) * 4096;  // 1024-byte aligned
    int i = 0;
    for (int t = pair; t < tiles; t += npairs, ++i) {
      const int buf = i & 1;
      if (!warp_wait(&tfull[buf], (i >> 1) & 1, err)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int mt = t / num_n, nt = t - mt * num_n;
      const int m = mt * 2 * HALF + (int)rank * HALF + q * 32 + lane;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      if (tma_out)
        epi_tile_tma(e, &tmY, N, m - lane, lane, base, half * (BN / 2), (half + 1) * (BN / 2), nt * BN, stg);
      else if (qkv_out)
        epi_tile_qkv_tma(e, tmQ, M, N, m - lane, lane, base, half * (BN / 2), (half + 1) * (BN / 2), nt * BN, stg);
      else
        epi_tile(e, M, N, m, base, half * (BN / 2), (half + 1) * (BN / 2), nt * BN);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&tempty[buf], 0);  // the leader's barrier
    }
    if (tma_out || qkv_out) tma_epi_drain(lane);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync();  // no remote arrive or MMA targets a CTA that has left
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  }
}

// Split-K: shared-memory staging of 128 x 128 f32 rows, float (r, c) at
// r * kSkRs + c + 8 * (c / 32).  The stride (4 mod 32) and the pad after each
// 32 columns keep every access pattern used here free of bank conflicts:
// 8 lanes on 8 rows at one column (TMEM copy), a warp along one row
// (workspace copies), 8 threads on 2 rows x 4 column blocks or 4 rows x 2
// heads (epilogue units).
constexpr int kSkRs = 164;
__device__ __forceinline__ int sk_off(int r, int c) { return r * kSkRs + c + 8 * (c >> 5); }

// Epilogue of one (row, CW-column) unit of the reduced rows staged in
// shared memory: CW = 64 for the epilogues that need whole 64-column heads,
// 32 otherwise.  Unit u covers staged row u / (BN / CW) = tile row
// row0 + that, columns (u % (BN / CW)) * CW of the BN-column tile.
template <int BN, int CW>
__device__ __forceinline__ void splitk_finish(const TcEpi &e, int M, int N, const float *stg, int row0, int mt,
                                              int nt, int u) {
  constexpr int UPR = BN / CW;
  const int rl = u / UPR, c0 = (u % UPR) * CW;
  const float4 *p4 = reinterpret_cast<const float4 *>(stg + sk_off(rl, c0));
  float v[CW];
#pragma unroll
  for (int j = 0; j < CW / 4; ++j) {
    const float4 x = p4[j + (j >= 8 ? 2 : 0)];  // the 8-float pad after 32 columns
    v[4 * j] = x.x;
    v[4 * j + 1] = x.y;
    v[4 * j + 2] = x.z;
    v[4 * j + 3] = x.w;
  }
  const int m = mt * TC_BM + row0 + rl, n0 = nt * BN + c0;
  if (m >= M || n0 >= N) return;
  if constexpr (CW == 64) {
    if (e.o.epi == EPI_KNORM)
      epi_row<64>(e, m, n0, v);
    else
      epi_qkv64(e, m, n0, v);
  } else {
    if (e.o.epi == EPI_ARGMAX)
      atomicMax(e.o.keys + m, epi_argmax32(e, m, n0, v));
    else
      epi_row<32>(e, m, n0, v);
  }
}

// Split-K GEMM for grids with few output tiles (decode-sized M): a cluster
// of S CTAs shares one 128 x BN output tile (BN = 128, or 64 when the
// narrower tiles still leave room for the split), CTA r of the cluster taking
// k-blocks [r * nkb / S, (r + 1) * nkb / S).  Every SM ingests at most ~64
// bytes per clock from L2, so a lone CTA walking all of K spends most of its
// time waiting for operands; S CTAs load and multiply S slices at once.
// Reduction through L2: every CTA writes its partial tile from TMEM to its
// own block of the caller's workspace (o.splitk_ws), one cluster
// barrier (release / acquire at cluster scope) orders those writes before
// the reads, and CTA r sums the S partials of tile rows [r * 128 / S,
// (r + 1) * 128 / S) in rank order and applies the epilogue.  Partial rows
// move through shared memory so that every global access of a warp covers
// whole contiguous rows: a thread storing its own accumulator row
// scatters each warp instruction over 32 rows and reaches a fraction of the
// SM's bandwidth (distributed shared memory behaves the same way).
// Under programmatic dependent launch the first weight tiles are requested
// before the wait for the previous kernel; only the activation tiles wait.
// Every mbarrier wait is bounded; a wait that gives up still reaches the
// cluster barrier.
template <int S, int BN>
__global__ void __launch_bounds__(TC_SPLITK_THREADS, 1)
    tc_gemm_splitk_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                          const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl, int M,
                          int N, int Kp, TcEpi e, int *err, int b_lo_zero) {
  constexpr int STAGES = 3;
  static_assert(BN == 64 || BN == 128, "tile widths of the split-K kernel");
  constexpr int LPR = BN / 4, RPI = 32 / LPR;  // lanes per 16-byte-chunked row, rows per warp instruction
  constexpr int A_BYTES = TC_BM * TC_BK * 2, B_BYTES = BN * TC_BK * 2;
  constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  constexpr uint32_t IDESC = umma_idesc(TC_BM, BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + STAGES * STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint32_t *tmem_slot = (uint32_t *)(tfull + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int tile = blockIdx.x / S, num_n = (N + BN - 1) / BN;
  const int mt = tile / num_n, nt = tile - mt * num_n;
  const int kper = Kp / TC_BK / S, kb0 = (int)rank * kper;
  float *tile_ws = e.o.splitk_ws + (size_t)tile * S * (128 * BN);
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // one 128-column f32 accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *(volatile uint32_t *)tmem_slot;

  if (warp == 0 && lane == 0) {
    // ── TMA producer: this CTA's K slice.  The weight (B) tiles of the first
    // stages are requested before the previous kernel has finished: no
    // kernel of the stream writes weights. ──
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmBh) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmBl) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmAh) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmAl) : "memory");
    const int pre = kper < STAGES ? kper : STAGES;
    for (int kk = 0; kk < pre; ++kk) {  // fresh barriers: every stage is free
      const int kx = (kb0 + kk) * TC_BK;
      uint8_t *st = smem + kk * STAGE_BYTES;
      mbar_expect_tx(&full[kk], b_lo_zero ? STAGE_BYTES - B_BYTES : STAGE_BYTES);
      tma_load_2d(st + 2 * A_BYTES, &tmBh, &full[kk], kx, nt * BN);
      if (!b_lo_zero) tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tmBl, &full[kk], kx, nt * BN);
    }
    pdl_wait();
    for (int kk = 0; kk < pre; ++kk) {
      const int kx = (kb0 + kk) * TC_BK;
      uint8_t *st = smem + kk * STAGE_BYTES;
      tma_load_2d(st, &tmAh, &full[kk], kx, mt * TC_BM);
      tma_load_2d(st + A_BYTES, &tmAl, &full[kk], kx, mt * TC_BM);
    }
    int stage = pre % STAGES;
    uint32_t phase = pre == STAGES ? 1u : 0u;
    bool ok = true;
    for (int kk = pre; kk < kper; ++kk) {
      if (!(ok = mbar_wait(&empty[stage], phase ^ 1, err))) break;
      const int kx = (kb0 + kk) * TC_BK;
      uint8_t *st = smem + stage * STAGE_BYTES;
      mbar_expect_tx(&full[stage], b_lo_zero ? STAGE_BYTES - B_BYTES : STAGE_BYTES);
      tma_load_2d(st, &tmAh, &full[stage], kx, mt * TC_BM);
      tma_load_2d(st + A_BYTES, &tmAl, &full[stage], kx, mt * TC_BM);
      tma_load_2d(st + 2 * A_BYTES, &tmBh, &full[stage], kx, nt * BN);
      if (!b_lo_zero) tma_load_2d(st + 2 * A_BYTES + B_BYTES, &tmBl, &full[stage], kx, nt * BN);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    // Drain: every issued stage consumed before the CTA moves on
    for (int s = 0; s < STAGES && ok; ++s) {
      ok = mbar_wait(&empty[stage], phase ^ 1, err);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
  } else {
    pdl_wait();  // global memory (the workspace, the epilogue's output) after the previous kernel
    if (warp == 1 && lane == 0) {
      // ── MMA issuer ──
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kk = 0; kk < kper; ++kk) {
        if (!(ok = mbar_wait(&full[stage], phase, err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint8_t *st = smem + stage * STAGE_BYTES;
        const uint64_t ah = umma_desc(st), al = umma_desc(st + A_BYTES);
        const uint64_t bh = umma_desc(st + 2 * A_BYTES), bl = umma_desc(st + 2 * A_BYTES + B_BYTES);
#pragma unroll
        for (int k = 0; k < TC_BK / 16; ++k) {
          const uint64_t adv = (uint64_t)((k * 32) >> 4);  // 16 bf16 = 32 bytes along K
          umma_bf16(tmem, ah + adv, bh + adv, IDESC, (kk | k) ? 1u : 0u);
          if (!b_lo_zero) umma_bf16(tmem, ah + adv, bl + adv, IDESC, 1u);
          umma_bf16(tmem, al + adv, bh + adv, IDESC, 1u);
        }
        umma_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) umma_commit(tfull);
    } else if (warp >= 4) {
      // ── partial tile -> this CTA's workspace block: warp q copies TMEM lanes
      // (rows) 32q.. into shared memory over the drained operand ring, then
      // writes them out one 512-byte row per instruction ──
      const int q = warp & 3;
      float *stg = reinterpret_cast<float *>(smem);
      if (warp_wait(tfull, 0, err)) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int row = q * 32 + lane;
        const uint32_t base = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(base + c, v);
          float4 *d4 = reinterpret_cast<float4 *>(stg + sk_off(row, c));
#pragma unroll
          for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        __syncwarp();
        float4 *dst = reinterpret_cast<float4 *>(tile_ws + (size_t)rank * (128 * BN));
        const int rl = lane / LPR, c4 = lane % LPR;
#pragma unroll 4
        for (int r = q * 32; r < q * 32 + 32; r += RPI)
          __stcg(dst + (r + rl) * LPR + c4, *reinterpret_cast<const float4 *>(stg + sk_off(r + rl, 4 * c4)));
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync();  // every CTA's partial tile is in the workspace

  if (warp >= 4) {
    // ── reduction of tile rows [rank * ROWS, (rank + 1) * ROWS): warp q sums
    // its ROWS / 4 rows over the S partials in rank order (lane = 4 columns
    // of a row, every load of a lane in flight at once), stages them, then
    // every epilogue thread takes (row, column-block) units ──
    constexpr int ROWS = TC_BM / S, RPW = ROWS / 4, IT = RPW / RPI;  // IT * S loads per lane
    const int q = warp & 3, row0 = (int)rank * ROWS, rl = lane / LPR, c4 = lane % LPR;
    float *stg = reinterpret_cast<float *>(smem);
    const float4 *src = reinterpret_cast<const float4 *>(tile_ws);
    float4 x[IT][S];
#pragma unroll
    for (int i = 0; i < IT; ++i)
#pragma unroll
      for (int r = 0; r < S; ++r)
        x[i][r] = __ldcg(src + (size_t)r * (128 * LPR) + (row0 + q * RPW + i * RPI + rl) * LPR + c4);
#pragma unroll
    for (int i = 0; i < IT; ++i) {
      float4 a = x[i][0];
#pragma unroll
      for (int r = 1; r < S; ++r) {
        a.x += x[i][r].x;
        a.y += x[i][r].y;
        a.z += x[i][r].z;
        a.w += x[i][r].w;
      }
      *reinterpret_cast<float4 *>(stg + sk_off(q * RPW + i * RPI + rl, 4 * c4)) = a;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
    const int epi = e.o.epi;
    const bool wide = epi == EPI_KNORM || epi == EPI_QKV || epi == EPI_QKV_DEC;
    const int units = ROWS * (BN / (wide ? 64 : 32));
#pragma unroll 1
    for (int u = threadIdx.x - 128; u < units; u += 128) {
      if (wide)
        splitk_finish<BN, 64>(e, M, N, stg, row0, mt, nt, u);
      else
        splitk_finish<BN, 32>(e, M, N, stg, row0, mt, nt, u);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}

// W (reference INT4 layout) -> bf16 hi/lo planes [N][Kp], K contiguous.
__global__ void prep_weight_kernel(Int4Weight W, int Kp, __nv_bfloat16 *hi, __nv_bfloat16 *lo) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)W.N * Kp) return;
  int n = (int)(idx / Kp), k = (int)(idx - (int64_t)n * Kp);
  float w = 0.0f;
  if (k < W.K && k < W.G * W.gs) {
    int p = k >> 1, g = k / W.gs;
    uint8_t b;
    float s;
    if (W.w2) {
      const int Nh = W.N >> 1;
      b = ((n & 1) ? W.w2 : W.w)[(int64_t)p * Nh + (n >> 1)];
      s = ((n & 1) ? W.s2 : W.s)[(int64_t)g * Nh + (n >> 1)];
    } else {
      b = W.w[(int64_t)p * W.N + n];
      s = W.s[(int64_t)g * W.N + n];
    }
    int code = (k & 1) ? sign_extend4(b >> 4) : sign_extend4(b & 0xF);
    w = (float)code * s;  // quant.rs:144-151
  }
  __nv_bfloat16 h = __float2bfloat16_rn(w);
  hi[idx] = h;
  lo[idx] = __float2bfloat16_rn(w - __bfloat162float(h));
}

// f32 rows [M][K] (stride ldx) -> bf16 hi/lo planes [M][Kp] (zero padded).
__global__ void split_rows_kernel(const float *__restrict__ x, int64_t ldx, int M, int K, int Kp,
                                  __nv_bfloat16 *hi, __nv_bfloat16 *lo) {
  int64_t idx = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (idx >= (int64_t)M * Kp) return;
  int m = (int)(idx / Kp), k = (int)(idx - (int64_t)m * Kp);
  __nv_bfloat16 h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v = (k + j < K) ? x[(int64_t)m * ldx + k + j] : 0.0f;
    h[j] = __float2bfloat16_rn(v);
    l[j] = __float2bfloat16_rn(v - __bfloat162float(h[j]));
  }
  *reinterpret_cast<uint2 *>(hi + idx) = *reinterpret_cast<uint2 *>(h);
  *reinterpret_cast<uint2 *>(lo + idx) = *reinterpret_cast<uint2 *>(l);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  }
  return fn;
}

int tc_sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

// Operand ring, barriers (under 1 KB), then eight 4 KB TMA output staging
// buffers (one per epilogue warp, 1024-byte aligned for the 128-byte swizzle).
constexpr size_t kTmaStageBytes = 1024 + 8 * 4096;
constexpr size_t tc_smem_bytes(int BN, int stages) {
  return 1024 + (size_t)stages * (2 * TC_BM * TC_BK * 2 + 2 * BN * TC_BK * 2) + kTmaStageBytes;
}
static_assert(tc_smem_bytes(128, 3) <= 232448 && tc_smem_bytes(256, 2) <= 232448,
              "exceeds the 227 KB of dynamic shared memory per block");
constexpr int TC_PAIR_STAGES = 3;
constexpr size_t tc_smem_pair_bytes() { return 1024 + (size_t)TC_PAIR_STAGES * (4 * 128 * TC_BK * 2) + kTmaStageBytes; }
static_assert(tc_smem_pair_bytes() <= 232448, "exceeds the 227 KB of dynamic shared memory per block");
constexpr size_t tc_smem_splitk_bytes() { return 1024 + (size_t)3 * (4 * 128 * TC_BK * 2) + 256; }
static_assert(tc_smem_splitk_bytes() <= 232448, "exceeds the 227 KB of dynamic shared memory per block");

// NEEDLE_NO_SPLITK=1 keeps every GEMM on the persistent kernels (for
// comparisons; results differ only in the order of the K summation).
bool splitk_disabled() {
  static const bool off = [] {
    const char *v = std::getenv("NEEDLE_NO_SPLITK");
    return v && *v && *v != '0';
  }();
  return off;
}

// Cluster size of the split-K kernel for `tiles` 128 x 128 output tiles over
// nkb k-blocks: the largest S in {8, 4, 2} that divides nkb and keeps all
// tiles' clusters resident at once (fits[i]: clusters of size 2 << i the
// device holds at a time); 1 (persistent kernel) when the tiles alone
// fill half the SMs.
int splitk_factor(int tiles, int nkb, int sms, const int fits[3]) {
  if (2 * tiles > sms) return 1;
  for (int i = 2; i >= 0; --i) {
    const int S = 2 << i;
    if (nkb % S == 0 && tiles <= fits[i]) return S;
  }
  return 1;
}

template <int S, int BN>
cudaError_t launch_splitk(const CUtensorMap *ah, const CUtensorMap *al, const CUtensorMap *bh, const CUtensorMap *bl,
                          int M, int N, int Kp, const TcEpi &e, int *err, int b_lo_zero, int tiles, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * S);
  cfg.blockDim = dim3(TC_SPLITK_THREADS);
  cfg.dynamicSmemBytes = tc_smem_splitk_bytes();
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  int na = 1;
  if (pdl_on()) {
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    na = 2;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, tc_gemm_splitk_kernel<S, BN>, *ah, *al, *bh, *bl, M, N, Kp, e, err, b_lo_zero);
}

}  // namespace

int tc_padded_k(int K) { return (K + TC_BK - 1) / TC_BK * TC_BK; }

size_t tc_splitk_ws_bytes() { return (size_t)tc_sm_count() * 128 * 128 * sizeof(float); }

cudaError_t tc_make_planes(const void *hi, const void *lo, int rows, int Kp, int box_rows, TcPlanes &out) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (((uintptr_t)hi & 15) || ((uintptr_t)lo & 15) || (Kp % TC_BK) || rows <= 0) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)Kp * 2};
  cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  cuuint32_t box64[2] = {(cuuint32_t)TC_BK, 64};
  for (int s = 0; s < 4; ++s) {
    unsigned char *m = s == 0 ? out.hi : s == 1 ? out.lo : s == 2 ? out.hi64 : out.lo64;
    CUresult r = fn(reinterpret_cast<CUtensorMap *>(m), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                    const_cast<void *>((s & 1) ? lo : hi), dims, strides, s < 2 ? box : box64, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  out.rows = rows;
  out.Kp = Kp;
  out.box_rows = box_rows;
  out.hi_ptr = hi;
  out.lo_ptr = lo;
  return cudaSuccess;
}

cudaError_t tma_map_f32(const void *base, int64_t rows, int cols, int box_rows, int box_cols, void *map) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (((uintptr_t)base & 15) || rows <= 0 || (cols % 4) || (box_cols % 4) || box_cols > 256 || box_rows > 256)
    return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(reinterpret_cast<CUtensorMap *>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base),
                  dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t tc_prep_weight(const Int4Weight &W, int Kp, void *hi, void *lo, cudaStream_t st) {
  int64_t n = (int64_t)W.N * Kp;
  prep_weight_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(W, Kp, (__nv_bfloat16 *)hi, (__nv_bfloat16 *)lo);
  return cudaGetLastError();
}

cudaError_t tc_split_rows(const float *x, int64_t ldx, int M, int K, int Kp, void *hi, void *lo, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (Kp % 4) return cudaErrorInvalidValue;
  int64_t n = (int64_t)M * Kp / 4;
  split_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, ldx, M, K, Kp, (__nv_bfloat16 *)hi,
                                                                   (__nv_bfloat16 *)lo);
  return cudaGetLastError();
}

namespace {
// TMA map of the f32 output of a store / residual / k-norm epilogue: 32 x 32
// boxes, 128-byte swizzle; 3-D ({col_block, M, N / col_block}) when the
// columns are split into blocks.  False when the layout does not allow one
// (the epilogue then stores per thread).
bool tma_map_out(const MatmulOut &o, int M, int N, CUtensorMap *map) {
  auto fn = encode_fn();
  if (!fn || !o.y || ((uintptr_t)o.y % 16) || (o.ldy % 4) || M <= 0) return false;
  cuuint32_t box[3] = {32, 32, 1}, es[3] = {1, 1, 1};
  CUresult r;
  if (o.col_block) {
    if ((o.col_block % 32) || (N % o.col_block) || (o.block_stride % 4)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)o.col_block, (cuuint64_t)M, (cuuint64_t)(N / o.col_block)};
    cuuint64_t strides[2] = {(cuuint64_t)o.ldy * 4, (cuuint64_t)o.block_stride * 4};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, o.y, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)o.ldy * 4};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, o.y, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r == CUDA_SUCCESS;
}

// TMA maps of the encoder QKV epilogue's six attention planes ({64, M, heads},
// plane stride slab rows); false when the planes' layout does not allow them.
bool tma_maps_qkv(const MatmulOut &o, int M, QkvMaps *qm) {
  auto fn = encode_fn();
  if (!fn || M <= 0 || o.slab < M) return false;
  for (int p = 0; p < 6; ++p) {
    if (!o.planes[p] || ((uintptr_t)o.planes[p] % 16)) return false;
    cuuint64_t dims[3] = {64, (cuuint64_t)M, (cuuint64_t)(p < 2 ? o.heads_q : o.heads_kv)};
    cuuint64_t strides[2] = {128, (cuuint64_t)o.slab * 128};
    cuuint32_t box[3] = {64, 32, 1}, es[3] = {1, 1, 1};
    if (fn(&qm->m[p], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, o.planes[p], dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  return true;
}

}  // namespace

// NEEDLE_NO_TMA_STORE=1 keeps every epilogue on per-thread stores (for
// comparisons; the residual then adds with one fused multiply-add).
bool tma_store_disabled() {
  static const bool off = [] {
    const char *v = std::getenv("NEEDLE_NO_TMA_STORE");
    return v && *v && *v != '0';
  }();
  return off;
}

cudaError_t tc_matmul(const TcPlanes &A, int M, const TcPlanes &B, int N, const MatmulOut &o, int *err,
                      cudaStream_t st, bool b_lo_zero) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (A.Kp != B.Kp || A.box_rows != TC_BM || B.box_rows != 128 || M > A.rows || N > B.rows)
    return cudaErrorInvalidValue;
  if (o.col_block && (o.col_block % 64)) return cudaErrorInvalidValue;
  if (o.epi == EPI_KNORM && (!o.col_block || !o.vec || (o.kv_block && (o.kv_block % o.col_block))))
    return cudaErrorInvalidValue;
  if (o.epi == EPI_ARGMAX) {
    if (!o.keys || !o.pos || (o.mask && o.mask_words * 64 < N)) return cudaErrorInvalidValue;
  } else if (o.epi == EPI_QKV) {
    if (N != (o.heads_q + 2 * o.heads_kv) * 64 || !o.pos || !o.q_norm || !o.k_norm || !o.rope_cos || !o.rope_sin ||
        M > o.slab)
      return cudaErrorInvalidValue;
    for (int i = 0; i < 6; ++i)
      if (!o.planes[i] || ((uintptr_t)o.planes[i] % 16)) return cudaErrorInvalidValue;
  } else if (o.epi == EPI_QKV_DEC) {
    if (N != (o.heads_q + 2 * o.heads_kv) * 64 || !o.pos || !o.q_norm || !o.k_norm || !o.rope_cos || !o.rope_sin ||
        !o.kcache || !o.vcache || o.cache_cap <= 0 || (o.ldy % 4) || ((uintptr_t)o.y % 16) ||
        ((uintptr_t)o.kcache % 16) || ((uintptr_t)o.vcache % 16))
      return cudaErrorInvalidValue;
  } else if (o.epi == EPI_ACT && o.planes[0]) {
    if (!o.planes[1] || ((uintptr_t)o.planes[0] % 16) || ((uintptr_t)o.planes[1] % 16) || (o.ldy % 8) ||
        o.col_block)
      return cudaErrorInvalidValue;
  } else if ((o.ldy % 4) || ((uintptr_t)o.y % 16) || (o.col_block && (o.block_stride % 4))) {
    return cudaErrorInvalidValue;
  }
  if (o.epi == EPI_ACT && (N & 1)) return cudaErrorInvalidValue;
  if (o.in_norm) return cudaErrorInvalidValue;  // input norm: CUDA-core matvec only
  TcEpi e{o, N};
  alignas(64) CUtensorMap ymap;
  std::memset(&ymap, 0, sizeof(ymap));
  const int y_tma = (o.epi == EPI_STORE || o.epi == EPI_RESID || o.epi == EPI_KNORM) && !tma_store_disabled() &&
                            tma_map_out(o, M, N, &ymap)
                        ? 1
                        : 0;
  alignas(64) QkvMaps qmaps;
  std::memset(&qmaps, 0, sizeof(qmaps));
  const int qkv_tma = o.epi == EPI_QKV && !tma_store_disabled() && tma_maps_qkv(o, M, &qmaps) ? 1 : 0;
  // setmaxnreg redistributes exactly the registers of a 168-register launch;
  // any other count would leave the increase waiting for registers that
  // never come, so such a build is refused here.
  static int regs[2] = {-1, -1};
  if (regs[0] < 0) {
    cudaFuncAttributes fa;
    cudaError_t ce = cudaFuncGetAttributes(&fa, tc_gemm_kernel<128, 3>);
    if (ce != cudaSuccess) return ce;
    regs[0] = fa.numRegs;
    ce = cudaFuncGetAttributes(&fa, tc_gemm_kernel<256, 2>);
    if (ce != cudaSuccess) return ce;
    regs[1] = fa.numRegs;
  }
  if (regs[0] != TC_REG_LAUNCH || regs[1] != TC_REG_LAUNCH) return cudaErrorInvalidKernelImage;
  static int pair_regs = -1;
  if (pair_regs < 0) {
    cudaFuncAttributes fa;
    cudaError_t ce = cudaFuncGetAttributes(&fa, tc_gemm_pair_kernel<TC_PAIR_STAGES>);
    if (ce != cudaSuccess) return ce;
    pair_regs = fa.numRegs;
  }
  const int sms = tc_sm_count(), num_m = (M + TC_BM - 1) / TC_BM;
  const auto *ah = reinterpret_cast<const CUtensorMap *>(A.hi), *al = reinterpret_cast<const CUtensorMap *>(A.lo);
  const auto *bh = reinterpret_cast<const CUtensorMap *>(B.hi), *bl = reinterpret_cast<const CUtensorMap *>(B.lo);
  const int tiles256 = num_m * ((N + 255) / 256);
  const int tiles_pair = ((M + 255) / 256) * ((N + 255) / 256);
  // Rounds of the grid: a CTA pair's 256 x 256 tile is twice the MMA work
  // per CTA of a 128 x 128 tile at the same operand bytes per CTA and
  // k-block, so a pair round takes about 1.5 single-CTA rounds.
  const int rounds1 = (num_m * ((N + 127) / 128) + sms - 1) / sms;
  const int rounds_pair = (tiles_pair + sms / 2 - 1) / (sms / 2);
  const bool pair_wins = tiles_pair >= sms || 3 * rounds_pair < 2 * rounds1;
  if (pair_wins && pair_regs == TC_REG_LAUNCH) {
    const int npairs = tiles_pair < sms / 2 ? tiles_pair : sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * npairs);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = tc_smem_pair_bytes();
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm_pair_kernel<TC_PAIR_STAGES>, *ah, *al, *bh, *bl, ymap, qmaps, M, N,
                              A.Kp, e, err, b_lo_zero ? 1 : 0, y_tma, qkv_tma);
  }
  if (tiles256 >= 2 * sms)
    return launch(tc_gemm_kernel<256, 2>, dim3(sms), dim3(TC_THREADS), tc_smem_bytes(256, 2), st, *ah, *al, *bh, *bl,
                  ymap, qmaps, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, y_tma, qkv_tma);
  const int tiles = num_m * ((N + 127) / 128);
  // clusters of 2, 4 and 8 split-K CTAs this device holds at once (0: the
  // split-K kernels are unavailable; both tile widths use the same shared
  // memory, so they fit alike)
  static int fits[64][3];
  static bool probed[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !probed[dev]) {
    const void *fs[3] = {(const void *)tc_gemm_splitk_kernel<2, 128>, (const void *)tc_gemm_splitk_kernel<4, 128>,
                         (const void *)tc_gemm_splitk_kernel<8, 128>};
    for (int i = 0; i < 3; ++i) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 << i);
      cfg.blockDim = dim3(TC_SPLITK_THREADS);
      cfg.dynamicSmemBytes = tc_smem_splitk_bytes();
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2 << i;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      fits[dev][i] = cudaOccupancyMaxActiveClusters(&n, fs[i], &cfg) == cudaSuccess ? n : 0;
    }
    cudaGetLastError();  // a failed query leaves no sticky error
    probed[dev] = true;
  }
  // 128 x 64 tiles when they still leave room for a split (half the partial
  // bytes and 5/8 of the operand bytes per CTA, twice the CTAs), else 128 x 128
  const bool can_split = o.splitk_ws && ((uintptr_t)o.splitk_ws % 16) == 0 && dev >= 0 && dev < 64 &&
                         !splitk_disabled();
  const int nkb = A.Kp / TC_BK, tiles64 = num_m * ((N + 63) / 64);
  int S = 1, bn = 128;
  if (can_split) {
    S = splitk_factor(tiles64, nkb, sms, fits[dev]);
    if (S > 1 && tiles64 * S <= sms) {
      bn = 64;
    } else {
      S = splitk_factor(tiles, nkb, sms, fits[dev]);
      if (tiles * S > sms) S = 1;  // the workspace holds one tile per SM
    }
  }
  if (bn == 64) {
    const auto *bh64 = reinterpret_cast<const CUtensorMap *>(B.hi64), *bl64 = reinterpret_cast<const CUtensorMap *>(B.lo64);
    if (S == 8) return launch_splitk<8, 64>(ah, al, bh64, bl64, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, tiles64, st);
    if (S == 4) return launch_splitk<4, 64>(ah, al, bh64, bl64, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, tiles64, st);
    return launch_splitk<2, 64>(ah, al, bh64, bl64, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, tiles64, st);
  }
  if (S == 8) return launch_splitk<8, 128>(ah, al, bh, bl, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, tiles, st);
  if (S == 4) return launch_splitk<4, 128>(ah, al, bh, bl, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, tiles, st);
  if (S == 2) return launch_splitk<2, 128>(ah, al, bh, bl, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, tiles, st);
  return launch(tc_gemm_kernel<128, 3>, dim3(tiles < sms ? tiles : sms), dim3(TC_THREADS), tc_smem_bytes(128, 3), st,
                *ah, *al, *bh, *bl, ymap, qmaps, M, N, A.Kp, e, err, b_lo_zero ? 1 : 0, y_tma, qkv_tma);
}

cudaError_t init_tc_kernels() {
  cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<128, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)tc_smem_bytes(128, 3));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc_gemm_kernel<256, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)tc_smem_bytes(256, 2));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc_gemm_pair_kernel<TC_PAIR_STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)tc_smem_pair_bytes());
  for (const void *f : {(const void *)tc_gemm_splitk_kernel<2, 128>, (const void *)tc_gemm_splitk_kernel<4, 128>,
                        (const void *)tc_gemm_splitk_kernel<8, 128>, (const void *)tc_gemm_splitk_kernel<2, 64>,
                        (const void *)tc_gemm_splitk_kernel<4, 64>, (const void *)tc_gemm_splitk_kernel<8, 64>})
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_splitk_bytes());
  return e;
}

}  // namespace ndl
