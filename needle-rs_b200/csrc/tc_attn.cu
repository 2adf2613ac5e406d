// tc_attn.cu — encoder self-attention on the tcgen05 tensor cores.
//
// Reference: self_attn_full (crates/needle-core/src/attn.rs:189-273): per
// token and Q head, scores = (q . k) * hd^-0.5 over every key of the request
// (bidirectional, GQA: Q head h reads KV head h / (H / KVH)), softmax, P V.
//
// Layout.  qkv_post_kernel turns the f32 output of the fused QKV projection
// into per-head bf16 planes with the ZCRMSNorm + RoPE of attn.rs:218-235
// applied in f32 first: Q [H][rows][64], K and V [KVH][rows][64], each as a
// hi/lo pair (hi = bf16(v), lo = bf16(v - hi)).
//
// Kernel.  Persistent.  A work item is two (Q head, 128-query tile) slots
// of one request that read the same KV head (the GQA heads of a KV head), so
// each K/V tile is loaded once for both.  384 threads in three warpgroups:
// warp 0 issues the TMA loads (the item's Q tiles, then K/V tiles of 128
// keys through a 2-stage ring), warp 1 allocates TMEM and issues the MMAs
// (the whole warp runs the issue loop and one elected lane issues each
// tcgen05 instruction; warps 2-3 idle), and warpgroups 1 / 2 run the
// softmax of slot a / slot b (thread = one query row, all 128 keys of a tile
// held in registers; the producer warpgroup hands its registers to them with
// setmaxnreg).  TMEM: S_a and S_b (128 columns each; P is written back over
// its own S), O_a and O_b (128 columns each).  Per key tile j and slot x:
//   S_x = Q_x K_j^T      tcgen05.mma M128 N128 K16, A and B K-major in smem
//   p = 2^(s*c - m)      c = hd^-0.5 * log2(e); m is raised only when a row's
//                        maximum passes it by more than 8, so p <= 256; p and
//                        the row sum share m, so their quotient is the
//                        reference's exp(s - max) / sum
//   P_x -> TMEM          bf16 hi/lo over S_x (tcgen05.st): keys 32c..32c+31
//                        in columns 32c..32c+15 (hi) and 32c+16..32c+31 (lo),
//                        the columns their own S values came from
//   O_x (+)= P_x V_j     A = P from TMEM, V read MN-major from its [key][dim]
//                        tiles: per 16 keys one M128 N128 K16 MMA of P_hi
//                        against [V_hi | V_lo] (the two planes as one
//                        128-wide operand) and one M128 N64 K16 MMA of P_lo
//                        against V_hi; O_x holds P V_hi + P_lo V_hi in its
//                        first 64 columns and P_hi V_lo in the next 64, summed
//                        when the row is written out.  O stays in TMEM and the
//                        softmax warps rescale it there when m moves
// The MMA warp issues S_a(0), S_b(0), then per tile PV_a(j), S_a(j+1),
// PV_b(j), S_b(j+1): while one slot's warps run the softmax, the tensor core
// works on the other slot.  Each product is the 3-term split hi*hi + hi*lo +
// lo*hi (about 1e-6 relative), so the f32 reference is matched within the
// logit tolerance.  Keys past the request's end get probability 0; query
// rows past it are computed on neighbouring rows and never stored.  Every TMA
// load fills only its own CTA's shared memory; every wait is bounded (error
// flag, then unwind).
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace ndl {
namespace {

using namespace tc;

constexpr int AT_BM = 128, AT_BN = 128, AT_HD = 64, AT_THREADS = 384;
// Registers a thread: launched at 168 (65,536 / 384, rounded down to 8),
// then the producer warpgroup drops to 56 and the two softmax warpgroups
// rise to 224: 128 x 56 + 256 x 224 = 384 x 168 = 64,512.
constexpr int AT_REG_LAUNCH = 168, AT_REG_PRODUCER = 56, AT_REG_SOFTMAX = 224;
static_assert(128 * AT_REG_PRODUCER + 256 * AT_REG_SOFTMAX == AT_THREADS * AT_REG_LAUNCH,
              "the register split must add up to the launch's registers");
constexpr int AT_TILE = AT_BM * AT_HD * 2;  // one 128 x 64 bf16 plane tile: 16 KB
constexpr int AT_Q = 0;                      // slot a hi, lo; slot b hi, lo
constexpr int AT_KV = 4 * AT_TILE;           // 2 stages x (K hi, K lo, V hi, V lo)
constexpr int AT_STAGE = 4 * AT_TILE;
constexpr int AT_STG = AT_KV + 2 * AT_STAGE;  // 8 x 4 KB output staging, one per softmax warp
constexpr int AT_BAR = AT_STG + 8 * 4096;
constexpr size_t AT_SMEM = 1024 + AT_BAR + 256;
constexpr float AT_RESCALE = 8.0f;  // log2 headroom before a row's reference point m is raised
static_assert(AT_SMEM <= 232448, "exceeds the 227 KB of dynamic shared memory per block");

__device__ __forceinline__ void norm_rope64(float &x0, float &x1, const float *__restrict__ nsc,
                                            const float *__restrict__ cr, const float *__restrict__ sr, bool rope,
                                            int lane) {
  // ZCRMSNorm over a 64-wide head held as (lane, lane + 32) pairs, then the
  // split-half rotation (norm.rs:23-30, rope.rs:63-75).
  float ss = x0 * x0 + x1 * x1;
  ss = warp_sum(ss);
  float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
  float a = ((1.0f + __ldg(nsc + lane)) * x0) * inv;
  float b = ((1.0f + __ldg(nsc + lane + 32)) * x1) * inv;
  if (rope) {
    float c = __ldg(cr + lane), s = __ldg(sr + lane);
    float l = a * c - b * s;
    float r = b * c + a * s;
    a = l;
    b = r;
  }
  x0 = a;
  x1 = b;
}

__device__ __forceinline__ void split_store(__nv_bfloat16 *hi, __nv_bfloat16 *lo, int64_t i, float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  hi[i] = h;
  lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
}

// One warp per (row, head) over the H + 2*KVH heads of a fused QKV row.
__global__ void qkv_post_kernel(const float *__restrict__ qkv, int rows, int slab, const int32_t *__restrict__ pos,
                                const float *__restrict__ qn, const float *__restrict__ kn,
                                const float *__restrict__ rc, const float *__restrict__ rs, AttnDims a,
                                __nv_bfloat16 *qh, __nv_bfloat16 *ql, __nv_bfloat16 *kh, __nv_bfloat16 *kl,
                                __nv_bfloat16 *vh, __nv_bfloat16 *vl) {
  const int heads = a.H + 2 * a.KVH;
  int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= (int64_t)rows * heads) return;
  const int lane = threadIdx.x & 31;
  const int row = (int)(w / heads), h = (int)(w % heads);
  const float *src = qkv + (int64_t)row * heads * AT_HD + h * AT_HD;
  float x0 = src[lane], x1 = src[lane + 32];
  const int p = pos[row];
  const float *cr = rc + (int64_t)p * 32, *sr = rs + (int64_t)p * 32;
  __nv_bfloat16 *dh, *dl;
  int64_t base;
  if (h < a.H) {
    norm_rope64(x0, x1, qn, cr, sr, true, lane);
    dh = qh;
    dl = ql;
    base = ((int64_t)h * slab + row) * AT_HD;
  } else if (h < a.H + a.KVH) {
    norm_rope64(x0, x1, kn, cr, sr, true, lane);
    dh = kh;
    dl = kl;
    base = ((int64_t)(h - a.H) * slab + row) * AT_HD;
  } else {
    dh = vh;
    dl = vl;
    base = ((int64_t)(h - a.H - a.KVH) * slab + row) * AT_HD;
  }
  split_store(dh, dl, base + lane, x0);
  split_store(dh, dl, base + lane + 32, x1);
}

// 32 x 32-bit columns of this thread's TMEM lane (tcgen05.st 32x32b.x32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 32 x 32-bit TMEM columns of this thread's lane into r (no wait).
__device__ __forceinline__ void tmem_ld32_raw(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 16 x 32-bit TMEM columns of this thread's lane (tcgen05.st 32x32b.x16).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 2^x with the approximate base-2 exponential instruction of the PTX ISA
// (a few ulp; subnormal results flush to zero, p < 2^-126 contributes
// nothing at f32 precision).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// f2pack / ffma2 / fadd2 / fsub2 / fmul2: packed f32 pairs (common.cuh).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// bf16 hi/lo split of two probabilities, packed as two bf16 per word (the
// lower key in the low half, as the TS-form MMA reads K).
__device__ __forceinline__ void split2(float p0, float p1, uint32_t &hi, uint32_t &lo) {
  __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
  float2 hf = __bfloat1622float2(h);
  __nv_bfloat162 l2 = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
  hi = *reinterpret_cast<uint32_t *>(&h);
  lo = *reinterpret_cast<uint32_t *>(&l2);
}

// P = 2^(s*c - m) for this thread's row of a 128-key tile held in sr,
// written over the row's S columns 32 keys at a time (hi in a chunk's first
// 16 columns, lo in the last 16), for the first nch chunks.  Returns the row
// sum.  MASK: keys at kvalid and beyond get probability 0.
template <bool MASK>
__device__ __forceinline__ float p_row(const uint32_t *sr, float c, float m, int kvalid, int nch, uint32_t tS) {
  // even and odd keys summed in the two lanes of ps, in key order
  uint64_t ps = f2pack(0.0f, 0.0f);
  const uint64_t cc = f2pack(c, c), nm = f2pack(-m, -m);
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    if (ch >= nch) break;  // keys the PV MMAs of this tile do not read
    uint32_t hw[16], lw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int k0 = ch * 32 + 2 * i;
      float t0, t1;
      f2unpack(ffma2(f2pack(__uint_as_float(sr[k0]), __uint_as_float(sr[k0 + 1])), cc, nm), t0, t1);
      float p0 = ex2(t0), p1 = ex2(t1);
      if (MASK) {
        p0 = k0 < kvalid ? p0 : 0.0f;
        p1 = k0 + 1 < kvalid ? p1 : 0.0f;
      }
      const uint64_t p2 = f2pack(p0, p1);
      ps = fadd2(ps, p2);
      const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
      const uint32_t hb = *reinterpret_cast<const uint32_t *>(&h);
      float l0, l1;
      f2unpack(fsub2(p2, f2pack(__uint_as_float(hb << 16), __uint_as_float(hb & 0xffff0000u))), l0, l1);
      const __nv_bfloat162 lb = __floats2bfloat162_rn(l0, l1);
      hw[i] = hb;
      lw[i] = *reinterpret_cast<const uint32_t *>(&lb);
    }
    tmem_st16(tS + 32 * ch, hw);
    tmem_st16(tS + 32 * ch + 16, lw);
  }
  float s0, s1;
  f2unpack(ps, s0, s1);
  return s0 + s1;
}

struct AttnItem {
  int req, qt[2], head[2], g;
  bool two;
};
__device__ __forceinline__ AttnItem decode_item(int4 v) {
  AttnItem it;
  it.req = v.x;
  it.qt[0] = v.y & 0xFFFF;
  it.qt[1] = (int)((unsigned)v.y >> 16);
  it.head[0] = v.z & 0xFFFF;
  it.head[1] = (int)((unsigned)v.z >> 16);
  it.g = v.w;
  it.two = it.head[1] != 0xFFFF;
  return it;
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    enc_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                       const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                       const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl,
                       const __grid_constant__ CUtensorMap tmOh, const __grid_constant__ CUtensorMap tmOl,
                       const int64_t *__restrict__ seq_off, const int4 *__restrict__ items, int n_items, int slab,
                       float *out, __nv_bfloat16 *out_hi, __nv_bfloat16 *out_lo, int ldp, int o_tma, AttnDims a,
                       int *err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = (uint64_t *)(sm + AT_BAR);
  uint64_t *q_full = bars, *q_empty = bars + 1;
  uint64_t *kv_full = bars + 2;   // [stage]
  uint64_t *kv_empty = bars + 4;  // [stage]
  uint64_t *s_full = bars + 6;    // [slot] S_x computed
  uint64_t *p_full = bars + 8;    // [slot] P_x written and O_x rescaled (128 arrivals)
  uint64_t *pv_done = bars + 10;  // [slot] PV_x complete: S_x may be overwritten
  uint64_t *o_done = bars + 12;   // [slot] the item's last PV_x complete
  uint64_t *o_free = bars + 14;   // [slot] O_x read by the epilogue (128 arrivals)
  uint32_t *tmem_slot = (uint32_t *)(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
      mbar_init(&pv_done[s], 1);
      mbar_init(&o_done[s], 1);
      mbar_init(&o_free[s], 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // S_a, S_b: 2 x 128 columns; O_a, O_b: 2 x 128 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *(volatile uint32_t *)tmem_slot;
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(AT_REG_PRODUCER));
    if (warp == 0) {
      if (lane == 0) {  // ── TMA producer ──
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++it) {
          const AttnItem item = decode_item(items[w]);
          const int64_t off = seq_off[item.req];
          const int T = (int)(seq_off[item.req + 1] - off);
          const int nk = (T + AT_BN - 1) / AT_BN;
          if (!(ok = mbar_wait(q_empty, (it & 1) ^ 1, err))) break;
          mbar_expect_tx(q_full, (item.two ? 4 : 2) * AT_TILE);
          for (int x = 0; x < (item.two ? 2 : 1); ++x) {
            const int qrow = item.head[x] * slab + (int)off + item.qt[x] * AT_BM;
            tma_load_2d(sm + AT_Q + 2 * x * AT_TILE, &tmQh, q_full, 0, qrow);
            tma_load_2d(sm + AT_Q + (2 * x + 1) * AT_TILE, &tmQl, q_full, 0, qrow);
          }
          for (int j = 0; j < nk; ++j) {
            if (!(ok = mbar_wait(&kv_empty[stage], phase ^ 1, err))) break;
            uint8_t *st = sm + AT_KV + stage * AT_STAGE;
            const int krow = item.g * slab + (int)off + j * AT_BN;
            mbar_expect_tx(&kv_full[stage], AT_STAGE);
            tma_load_2d(st, &tmKh, &kv_full[stage], 0, krow);
            tma_load_2d(st + AT_TILE, &tmKl, &kv_full[stage], 0, krow);
            tma_load_2d(st + 2 * AT_TILE, &tmVh, &kv_full[stage], 0, krow);
            tma_load_2d(st + 3 * AT_TILE, &tmVl, &kv_full[stage], 0, krow);
            if (++stage == 2) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        // drain: every issued copy consumed before the CTA exits
        for (int s = 0; s < 2 && ok; ++s) {
          ok = mbar_wait(&kv_empty[stage], phase ^ 1, err);
          if (++stage == 2) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) mbar_wait(q_empty, (it & 1) ^ 1, err);
      }
    } else if (warp == 1) {
      {  // ── MMA issuer: the whole warp runs the loop, one elected lane issues ──
        constexpr uint32_t ID_PV2 = umma_idesc(AT_BM, 2 * AT_HD, true);  // P_hi x [V_hi | V_lo]
        constexpr uint32_t ID_PV = umma_idesc(AT_BM, AT_HD, true);       // P_lo x V_hi
        // per-slot phase counters (scalars: x is 0 or 1)
        uint32_t pv_issued0 = 0, pv_issued1 = 0, pv_waited0 = 0, pv_waited1 = 0, p_seen0 = 0, p_seen1 = 0;
        uint32_t items0 = 0, items1 = 0;
        // Operand descriptors from one base.  Every operand here has the
        // same high word (SBO 1024 bytes, version, 128-byte swizzle); the
        // low word is the start address >> 4 plus the LBO field.  A K step
        // adds 32 bytes (2) to a K-major start address and 16 rows of 128
        // bytes (128) to an MN-major one.
        const uint32_t s16 = smem_u32(sm) >> 4;
        const uint64_t dhi = umma_desc(sm) & 0xFFFFFFFF00000000ull;
        auto kmaj = [&](uint32_t a16) { return dhi | (uint64_t)(a16 | (1u << 16)); };
        auto mnmaj = [&](uint32_t a16, uint32_t lbo16) { return dhi | (uint64_t)(a16 | (lbo16 << 16)); };
        // S_x = Q_x K^T from stage st, once the slot's previous PV (which reads
        // P over S_x) has completed.
        auto issue_s = [&](int x, int st, int ns) -> bool {
          const uint32_t waited = x ? pv_waited1 : pv_waited0;
          if ((x ? pv_issued1 : pv_issued0) > waited) {
            if (!warp_wait(&pv_done[x], waited & 1, err)) return false;
            if (x) ++pv_waited1; else ++pv_waited0;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t qh = s16 + (uint32_t)((AT_Q + 2 * x * AT_TILE) >> 4), ql = qh + (AT_TILE >> 4);
          const uint32_t kh = s16 + (uint32_t)((AT_KV + st * AT_STAGE) >> 4), kl = kh + (AT_TILE >> 4);
          const uint32_t d = tmem + (uint32_t)(x * AT_BN);
          const uint32_t id_s = umma_idesc(AT_BM, ns);  // the tile's first ns keys (a multiple of 16)
#pragma unroll 1
          for (int ks = 0; ks < AT_HD / 16; ++ks) {
            umma_bf16_e(d, kmaj(qh + 2 * ks), kmaj(kh + 2 * ks), id_s, ks ? 1u : 0u);
            umma_bf16_e(d, kmaj(qh + 2 * ks), kmaj(kl + 2 * ks), id_s, 1u);
            umma_bf16_e(d, kmaj(ql + 2 * ks), kmaj(kh + 2 * ks), id_s, 1u);
          }
          umma_commit_e(&s_full[x]);
          return true;
        };
        // O_x (+)= P_x V from stage st, once the softmax has written P_x (and,
        // on an item's first tile, the previous item's O_x has been read out).
        auto issue_pv = [&](int x, int st, int j, bool last, int nks) -> bool {
          const uint32_t seen = x ? p_seen1 : p_seen0;
          if (!warp_wait(&p_full[x], seen & 1, err)) return false;
          if (x) ++p_seen1; else ++p_seen0;
          const uint32_t items = x ? items1 : items0;
          if (j == 0 && items > 0 && !warp_wait(&o_free[x], (items - 1) & 1, err)) return false;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          // V_lo sits one plane tile (AT_TILE bytes) after V_hi: the second MN atom
          const uint32_t v16 = s16 + (uint32_t)((AT_KV + st * AT_STAGE + 2 * AT_TILE) >> 4);
          const uint32_t d = tmem + 256u + (uint32_t)(x * 2 * AT_HD);
          const uint32_t pbase = tmem + (uint32_t)(x * AT_BN);
          const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll 1
          for (int ks = 0; ks < nks; ++ks) {
            // keys 16ks..16ks+15: chunk ks/2, hi at 32(ks/2) + 8(ks%2), lo 16 columns on
            const uint32_t ph = pbase + 32u * (ks >> 1) + 8u * (ks & 1), pl = ph + 16u;
            umma_bf16_ts_e(d, ph, mnmaj(v16 + 128 * ks, AT_TILE >> 4), ID_PV2, ks ? 1u : acc0);
            umma_bf16_ts_e(d, pl, mnmaj(v16 + 128 * ks, 1), ID_PV, 1u);
          }
          umma_commit_e(&pv_done[x]);
          if (x) ++pv_issued1; else ++pv_issued0;
          if (last) umma_commit_e(&o_done[x]);
          return true;
        };
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++it) {
          const AttnItem item = decode_item(items[w]);
          const int T = (int)(seq_off[item.req + 1] - seq_off[item.req]);
          const int nk = (T + AT_BN - 1) / AT_BN;
          // keys of tile j that belong to the request, as S columns (a
          // multiple of 16) and as 16-key PV steps
          auto tile_ns = [&](int j) { return min(AT_BN, (T - j * AT_BN + 15) & ~15); };
          if (!(ok = warp_wait(q_full, it & 1, err))) break;
          if (!(ok = warp_wait(&kv_full[stage], phase, err))) break;
          if (!(ok = issue_s(0, stage, tile_ns(0)))) break;
          if (item.two && !(ok = issue_s(1, stage, tile_ns(0)))) break;
          if (nk == 1) umma_commit_e(q_empty);  // every S of the item issued
          for (int j = 0; j < nk && ok; ++j) {
            const int cur = stage;
            const int nxt = stage ^ 1;
            const uint32_t nph = stage == 1 ? phase ^ 1 : phase;
            const bool more = j + 1 < nk, last = j + 1 == nk;
            const int nks = tile_ns(j) >> 4, ns1 = more ? tile_ns(j + 1) : 0;
            if (!(ok = issue_pv(0, cur, j, last, nks))) break;
            if (more) {
              if (!(ok = warp_wait(&kv_full[nxt], nph, err))) break;
              if (!(ok = issue_s(0, nxt, ns1))) break;
            }
            if (item.two) {
              if (!(ok = issue_pv(1, cur, j, last, nks))) break;
              if (more && !(ok = issue_s(1, nxt, ns1))) break;
            }
            if (j + 2 == nk) umma_commit_e(q_empty);
            umma_commit_e(&kv_empty[cur]);  // every S and PV reading K_j / V_j issued before this commit
            stage = nxt;
            phase = nph;
          }
          if (ok) {
            ++items0;
            if (item.two) ++items1;
          }
        }
      }
    }
  } else {  // ── softmax: warps 4-7 slot a, warps 8-11 slot b ──
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(AT_REG_SOFTMAX));
    const int quarter = warp & 3, x = (warp - 4) >> 2;
    const int r = quarter * 32 + lane;  // TMEM lane = query row of the tile
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lanes + (uint32_t)(x * AT_BN), tO = tmem + lanes + 256u + (uint32_t)(x * 2 * AT_HD);
    const float c = a.scale * 1.4426950408889634f;  // hd^-0.5 * log2(e)
    uint32_t s_seen = 0, o_seen = 0;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      const AttnItem item = decode_item(items[w]);
      if (x == 1 && !item.two) continue;
      const int64_t off = seq_off[item.req];
      const int T = (int)(seq_off[item.req + 1] - off);
      const int nk = (T + AT_BN - 1) / AT_BN;
      float m = -INFINITY, l = 0.0f;
      bool ok = true;
      for (int j = 0; j < nk; ++j) {
        if (!(ok = warp_wait(&s_full[x], s_seen & 1, err))) break;
        ++s_seen;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int kvalid = T - j * AT_BN;  // keys of this tile that belong to the request (>= 1)
        // 32-key chunks the PV MMAs read (warp-uniform).  All 128 columns
        // are loaded: those past the S MMA's columns hold stale values that
        // the mask excludes.
        const int nch = kvalid >= AT_BN ? 4 : (kvalid + 31) >> 5;
        uint32_t sr[128];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32_raw(tS + 32 * q, sr + 32 * q);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (kvalid >= AT_BN) {
#pragma unroll
          for (int e = 0; e < 128; e += 2)
            mx[(e >> 1) & 3] = fmax3(mx[(e >> 1) & 3], __uint_as_float(sr[e]), __uint_as_float(sr[e + 1]));
        } else {
#pragma unroll
          for (int e = 0; e < 128; ++e)
            if (e < kvalid) mx[e & 3] = fmaxf(mx[e & 3], __uint_as_float(sr[e]));
        }
        const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * c;
        float corr = 1.0f;
        const bool resc = j == 0 || mt > m + AT_RESCALE;
        if (resc) {
          corr = ex2(m - mt);  // 0 on the first tile (m = -inf)
          m = mt;
        }
        const float psum =
            kvalid >= AT_BN ? p_row<false>(sr, c, m, kvalid, 4, tS) : p_row<true>(sr, c, m, kvalid, nch, tS);
        l = l * corr + psum;
        // O_x *= corr (PV_x(j-1) completed before S_x(j) was issued).  The
        // tcgen05 loads and stores are warp-collective, so the whole warp
        // takes this branch when any of its rows moved m (corr = 1 elsewhere).
        if (__any_sync(0xffffffffu, resc && j > 0)) {
          uint32_t ov[128];
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_ld32_raw(tO + 32 * q, ov + 32 * q);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          const uint64_t cr2 = f2pack(corr, corr);
#pragma unroll
          for (int e = 0; e < 128; e += 2) {
            float a0, a1;
            f2unpack(fmul2(f2pack(__uint_as_float(ov[e]), __uint_as_float(ov[e + 1])), cr2), a0, a1);
            ov[e] = __float_as_uint(a0);
            ov[e + 1] = __float_as_uint(a1);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_st32(tO + 32 * q, ov + 32 * q);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&p_full[x]);
      }
      if (!ok) break;
      if (!warp_wait(&o_done[x], o_seen & 1, err)) break;  // the item's last PV_x
      ++o_seen;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t ov[128];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld32_raw(tO + 32 * q, ov + 32 * q);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&o_free[x]);  // O_x may take the next item's PV
#pragma unroll
      for (int e = 0; e < 64; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) + __uint_as_float(ov[64 + e]));
      const int qt = x ? item.qt[1] : item.qt[0], head = x ? item.head[1] : item.head[0];
      const int qr = qt * AT_BM + r;
      const int row0 = qt * AT_BM + quarter * 32;  // the warp's first query row
      if (o_tma && row0 + 32 <= T) {
        // all 32 rows of the warp belong to the request: the hi and lo
        // planes leave as two 32-row x 64-column TMA boxes, staged in the
        // warp's 4 KB buffer with the 128-byte swizzle (16-byte chunk j of
        // row r at r * 128 + ((j ^ (r & 7)) << 4))
        const float inv = 1.0f / l;
        uint8_t *stg = sm + AT_STG + (warp - 4) * 4096, *srow = stg + lane * 128;
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          if (lane == 0) bulk_wait_read_all();  // the warp's previous box has left stg
          __syncwarp();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              split2(__uint_as_float(ov[8 * e + 2 * q]) * inv, __uint_as_float(ov[8 * e + 2 * q + 1]) * inv, hw[q],
                     lw[q]);
            *reinterpret_cast<uint4 *>(srow + ((e ^ (lane & 7)) << 4)) =
                part ? make_uint4(lw[0], lw[1], lw[2], lw[3]) : make_uint4(hw[0], hw[1], hw[2], hw[3]);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(part ? &tmOl : &tmOh, stg, head * AT_HD, (int)off + row0);
            bulk_commit();
          }
        }
      } else if (qr < T) {
        const float inv = 1.0f / l;
        if (out_hi) {  // bf16 hi/lo planes of the O projection's input
          const int64_t base = (off + qr) * (int64_t)ldp + head * AT_HD;
          uint4 *dh = reinterpret_cast<uint4 *>(out_hi + base), *dl = reinterpret_cast<uint4 *>(out_lo + base);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              split2(__uint_as_float(ov[8 * e + 2 * q]) * inv, __uint_as_float(ov[8 * e + 2 * q + 1]) * inv, hw[q],
                     lw[q]);
            dh[e] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            dl[e] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
        } else {
          float4 *dst = reinterpret_cast<float4 *>(out + (off + qr) * (int64_t)(a.H * AT_HD) + head * AT_HD);
#pragma unroll
          for (int e = 0; e < 16; ++e)
            dst[e] = make_float4(__uint_as_float(ov[4 * e]) * inv, __uint_as_float(ov[4 * e + 1]) * inv,
                                 __uint_as_float(ov[4 * e + 2]) * inv, __uint_as_float(ov[4 * e + 3]) * inv);
        }
      }
    }
  }
  if (warp >= 4 && o_tma && lane == 0) bulk_wait_all();  // this warp's output boxes written
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

}  // namespace

cudaError_t attn_planes_make(void *const bufs[6], int H, int KVH, int slab, AttnPlanes &p) {
  p.slab = slab;
  for (int i = 0; i < 6; ++i) p.buf[i] = bufs[i];
  cudaError_t e = tc_make_planes(bufs[0], bufs[1], H * slab, 64, 128, p.q);
  if (e == cudaSuccess) e = tc_make_planes(bufs[2], bufs[3], KVH * slab, 64, 128, p.k);
  if (e == cudaSuccess) e = tc_make_planes(bufs[4], bufs[5], KVH * slab, 64, 128, p.v);
  return e;
}

cudaError_t qkv_post(const float *qkv, int rows, const int32_t *pos, const float *q_norm, const float *k_norm,
                     const float *rope_cos, const float *rope_sin, AttnDims a, const AttnPlanes &p, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (a.HD != 64 || rows > p.slab) return cudaErrorInvalidValue;
  int64_t threads = (int64_t)rows * (a.H + 2 * a.KVH) * 32;
  auto B = [&](int i) { return (__nv_bfloat16 *)p.buf[i]; };
  qkv_post_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(qkv, rows, p.slab, pos, q_norm, k_norm, rope_cos,
                                                                       rope_sin, a, B(0), B(1), B(2), B(3), B(4),
                                                                       B(5));
  return cudaGetLastError();
}

cudaError_t encoder_attention_tc(const AttnPlanes &p, const int64_t *seq_off, const void *items, int n_items,
                                 float *out, void *out_hi, void *out_lo, int ldp, int out_rows, AttnDims a, int *err,
                                 cudaStream_t st) {
  if (n_items <= 0) return cudaSuccess;
  if (a.HD != 64 || (a.H % a.KVH)) return cudaErrorInvalidValue;
  if (out_hi && (!out_lo || (ldp % 8) || ((uintptr_t)out_hi % 16) || ((uintptr_t)out_lo % 16)))
    return cudaErrorInvalidValue;
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = n_items < sms ? n_items : sms;
  // setmaxnreg redistributes exactly the registers of a 168-register launch;
  // any other count would leave the increase waiting for registers that
  // never come, so such a build is refused here.
  static int regs = -1;
  if (regs < 0) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, enc_attn_tc_kernel);
    if (e != cudaSuccess) return e;
    regs = fa.numRegs;
  }
  if (regs != AT_REG_LAUNCH) return cudaErrorInvalidKernelImage;
  // output planes as TMA boxes of 32 rows x 64 columns, when they allow it
  alignas(64) TcPlanes om;
  std::memset(om.hi, 0, sizeof(om.hi));
  std::memset(om.lo, 0, sizeof(om.lo));
  const int o_tma = out_hi && out_rows > 0 && (ldp % 64) == 0 && !tma_store_disabled() &&
                            tc_make_planes(out_hi, out_lo, out_rows, ldp, 32, om) == cudaSuccess
                        ? 1
                        : 0;
  auto M = [](const unsigned char *m) { return *reinterpret_cast<const CUtensorMap *>(m); };
  enc_attn_tc_kernel<<<grid, AT_THREADS, AT_SMEM, st>>>(
      M(p.q.hi), M(p.q.lo), M(p.k.hi), M(p.k.lo), M(p.v.hi), M(p.v.lo), M(om.hi), M(om.lo), seq_off,
      (const int4 *)items, n_items, p.slab, out, (__nv_bfloat16 *)out_hi, (__nv_bfloat16 *)out_lo, ldp, o_tma, a, err);
  return cudaGetLastError();
}

cudaError_t init_tc_attn_kernels() {
  return cudaFuncSetAttribute(enc_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AT_SMEM);
}

}  // namespace ndl
