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
// Kernel.  Persistent; a work item is (request, 128-query tile, Q head).
// 320 threads: warp 0 TMA (Q tile once, then K/V tiles of 128 keys through a
// 2-stage ring), warp 1 TMEM allocation + MMA issue, warps 2-9 softmax in two
// warpgroups: thread = one query row and one half (64 keys) of each S tile;
// the halves exchange row maxima through shared memory and split the 64
// output columns.  Per key tile j:
//   S_j = Q K_j^T                       tcgen05.mma M128 N128 K16, A and B
//                                       K-major, f32 in TMEM (2 buffers, so
//                                       S_{j+1} runs during softmax_j)
//   p = exp(S*scale - m) (hardware exp2), online max/sum per row in registers
//   P_j -> TMEM as bf16 hi/lo over its own S buffer (tcgen05.st)
//   O_j = P_j V_j                       M128 N64 K16, A = P from TMEM, V read
//                                       MN-major straight from its [key][dim]
//                                       tile, into one of two O buffers
//   O = O * exp(m_old - m_new) + O_j    in registers, one tile behind, so PV_j
//                                       runs during the softmax of tile j+1
// Each product is the 3-term split hi*hi + hi*lo + lo*hi (about 1e-6
// relative), so the f32 reference is matched within the logit tolerance.
// Keys past the request's end get probability 0; query rows past it are
// computed on neighbouring rows and never stored.  TMA loads never use
// cluster multicast; every wait is bounded (error flag, then unwind).
#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace ndl {
namespace {

using namespace tc;

constexpr int AT_BM = 128, AT_BN = 128, AT_HD = 64, AT_THREADS = 320;
constexpr int AT_TILE = AT_BM * AT_HD * 2;              // one 128 x 64 bf16 plane tile: 16 KB
constexpr int AT_Q = 0;                                  // Q hi, Q lo
constexpr int AT_KV = 2 * AT_TILE;                       // 2 stages x (K hi, K lo, V hi, V lo)
constexpr int AT_STAGE = 4 * AT_TILE;
constexpr int AT_XCH = AT_KV + 2 * AT_STAGE;             // row-max / row-sum exchange [2][128] f32
constexpr int AT_BAR = AT_XCH + 2 * 128 * 4;
constexpr size_t AT_SMEM = 1024 + AT_BAR + 256;
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

// tcgen05.mma kind::f16 with the A operand in TMEM (M lanes, K packed two
// bf16 per 32-bit column) and B from shared memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

// Rendezvous of the 256 softmax threads on an mbarrier (a bounded wait, so a
// warpgroup that unwinds on an error can never strand the other).
__device__ __forceinline__ bool xsync(uint64_t *bar, uint32_t &uses, int *err) {
  mbar_arrive(bar);
  return mbar_wait(bar, (uses++) & 1, err);
}

// Two x32 TMEM loads (64 consecutive columns) with a single wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float *v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr + 32));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    enc_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                       const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                       const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl,
                       const int64_t *__restrict__ seq_off, const int4 *__restrict__ items, int n_items, int slab,
                       float *out, __nv_bfloat16 *out_hi, __nv_bfloat16 *out_lo, int ldp, AttnDims a, int *err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *q_full = (uint64_t *)(sm + AT_BAR);
  uint64_t *q_empty = q_full + 1;
  uint64_t *kv_full = q_full + 2;   // [2]
  uint64_t *kv_empty = q_full + 4;  // [2]
  uint64_t *s_full = q_full + 6;    // [2]
  uint64_t *s_empty = q_full + 8;   // [2]  S/P buffer free (PV of its tile done)
  uint64_t *p_full = q_full + 10;   // [2]  P written over the S buffer
  uint64_t *o_full = q_full + 12;   // [2]
  uint64_t *o_empty = q_full + 14;  // [2]
  uint64_t *xbar = q_full + 16;     // the two softmax warpgroups' exchange rendezvous
  uint32_t *tmem_slot = (uint32_t *)(q_full + 17);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rep = a.H / a.KVH;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 1);
      mbar_init(&p_full[s], 256);
      mbar_init(&o_full[s], 1);
      mbar_init(&o_empty[s], 256);
    }
    mbar_init(xbar, 256);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // S/P: 2 x 128 columns, O: 2 x 64 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *(volatile uint32_t *)tmem_slot;
  const uint32_t t_o = tmem + 256;  // O buffer b at t_o + 64 b

  if (warp == 0) {
    if (lane == 0) {  // ── TMA producer ──
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++it) {
        const int4 item = items[w];
        const int64_t off = seq_off[item.x];
        const int T = (int)(seq_off[item.x + 1] - off);
        const int nk = (T + AT_BN - 1) / AT_BN, g = item.z / rep;
        if (!(ok = mbar_wait(q_empty, (it & 1) ^ 1, err))) break;
        mbar_expect_tx(q_full, 2 * AT_TILE);
        const int qrow = item.z * slab + (int)off + item.y * AT_BM;
        tma_load_2d(sm + AT_Q, &tmQh, q_full, 0, qrow);
        tma_load_2d(sm + AT_Q + AT_TILE, &tmQl, q_full, 0, qrow);
        for (int j = 0; j < nk; ++j) {
          if (!(ok = mbar_wait(&kv_empty[stage], phase ^ 1, err))) break;
          uint8_t *st = sm + AT_KV + stage * AT_STAGE;
          const int krow = g * slab + (int)off + j * AT_BN;
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
    if (lane == 0) {  // ── MMA issuer ──
      constexpr uint32_t ID_S = umma_idesc(AT_BM, AT_BN);
      constexpr uint32_t ID_PV = umma_idesc(AT_BM, AT_HD, true);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t jj = 0, pv = 0;
      int it = 0;
      bool ok = true;
      int pv_stage = 0, pv_sb = 0;
      // O_t = P_t V_t for the tile t whose S/P buffer is `sb` and whose K/V
      // sit in stage `st`; O_t goes to O buffer (pv & 1).
      auto do_pv = [&](int st, int sb) -> bool {
        const int ob = pv & 1;
        if (!mbar_wait(&p_full[sb], (pv >> 1) & 1, err) || !mbar_wait(&o_empty[ob], ((pv >> 1) & 1) ^ 1, err))
          return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint8_t *kvs = sm + AT_KV + st * AT_STAGE;
        const uint32_t d = t_o + (uint32_t)(ob * AT_HD);
        const uint32_t ph = tmem + (uint32_t)(sb * AT_BN), pl = ph + 64;
#pragma unroll
        for (int ks = 0; ks < AT_BN / 16; ++ks) {
          const uint64_t vh = umma_desc_mn(kvs + 2 * AT_TILE + ks * 2048);
          const uint64_t vl = umma_desc_mn(kvs + 3 * AT_TILE + ks * 2048);
          umma_bf16_ts(d, ph + ks * 8, vh, ID_PV, ks ? 1u : 0u);
          umma_bf16_ts(d, ph + ks * 8, vl, ID_PV, 1u);
          umma_bf16_ts(d, pl + ks * 8, vh, ID_PV, 1u);
        }
        umma_commit(&o_full[ob]);
        umma_commit(&s_empty[sb]);   // the S/P buffer may take the tile after next
        umma_commit(&kv_empty[st]);  // S and PV of this tile are done with its K/V
        ++pv;
        return true;
      };
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++it) {
        const int4 item = items[w];
        const int T = (int)(seq_off[item.x + 1] - seq_off[item.x]);
        const int nk = (T + AT_BN - 1) / AT_BN;
        if (!(ok = mbar_wait(q_full, it & 1, err))) break;
        for (int j = 0; j < nk && ok; ++j) {
          const int sb = jj & 1;
          if (!(ok = mbar_wait(&kv_full[stage], phase, err))) break;
          if (!(ok = mbar_wait(&s_empty[sb], ((jj >> 1) & 1) ^ 1, err))) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          uint8_t *kvs = sm + AT_KV + stage * AT_STAGE;
          const uint32_t d = tmem + (uint32_t)(sb * AT_BN);
#pragma unroll
          for (int ks = 0; ks < AT_HD / 16; ++ks) {
            const uint64_t adv = (uint64_t)((ks * 32) >> 4);
            const uint64_t qh = umma_desc(sm + AT_Q) + adv, ql = umma_desc(sm + AT_Q + AT_TILE) + adv;
            const uint64_t kh = umma_desc(kvs) + adv, kl = umma_desc(kvs + AT_TILE) + adv;
            umma_bf16(d, qh, kh, ID_S, ks ? 1u : 0u);
            umma_bf16(d, qh, kl, ID_S, 1u);
            umma_bf16(d, ql, kh, ID_S, 1u);
          }
          umma_commit(&s_full[sb]);
          if (j == nk - 1) umma_commit(q_empty);
          ++jj;
          if (j > 0 && !(ok = do_pv(pv_stage, pv_sb))) break;
          pv_stage = stage;
          pv_sb = sb;
          if (++stage == 2) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) ok = do_pv(pv_stage, pv_sb);
      }
    }
  } else {  // ── softmax: warps 2-9, two warpgroups ──
    const int quarter = warp & 3, wg = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // TMEM lane = query row of the tile
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    float *xch = (float *)(sm + AT_XCH);  // [2 groups][128]: row maxima, then row sums
    uint32_t jj = 0, pv = 0, xu = 0;
    // O += O_t (computed by the MMA with the row maxima of tile t), after
    // rescaling the running sum by corr_t = exp(m_{t-1} - m_t).
    float o[32];
    auto add_o = [&](float corr) -> bool {
      const int ob = pv & 1;
      if (!mbar_wait(&o_full[ob], (pv >> 1) & 1, err)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float v[32];
      tmem_ld32(t_o + lanes + (uint32_t)(ob * AT_HD + wg * 32), v);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&o_empty[ob]);
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = o[e] * corr + v[e];
      ++pv;
      return true;
    };
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      const int4 item = items[w];
      const int64_t off = seq_off[item.x];
      const int T = (int)(seq_off[item.x + 1] - off);
      const int nk = (T + AT_BN - 1) / AT_BN;
      float m = -INFINITY, l = 0.0f, corr_prev = 0.0f;
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = 0.0f;
      bool ok = true;
      for (int j = 0; j < nk; ++j) {
        const int sb = jj & 1;
        if (!(ok = mbar_wait(&s_full[sb], (jj >> 1) & 1, err))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float v[64];
        tmem_ld64(tmem + lanes + (uint32_t)(sb * AT_BN + wg * 64), v);
        const int kvalid = T - j * AT_BN - wg * 64;  // keys of this half that belong to the request
        float mx = -INFINITY;
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          v[e] *= a.scale;
          if (e < kvalid) mx = fmaxf(mx, v[e]);
        }
        xch[wg * 128 + r] = mx;
        // after this rendezvous both halves hold their S in registers, so P
        // may overwrite the S buffer
        if (!(ok = xsync(xbar, xu, err))) break;
        const float m_new = fmaxf(m, fmaxf(mx, xch[(wg ^ 1) * 128 + r]));
        if (!(ok = xsync(xbar, xu, err))) break;  // both halves read before the next write
        const float corr = expf(m - m_new);       // 0 on the first tile (m = -inf)
        // Probabilities with the hardware exp2 intrinsic: __expf's error,
        // 2 + |1.17 x| ulp for x = s - max <= 0, is ~1e-6 relative where p is
        // not negligible, far inside the logit tolerance.
        float psum = 0.0f;
        uint32_t ph[32], pl[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float p0 = (2 * i < kvalid) ? __expf(v[2 * i] - m_new) : 0.0f;
          float p1 = (2 * i + 1 < kvalid) ? __expf(v[2 * i + 1] - m_new) : 0.0f;
          psum += p0 + p1;
          __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
          float2 hf = __bfloat1622float2(h);
          __nv_bfloat162 lo = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
          ph[i] = *reinterpret_cast<uint32_t *>(&h);
          pl[i] = *reinterpret_cast<uint32_t *>(&lo);
        }
        // P over the S buffer: hi plane in columns [0, 64), lo in [64, 128),
        // this half's 64 keys at column offset wg * 32
        const uint32_t tp = tmem + lanes + (uint32_t)(sb * AT_BN + wg * 32);
        tmem_st32(tp, ph);
        tmem_st32(tp + 64, pl);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&p_full[sb]);
        l = l * corr + psum;
        m = m_new;
        ++jj;
        if (j > 0 && !(ok = add_o(corr_prev))) break;  // O of the previous tile
        corr_prev = corr;
      }
      if (!ok || !add_o(corr_prev)) break;
      // combine the two halves' row sums
      xch[wg * 128 + r] = l;
      if (!xsync(xbar, xu, err)) break;
      const float ltot = l + xch[(wg ^ 1) * 128 + r];
      if (!xsync(xbar, xu, err)) break;  // the exchange area is reused by the next item
      const int qr = item.y * AT_BM + r;
      if (qr < T) {
        const float inv = 1.0f / ltot;
        if (out_hi) {  // bf16 hi/lo planes of the O projection's input
          const int64_t base = (off + qr) * (int64_t)ldp + item.z * AT_HD + wg * 32;
          uint32_t hw[16], lw[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0 = o[2 * e] * inv, x1 = o[2 * e + 1] * inv;
            __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
            float2 hf = __bfloat1622float2(h);
            __nv_bfloat162 lo = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
            hw[e] = *reinterpret_cast<uint32_t *>(&h);
            lw[e] = *reinterpret_cast<uint32_t *>(&lo);
          }
          uint4 *dh = reinterpret_cast<uint4 *>(out_hi + base), *dl = reinterpret_cast<uint4 *>(out_lo + base);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            dh[e] = make_uint4(hw[4 * e], hw[4 * e + 1], hw[4 * e + 2], hw[4 * e + 3]);
            dl[e] = make_uint4(lw[4 * e], lw[4 * e + 1], lw[4 * e + 2], lw[4 * e + 3]);
          }
        } else {
          float4 *dst =
              reinterpret_cast<float4 *>(out + (off + qr) * (int64_t)(a.H * AT_HD) + item.z * AT_HD + wg * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dst[e] = make_float4(o[4 * e] * inv, o[4 * e + 1] * inv, o[4 * e + 2] * inv, o[4 * e + 3] * inv);
        }
      }
    }
  }
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
                                 float *out, void *out_hi, void *out_lo, int ldp, AttnDims a, int *err,
                                 cudaStream_t st) {
  if (n_items <= 0) return cudaSuccess;
  if (a.HD != 64 || (a.H % a.KVH)) return cudaErrorInvalidValue;
  if (out_hi && (!out_lo || (ldp % 8) || ((uintptr_t)out_hi % 16) || ((uintptr_t)out_lo % 16)))
    return cudaErrorInvalidValue;
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = n_items < sms ? n_items : sms;
  auto M = [](const unsigned char *m) { return *reinterpret_cast<const CUtensorMap *>(m); };
  enc_attn_tc_kernel<<<grid, AT_THREADS, AT_SMEM, st>>>(M(p.q.hi), M(p.q.lo), M(p.k.hi), M(p.k.lo), M(p.v.hi),
                                                        M(p.v.lo), seq_off, (const int4 *)items, n_items, p.slab, out,
                                                        (__nv_bfloat16 *)out_hi, (__nv_bfloat16 *)out_lo, ldp, a, err);
  return cudaGetLastError();
}

cudaError_t init_tc_attn_kernels() {
  return cudaFuncSetAttribute(enc_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AT_SMEM);
}

}  // namespace ndl
