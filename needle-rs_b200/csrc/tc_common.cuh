// tc_common.cuh — PTX helpers for the tcgen05 / TMA kernels (sm_100a).
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace ndl {
namespace tc {


__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: mbarrier.try_wait already suspends the thread in hardware
// until the phase completes or a short timeout, so it is polled without a
// sleep.  Gives up (sets *err, returns false) after kWaitNs of wall time, or
// as soon as another role of the kernel has given up.
constexpr uint64_t kWaitNs = 4000000000ull;  // 4 s
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, int *err) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 255) == 0) {
      if (*(volatile int *)err) return false;
      if (globaltimer_ns() - t0 > kWaitNs) {
        atomicExch(err, 1);
        return false;
      }
    }
  }
}

// Bounded wait that ignores the error flag: after a wait gave up, lets the
// asynchronous copies already started into this CTA's shared memory land
// before the CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t *b, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; !mbar_try_wait(b, parity); ++i)
    if ((i & 255) == 255 && globaltimer_ns() - t0 > kWaitNs) return;
}

// Bounded wait with one outcome for the whole (converged) warp, so that a
// timeout can never split a warp ahead of a warp-collective tcgen05
// instruction.
__device__ __forceinline__ bool warp_wait(uint64_t *b, uint32_t parity, int *err) {
  return __all_sync(0xffffffffu, mbar_wait(b, parity, err));
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ── TMA stores from shared memory (the output side of the epilogues) ──
// 2-D / 3-D tile store, and the 2-D / 3-D tile reduce-add (global += smem,
// element type of the tensor map), from this CTA's shared memory.  Each
// call joins the thread's current bulk group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared-memory sources of every committed bulk group have been read.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every committed bulk group has completed (its global writes are done).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ── CTA pairs (a cluster of two CTAs sharing one tcgen05.mma.cta_group::2) ──
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared-memory address of the same variable in CTA 0 of the pair (the
// address bit that selects the peer cleared).
__device__ __forceinline__ uint32_t pair_leader_addr(const void *p) { return smem_u32(p) & 0xFEFFFFFFu; }
// TMA 2-D load into this CTA's own shared memory whose completed bytes are
// counted on the pair leader's mbarrier.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t leader_bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
// Arrive on the mbarrier at the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t *b, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(b)), "r"(rank));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

// UMMA shared-memory descriptor: K-major operand, 128-byte swizzle, 8-row
// atoms of 1024 bytes stacked along M/N (SBO = 1024 B), version 1 (sm100).
__device__ __forceinline__ uint64_t umma_desc(const void *smem) {
  uint64_t addr = smem_u32(smem);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;          // start address
  d |= (uint64_t)1 << 16;                // LBO (ignored for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;      // SBO
  d |= (uint64_t)1 << 46;                // version
  d |= (uint64_t)2 << 61;                // SWIZZLE_128B
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 x bf16 -> f32, A
// K-major, B K-major (or MN-major when b_mn), shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N, bool b_mn = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// UMMA descriptor of an MN-major operand with 128-byte swizzle whose MN
// extent is one 64-element atom: rows of 128 bytes = 64 bf16 along MN, one
// row per K index, 8-row (8 K) groups of 1024 bytes (SBO).
// lbo: byte stride between consecutive 64-element MN atoms when the operand
// spans more than one (N = 128 reads the atom at smem + lbo as elements
// 64..127).
__device__ __forceinline__ uint64_t umma_desc_mn(const void *smem, uint32_t lbo = 16) {
  uint64_t addr = smem_u32(smem);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;                 // start address
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;  // LBO: stride between 64-element MN atoms
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO: stride between 8-row K groups
  d |= (uint64_t)1 << 46;            // version
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

// tcgen05.mma issued by the pair leader over both CTAs: A rows and B columns
// split between the CTAs' shared memory at the same offsets, D split by rows
// between their TMEM.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                               uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Arrive on the mbarrier at this offset in both CTAs of the pair once the
// pair's earlier MMAs complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

// The same MMAs and commits issued by the one lane that elect.sync picks from
// a converged warp.  The whole warp runs the issue loop, so descriptors and
// TMEM addresses are warp-uniform values.  Measured on B200: loops issuing
// M128 N128 MMAs from a single-lane branch kept the tensor pipe 0.5-0.7
// busy, the same loops issued warp-wide 0.9-1.0.
__device__ __forceinline__ void umma_bf16_e(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// A operand in TMEM (M lanes, K packed two bf16 per 32-bit column).
__device__ __forceinline__ void umma_bf16_ts_e(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                               uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_bf16_pair_e(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                                 uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit_e(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair_e(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}


}  // namespace tc
}  // namespace ndl
