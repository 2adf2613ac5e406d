// common.cuh — shared device helpers for the needle B200 kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ndl {

// Additive mask value of a blocked vocabulary entry (constrained.rs:93-116).
constexpr float kMaskBlocked = -1e9f;

// f32::total_cmp order (IEEE totalOrder) as an unsigned key.
__device__ __forceinline__ uint32_t total_order_key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Packed argmax key: larger logit wins, then larger index ("last maximal
// index", the result of Iterator::max_by in engine.rs:299-304).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  return ((unsigned long long)total_order_key(v) << 32) | idx;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ int sign_extend4(uint32_t nib) {
  return (int)(nib << 28) >> 28;
}

// Packed pairs of f32 (sm_100 two-lane FMA / add / sub / mul: each lane
// rounds exactly as the scalar instruction).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float &a, float &b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Programmatic dependent launch.  pdl_trigger lets the next kernel of the
// stream start its CTAs; pdl_wait blocks until the previous kernel of the
// stream has completed and its writes are visible.  Both are no-ops in a
// kernel launched without the programmatic-serialization attribute.  A kernel
// launched with it calls pdl_wait before its first global-memory access.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Whether launches from this host thread currently use programmatic
// dependent launch (set_pdl in kernels.h).
bool pdl_on();

// <<<grid, block, smem, st>>> launch, with the programmatic-serialization
// attribute while pdl_on().
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  if (pdl_on()) {
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, k, static_cast<Args &&>(args)...);
}

}  // namespace ndl
