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

}  // namespace ndl
