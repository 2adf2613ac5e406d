// ffn_noalloc.cu — the gated MLP block without any device allocation.
//
// needle_ffn_forward allocates its [T][d_ff] hidden activation (and, for tall
// inputs, tensor-core staging buffers) from the CUDA memory pool on every
// call.  Some callers cannot do that: a host that hands the library a fixed
// device-memory budget up front and forbids allocations afterwards, real-time
// or latency-critical callers that cannot take an allocator call (or an
// out-of-memory failure) in the middle of a step, and embedders that run the
// library beside their own memory manager.  needle_ffn_forward_noalloc serves
// them: it keeps the hidden activation in a fixed device array compiled into
// the library and computes the MLP on the CUDA cores, so a call allocates
// nothing.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "../../include/needle_b200.h"
#include "capi_internal.h"
#include "kernels.h"

namespace {

// Capacity of the fixed hidden-activation array: T * d_ff floats (4 MiB;
// e.g. 512 tokens at d_ff = 2048).  Every GPU that loads the library holds
// this array until the process exits.
constexpr size_t kNoAllocHiddenFloats = size_t(1) << 20;

static __device__ __align__(256) float g_ffn_hidden[kNoAllocHiddenFloats];

// The host-side name of g_ffn_hidden is only a stand-in, not a device
// address: each call looks up the current device's address with
// cudaGetSymbolAddress (cheap, allocates nothing), so an address never
// outlives the context it came from.  Kernel attributes are set once per
// device.
std::mutex g_mu;
bool g_kernels_ready[64] = {false};

bool setup_device(int dev, float **hidden) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_ffn_hidden);
  if (e != cudaSuccess) {
    ndl::capi_set_last_error(std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    return false;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_kernels_ready[dev]) {
    e = ndl::init_kernels();
    if (e != cudaSuccess) {
      ndl::capi_set_last_error(std::string("kernel set-up failed: ") + cudaGetErrorString(e));
      return false;
    }
    g_kernels_ready[dev] = true;
  }
  *hidden = (float *)p;
  return true;
}

}  // namespace

extern "C" int needle_ffn_forward_noalloc(const float *x, size_t T, size_t d_model, size_t d_ff,
                                          const uint8_t *gate_data, const float *gate_scales,
                                          const uint8_t *up_data, const float *up_scales, const uint8_t *down_data,
                                          const float *down_scales, int activation, float *out, void *stream) {
  using namespace ndl;
  capi_clear_last_error();
  if (!x || !gate_data || !gate_scales || !up_data || !up_scales || !down_data || !down_scales || !out || T == 0 ||
      d_model == 0 || d_ff == 0 || activation < 0 || activation > 2 || d_model > (1u << 20) || d_ff > (1u << 20)) {
    capi_set_last_error("invalid ffn arguments");
    return -1;
  }
  if (T > kNoAllocHiddenFloats / d_ff) {
    capi_set_last_error("needle_ffn_forward_noalloc: T * d_ff = " + std::to_string(T * d_ff) +
                        " exceeds the fixed hidden buffer of " + std::to_string(kNoAllocHiddenFloats) + " floats");
    return -1;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    capi_set_last_error("no current CUDA device");
    return -1;
  }
  float *hidden = nullptr;
  if (!setup_device(dev, &hidden)) return -1;
  cudaStream_t st = (cudaStream_t)stream;
  const int gs1 = (int)(d_model < 32 ? d_model : 32), gs2 = (int)(d_ff < 32 ? d_ff : 32);
  const int G1 = (int)((d_model + gs1 - 1) / gs1), G2 = (int)((d_ff + gs2 - 1) / gs2);
  // gate and up in one pass, (gate_i, up_i) interleaved; the epilogue writes
  // act(gate) * up into every element of the [T][d_ff] hidden array, so
  // nothing left by an earlier call is read.
  Int4Weight gu{gate_data, gate_scales, (int)d_model, (int)(2 * d_ff), G1, gs1};
  gu.w2 = up_data;
  gu.s2 = up_scales;
  MatmulOut a;
  a.y = hidden;
  a.ldy = (int64_t)d_ff;
  a.epi = EPI_ACT;
  a.act = activation;
  Int4Weight dn{down_data, down_scales, (int)d_ff, (int)d_model, G2, gs2};
  MatmulOut o;
  o.y = out;
  o.ldy = (int64_t)d_model;
  // up to 8 tokens the matvec kernels hold x in shared memory: refuse what
  // does not fit with the reason, not a bare launch error
  const size_t need = std::max(int4_matmul_smem((int)T, gu, a), int4_matmul_smem((int)T, dn, o));
  if (need > (size_t)kMaxDynSmem) {
    capi_set_last_error("needle_ffn_forward_noalloc: " + std::to_string(T) + " tokens at d_model " +
                        std::to_string(d_model) + ", d_ff " + std::to_string(d_ff) + " need " + std::to_string(need) +
                        " bytes of shared memory per block; the limit is " + std::to_string(kMaxDynSmem) +
                        " (up to 8 tokens a block holds every token's input row)");
    return -1;
  }
  cudaError_t e = int4_matmul(x, (int64_t)d_model, (int)T, gu, a, st);
  if (e == cudaSuccess) e = int4_matmul(hidden, (int64_t)d_ff, (int)T, dn, o, st);
  if (e != cudaSuccess) {
    capi_set_last_error(std::string("CUDA error: ") + cudaGetErrorString(e));
    return -1;
  }
  return 0;
}
