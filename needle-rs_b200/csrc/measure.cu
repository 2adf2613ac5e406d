// measure.cu — a streaming-read probe that the benchmark uses to report the
// device's read ceiling beside the measured copy bandwidth: a read-dominated
// kernel (decoder cross-attention reads 2.4 GB and writes 4 MB per launch) is
// bounded by the read stream, which runs faster than a copy.
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

__global__ void fill_kernel(float4 *x, int64_t n4) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const uint32_t h = (uint32_t)i * 2654435761u;
    x[i] = make_float4((float)(h & 0xffff), (float)(h >> 16), (float)(i & 1023), 1.0f);
  }
}

// Grid-stride sum of float4 loads, four loads in flight per thread.
__global__ void __launch_bounds__(256) read_stream_kernel(const float4 *__restrict__ x, int64_t n4, float *out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float acc = 0.0f;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(x + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) acc += v[u].x + v[u].y + v[u].z + v[u].w;
  }
  for (; i < n4; i += stride) {
    const float4 v = __ldg(x + i);
    acc += v.x + v.y + v.z + v.w;
  }
  out[(int64_t)blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

}  // namespace

extern "C" int needle_hbm_read_gbs(size_t bytes, int iters, double *gbs) {
  if (!gbs || bytes < (1u << 20) || iters <= 0) return -1;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return -1;
  const int64_t n4 = (int64_t)(bytes / 16);
  const int grid = 4 * sms;
  float4 *x = nullptr;
  float *out = nullptr;
  cudaEvent_t a = nullptr, b = nullptr;
  int rc = -1;
  if (cudaMalloc(&x, (size_t)n4 * 16) == cudaSuccess && cudaMalloc(&out, (size_t)grid * 256 * 4) == cudaSuccess &&
      cudaEventCreate(&a) == cudaSuccess && cudaEventCreate(&b) == cudaSuccess) {
    fill_kernel<<<grid, 256>>>(x, n4);
    for (int w = 0; w < 3; ++w) read_stream_kernel<<<grid, 256>>>(x, n4, out);
    cudaEventRecord(a);
    for (int it = 0; it < iters; ++it) read_stream_kernel<<<grid, 256>>>(x, n4, out);
    cudaEventRecord(b);
    float ms = 0.0f;
    if (cudaEventSynchronize(b) == cudaSuccess && cudaEventElapsedTime(&ms, a, b) == cudaSuccess && ms > 0.0f) {
      *gbs = (double)n4 * 16.0 * iters / (ms * 1e6);
      rc = 0;
    }
  }
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  cudaFree(out);
  cudaFree(x);
  return cudaGetLastError() == cudaSuccess ? rc : -1;
}
