// Plain streaming-read kernel: the HBM read ceiling a memory-bound kernel of this library
// (the split-KV decode) is measured against, next to the driver's copy bandwidth.
//
// Every thread of a grid sized to the SMs reads 16-byte chunks of one contiguous buffer in
// a grid-stride loop, four independent loads in flight per iteration, and folds them into
// one XOR word per CTA (so the loads cannot be dropped); nothing else touches memory. Bytes
// per launch = `bytes` (a multiple of 16). Reads only; `sink` receives one word per CTA.
#include "common.cuh"
#include "kernels.cuh"

namespace hyt {
namespace {

constexpr int kProbeThreads = 512;

__global__ void __launch_bounds__(kProbeThreads) read_probe_kernel(const uint4* __restrict__ src,
                                                                   size_t chunks, uint32_t* sink) {
  const size_t stride = size_t(gridDim.x) * kProbeThreads;
  size_t i = size_t(blockIdx.x) * kProbeThreads + threadIdx.x;
  uint32_t acc = 0;
  for (; i + 3 * stride < chunks; i += 4 * stride) {
    const uint4 a = __ldcs(src + i), b = __ldcs(src + i + stride);
    const uint4 c = __ldcs(src + i + 2 * stride), d = __ldcs(src + i + 3 * stride);
    acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
  }
  for (; i < chunks; i += stride) {
    const uint4 a = __ldcs(src + i);
    acc ^= a.x ^ a.y ^ a.z ^ a.w;
  }
  __shared__ uint32_t red[kProbeThreads / 32];
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t v = 0;
    for (int w = 0; w < kProbeThreads / 32; ++w) v ^= red[w];
    sink[blockIdx.x] = v;
  }
}

}  // namespace

cudaError_t run_read_probe(const void* src, size_t bytes, uint32_t* sink, int ctas, cudaStream_t stream) {
  read_probe_kernel<<<ctas, kProbeThreads, 0, stream>>>(static_cast<const uint4*>(src), bytes / 16, sink);
  return cudaGetLastError();
}

}  // namespace hyt
