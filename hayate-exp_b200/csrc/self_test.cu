// Self-test of the bounded pipeline wait every kernel of this library uses.
//
// One CTA of two warps. Warp 0 waits on an mbarrier that nothing arrives at (count 1,
// no thread arrives, no copy is addressed to it), so its wait runs out after the 1 s
// limit, sets HYT_DEVERR_WAIT_TIMEOUT and the CTA's abort flag, and returns. Warp 1
// then waits on a second such barrier and must return at once through the abort flag,
// the path that keeps a CTA with several waiting roles from paying the limit once per
// role. No copy or tensor-core operation is ever in flight, so the kernel exits clean
// and the context stays usable; the host reads the status from the error word.
#include "common.cuh"
#include "kernels.cuh"

namespace hyt {
namespace {

__global__ void __launch_bounds__(64) wait_self_test_kernel(int32_t* error_word, int64_t* elapsed_ns) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int s_abort;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t start = global_ns();
  if (warp == 0) mbar_wait(&bars[0], 0, error_word, &s_abort);
  __syncthreads();
  const uint64_t first = global_ns();
  if (warp == 1) mbar_wait(&bars[1], 0, error_word, &s_abort);
  __syncthreads();
  if (threadIdx.x == 0) {
    elapsed_ns[0] = static_cast<int64_t>(first - start);
    elapsed_ns[1] = static_cast<int64_t>(global_ns() - first);
  }
}

}  // namespace

cudaError_t run_wait_self_test(int32_t* error_word, int64_t* elapsed_ns, cudaStream_t stream) {
  wait_self_test_kernel<<<1, 64, 0, stream>>>(error_word, elapsed_ns);
  return cudaGetLastError();
}

}  // namespace hyt
