// Self-test of the bounded wait that every fused kernel builds on.
//
// A one-block kernel waits on an mbarrier that nothing ever arrives at, with
// the same wait_parity_limit the kernels use (only the cycle limit is the
// caller's), and records how the wait ended.  In the second case another warp
// of the block raises the abort flag, which must end the wait early.  The
// kernel then finishes normally, so the test observes a timed-out wait and a
// usable context without any fault or hang.
#include <cuda_runtime.h>

#include "mhc_b200.h"
#include "mhc_sm100.cuh"

namespace mhc {

using namespace sm100;

// out[0] = 1 if the wait returned false (gave up), out[1] = elapsed cycles
__global__ void __launch_bounds__(64, 1) selftest_wait_kernel(long long limit, int use_abort, long long *out) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    abort_flag = 0;
  }
  fence_mbar_init_cluster();
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    // parity 0 completes only when the single expected arrival happens; none does
    const bool ok = wait_parity_limit<false>(b, 0u, &abort_flag, limit);
    out[0] = ok ? 0 : 1;
    out[1] = clock64() - t0;
  } else if (threadIdx.x == 32 && use_abort) {
    // raise the abort flag after a short delay (well inside the limit)
    const long long t0 = clock64();
    while (clock64() - t0 < 200000) {
    }
    *reinterpret_cast<volatile int *>(&abort_flag) = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_arrive(b);  // complete the phase before the block exits
}

}  // namespace mhc

extern "C" int mhc_selftest_bounded_wait(long long limit_cycles, int use_abort, long long *result) {
  if (limit_cycles <= 0 || limit_cycles > 4000000000LL || !result) return MHC_ERR_SHAPE;
  long long *d = nullptr;
  if (cudaMalloc(&d, 2 * sizeof(long long)) != cudaSuccess) return MHC_ERR_CUDA;
  mhc::selftest_wait_kernel<<<1, 64>>>(limit_cycles, use_abort, d);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(result, d, 2 * sizeof(long long), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return e == cudaSuccess ? MHC_OK : MHC_ERR_CUDA;
}
