// Self-test of the bounded wait and of the give-up path every fused kernel
// builds on.
//
// A one-block kernel waits on an mbarrier that nothing ever arrives at, with
// the same wait_parity_limit the kernels use (only the cycle limit is the
// caller's), and records how the wait ended.  In the second case another warp
// of the block raises the abort flag, which must end the wait early.  When the
// wait gives up, the kernel goes through the same steps as a fused kernel
// whose wait ran out: report_give_up (device error word and, if registered,
// the pinned host error flag) and NaN over the output it owns (`poison`).
// The kernel then finishes normally, so the test observes a timed-out wait, a
// reported error, poisoned output and a usable context without any fault or
// hang.
#include <cuda_runtime.h>

#include "mhc_b200.h"
#include "mhc_kernels.h"
#include "mhc_sm100.cuh"

namespace mhc {

__device__ int g_selftest_error = 0;  // error word of the self-test kernel

using namespace sm100;

constexpr int SELFTEST_ERR = 99;

// out[0] = 1 if the wait returned false (gave up), out[1] = elapsed cycles
__global__ void __launch_bounds__(64, 1)
selftest_wait_kernel(long long limit, int use_abort, long long *out, float *poison, long long poison_n,
                     int *err_flag) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  __shared__ int gave_up;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    abort_flag = 0;
    gave_up = 0;
  }
  fence_mbar_init_cluster();
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    // parity 0 completes only when the single expected arrival happens; none does
    const bool ok = wait_parity_limit<false>(b, 0u, &abort_flag, limit);
    out[0] = ok ? 0 : 1;
    out[1] = clock64() - t0;
    if (!ok) {
      gave_up = 1;
      report_give_up(&g_selftest_error, err_flag, SELFTEST_ERR);
    }
  } else if (threadIdx.x == 32 && use_abort) {
    // raise the abort flag after a short delay (well inside the limit)
    const long long t0 = clock64();
    while (clock64() - t0 < 200000) {
    }
    *reinterpret_cast<volatile int *>(&abort_flag) = 1;
  }
  __syncthreads();
  if (gave_up && poison != nullptr) {
    const float qnan = __int_as_float(0x7fc00000);
    for (long long i = threadIdx.x; i < poison_n; i += blockDim.x) poison[i] = qnan;
  }
  if (threadIdx.x == 0) mbar_arrive(b);  // complete the phase before the block exits
}

int read_selftest_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_selftest_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_selftest_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace mhc

extern "C" int mhc_selftest_bounded_wait(long long limit_cycles, int use_abort, long long *result, float *poison,
                                         long long poison_n) {
  if (limit_cycles <= 0 || limit_cycles > 4000000000LL || !result) return MHC_ERR_SHAPE;
  if (poison_n < 0 || (poison_n > 0 && !poison)) return MHC_ERR_SHAPE;
  long long *d = nullptr;
  if (cudaMalloc(&d, 2 * sizeof(long long)) != cudaSuccess) return MHC_ERR_CUDA;
  mhc::selftest_wait_kernel<<<1, 64>>>(limit_cycles, use_abort, d, poison, poison_n, mhc::host_error_flag());
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(result, d, 2 * sizeof(long long), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return e == cudaSuccess ? MHC_OK : MHC_ERR_CUDA;
}
