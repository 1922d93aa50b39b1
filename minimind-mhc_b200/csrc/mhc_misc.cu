// Stand-alone Sinkhorn-Knopp (forward and backward-by-recompute, one thread per
// matrix), the StreamExpand copy / its reduction, and the row RMSNorm of the
// generic post + pre path.
#include "mhc_device.cuh"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"

namespace mhc {

template <int N>
__global__ void __launch_bounds__(128)
sinkhorn_fwd_kernel(const void *__restrict__ M, int mdt, void *__restrict__ Y, int ydt,
                    int64_t batch, int iters, float eps) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float p[N * N];
MHC_UNROLL_N
  for (int k = 0; k < N * N; ++k) p[k] = load_dyn(M, mdt, b * N * N + k);
  sinkhorn_fwd<N>(p, iters, eps);
MHC_UNROLL_N
  for (int k = 0; k < N * N; ++k) store_dyn(Y, ydt, b * N * N + k, p[k]);
}

template <int N>
__global__ void __launch_bounds__(128)
sinkhorn_bwd_kernel(const void *__restrict__ M, int mdt, const void *__restrict__ dY, int gdt,
                    void *__restrict__ dM, int dmdt, int64_t batch, int iters, float eps, int TB) {
  extern __shared__ float traj[];  // [checkpoints][N*N][TB]
  const int t = threadIdx.x;
  const int64_t b = (int64_t)blockIdx.x * TB + t;
  if (t >= TB || b >= batch) return;
  float m[N * N], g[N * N];
MHC_UNROLL_N
  for (int k = 0; k < N * N; ++k) {
    m[k] = load_dyn(M, mdt, b * N * N + k);
    g[k] = load_dyn(dY, gdt, b * N * N + k);
  }
  sinkhorn_bwd<N>(m, g, iters, eps, traj + t, TB);
MHC_UNROLL_N
  for (int k = 0; k < N * N; ++k) store_dyn(dM, dmdt, b * N * N + k, g[k]);
}

size_t sinkhorn_bwd_smem_per_item(int n, int iters) {
  return (size_t)sk_ckpt_count(n, iters) * n * n * 4;
}

cudaError_t launch_sinkhorn_fwd(int n, const void *M, int m_dtype, void *Y, int y_dtype,
                                int64_t batch, int iters, float eps, cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  return with_n(n, [&](auto nn) {
    constexpr int N = decltype(nn)::value;
    const unsigned grid = (unsigned)((batch + 127) / 128);
    sinkhorn_fwd_kernel<N><<<grid, 128, 0, stream>>>(M, m_dtype, Y, y_dtype, batch, iters, eps);
    return cudaGetLastError();
  });
}

cudaError_t launch_sinkhorn_bwd(int n, const void *M, int m_dtype, const void *dY, int dy_dtype,
                                void *dM, int dm_dtype, int64_t batch, int iters, float eps,
                                cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  const size_t per = sinkhorn_bwd_smem_per_item(n, iters);
  int TB = (int)((96 * 1024) / per);
  if (TB > 128) TB = 128;
  if (TB < 1) TB = 1;
  const size_t smem = per * TB;
  return with_n(n, [&](auto nn) {
    constexpr int N = decltype(nn)::value;
    auto kern = sinkhorn_bwd_kernel<N>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)((batch + TB - 1) / TB);
    kern<<<grid, 128, smem, stream>>>(M, m_dtype, dY, dy_dtype, dM, dm_dtype, batch, iters, eps, TB);
    return cudaGetLastError();
  });
}

// out[t, i*C + c] = x[t, c]
template <typename T>
__global__ void __launch_bounds__(256)
expand_fwd_kernel(const T *__restrict__ x, T *__restrict__ out, int64_t T_, int n, int C, bool vec) {
  const int64_t nC = (int64_t)n * C;
  if (vec) {
    constexpr int VEC = 16 / sizeof(T);
    const int vpt = C / VEC;
    const int64_t items = T_ * vpt;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
         it += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = it / vpt;
      const int v = (int)(it - t * vpt);
      const uint4 r = ldg_stream(x + t * C + (int64_t)v * VEC);
      for (int i = 0; i < n; ++i) stg_stream(out + t * nC + (int64_t)i * C + (int64_t)v * VEC, r);
    }
  } else {
    const int64_t items = T_ * C;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
         it += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = it / C;
      const int c = (int)(it - t * C);
      const T v = x[it];
      for (int i = 0; i < n; ++i) out[t * nC + (int64_t)i * C + c] = v;
    }
  }
}

// dx[t, c] = sum_i dout[t, i*C + c]
template <typename T>
__global__ void __launch_bounds__(256)
expand_bwd_kernel(const T *__restrict__ dout, T *__restrict__ dx, int64_t T_, int n, int C) {
  const int64_t nC = (int64_t)n * C;
  const int64_t items = T_ * C;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = it / C;
    const int c = (int)(it - t * C);
    float a = 0.f;
    for (int i = 0; i < n; ++i) a += to_f(dout[t * nC + (int64_t)i * C + c]);
    dx[it] = from_f<T>(a);
  }
}

cudaError_t launch_expand_fwd(int dtype, const void *x, void *out, int64_t T, int n, int C,
                              cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int sms = device_sm_count();
  return with_dtype(dtype, [&](auto tag) {
    using Tx = decltype(tag);
    constexpr int VEC = 16 / sizeof(Tx);
    const bool vec = C % VEC == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0;
    const int64_t items = T * (vec ? C / VEC : C);
    expand_fwd_kernel<Tx><<<grid_for(items, 256, sms, 16), 256, 0, stream>>>(
        (const Tx *)x, (Tx *)out, T, n, C, vec);
    return cudaGetLastError();
  });
}

cudaError_t launch_expand_bwd(int dtype, const void *dout, void *dx, int64_t T, int n, int C,
                              cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int sms = device_sm_count();
  return with_dtype(dtype, [&](auto tag) {
    using Tx = decltype(tag);
    expand_bwd_kernel<Tx><<<grid_for(T * C, 256, sms, 16), 256, 0, stream>>>(
        (const Tx *)dout, (Tx *)dx, T, n, C);
    return cudaGetLastError();
  });
}

// y[t, c] = z[t, c] * rsqrt(mean_c z[t, :]^2 + eps) * w[c], one warp per row;
// the mean is taken over the z values as stored.
__global__ void __launch_bounds__(256)
rmsnorm_rows_kernel(const void *__restrict__ z, int zdt, const void *__restrict__ w, int wdt, float eps,
                    void *__restrict__ y, int64_t T, int C) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += nwarps) {
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float v = load_dyn(z, zdt, t * C + c);
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)C + eps);
    for (int c = lane; c < C; c += 32)
      store_dyn(y, zdt, t * C + c, load_dyn(z, zdt, t * C + c) * r * load_dyn(w, wdt, c));
  }
}

// The same with 16-byte vectors (16-bit z, C a multiple of 8, aligned rows):
// a warp keeps VPL vectors of each of two rows in registers (one HBM read of
// z) and reduces the two rows together, so their loads and shuffles overlap.
template <typename Tz, typename Tw, int VPL>
__global__ void __launch_bounds__(256)
rmsnorm_rows_vec_kernel(const Tz *__restrict__ z, const Tw *__restrict__ w, float eps, Tz *__restrict__ y,
                        int64_t T, int C) {
  constexpr int VEC = 8;
  extern __shared__ float ws[];  // the norm weight in fp32, staged once per block
  for (int c = threadIdx.x; c < C; c += blockDim.x) ws[c] = to_f(w[c]);
  __syncthreads();
  const int lane = threadIdx.x & 31, nv = C / VEC;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2; t0 < T; t0 += nwarps * 2) {
    Pack<Tz> pk[2][VPL];
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
      for (int u = 0; u < VPL; ++u) {
        const int v = lane + 32 * u;
        pk[r][u].raw = (t0 + r < T && v < nv) ? ldg_stream(z + (t0 + r) * C + v * VEC) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int u = 0; u < VPL; ++u)
#pragma unroll
        for (int e = 0; e < VEC; ++e) ss[r] = fmaf(pk[r][u].get(e), pk[r][u].get(e), ss[r]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], o);
      ss[1] += __shfl_xor_sync(0xffffffffu, ss[1], o);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (t0 + r >= T) continue;
      const float rr = rsqrtf(ss[r] / (float)C + eps);
#pragma unroll
      for (int u = 0; u < VPL; ++u) {
        const int v = lane + 32 * u;
        if (v >= nv) continue;
        const float4 w0 = *reinterpret_cast<const float4 *>(ws + v * VEC);
        const float4 w1 = *reinterpret_cast<const float4 *>(ws + v * VEC + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        Pack<Tz> o;
#pragma unroll
        for (int e = 0; e < VEC; ++e) o.set(e, pk[r][u].get(e) * rr * wv[e]);
        stg_stream(y + (t0 + r) * C + v * VEC, o.raw);
      }
    }
  }
}

cudaError_t launch_rmsnorm_rows(int z_dtype, const void *z, const void *w, int w_dtype, float eps, void *y,
                                int64_t T, int C, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const unsigned grid = grid_for(T * 32, 256, device_sm_count(), 16);
  const size_t smem = (size_t)C * 4;
  const bool vec = z_dtype != MHC_F32 && C % 8 == 0 && C <= 2048 && ((uintptr_t)z & 15) == 0 &&
                   ((uintptr_t)y & 15) == 0;
  if (vec) {
    const int vpl = (C / 8 + 31) / 32;  // vectors of a row per lane
    auto go = [&](auto vtag) -> cudaError_t {
      constexpr int VPL = decltype(vtag)::value;
      const unsigned g2 = grid_for((T + 1) / 2 * 32, 256, device_sm_count(), 16);
      return with_dtype(w_dtype, [&](auto wtag) -> cudaError_t {
        using Tw = decltype(wtag);
        if (z_dtype == MHC_BF16)
          rmsnorm_rows_vec_kernel<__nv_bfloat16, Tw, VPL><<<g2, 256, smem, stream>>>(
              (const __nv_bfloat16 *)z, (const Tw *)w, eps, (__nv_bfloat16 *)y, T, C);
        else
          rmsnorm_rows_vec_kernel<__half, Tw, VPL><<<g2, 256, smem, stream>>>((const __half *)z, (const Tw *)w, eps,
                                                                             (__half *)y, T, C);
        return cudaGetLastError();
      });
    };
    if (vpl <= 1) return go(IC<1>{});
    if (vpl <= 2) return go(IC<2>{});
    if (vpl <= 3) return go(IC<3>{});
    if (vpl <= 4) return go(IC<4>{});
    if (vpl <= 8) return go(IC<8>{});
  }
  rmsnorm_rows_kernel<<<grid, 256, 0, stream>>>(z, z_dtype, w, w_dtype, eps, y, T, C);
  return cudaGetLastError();
}

}  // namespace mhc
