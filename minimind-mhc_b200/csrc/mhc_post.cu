// Post / res merge (forward) and its backward.
//
// post_fwd_kernel streams one 16-byte vector of every stream per item:
//   out[i, v] = sum_j H_res[i,j] x[j, v] + H_post[i] f[v]
// with the block's per-token coefficients staged once in shared memory (fp32).
//
// post_bwd_kernel runs one warp per token: the per-token reductions over C
// (dH_res, dH_post) are lane partial sums followed by a warp reduction; dx and
// df are streamed out in the same pass.
#include "mhc_device.cuh"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"

namespace mhc {

// Stage the block's per-token coefficients in shared memory (fp32).  With
// SK, h_res holds H_res logits: one thread per token runs Sinkhorn-Knopp in
// registers, writes the normalised matrix back to shared memory and, when
// h_res_out is given, to global memory for the backward pass.
template <int N, bool HAS_RES, bool SK>
__device__ __forceinline__ int stage_post_coefs(float *cs, const void *h_res, int hr_dt, const void *h_post,
                                                int hp_dt, int64_t T, int64_t tok0, int TB, int sk_iters,
                                                float sk_eps, void *h_res_out) {
  constexpr int NCOEF = (HAS_RES ? N * N : 0) + N;
  const int tb = (int)((T - tok0) < TB ? (T - tok0) : TB);
  for (int i = threadIdx.x; i < tb * NCOEF; i += blockDim.x) {
    const int t = i / NCOEF, k = i - t * NCOEF;
    const int64_t tok = tok0 + t;
    float v;
    if (HAS_RES && k < N * N) v = load_dyn(h_res, hr_dt, tok * (N * N) + k);
    else v = load_dyn(h_post, hp_dt, tok * N + (k - (HAS_RES ? N * N : 0)));
    cs[i] = v;
  }
  if constexpr (HAS_RES && SK) {
    __syncthreads();
    for (int t = threadIdx.x; t < tb; t += blockDim.x) {
      float p[N * N];
      MHC_UNROLL_N
      for (int k = 0; k < N * N; ++k) p[k] = cs[t * NCOEF + k];
      sinkhorn_fwd<N>(p, sk_iters, sk_eps);
      MHC_UNROLL_N
      for (int k = 0; k < N * N; ++k) {
        cs[t * NCOEF + k] = p[k];
        if (h_res_out) store_dyn(h_res_out, hr_dt, (tok0 + t) * (N * N) + k, p[k]);
      }
    }
  }
  __syncthreads();
  return tb;
}

// 16-byte vector path (x / out in Tx, f in Tf).
template <int N, typename Tx, typename Tf, bool HAS_RES, bool SK>
__global__ void __launch_bounds__(256)
post_fwd_kernel(const Tx *__restrict__ x, const void *__restrict__ h_res, int hr_dt,
                const void *__restrict__ h_post, int hp_dt, const Tf *__restrict__ f,
                Tx *__restrict__ out, int64_t T, int C, int TB, int sk_iters, float sk_eps,
                void *__restrict__ h_res_out) {
  constexpr int VEC = 16 / sizeof(Tx);
  constexpr int NCOEF = (HAS_RES ? N * N : 0) + N;
  extern __shared__ float cs[];  // [TB][NCOEF]
  grid_dep_launch();
  grid_dep_wait();
  const int64_t tok0 = (int64_t)blockIdx.x * TB;
  const int tb = stage_post_coefs<N, HAS_RES, SK>(cs, h_res, hr_dt, h_post, hp_dt, T, tok0, TB, sk_iters,
                                                  sk_eps, h_res_out);
  const int vpt = C / VEC;
  const int64_t nC = (int64_t)N * C;
  const int items = tb * vpt;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int t = it / vpt, v = it - t * vpt;
    const int64_t tok = tok0 + t;
    const float *H = cs + t * NCOEF;
    const float *hp = H + (HAS_RES ? N * N : 0);
    const Tx *xr = x + tok * nC + (int64_t)v * VEC;
    Tx *orow = out + tok * nC + (int64_t)v * VEC;
    Pack<Tx> px[N];
#pragma unroll
    for (int j = 0; j < N; ++j) px[j].raw = ldg_stream(xr + (int64_t)j * C);
    float fv[VEC];
    load_vec_stream<Tf, VEC>(f + tok * C + (int64_t)v * VEC, fv);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      Pack<Tx> o;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        float a;
        if constexpr (HAS_RES) {
          a = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) a = fmaf(H[i * N + j], px[j].get(e), a);
        } else {
          a = px[i].get(e);
        }
        o.set(e, fmaf(hp[i], fv[e], a));
      }
      stg_stream(orow + (int64_t)i * C, o.raw);
    }
  }
}

// Element-wise path for any dtype combination / alignment.
template <int N, bool HAS_RES, bool SK>
__global__ void __launch_bounds__(256)
post_fwd_scalar_kernel(const void *__restrict__ x, int x_dt, const void *__restrict__ h_res, int hr_dt,
                       const void *__restrict__ h_post, int hp_dt, const void *__restrict__ f, int f_dt,
                       void *__restrict__ out, int64_t T, int C, int TB, int sk_iters, float sk_eps,
                       void *__restrict__ h_res_out) {
  constexpr int NCOEF = (HAS_RES ? N * N : 0) + N;
  extern __shared__ float cs[];
  grid_dep_launch();
  grid_dep_wait();
  const int64_t tok0 = (int64_t)blockIdx.x * TB;
  const int tb = stage_post_coefs<N, HAS_RES, SK>(cs, h_res, hr_dt, h_post, hp_dt, T, tok0, TB, sk_iters,
                                                  sk_eps, h_res_out);
  const int64_t nC = (int64_t)N * C;
  const int items = tb * C;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int t = it / C, c = it - t * C;
    const int64_t tok = tok0 + t;
    const float *H = cs + t * NCOEF;
    const float *hp = H + (HAS_RES ? N * N : 0);
    float xv[N];
    for (int j = 0; j < N; ++j) xv[j] = load_dyn(x, x_dt, tok * nC + (int64_t)j * C + c);
    const float fv = load_dyn(f, f_dt, tok * C + c);
    for (int i = 0; i < N; ++i) {
      float a;
      if constexpr (HAS_RES) {
        a = 0.f;
        for (int j = 0; j < N; ++j) a = fmaf(H[i * N + j], xv[j], a);
      } else {
        a = xv[i];
      }
      store_dyn(out, x_dt, tok * nC + (int64_t)i * C + c, fmaf(hp[i], fv, a));
    }
  }
}

// Backward, one warp per token.  Vector path (Tx / Tf packs).  The token's
// coefficients sit in a per-warp shared-memory slot (read by broadcast), which
// leaves the registers to the accumulators and to one whole round of loads:
// every lane issues its n dout vectors, n x vectors and its f vector before any
// arithmetic.  At n = 4 that fits three 256-thread blocks per SM.
template <int N, typename Tx, typename Tf, bool HAS_RES>
__global__ void __launch_bounds__(256, N <= 4 ? 3 : 1)
post_bwd_kernel(const Tx *__restrict__ dout, const Tx *__restrict__ x, const void *__restrict__ h_res,
                int hr_dt, const void *__restrict__ h_post, int hp_dt, const Tf *__restrict__ f,
                Tx *__restrict__ dx, void *__restrict__ dh_res, void *__restrict__ dh_post,
                Tf *__restrict__ df, int64_t T, int C) {
  constexpr int VEC = 16 / sizeof(Tx);
  constexpr int NR = HAS_RES ? N * N : 0;   // H_res entries
  constexpr int NH = HAS_RES ? N * N : 1;
  constexpr int NCO = NR + N;                // H_res then H_post
  __shared__ float cs_all[8][NCO];
  const int lane = threadIdx.x & 31;
  float *cs = cs_all[threadIdx.x >> 5];
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nC = (int64_t)N * C;
  const int vpt = C / VEC;
  for (int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); tok < T;
       tok += nwarps) {
    __syncwarp();  // the previous token's coefficient reads are done
    for (int k = lane; k < NCO; k += 32)
      cs[k] = k < NR ? load_dyn(h_res, hr_dt, tok * (N * N) + k) : load_dyn(h_post, hp_dt, tok * N + (k - NR));
    __syncwarp();
    const float *H = cs;
    const float *hp = cs + NR;
    float aH[NH], ahp[N];
    MHC_UNROLL_N
    for (int k = 0; k < NH; ++k) aH[k] = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) ahp[i] = 0.f;
    const Tx *gr = dout + tok * nC;
    const Tx *xr = x + tok * nC;
    for (int v = lane; v < vpt; v += 32) {
      const int64_t off = (int64_t)v * VEC;
      Pack<Tx> pg[N], px[HAS_RES ? N : 1];
#pragma unroll
      for (int i = 0; i < N; ++i) pg[i].raw = ldg_stream(gr + (int64_t)i * C + off);
      if constexpr (HAS_RES) {
#pragma unroll
        for (int j = 0; j < N; ++j) px[j].raw = ldg_stream(xr + (int64_t)j * C + off);
      }
      float fv[VEC];
      load_vec_stream<Tf, VEC>(f + tok * C + off, fv);
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int e = 0; e < VEC; ++e) ahp[i] = fmaf(pg[i].get(e), fv[e], ahp[i]);
      if (df) {
        float d[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          float a = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) a = fmaf(hp[i], pg[i].get(e), a);
          d[e] = a;
        }
        store_vec_stream<Tf, VEC>(df + tok * C + off, d);
      }
      if constexpr (HAS_RES) {
        // dH_res[i][j] += <g_i, x_j>;  dx_j = sum_i H[i][j] g_i
#pragma unroll
        for (int j = 0; j < N; ++j) {
#pragma unroll
          for (int i = 0; i < N; ++i)
#pragma unroll
            for (int e = 0; e < VEC; ++e) aH[i * N + j] = fmaf(pg[i].get(e), px[j].get(e), aH[i * N + j]);
          if (dx) {
            Pack<Tx> o;
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              float a = 0.f;
#pragma unroll
              for (int i = 0; i < N; ++i) a = fmaf(H[i * N + j], pg[i].get(e), a);
              o.set(e, a);
            }
            stg_stream(dx + tok * nC + (int64_t)j * C + off, o.raw);
          }
        }
      } else if (dx) {
#pragma unroll
        for (int i = 0; i < N; ++i) stg_stream(dx + tok * nC + (int64_t)i * C + off, pg[i].raw);
      }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) ahp[i] = warp_sum(ahp[i]);
    if constexpr (HAS_RES) {
      MHC_UNROLL_N
      for (int k = 0; k < N * N; ++k) aH[k] = warp_sum(aH[k]);
    }
    if (lane == 0) {
      if (dh_post) {
#pragma unroll
        for (int i = 0; i < N; ++i) store_dyn(dh_post, hp_dt, tok * N + i, ahp[i]);
      }
      if (HAS_RES && dh_res) {
        MHC_UNROLL_N
        for (int k = 0; k < N * N; ++k) store_dyn(dh_res, hr_dt, tok * (N * N) + k, aH[k]);
      }
    }
  }
}

// Element-wise backward for any dtype combination / alignment.
template <int N, bool HAS_RES>
__global__ void __launch_bounds__(256)
post_bwd_scalar_kernel(const void *__restrict__ dout, const void *__restrict__ x, int x_dt,
                       const void *__restrict__ h_res, int hr_dt, const void *__restrict__ h_post,
                       int hp_dt, const void *__restrict__ f, int f_dt, void *__restrict__ dx,
                       void *__restrict__ dh_res, void *__restrict__ dh_post, void *__restrict__ df,
                       int64_t T, int C) {
  constexpr int NH = HAS_RES ? N * N : 1;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nC = (int64_t)N * C;
  for (int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); tok < T;
       tok += nwarps) {
    float H[NH], hp[N], aH[NH], ahp[N];
    for (int k = 0; k < NH; ++k) {
      H[k] = HAS_RES ? load_dyn(h_res, hr_dt, tok * (N * N) + k) : 0.f;
      aH[k] = 0.f;
    }
    for (int i = 0; i < N; ++i) {
      hp[i] = load_dyn(h_post, hp_dt, tok * N + i);
      ahp[i] = 0.f;
    }
    for (int c = lane; c < C; c += 32) {
      float g[N];
      for (int i = 0; i < N; ++i) g[i] = load_dyn(dout, x_dt, tok * nC + (int64_t)i * C + c);
      const float fv = load_dyn(f, f_dt, tok * C + c);
      float d = 0.f;
      for (int i = 0; i < N; ++i) {
        ahp[i] = fmaf(g[i], fv, ahp[i]);
        d = fmaf(hp[i], g[i], d);
      }
      if (df) store_dyn(df, f_dt, tok * C + c, d);
      for (int j = 0; j < N; ++j) {
        if constexpr (HAS_RES) {
          const float xj = load_dyn(x, x_dt, tok * nC + (int64_t)j * C + c);
          float a = 0.f;
          for (int i = 0; i < N; ++i) {
            aH[i * N + j] = fmaf(g[i], xj, aH[i * N + j]);
            a = fmaf(H[i * N + j], g[i], a);
          }
          if (dx) store_dyn(dx, x_dt, tok * nC + (int64_t)j * C + c, a);
        } else {
          if (dx) store_dyn(dx, x_dt, tok * nC + (int64_t)j * C + c, g[j]);
        }
      }
    }
    for (int i = 0; i < N; ++i) ahp[i] = warp_sum(ahp[i]);
    if constexpr (HAS_RES) {
      for (int k = 0; k < N * N; ++k) aH[k] = warp_sum(aH[k]);
    }
    if (lane == 0) {
      if (dh_post)
        for (int i = 0; i < N; ++i) store_dyn(dh_post, hp_dt, tok * N + i, ahp[i]);
      if (HAS_RES && dh_res)
        for (int k = 0; k < N * N; ++k) store_dyn(dh_res, hr_dt, tok * (N * N) + k, aH[k]);
    }
  }
}

namespace {
// (Tx, Tf) pairs with a 16-byte vector instance.
template <typename F>
cudaError_t with_vec_pair(int x_dt, int f_dt, F &&fn) {
  if (x_dt == f_dt) return with_dtype(x_dt, [&](auto t) { return fn(t, t); });
  if (x_dt == MHC_F32 && f_dt == MHC_BF16) return fn(float{}, __nv_bfloat16{});
  return fn(float{}, __half{});
}
bool is_vec_pair(int x_dt, int f_dt) {
  return x_dt == f_dt || (x_dt == MHC_F32 && (f_dt == MHC_BF16 || f_dt == MHC_F16));
}
bool a16(const void *p) { return ((uintptr_t)p & 15) == 0; }
}  // namespace

cudaError_t launch_post_fwd(int n, int x_dtype, const void *x, const void *h_res, int h_res_dtype,
                            const void *h_post, int h_post_dtype, const void *f, int f_dtype,
                            void *out, int64_t T, int C, int res_is_logits, int sk_iters,
                            float sk_eps, void *h_res_out, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int xvec = x_dtype == MHC_F32 ? 4 : 8;
  const bool vecok = is_vec_pair(x_dtype, f_dtype) && C % xvec == 0 && a16(x) && a16(f) && a16(out);
  const int vpt = vecok ? C / xvec : C;
  int TB = (1024 + vpt - 1) / vpt;
  if (TB > 64) TB = 64;
  if (TB < 1) TB = 1;
  const unsigned grid = (unsigned)((T + TB - 1) / TB);
  const bool sk = h_res != nullptr && res_is_logits != 0;
  return with_n(n, [&](auto nn) {
    constexpr int N = decltype(nn)::value;
    const size_t smem = (size_t)TB * ((h_res ? N * N : 0) + N) * 4;
    auto go = [&](auto kern, auto... args) {
      if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
      }
      // programmatic dependent launch: the kernel waits (griddepcontrol) for
      // the previous kernel of the stream before its first global read
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cfg.gridDim = dim3(grid, 1, 1);
      cfg.blockDim = dim3(256, 1, 1);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
      if (e != cudaSuccess) return e;
      return cudaGetLastError();
    };
    if (!vecok) {
      if (sk)
        return go(post_fwd_scalar_kernel<N, true, true>, x, x_dtype, h_res, h_res_dtype, h_post, h_post_dtype,
                  f, f_dtype, out, T, C, TB, sk_iters, sk_eps, h_res_out);
      if (h_res)
        return go(post_fwd_scalar_kernel<N, true, false>, x, x_dtype, h_res, h_res_dtype, h_post, h_post_dtype,
                  f, f_dtype, out, T, C, TB, sk_iters, sk_eps, h_res_out);
      return go(post_fwd_scalar_kernel<N, false, false>, x, x_dtype, h_res, h_res_dtype, h_post, h_post_dtype,
                f, f_dtype, out, T, C, TB, sk_iters, sk_eps, h_res_out);
    }
    return with_vec_pair(x_dtype, f_dtype, [&](auto tx, auto tf) {
      using Tx = decltype(tx);
      using Tf = decltype(tf);
      if (sk)
        return go(post_fwd_kernel<N, Tx, Tf, true, true>, (const Tx *)x, h_res, h_res_dtype, h_post,
                  h_post_dtype, (const Tf *)f, (Tx *)out, T, C, TB, sk_iters, sk_eps, h_res_out);
      if (h_res)
        return go(post_fwd_kernel<N, Tx, Tf, true, false>, (const Tx *)x, h_res, h_res_dtype, h_post,
                  h_post_dtype, (const Tf *)f, (Tx *)out, T, C, TB, sk_iters, sk_eps, h_res_out);
      return go(post_fwd_kernel<N, Tx, Tf, false, false>, (const Tx *)x, h_res, h_res_dtype, h_post,
                h_post_dtype, (const Tf *)f, (Tx *)out, T, C, TB, sk_iters, sk_eps, h_res_out);
    });
  });
}

cudaError_t launch_post_bwd(int n, int x_dtype, const void *dout, const void *x, const void *h_res,
                            int h_res_dtype, const void *h_post, int h_post_dtype, const void *f,
                            int f_dtype, void *dx, void *dh_res, void *dh_post, void *df,
                            int64_t T, int C, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int sms = device_sm_count();
  const int xvec = x_dtype == MHC_F32 ? 4 : 8;
  const bool vecok = is_vec_pair(x_dtype, f_dtype) && C % xvec == 0 && a16(x) && a16(dout) &&
                     a16(f) && a16(dx) && a16(df);
  const unsigned grid = grid_for(T * 32, 256, sms, 6);
  return with_n(n, [&](auto nn) {
    constexpr int N = decltype(nn)::value;
    auto go = [&](auto kern, auto... args) {
      kern<<<grid, 256, 0, stream>>>(args...);
      return cudaGetLastError();
    };
    if (!vecok) {
      if (h_res)
        return go(post_bwd_scalar_kernel<N, true>, dout, x, x_dtype, h_res, h_res_dtype, h_post,
                  h_post_dtype, f, f_dtype, dx, dh_res, dh_post, df, T, C);
      return go(post_bwd_scalar_kernel<N, false>, dout, x, x_dtype, h_res, h_res_dtype, h_post,
                h_post_dtype, f, f_dtype, dx, dh_res, dh_post, df, T, C);
    }
    return with_vec_pair(x_dtype, f_dtype, [&](auto tx, auto tf) {
      using Tx = decltype(tx);
      using Tf = decltype(tf);
      if (h_res)
        return go(post_bwd_kernel<N, Tx, Tf, true>, (const Tx *)dout, (const Tx *)x, h_res, h_res_dtype,
                  h_post, h_post_dtype, (const Tf *)f, (Tx *)dx, dh_res, dh_post, (Tf *)df, T, C);
      return go(post_bwd_kernel<N, Tx, Tf, false>, (const Tx *)dout, (const Tx *)x, h_res, h_res_dtype,
                h_post, h_post_dtype, (const Tf *)f, (Tx *)dx, dh_res, dh_post, (Tf *)df, T, C);
    });
  });
}

}  // namespace mhc
