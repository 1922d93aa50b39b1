// Forward coefficient stage and pre-aggregate (generic CUDA-core path).
//
// coef_fwd_kernel: per block a tile of TM tokens; the n*C reduction is streamed
// in 128-byte column chunks through shared memory (x converted to fp32, phi
// transposed to fp32); each thread owns RT tokens x RJ projection columns in
// registers, so a phi element staged once is reused by every token of the tile.
// The unweighted sum of squares is accumulated while staging x.  The epilogue
// (one thread per token) applies 1/rms, the sigmoid gates and, for the full
// layer, Sinkhorn-Knopp in registers.
//
// aggregate_kernel: z[t,c] = sum_i w[t,i] x[t,i*C+c] with 16-byte vectors.
#include "mhc_device.cuh"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"

namespace mhc {

template <int N, int MODE, typename Tx>
struct CoefCfg {
  static constexpr int FD = Dims<N, MODE>::FD;
  static constexpr int JG = FD <= 32 ? 4 : (FD <= 96 ? 8 : 32);  // column groups per warp
  static constexpr int RJ = (FD + JG - 1) / JG;                  // columns per thread
  // tokens per thread and block size: fp32 x takes 4 tokens per thread in
  // 128-thread blocks (twice the FMAs per shared-memory load: the fp32 kernel
  // is bound by shared-memory wavefronts), 16-bit x 2 in 256-thread blocks
  static constexpr int RT = sizeof(Tx) == 4 ? 4 : 2;
  static constexpr int TG = 32 / JG;                             // token groups per warp
  static constexpr int TPW = TG * RT;                            // tokens per warp
  static constexpr int THREADS = sizeof(Tx) == 4 ? 128 : 256;
  static constexpr int TM = (THREADS / 32) * TPW;                // tokens per block
  static constexpr int VEC = 16 / sizeof(Tx);
  static constexpr int KC = 8 * VEC;                             // 128 bytes of a row
  static constexpr int XS = KC + 4;                              // smem row stride (floats)
  static constexpr int FDP = JG * RJ;
  static constexpr int SEGS = TM * 8;                            // 16 B segments per chunk
  static constexpr int SEG_IT = (SEGS + THREADS - 1) / THREADS;
  static constexpr int PH_IT = (KC * FD + THREADS - 1) / THREADS;  // phi elements per thread per chunk
  static constexpr int MRS = FD + 1;
  static constexpr int NPAR = 3 + 2 * N + N * N;
  static constexpr size_t SMEM_X = size_t(TM) * XS * 4;
  static constexpr size_t SMEM_MR = size_t(TM) * MRS * 4;
  static constexpr size_t SMEM_A = SMEM_X > SMEM_MR ? SMEM_X : SMEM_MR;
  static constexpr size_t SMEM_P = size_t(FDP) * XS * 4;
  static constexpr size_t SMEM = SMEM_A + SMEM_P + size_t(TM) * 4 + size_t(NPAR) * 4;
};

// Parameter vector in shared memory: [0] alpha_pre (head: alpha), [1] alpha_post,
// [2] alpha_res, [3, 3+N) bias_pre (head: bias), [3+N, 3+2N) bias_post,
// [3+2N, 3+2N+N^2) bias_res.
template <int N, int MODE>
__device__ __forceinline__ void load_params(float *par, const CoefParams &p, int tid, int nthreads) {
  constexpr int NPAR = 3 + 2 * N + N * N;
  for (int i = tid; i < NPAR; i += nthreads) {
    float v = 0.f;
    const int dt = p.param_dtype;
    if (i == 0) v = load_dyn(p.alpha_pre, dt, 0);
    else if (i == 1) { if (MODE != HEAD) v = load_dyn(p.alpha_post, dt, 0); }
    else if (i == 2) { if (MODE == FULL) v = load_dyn(p.alpha_res, dt, 0); }
    else if (i < 3 + N) v = load_dyn(p.bias_pre, dt, i - 3);
    else if (i < 3 + 2 * N) { if (MODE != HEAD) v = load_dyn(p.bias_post, dt, i - 3 - N); }
    else { if (MODE == FULL) v = load_dyn(p.bias_res, dt, i - 3 - 2 * N); }
    par[i] = v;
  }
}

template <int N, int MODE, typename Tx>
__global__ void __launch_bounds__(256)
coef_fwd_kernel(const Tx *__restrict__ x, int64_t T, int nC, const void *__restrict__ phi,
                CoefParams p, void *h_pre, void *h_post, void *h_res, int coef_dtype,
                float *__restrict__ inv_rms, float *__restrict__ mixes, float *__restrict__ gate_ws,
                bool vecok) {
  using Cf = CoefCfg<N, MODE, Tx>;
  constexpr int FD = Cf::FD, TM = Cf::TM, XS = Cf::XS, KC = Cf::KC, VEC = Cf::VEC;
  extern __shared__ float4 smem4[];
  float *smem = reinterpret_cast<float *>(smem4);
  float *xs = smem;                                 // [TM][XS], later mr[TM][MRS]
  float *ps = smem + Cf::SMEM_A / 4;                // [FDP][XS]
  float *ssq_s = ps + Cf::FDP * XS;                 // [TM]
  float *par = ssq_s + TM;                          // [NPAR]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tok0 = (int64_t)blockIdx.x * TM;
  load_params<N, MODE>(par, p, tid, Cf::THREADS);
  for (int i = tid; i < (Cf::FDP - FD) * XS; i += Cf::THREADS) ps[FD * XS + i] = 0.f;

  const int nchunks = (nC + KC - 1) / KC;
  uint4 pre[Cf::SEG_IT];     // raw Tx elements of the next chunk
  float phv[Cf::PH_IT];      // phi elements of the next chunk (loaded a chunk ahead: the loads'
                             // latency overlaps the FMA loop instead of stalling every chunk)
  float ssq_part[Cf::SEG_IT];
#pragma unroll
  for (int s = 0; s < Cf::SEG_IT; ++s) ssq_part[s] = 0.f;

  auto load_chunk = [&](int kc) {
    const int k0 = kc * KC;
#pragma unroll
    for (int s = 0; s < Cf::SEG_IT; ++s) {
      const int seg = tid + s * Cf::THREADS;
      const int row = seg >> 3, sg = seg & 7;
      const int64_t tok = tok0 + row;
      const int k = k0 + sg * VEC;
      pre[s] = make_uint4(0u, 0u, 0u, 0u);
      if (vecok) {
        if (seg < Cf::SEGS && tok < T && k < nC) pre[s] = ldg_keep(x + tok * nC + k);
      } else {
        Tx *e8 = reinterpret_cast<Tx *>(&pre[s]);
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (seg < Cf::SEGS && tok < T && k + e < nC) e8[e] = x[tok * nC + k + e];
      }
    }
    const int dt = p.param_dtype;
#pragma unroll
    for (int u = 0; u < Cf::PH_IT; ++u) {
      const int e = tid + u * Cf::THREADS;
      const int kk = e / FD, j = e - kk * FD;
      phv[u] = (e < KC * FD && k0 + kk < nC) ? load_dyn(phi, dt, (int64_t)(k0 + kk) * FD + j) : 0.f;
    }
  };

  const int tg = lane / Cf::JG, jg = lane % Cf::JG;
  float acc[Cf::RT][Cf::RJ];
#pragma unroll
  for (int r = 0; r < Cf::RT; ++r)
#pragma unroll
    for (int q = 0; q < Cf::RJ; ++q) acc[r][q] = 0.f;

  load_chunk(0);
  for (int kc = 0; kc < nchunks; ++kc) {
    __syncthreads();
    // stage x (fp32) and accumulate squares
#pragma unroll
    for (int s = 0; s < Cf::SEG_IT; ++s) {
      const int seg = tid + s * Cf::THREADS;
      if (seg < Cf::SEGS) {
        const int row = seg >> 3, sg = seg & 7;
        float v[VEC];
        Pack<Tx> pk;
        pk.raw = pre[s];
        pk.to_float(v);
        float *dst = xs + row * XS + sg * VEC;
#pragma unroll
        for (int e = 0; e < VEC; e += 4) {
          *reinterpret_cast<float4 *>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
          ssq_part[s] += v[e] * v[e] + v[e + 1] * v[e + 1] + v[e + 2] * v[e + 2] + v[e + 3] * v[e + 3];
        }
      }
    }
    // stage phi^T chunk (fp32), loaded with the chunk's x
#pragma unroll
    for (int u = 0; u < Cf::PH_IT; ++u) {
      const int e = tid + u * Cf::THREADS;
      if (e < KC * FD) {
        const int kk = e / FD, j = e - kk * FD;
        ps[j * XS + kk] = phv[u];
      }
    }
    __syncthreads();
    if (kc + 1 < nchunks) load_chunk(kc + 1);
    // register-tiled FMA over the chunk
    const float *xr0 = xs + (warp * Cf::TPW + tg) * XS;
    const float *pr0 = ps + jg * XS;
#pragma unroll 4
    for (int kk = 0; kk < KC; kk += 4) {
      float4 xv[Cf::RT];
#pragma unroll
      for (int r = 0; r < Cf::RT; ++r) xv[r] = *reinterpret_cast<const float4 *>(xr0 + r * Cf::TG * XS + kk);
#pragma unroll
      for (int q = 0; q < Cf::RJ; ++q) {
        const float4 pv = *reinterpret_cast<const float4 *>(pr0 + q * Cf::JG * XS + kk);
#pragma unroll
        for (int r = 0; r < Cf::RT; ++r) {
          float a = acc[r][q];
          a = fmaf(xv[r].x, pv.x, a);
          a = fmaf(xv[r].y, pv.y, a);
          a = fmaf(xv[r].z, pv.z, a);
          a = fmaf(xv[r].w, pv.w, a);
          acc[r][q] = a;
        }
      }
    }
  }
  __syncthreads();
  // raw projections -> smem (aliases the x stage)
  float *mr = xs;
#pragma unroll
  for (int r = 0; r < Cf::RT; ++r)
#pragma unroll
    for (int q = 0; q < Cf::RJ; ++q) {
      const int j = jg + Cf::JG * q;
      if (j < FD) mr[(warp * Cf::TPW + tg + Cf::TG * r) * Cf::MRS + j] = acc[r][q];
    }
#pragma unroll
  for (int s = 0; s < Cf::SEG_IT; ++s) {
    float v = ssq_part[s];
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    const int seg = tid + s * Cf::THREADS;
    if ((lane & 7) == 0 && seg < Cf::SEGS) ssq_s[seg >> 3] = v;
  }
  __syncthreads();

  // per-token epilogue
  for (int t = tid; t < TM; t += Cf::THREADS) {
    const int64_t tok = tok0 + t;
    if (tok >= T) continue;
    const float inv = rsqrtf(ssq_s[t] / (float)nC + p.rms_eps);
    inv_rms[tok] = inv;
    float m[FD];
    MHC_UNROLL_N
    for (int j = 0; j < FD; ++j) {
      m[j] = mr[t * Cf::MRS + j] * inv;
      mixes[tok * FD + j] = m[j];
    }
    if constexpr (MODE == HEAD) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float a = __fadd_rn(__fmul_rn(m[i], par[0]), par[3 + i]);
        gate_ws[tok * N + i] = sigmoidf_(a) + p.pre_eps;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float hp = sigmoidf_(__fadd_rn(__fmul_rn(m[i], par[0]), par[3 + i])) + p.pre_eps;
        const float ho = sigmoidf_(__fadd_rn(__fmul_rn(m[N + i], par[1]), par[3 + N + i])) * p.post_mult;
        gate_ws[tok * N + i] = hp;
        if (h_pre) store_dyn(h_pre, coef_dtype, tok * N + i, hp);
        if (h_post) store_dyn(h_post, coef_dtype, tok * N + i, ho);
      }
      if constexpr (MODE == FULL) {
        float L[N * N];
        MHC_UNROLL_N
        for (int k = 0; k < N * N; ++k) L[k] = __fadd_rn(__fmul_rn(m[2 * N + k], par[2]), par[3 + 2 * N + k]);
        if (p.apply_sinkhorn) sinkhorn_fwd<N>(L, p.sk_iters, p.sk_eps);
        if (h_res) {
          MHC_UNROLL_N
          for (int k = 0; k < N * N; ++k) store_dyn(h_res, coef_dtype, tok * N * N + k, L[k]);
        }
      }
    }
  }
}

template <int N, typename Tx, bool VECOK>
__global__ void __launch_bounds__(256)
aggregate_kernel(const Tx *__restrict__ x, const float *__restrict__ w, Tx *__restrict__ z,
                 int64_t T, int C) {
  constexpr int VEC = VECOK ? 16 / sizeof(Tx) : 1;
  const int vpt = C / VEC;
  const int64_t items = T * vpt;
  const int64_t nC = (int64_t)N * C;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = it / vpt;
    const int v = (int)(it - t * vpt);
    float wv[N];
#pragma unroll
    for (int i = 0; i < N; ++i) wv[i] = __ldg(w + t * N + i);
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    const Tx *xr = x + t * nC + (int64_t)v * VEC;
    if constexpr (VECOK) {
      Pack<Tx> pk[N];
#pragma unroll
      for (int i = 0; i < N; ++i) pk[i].raw = ldg_keep(xr + (int64_t)i * C);
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = fmaf(wv[i], pk[i].get(e), acc[e]);
      Pack<Tx> o;
#pragma unroll
      for (int e = 0; e < VEC; ++e) o.set(e, acc[e]);
      stg(z + t * C + (int64_t)v * VEC, o.raw);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) acc[0] = fmaf(wv[i], to_f(xr[(int64_t)i * C]), acc[0]);
      z[t * C + v] = from_f<Tx>(acc[0]);
    }
  }
}

// n == 1 head: out = x * inv_rms (plain unweighted RMSNorm), one warp per token.
template <typename Tx>
__global__ void __launch_bounds__(256)
head1_fwd_kernel(const Tx *__restrict__ x, Tx *__restrict__ out, float *__restrict__ inv_rms,
                 int64_t T, int C, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    const Tx *xr = x + t * C;
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float v = to_f(xr[c]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)C + eps);
    if (lane == 0) inv_rms[t] = inv;
    for (int c = lane; c < C; c += 32) out[t * C + c] = from_f<Tx>(to_f(xr[c]) * inv);
  }
}

template <typename Tx>
__global__ void __launch_bounds__(256)
head1_bwd_kernel(const Tx *__restrict__ x, const float *__restrict__ inv_rms,
                 const Tx *__restrict__ dout, Tx *__restrict__ dx, int64_t T, int C) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    const Tx *xr = x + t * C;
    const Tx *gr = dout + t * C;
    const float inv = inv_rms[t];
    float dot = 0.f;
    for (int c = lane; c < C; c += 32) dot += to_f(xr[c]) * to_f(gr[c]);
    dot = warp_sum(dot);
    const float k = inv * inv * inv * dot / (float)C;
    for (int c = lane; c < C; c += 32) dx[t * C + c] = from_f<Tx>(inv * to_f(gr[c]) - k * to_f(xr[c]));
  }
}

cudaError_t launch_coef_fwd(int mode, int n, int x_dtype, const void *x, int64_t T, int C,
                            const void *phi, const CoefParams &p, void *h_pre, void *h_post,
                            void *h_res, int coef_dtype, float *inv_rms, float *mixes,
                            float *gate_ws, int sm_count, cudaStream_t stream) {
  (void)sm_count;
  return with_mode(mode, [&](auto md) {
    constexpr int MODE = decltype(md)::value;
    return with_n(n, [&](auto nn) {
      constexpr int N = decltype(nn)::value;
      return with_dtype(x_dtype, [&](auto tag) {
        using Tx = decltype(tag);
        using Cf = CoefCfg<N, MODE, Tx>;
        const int nC = n * C;
        const bool vecok = ((int64_t)nC * (int64_t)sizeof(Tx)) % 16 == 0 &&
                           (reinterpret_cast<uintptr_t>(x) & 15) == 0;
        const unsigned grid = (unsigned)((T + Cf::TM - 1) / Cf::TM);
        if (grid == 0) return cudaSuccess;
        auto kern = coef_fwd_kernel<N, MODE, Tx>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)Cf::SMEM);
        if (e != cudaSuccess) return e;
        kern<<<grid, Cf::THREADS, Cf::SMEM, stream>>>(reinterpret_cast<const Tx *>(x), T, nC, phi, p,
                                                      h_pre, h_post, h_res, coef_dtype, inv_rms,
                                                      mixes, gate_ws, vecok);
        return cudaGetLastError();
      });
    });
  });
}

cudaError_t launch_aggregate(int n, int x_dtype, const void *x, const float *w, void *z,
                             int64_t T, int C, cudaStream_t stream) {
  const int sms = device_sm_count();
  return with_n(n, [&](auto nn) {
    constexpr int N = decltype(nn)::value;
    return with_dtype(x_dtype, [&](auto tag) {
      using Tx = decltype(tag);
      constexpr int VEC = 16 / sizeof(Tx);
      const bool vecok = C % VEC == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(z) & 15) == 0;
      const int64_t items = T * (vecok ? C / VEC : C);
      if (items == 0) return cudaSuccess;
      const unsigned grid = grid_for(items, 256, sms, 16);
      if (vecok)
        aggregate_kernel<N, Tx, true><<<grid, 256, 0, stream>>>(
            reinterpret_cast<const Tx *>(x), w, reinterpret_cast<Tx *>(z), T, C);
      else
        aggregate_kernel<N, Tx, false><<<grid, 256, 0, stream>>>(
            reinterpret_cast<const Tx *>(x), w, reinterpret_cast<Tx *>(z), T, C);
      return cudaGetLastError();
    });
  });
}

cudaError_t launch_head1_fwd(int x_dtype, const void *x, void *out, float *inv_rms, int64_t T,
                             int C, float rms_eps, cudaStream_t stream) {
  const int sms = device_sm_count();
  return with_dtype(x_dtype, [&](auto tag) {
    using Tx = decltype(tag);
    if (T == 0) return cudaSuccess;
    const unsigned grid = grid_for(T * 32, 256, sms, 16);
    head1_fwd_kernel<Tx><<<grid, 256, 0, stream>>>(reinterpret_cast<const Tx *>(x),
                                                   reinterpret_cast<Tx *>(out), inv_rms, T, C, rms_eps);
    return cudaGetLastError();
  });
}

cudaError_t launch_head1_bwd(int x_dtype, const void *x, const float *inv_rms, const void *dout,
                             void *dx, int64_t T, int C, cudaStream_t stream) {
  const int sms = device_sm_count();
  return with_dtype(x_dtype, [&](auto tag) {
    using Tx = decltype(tag);
    if (T == 0) return cudaSuccess;
    const unsigned grid = grid_for(T * 32, 256, sms, 16);
    head1_bwd_kernel<Tx><<<grid, 256, 0, stream>>>(reinterpret_cast<const Tx *>(x), inv_rms,
                                                   reinterpret_cast<const Tx *>(dout),
                                                   reinterpret_cast<Tx *>(dx), T, C);
    return cudaGetLastError();
  });
}

}  // namespace mhc
