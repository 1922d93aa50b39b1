// Device-side building blocks shared by the mHC kernels: dtype conversion,
// 16-byte vector packs, the per-token coefficient epilogue and the Sinkhorn-Knopp
// forward / backward in registers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "mhc_b200.h"

// Loops whose trip count grows with the stream count n are fully unrolled only
// for n <= 4 (the register-resident fast case); larger n keeps them rolled so the
// per-token matrices live in local memory instead of exploding code size.
#define MHC_UNROLL_N _Pragma("unroll (N <= 4 ? 256 : 1)")

namespace mhc {

// Variants of the layer.  FULL: H_pre, H_post, H_res (FD = 2n + n^2).
// NOHRES: H_pre, H_post (FD = 2n).  HEAD: one gate set (FD = n).
enum Mode { FULL = 0, NOHRES = 1, HEAD = 2 };

template <int N, int MODE>
struct Dims {
  static constexpr int FD = MODE == FULL ? 2 * N + N * N : (MODE == NOHRES ? 2 * N : N);
};

// ---------------------------------------------------------------------------
// scalar conversions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// Load / store one element of a runtime-typed buffer (used for the small
// per-token and per-parameter tensors whose dtype follows the caller).
__device__ __forceinline__ float load_dyn(const void *p, int dtype, int64_t i) {
  switch (dtype) {
    case MHC_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    case MHC_F16: return __half2float(reinterpret_cast<const __half *>(p)[i]);
    default: return reinterpret_cast<const float *>(p)[i];
  }
}
__device__ __forceinline__ void store_dyn(void *p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case MHC_BF16: reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
    case MHC_F16: reinterpret_cast<__half *>(p)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<float *>(p)[i] = v; break;
  }
}

// ---------------------------------------------------------------------------
// 16-byte packs: VEC elements of T in one uint4
// ---------------------------------------------------------------------------
template <typename T>
struct Pack {
  static constexpr int VEC = 16 / sizeof(T);
  uint4 raw;
  __device__ __forceinline__ float get(int i) const {
    const T *e = reinterpret_cast<const T *>(&raw);
    return to_f(e[i]);
  }
  __device__ __forceinline__ void set(int i, float v) {
    T *e = reinterpret_cast<T *>(&raw);
    e[i] = from_f<T>(v);
  }
  __device__ __forceinline__ void to_float(float (&o)[VEC]) const {
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = get(i);
  }
};

// Read-only vector loads.  `ldg_stream` marks data that is read exactly once
// (evict-first), `ldg_keep` data another kernel re-reads soon.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  return __ldcs(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ uint4 ldg_keep(const void *p) {
  return __ldg(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ void stg_stream(void *p, uint4 v) {
  __stcs(reinterpret_cast<uint4 *>(p), v);
}
__device__ __forceinline__ void stg(void *p, uint4 v) {
  *reinterpret_cast<uint4 *>(p) = v;
}

// V elements of T as fp32, read once (streaming).  V*sizeof(T) is 8 or 16 bytes.
template <typename T, int V>
__device__ __forceinline__ void load_vec_stream(const T *p, float (&o)[V]) {
  constexpr int BYTES = V * (int)sizeof(T);
  static_assert(BYTES == 16 || BYTES == 8, "vector width");
  if constexpr (BYTES == 16) {
    uint4 r = __ldcs(reinterpret_cast<const uint4 *>(p));
    const T *e = reinterpret_cast<const T *>(&r);
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = to_f(e[i]);
  } else {
    uint2 r = __ldcs(reinterpret_cast<const uint2 *>(p));
    const T *e = reinterpret_cast<const T *>(&r);
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = to_f(e[i]);
  }
}

template <typename T, int V>
__device__ __forceinline__ void store_vec_stream(T *p, const float (&v)[V]) {
  constexpr int BYTES = V * (int)sizeof(T);
  static_assert(BYTES == 16 || BYTES == 8, "vector width");
  if constexpr (BYTES == 16) {
    uint4 r;
    T *e = reinterpret_cast<T *>(&r);
#pragma unroll
    for (int i = 0; i < V; ++i) e[i] = from_f<T>(v[i]);
    __stcs(reinterpret_cast<uint4 *>(p), r);
  } else {
    uint2 r;
    T *e = reinterpret_cast<T *>(&r);
#pragma unroll
    for (int i = 0; i < V; ++i) e[i] = from_f<T>(v[i]);
    __stcs(reinterpret_cast<uint2 *>(p), r);
  }
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the previous kernel of the stream is still
// running; it must call grid_dep_wait() before reading anything an earlier
// kernel wrote (the wait returns at once when there is no such kernel).
// grid_dep_launch() lets the next kernel of the stream start early.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Hardware reciprocal (rcp.approx.ftz.f32, within 1 ulp for normal inputs).
// The reference's Triton kernels divide with Triton's default fp32 division,
// which is approximate as well (model/mhc_fused.py:86-91, 210, 252-253); the
// IEEE-rounded reciprocal is a multi-instruction sequence that made the
// 20-iteration Sinkhorn about 3.5x slower.
__device__ __forceinline__ float fast_rcp(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float sigmoidf_(float v) { return fast_rcp(1.0f + __expf(-v)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Sinkhorn-Knopp on an N x N matrix held in registers (row-major p[i*N+j]).
// Same step order as the reference: softmax(-1) + eps, column normalisation,
// then (iters - 1) x [row, column] normalisations, each x / (sum + eps).  Each
// normalisation takes one hardware reciprocal of (sum + eps) per row / column
// and multiplies by it (within 2 ulp of a per-element division).
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ void sk_row_norm(float (&p)[N * N], float eps) {
MHC_UNROLL_N
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) s += p[i * N + j];
    const float r = fast_rcp(s + eps);
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) p[i * N + j] = p[i * N + j] * r;
  }
}

template <int N>
__device__ __forceinline__ void sk_col_norm(float (&p)[N * N], float eps) {
MHC_UNROLL_N
  for (int j = 0; j < N; ++j) {
    float s = 0.f;
MHC_UNROLL_N
    for (int i = 0; i < N; ++i) s += p[i * N + j];
    const float r = fast_rcp(s + eps);
MHC_UNROLL_N
    for (int i = 0; i < N; ++i) p[i * N + j] = p[i * N + j] * r;
  }
}

// Row softmax; returns the probabilities (without the +eps).
template <int N>
__device__ __forceinline__ void sk_softmax_rows(float (&p)[N * N]) {
MHC_UNROLL_N
  for (int i = 0; i < N; ++i) {
    float mx = p[i * N];
MHC_UNROLL_N
    for (int j = 1; j < N; ++j) mx = fmaxf(mx, p[i * N + j]);
    float s = 0.f;
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) {
      const float e = __expf(p[i * N + j] - mx);
      p[i * N + j] = e;
      s += e;
    }
    const float r = fast_rcp(s);
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) p[i * N + j] = p[i * N + j] * r;
  }
}

template <int N>
__device__ __forceinline__ void sinkhorn_fwd(float (&p)[N * N], int iters, float eps) {
  sk_softmax_rows<N>(p);
MHC_UNROLL_N
  for (int k = 0; k < N * N; ++k) p[k] += eps;
  sk_col_norm<N>(p, eps);
  for (int it = 1; it < iters; ++it) {
    sk_row_norm<N>(p, eps);
    sk_col_norm<N>(p, eps);
  }
}

// Backward of x -> x / (rowsum(x) + eps) given the step's input `a` and its
// output `b`: da[i][j] = (db[i][j] - sum_j' db[i][j'] b[i][j']) / (r_i + eps).
template <int N>
__device__ __forceinline__ void sk_row_norm_bwd(const float (&a)[N * N], float (&g)[N * N], float eps) {
MHC_UNROLL_N
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) s += a[i * N + j];
    const float r = fast_rcp(s + eps);
    float dot = 0.f;
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) dot += g[i * N + j] * (a[i * N + j] * r);
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) g[i * N + j] = (g[i * N + j] - dot) * r;
  }
}

template <int N>
__device__ __forceinline__ void sk_col_norm_bwd(const float (&a)[N * N], float (&g)[N * N], float eps) {
MHC_UNROLL_N
  for (int j = 0; j < N; ++j) {
    float s = 0.f;
MHC_UNROLL_N
    for (int i = 0; i < N; ++i) s += a[i * N + j];
    const float r = fast_rcp(s + eps);
    float dot = 0.f;
MHC_UNROLL_N
    for (int i = 0; i < N; ++i) dot += g[i * N + j] * (a[i * N + j] * r);
MHC_UNROLL_N
    for (int i = 0; i < N; ++i) g[i * N + j] = (g[i * N + j] - dot) * r;
  }
}

// Sinkhorn backward by recompute with checkpoints.  The forward is
// A_0 = softmax(m) + eps, B_t = colnorm(A_t), A_{t+1} = rownorm(B_t) and the
// output is B_{steps-1}.  Only every K-th state is kept in `traj` (caller
// scratch, sk_ckpt_count(N, iters) matrices of N*N floats, consecutive floats
// `tstride` apart so a block can interleave threads): checkpoint 0 is A_0 and
// checkpoint c >= 1 is B_{cK-1}.  The reverse sweep recomputes each segment of
// K states into registers from its checkpoint with the same operations in the
// same order, so every recomputed state equals the forward one bit for bit.
// On entry `m` holds the logits and `g` the gradient w.r.t. the output; on
// exit `g` holds the gradient w.r.t. the logits.
template <int N>
__host__ __device__ constexpr int sk_ckpt_every() { return N <= 4 ? 4 : 1; }

__host__ __device__ inline int sk_ckpt_count(int n, int iters) {
  const int steps = iters < 1 ? 1 : iters;
  const int k = n <= 4 ? 4 : 1;
  return (steps + k - 1) / k;
}

template <int N>
__device__ void sinkhorn_bwd(const float (&m)[N * N], float (&g)[N * N], int iters, float eps,
                             float *traj, int tstride) {
  constexpr int K = sk_ckpt_every<N>();
  constexpr int NN = N * N;
  const int steps = iters < 1 ? 1 : iters;
  {
    float p[NN];
MHC_UNROLL_N
    for (int k = 0; k < NN; ++k) p[k] = m[k];
    sk_softmax_rows<N>(p);
MHC_UNROLL_N
    for (int k = 0; k < NN; ++k) {
      p[k] += eps;  // A_0
      traj[k * tstride] = p[k];
    }
    for (int it = 0; it + 1 < steps; ++it) {
      sk_col_norm<N>(p, eps);  // B_it
      if ((it + 1) % K == 0) {
        float *slot = traj + (size_t)((it + 1) / K) * NN * tstride;
MHC_UNROLL_N
        for (int k = 0; k < NN; ++k) slot[k * tstride] = p[k];
      }
      sk_row_norm<N>(p, eps);  // A_{it+1}
    }
  }
  // reverse sweep, one segment of K states at a time
  for (int c = (steps + K - 1) / K - 1; c >= 0; --c) {
    const int base = c * K;
    const float *slot = traj + (size_t)c * NN * tstride;
    float a[K][NN];  // A_base .. A_{base+K-1}
MHC_UNROLL_N
    for (int k = 0; k < NN; ++k) a[0][k] = slot[k * tstride];
    if (c > 0) sk_row_norm<N>(a[0], eps);  // A_base = rownorm(B_{base-1})
    // states past the last step are computed too (cheaper than a branch that
    // keeps `a` out of registers) and never used
#pragma unroll
    for (int u = 1; u < K; ++u) {
MHC_UNROLL_N
      for (int k = 0; k < NN; ++k) a[u][k] = a[u - 1][k];
      sk_col_norm<N>(a[u], eps);
      sk_row_norm<N>(a[u], eps);
    }
#pragma unroll
    for (int u = K - 1; u >= 1; --u) {
      if (base + u < steps) {
        sk_col_norm_bwd<N>(a[u], g, eps);  // through B_it = colnorm(A_it)
        float b[NN];                       // B_{it-1} = colnorm(A_{it-1})
MHC_UNROLL_N
        for (int k = 0; k < NN; ++k) b[k] = a[u - 1][k];
        sk_col_norm<N>(b, eps);
        sk_row_norm_bwd<N>(b, g, eps);     // through A_it = rownorm(B_{it-1})
      }
    }
    sk_col_norm_bwd<N>(a[0], g, eps);      // the segment's first state
    if (c > 0) {
      float b[NN];                         // B_{base-1}: the checkpoint itself
MHC_UNROLL_N
      for (int k = 0; k < NN; ++k) b[k] = slot[k * tstride];
      sk_row_norm_bwd<N>(b, g, eps);
    }
  }
  // softmax backward (dA_0 = dS_0)
  float s0[NN];
MHC_UNROLL_N
  for (int k = 0; k < NN; ++k) s0[k] = m[k];
  sk_softmax_rows<N>(s0);
MHC_UNROLL_N
  for (int i = 0; i < N; ++i) {
    float dot = 0.f;
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) dot += g[i * N + j] * s0[i * N + j];
MHC_UNROLL_N
    for (int j = 0; j < N; ++j) g[i * N + j] = s0[i * N + j] * (g[i * N + j] - dot);
  }
}

// ---------------------------------------------------------------------------
// Layer constants handed to the kernels
// ---------------------------------------------------------------------------
struct CoefArgs {
  const void *alpha_pre, *bias_pre, *alpha_post, *bias_post, *alpha_res, *bias_res;
  int param_dtype;
  float post_mult, pre_eps, rms_eps, sk_eps;
  int apply_sinkhorn, sk_iters;
};

}  // namespace mhc
