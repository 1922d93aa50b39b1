// Backward of the coefficient stage + pre-aggregate (generic CUDA-core path).
//
// Launches, no atomics (deterministic):
//  K1a coef_dots_kernel: per token, the dot products <dz, x_i>: a streaming
//     pass over x and dz, one warp per token with every load of a round in
//     flight before the first FMA.
//  K1 coef_bwd_kernel  : one thread per token runs the gate / Sinkhorn
//     backward (the Sinkhorn trajectory is recomputed, every 4th state kept in
//     shared memory) and
//     writes dm = dL/dmixes, the RMS-backward row coefficient and the
//     aggregation weights.  Per-block sums of the alpha / bias gradients go to
//     the workspace.  (Without K1a's dots it computes them itself, one warp per
//     token.)
//  K2 dx_dphi_kernel   : grid (k-chunks x token splits).  For its k-chunk a block
//     keeps phi^T in shared memory and, per 32-token tile (dm scaled by the
//     token's 1/rms when staged),
//       dx = (inv*dm) @ phi^T - rowb*x + w_i*dz + dx_add
//     and accumulates dphi[k, :] += x[t,k] * (inv*dm)[t,:] in registers
//     (register-tiled: 2 columns x up to 16 projection columns per thread,
//     the tile's tokens split over warp groups, whose partials are summed in
//     a fixed order at the end).
//  K3 reduce kernels   : fixed-order sums of the per-split dphi partials and of
//     the per-block alpha / bias partials.
#include "mhc_device.cuh"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"
#include "mhc_sm100.cuh"

namespace mhc {

static inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static inline int fd_of(int mode, int n) {
  return mode == FULL ? 2 * n + n * n : (mode == NOHRES ? 2 * n : n);
}

// number of per-block coefficient partials: 3 alphas + FD biases
static inline int ng_of(int mode, int n) { return 3 + fd_of(mode, n); }

static inline int k2_kc_of(int fd) { return fd <= 96 ? 64 : 16; }

PreBwdPlan plan_pre_bwd(int mode, int n, int64_t T, int C, int sk_iters, int sm_count) {
  PreBwdPlan p{};
  p.fd = fd_of(mode, n);
  const int64_t nC = (int64_t)n * C;
  int tokens = 32;
  if (mode == FULL) {
    const size_t per = (size_t)sk_ckpt_count(n, sk_iters) * n * n * 4;
    const size_t budget = 96 * 1024;
    int t = (int)(budget / per);
    if (t < 1) t = (per <= 200 * 1024) ? 1 : 0;  // 0 => unsupported
    if (t < tokens) tokens = t;
  }
  p.k1_tokens = tokens;
  p.k1_blocks = tokens > 0 ? (int)((T + tokens - 1) / tokens) : 0;
  p.k2_kc = k2_kc_of(p.fd);
  p.k2_kblocks = (int)((nC + p.k2_kc - 1) / p.k2_kc);
  const int64_t tiles = (T + 31) / 32;
  int64_t target = (int64_t)(sm_count > 0 ? sm_count : 148) * 8 / (p.k2_kblocks > 0 ? p.k2_kblocks : 1);
  if (target < 1) target = 1;
  if (target > tiles) target = tiles;
  if (target > 64) target = 64;
  if (target < 1) target = 1;
  p.k2_tsplits = (int)target;
  size_t off = 0;
  p.off_dm = off;        off = align256(off + (size_t)T * p.fd * 4);
  p.off_rowb = off;      off = align256(off + (size_t)T * 4);
  p.off_gate = off;      off = align256(off + (size_t)T * n * 4);
  p.off_dphi_part = off; off = align256(off + (size_t)p.k2_tsplits * nC * p.fd * 4);
  p.off_coef_part = off; off = align256(off + (size_t)(p.k1_blocks > 0 ? p.k1_blocks : 1) * ng_of(mode, n) * 4);
  p.off_dots = off;      off = align256(off + (size_t)T * n * 4);
  p.total = off;
  return p;
}

// ---------------------------------------------------------------------------
// K1a
// ---------------------------------------------------------------------------
// dots[t, i] = <dz[t, :], x[t, i*C : (i+1)*C]>.  One warp per token; a round
// takes U 16-byte vectors per lane of dz and of every stream (5 U loads in
// flight per lane at n = 4) before any FMA.  x streams through L2 (evict
// first); dz keeps the default policy, the dx kernel reads it again.
template <int N, typename Tx>
__global__ void __launch_bounds__(256)
coef_dots_kernel(const Tx *__restrict__ x, const Tx *__restrict__ dz, int64_t T, int C,
                 float *__restrict__ dots, bool vecok) {
  constexpr int VEC = 16 / sizeof(Tx);
  constexpr int U = N <= 4 ? 3 : 1;  // rounds of loads stay within ~64 registers
  const int lane = threadIdx.x & 31;
  const int64_t wg = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nC = (int64_t)N * C;
  for (int64_t tok = wg; tok < T; tok += nw) {
    float d[N];
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = 0.f;
    const Tx *xr = x + tok * nC;
    const Tx *gr = dz + tok * C;
    if (vecok) {
      const int vpt = C / VEC;
      for (int v0 = lane; v0 < vpt; v0 += 32 * U) {
        uint4 g[U], xv[N][U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int v = v0 + u * 32;
          if (v < vpt) {
            g[u] = ldg_keep(gr + (int64_t)v * VEC);
#pragma unroll
            for (int i = 0; i < N; ++i) xv[i][u] = ldg_stream(xr + (int64_t)i * C + (int64_t)v * VEC);
          } else {
            g[u] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int i = 0; i < N; ++i) xv[i][u] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          Pack<Tx> pg;
          pg.raw = g[u];
          float gf[VEC];
          pg.to_float(gf);
#pragma unroll
          for (int i = 0; i < N; ++i) {
            Pack<Tx> px;
            px.raw = xv[i][u];
#pragma unroll
            for (int e = 0; e < VEC; ++e) d[i] = fmaf(gf[e], px.get(e), d[i]);
          }
        }
      }
    } else {
      for (int c = lane; c < C; c += 32) {
        const float g = to_f(gr[c]);
#pragma unroll
        for (int i = 0; i < N; ++i) d[i] = fmaf(g, to_f(xr[(int64_t)i * C + c]), d[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = warp_sum(d[i]);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < N; ++i) dots[tok * N + i] = d[i];
    }
  }
}

// ---------------------------------------------------------------------------
// K1
// ---------------------------------------------------------------------------
template <int N, int MODE, typename Tx>
__global__ void __launch_bounds__(256)
coef_bwd_kernel(const Tx *__restrict__ x, int64_t T, int C, CoefParams p,
                const float *__restrict__ inv_rms, const float *__restrict__ mixes,
                const Tx *__restrict__ dz, const void *dh_pre, const void *dh_post,
                const void *dh_res, int coef_dtype, int TB,
                float *__restrict__ dm_ws, float *__restrict__ rowb_ws, float *__restrict__ gate_ws,
                float *__restrict__ coef_part, bool vecok, const float *__restrict__ dots_in) {
  constexpr int FD = Dims<N, MODE>::FD;
  constexpr int NG = 3 + FD;
  constexpr int NPAR = 3 + 2 * N + N * N;
  constexpr int VEC = 16 / sizeof(Tx);
  extern __shared__ float4 smem4[];
  float *smem = reinterpret_cast<float *>(smem4);
  float *par = smem;                     // [NPAR]
  float *dots = par + NPAR;              // [TB][N]
  float *pg = dots + TB * N;             // [TB][NG]
  float *traj = pg + TB * NG;            // [checkpoints][N*N][TB]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tok0 = (int64_t)blockIdx.x * TB;
  const int64_t nC = (int64_t)N * C;
  for (int i = tid; i < NPAR; i += blockDim.x) {
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

  // phase 1: <dz, x_i> per token, one warp per token (unless K1a made them)
  const int vpt = vecok ? C / VEC : C;
  for (int t = warp; !dots_in && t < TB; t += (blockDim.x >> 5)) {
    const int64_t tok = tok0 + t;
    float d[N];
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = 0.f;
    if (tok < T) {
      const Tx *xr = x + tok * nC;
      const Tx *gr = dz + tok * C;
      for (int v = lane; v < vpt; v += 32) {
        const int64_t off = vecok ? (int64_t)v * VEC : v;
        if (vecok) {
          Pack<Tx> pgz;
          pgz.raw = ldg_keep(gr + off);
          float g[VEC];
          pgz.to_float(g);
#pragma unroll
          for (int i = 0; i < N; ++i) {
            Pack<Tx> px;
            px.raw = ldg_keep(xr + (int64_t)i * C + off);
#pragma unroll
            for (int e = 0; e < VEC; ++e) d[i] = fmaf(g[e], px.get(e), d[i]);
          }
        } else {
          const float g = to_f(gr[off]);
#pragma unroll
          for (int i = 0; i < N; ++i) d[i] = fmaf(g, to_f(xr[(int64_t)i * C + off]), d[i]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = warp_sum(d[i]);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < N; ++i) dots[t * N + i] = d[i];
    }
  }
  __syncthreads();

  // phase 2: one thread per token
  for (int t = tid; t < TB; t += blockDim.x) {
    const int64_t tok = tok0 + t;
    float *g_out = pg + t * NG;
    for (int k = 0; k < NG; ++k) g_out[k] = 0.f;
    if (tok >= T) continue;
    float m[FD], dm[FD];
    MHC_UNROLL_N
    for (int j = 0; j < FD; ++j) {
      m[j] = mixes[tok * FD + j];
      dm[j] = 0.f;
    }
    const float inv = inv_rms[tok];
    if constexpr (MODE == HEAD) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float s = sigmoidf_(__fadd_rn(__fmul_rn(m[i], par[0]), par[3 + i]));
        gate_ws[tok * N + i] = s + p.pre_eps;
        const float da = (dots_in ? dots_in[tok * N + i] : dots[t * N + i]) * s * (1.f - s);
        dm[i] = par[0] * da;
        g_out[0] += da * m[i];
        g_out[3 + i] = da;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float sp = sigmoidf_(__fadd_rn(__fmul_rn(m[i], par[0]), par[3 + i]));
        gate_ws[tok * N + i] = sp + p.pre_eps;
        float gp = dots_in ? dots_in[tok * N + i] : dots[t * N + i];
        if (dh_pre) gp += load_dyn(dh_pre, coef_dtype, tok * N + i);
        const float dpre = gp * sp * (1.f - sp);
        dm[i] = par[0] * dpre;
        g_out[0] += dpre * m[i];
        g_out[3 + i] = dpre;
        const float so = sigmoidf_(__fadd_rn(__fmul_rn(m[N + i], par[1]), par[3 + N + i]));
        const float go = dh_post ? load_dyn(dh_post, coef_dtype, tok * N + i) : 0.f;
        const float dpost = go * so * (1.f - so) * p.post_mult;
        dm[N + i] = par[1] * dpost;
        g_out[1] += dpost * m[N + i];
        g_out[3 + N + i] = dpost;
      }
      if constexpr (MODE == FULL) {
        float gl[N * N];
        MHC_UNROLL_N
        for (int k = 0; k < N * N; ++k) gl[k] = dh_res ? load_dyn(dh_res, coef_dtype, tok * (N * N) + k) : 0.f;
        if (p.apply_sinkhorn && dh_res) {
          float L[N * N];
          MHC_UNROLL_N
          for (int k = 0; k < N * N; ++k) L[k] = __fadd_rn(__fmul_rn(m[2 * N + k], par[2]), par[3 + 2 * N + k]);
          sinkhorn_bwd<N>(L, gl, p.sk_iters, p.sk_eps, traj + t, TB);
        }
        MHC_UNROLL_N
        for (int k = 0; k < N * N; ++k) {
          dm[2 * N + k] = par[2] * gl[k];
          g_out[2] += gl[k] * m[2 * N + k];
          g_out[3 + 2 * N + k] = gl[k];
        }
      }
    }
    float s = 0.f;
    MHC_UNROLL_N
    for (int j = 0; j < FD; ++j) {
      s = fmaf(dm[j], m[j], s);
      dm_ws[tok * FD + j] = dm[j];
    }
    rowb_ws[tok] = inv * inv * s / (float)nC;
  }
  __syncthreads();
  // phase 3: fixed-order per-block sums of the coefficient gradients
  for (int k = tid; k < NG; k += blockDim.x) {
    float a = 0.f;
    for (int t = 0; t < TB; ++t) a += pg[t * NG + k];
    coef_part[(int64_t)blockIdx.x * NG + k] = a;
  }
}

// ---------------------------------------------------------------------------
// K2
// ---------------------------------------------------------------------------
// Shared-memory floats the kernel below needs (the staging buffers, or the
// dphi reduction over the token groups at the end, whichever is larger).
template <int N, int MODE>
struct DxDphiCfg {
  static constexpr int FD = Dims<N, MODE>::FD;
  static constexpr int KC = FD <= 96 ? 64 : 16;    // columns k per block
  static constexpr int TT = 32;                    // tokens per tile
  static constexpr int XSW = KC;                   // x tile row stride (floats)
  // dphi register tiling (KC = 64): lane = column pair, warp = (j group, token group)
  static constexpr bool RT = KC == 64;
  static constexpr int JH = FD <= 16 ? 1 : (FD <= 32 ? 2 : (FD <= 64 ? 4 : 8));
  static constexpr int JR = (FD + JH - 1) / JH;    // projection columns per thread
  static constexpr int TG = 8 / JH;                // token groups
  static constexpr int STAGE = FD * KC + TT * XSW + TT * FD + 2 * TT + TT * N;
  static constexpr int FDP = FD + 1;              // reduction row stride (odd: fewer bank conflicts)
  static constexpr int RED = RT ? TG * KC * FDP : 0;
  static constexpr int SMEM_FLOATS = STAGE > RED ? STAGE : RED;
};

template <int N, int MODE, typename Tx>
__global__ void __launch_bounds__(256)
dx_dphi_kernel(const Tx *__restrict__ x, int64_t T, int C, const void *__restrict__ phi, int pdt,
               const float *__restrict__ inv_rms, const float *__restrict__ dm_ws,
               const float *__restrict__ rowb_ws, const float *__restrict__ gate_ws,
               const Tx *__restrict__ dz, const Tx *__restrict__ dx_add, Tx *__restrict__ dx,
               float *__restrict__ dphi_part, int tsplits, bool xvec) {
  using Cf = DxDphiCfg<N, MODE>;
  constexpr int FD = Cf::FD, KC = Cf::KC, TT = Cf::TT, XSW = Cf::XSW;
  constexpr int JGRP = 256 / KC;               // token rows of the dx pass per column
  constexpr int RR = TT / JGRP;                // dx rows per thread
  constexpr int RJ = (FD + JGRP - 1) / JGRP;   // dphi columns per thread without the tiling
  constexpr int JH = Cf::JH, JR = Cf::JR, TG = Cf::TG;
  extern __shared__ float4 smem4[];
  float *smem = reinterpret_cast<float *>(smem4);
  float *psT = smem;                  // [FD][KC]
  float *xs = psT + FD * KC;          // [TT][XSW]
  float *dms = xs + TT * XSW;         // [TT][FD]: inv * dm
  float *trow = dms + TT * FD;        // [TT]
  float *tgate = trow + 2 * TT;       // [TT][N]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kk = tid % KC, jgrp = tid / KC;
  const int64_t nC = (int64_t)N * C;
  const int64_t k0 = (int64_t)blockIdx.x * KC;
  const int64_t kglob = k0 + kk;
  const bool kvalid = kglob < nC;
  const int stream_i = kvalid ? (int)(kglob / C) : 0;
  const int cc = kvalid ? (int)(kglob - (int64_t)stream_i * C) : 0;
  // dphi tiling: columns 2*lane, 2*lane+1; projection columns jh*JR + q; tokens tg + TG*u
  const int jh = warp % JH, tg = warp / JH;

  for (int e = tid; e < KC * FD; e += blockDim.x) {
    const int r = e / FD, j = e - r * FD;
    float v = 0.f;
    if (k0 + r < nC) v = load_dyn(phi, pdt, (k0 + r) * FD + j);
    psT[j * KC + r] = v;
  }

  // token range of this split
  const int64_t tiles = (T + TT - 1) / TT;
  const int64_t tiles_per = (tiles + tsplits - 1) / tsplits;
  const int64_t tile_beg = (int64_t)blockIdx.y * tiles_per;
  int64_t tile_end = tile_beg + tiles_per;
  if (tile_end > tiles) tile_end = tiles;

  float acc[Cf::RT ? 2 * JR : RJ];
#pragma unroll
  for (int q = 0; q < (Cf::RT ? 2 * JR : RJ); ++q) acc[q] = 0.f;
  // this thread's phi column (k = kglob), the same for every tile: in
  // registers for the usual projection widths, else read from shared memory
  constexpr bool PREG = FD <= 32;
  __syncthreads();
  float pcol[PREG ? FD : 1];
  if constexpr (PREG) {
#pragma unroll
    for (int j = 0; j < FD; ++j) pcol[j] = psT[j * KC + kk];
  }

  for (int64_t tile = tile_beg; tile < tile_end; ++tile) {
    const int64_t t0 = tile * TT;
    __syncthreads();
    if (xvec) {
      // 4-byte elements, nC % 4 == 0, 16-byte aligned x: 16-byte vectors
      constexpr int V4 = TT * KC / 4;
      for (int e = tid; e < V4; e += blockDim.x) {
        const int r = e / (KC / 4), c = (e - r * (KC / 4)) * 4;
        const int64_t tok = t0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tok < T && k0 + c < nC) v = __ldg(reinterpret_cast<const float4 *>(x + tok * nC + k0 + c));
        *reinterpret_cast<float4 *>(xs + r * XSW + c) = v;
      }
    } else {
      for (int e = tid; e < TT * KC; e += blockDim.x) {
        const int r = e / KC, c = e - r * KC;
        const int64_t tok = t0 + r;
        float v = 0.f;
        if (tok < T && k0 + c < nC) v = to_f(x[tok * nC + k0 + c]);
        xs[r * XSW + c] = v;
      }
    }
    // dm scaled by the token's 1/rms: dx = (inv dm) . phi^T, dphi = x^T (inv dm)
    for (int e = tid; e < TT * FD; e += blockDim.x) {
      const int r = e / FD;
      const int64_t tok = t0 + r;
      dms[e] = tok < T ? dm_ws[t0 * FD + e] * inv_rms[tok] : 0.f;
    }
    for (int e = tid; e < TT; e += blockDim.x) {
      const int64_t tok = t0 + e;
      trow[e] = tok < T ? rowb_ws[tok] : 0.f;
    }
    for (int e = tid; e < TT * N; e += blockDim.x) {
      const int64_t tok = t0 + e / N;
      tgate[e] = tok < T ? gate_ws[t0 * N + e] : 0.f;
    }
    __syncthreads();
    // dx for rows jgrp + JGRP*r, column kk.  Every global load of the tile's
    // rows is issued before the arithmetic, so their latencies overlap.
    if (kvalid) {
      float dzv[RR], dav[RR];
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        const int64_t tok = t0 + jgrp + JGRP * r;
        dzv[r] = tok < T ? to_f(dz[tok * C + cc]) : 0.f;
        dav[r] = (dx_add && tok < T) ? to_f(dx_add[tok * nC + kglob]) : 0.f;
      }
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        const int row = jgrp + JGRP * r;
        const int64_t tok = t0 + row;
        if (tok >= T) continue;
        float a = 0.f;
        if constexpr (!PREG) {
#pragma unroll 8
          for (int j = 0; j < FD; ++j) a = fmaf(dms[row * FD + j], psT[j * KC + kk], a);
        } else if constexpr (FD % 4 == 0) {
#pragma unroll
          for (int j = 0; j < FD; j += 4) {
            const float4 d4 = *reinterpret_cast<const float4 *>(dms + row * FD + j);  // one row: broadcast
            a = fmaf(d4.x, pcol[j], a);
            a = fmaf(d4.y, pcol[j + 1], a);
            a = fmaf(d4.z, pcol[j + 2], a);
            a = fmaf(d4.w, pcol[j + 3], a);
          }
        } else {
#pragma unroll
          for (int j = 0; j < FD; ++j) a = fmaf(dms[row * FD + j], pcol[j], a);
        }
        float v = a - trow[row] * xs[row * XSW + kk];
        v = fmaf(tgate[row * N + stream_i], dzv[r], v);
        v += dav[r];
        dx[tok * nC + kglob] = from_f<Tx>(v);
      }
    }
    if constexpr (Cf::RT) {
      // dphi[k, j] += sum_t x[t, k] (inv dm)[t, j]: 2 columns x JR projection
      // columns per thread, the tile's tokens split over TG warp groups (one
      // 8-byte x load and JR/4 broadcast dm loads per 2*JR FMAs)
#pragma unroll 2
      for (int u = 0; u < TT / TG; ++u) {
        const int t = tg + TG * u;
        const float2 x2 = *reinterpret_cast<const float2 *>(xs + t * XSW + 2 * lane);
        const float *drow = dms + t * FD + jh * JR;
        if constexpr (JR % 4 == 0 && FD % 4 == 0) {
#pragma unroll
          for (int q = 0; q < JR; q += 4) {
            const float4 d4 = *reinterpret_cast<const float4 *>(drow + q);
            acc[q] = fmaf(x2.x, d4.x, acc[q]);
            acc[q + 1] = fmaf(x2.x, d4.y, acc[q + 1]);
            acc[q + 2] = fmaf(x2.x, d4.z, acc[q + 2]);
            acc[q + 3] = fmaf(x2.x, d4.w, acc[q + 3]);
            acc[JR + q] = fmaf(x2.y, d4.x, acc[JR + q]);
            acc[JR + q + 1] = fmaf(x2.y, d4.y, acc[JR + q + 1]);
            acc[JR + q + 2] = fmaf(x2.y, d4.z, acc[JR + q + 2]);
            acc[JR + q + 3] = fmaf(x2.y, d4.w, acc[JR + q + 3]);
          }
        } else if constexpr (JR % 2 == 0 && FD % 2 == 0) {
#pragma unroll
          for (int q = 0; q < JR; q += 2) {
            const float2 d2 = *reinterpret_cast<const float2 *>(drow + q);
            acc[q] = fmaf(x2.x, d2.x, acc[q]);
            acc[q + 1] = fmaf(x2.x, d2.y, acc[q + 1]);
            acc[JR + q] = fmaf(x2.y, d2.x, acc[JR + q]);
            acc[JR + q + 1] = fmaf(x2.y, d2.y, acc[JR + q + 1]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < JR; ++q) {
            if (jh * JR + q < FD) {
              const float d = drow[q];
              acc[q] = fmaf(x2.x, d, acc[q]);
              acc[JR + q] = fmaf(x2.y, d, acc[JR + q]);
            }
          }
        }
      }
    } else {
      // dphi[k, j] += sum_t x[t, k] (inv dm)[t, j] for this thread's
      // consecutive columns j = jgrp * RJ + q
#pragma unroll 4
      for (int t = 0; t < TT; ++t) {
        const float xv = xs[t * XSW + kk];
#pragma unroll
        for (int q = 0; q < RJ; ++q) {
          const int j = jgrp * RJ + q;
          if (j < FD) acc[q] = fmaf(xv, dms[t * FD + j], acc[q]);
        }
      }
    }
  }
  if constexpr (Cf::RT) {
    // the token groups' partials, summed in a fixed order (deterministic)
    __syncthreads();
    constexpr int FDP = Cf::FDP;
    float *red = smem;  // [TG][KC][FDP]
#pragma unroll
    for (int q = 0; q < JR; ++q) {
      const int j = jh * JR + q;
      if (j < FD) {
        red[(tg * KC + 2 * lane) * FDP + j] = acc[q];
        red[(tg * KC + 2 * lane + 1) * FDP + j] = acc[JR + q];
      }
    }
    __syncthreads();
    for (int e = tid; e < KC * FD; e += blockDim.x) {
      const int col = e / FD, j = e - col * FD;
      if (k0 + col >= nC) continue;
      float v = red[col * FDP + j];
#pragma unroll
      for (int g = 1; g < TG; ++g) v += red[(g * KC + col) * FDP + j];
      dphi_part[((int64_t)blockIdx.y * nC + k0) * FD + e] = v;
    }
  } else if (kvalid) {
    float *dst = dphi_part + ((int64_t)blockIdx.y * nC + kglob) * FD;
#pragma unroll
    for (int q = 0; q < RJ; ++q) {
      const int j = jgrp * RJ + q;
      if (j < FD) dst[j] = acc[q];
    }
  }
}

// 16-byte asynchronous global -> shared copy; `bytes` < 16 fills the rest of
// the 16 bytes with zeros (0: nothing is read, `src` need only be a valid
// address).
__device__ __forceinline__ void cp_async16(void *dst, const void *src, int bytes) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N_>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N_) : "memory"); }

template <typename Tx>
__device__ __forceinline__ float2 ld2f(const Tx *p) {
  if constexpr (sizeof(Tx) == 4) {
    return *reinterpret_cast<const float2 *>(p);
  } else {
    return make_float2(to_f(p[0]), to_f(p[1]));
  }
}

template <typename Tx>
__device__ __forceinline__ void st2(Tx *p, float a, float b) {
  if constexpr (sizeof(Tx) == 4) {
    *reinterpret_cast<float2 *>(p) = make_float2(a, b);
  } else {
    Tx h[2] = {from_f<Tx>(a), from_f<Tx>(b)};
    *reinterpret_cast<uint32_t *>(p) = *reinterpret_cast<const uint32_t *>(h);
  }
}

// The same computation as dx_dphi_kernel at KC = 64 with the tile loads
// software-pipelined: every input of tile i+1 (x, dz, dx_add in the
// activation dtype; dm, 1/rms, rowb, the weights in fp32) is copied into the
// other half of a double-buffered shared-memory stage with cp.async while
// tile i is computed, so the global-memory latency hides behind the FMAs
// instead of stalling each tile.  Needs C % 64 == 0 (a block's 64 columns lie
// in one stream) and 16-byte aligned x, dz, dx_add and inv_rms.
template <int N, int MODE, typename Tx>
struct PipeCfg {
  using Cf = DxDphiCfg<N, MODE>;
  static constexpr int FD = Cf::FD, KC = 64, TT = 32;
  static constexpr int XB = TT * KC * (int)sizeof(Tx);  // one x / dz / dx_add tile (bytes)
  static constexpr int DMB = ((TT * FD * 4 + 15) / 16) * 16, VB = TT * 4, GB = ((TT * N * 4 + 15) / 16) * 16;
  static constexpr int SB = 3 * XB + DMB + 2 * VB + GB;  // one stage
  static constexpr int PHI = FD * KC * 4;
  static constexpr int BYTES = PHI + 2 * SB > Cf::RED * 4 ? PHI + 2 * SB : Cf::RED * 4;
  // packed fp32 pairs (fma.rn.f32x2) where the widths allow; then a thread's
  // dx is two adjacent columns (one dm row broadcast serves both)
  static constexpr bool PAIR = FD <= 32 && FD % 4 == 0 && Cf::JR % 4 == 0;
  // blocks per SM the registers are sized for
  static constexpr int MINB = PAIR ? 2 : (Cf::JR <= 12 ? 3 : 2);
};

template <int N, int MODE, typename Tx>
__global__ void __launch_bounds__(256, (PipeCfg<N, MODE, Tx>::MINB))
dx_dphi_pipe_kernel(const Tx *__restrict__ x, int64_t T, int C, const void *__restrict__ phi, int pdt,
                    const float *__restrict__ inv_rms, const float *__restrict__ dm_ws,
                    const float *__restrict__ rowb_ws, const float *__restrict__ gate_ws,
                    const Tx *__restrict__ dz, const Tx *__restrict__ dx_add, Tx *__restrict__ dx,
                    float *__restrict__ dphi_part, int tsplits) {
  using Cf = DxDphiCfg<N, MODE>;
  using Pc = PipeCfg<N, MODE, Tx>;
  static_assert(Cf::RT && Cf::KC == 64, "pipelined path: 64 columns per block");
  constexpr int FD = Cf::FD, KC = 64, TT = 32, JH = Cf::JH, JR = Cf::JR, TG = Cf::TG;
  constexpr int JGRP = 256 / KC, RR = TT / JGRP;
  constexpr int EPV = 16 / (int)sizeof(Tx);   // elements per 16-byte vector
  constexpr int VPR = KC / EPV;               // vectors per tile row
  extern __shared__ float4 smem4[];
  uint8_t *sm = reinterpret_cast<uint8_t *>(smem4);
  float *psT = reinterpret_cast<float *>(sm);  // [FD][KC]
  auto stage = [&](int b) { return sm + Pc::PHI + b * Pc::SB; };

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kk = tid % KC, jgrp = tid / KC;
  const int64_t nC = (int64_t)N * C;
  const int64_t k0 = (int64_t)blockIdx.x * KC;
  const int64_t kglob = k0 + kk;
  const int stream_i = (int)(k0 / C);
  const int c0 = (int)(k0 - (int64_t)stream_i * C);
  const int jh = warp % JH, tg = warp / JH;

  const int64_t tiles = (T + TT - 1) / TT;
  const int64_t tiles_per = (tiles + tsplits - 1) / tsplits;
  const int64_t tile_beg = (int64_t)blockIdx.y * tiles_per;
  int64_t tile_end = tile_beg + tiles_per;
  if (tile_end > tiles) tile_end = tiles;

  // all inputs of one tile into stage b (one commit group)
  auto issue = [&](int64_t tile, int b) {
    uint8_t *st = stage(b);
    uint8_t *xb = st, *zb = st + Pc::XB, *ab = st + 2 * Pc::XB, *db = st + 3 * Pc::XB;
    uint8_t *ib = db + Pc::DMB, *rb = ib + Pc::VB, *gb = rb + Pc::VB;
    const int64_t t0 = tile * TT;
    for (int e = tid; e < TT * VPR; e += 256) {
      const int r = e / VPR, v = e - r * VPR;
      const int64_t tok = t0 + r;
      const bool ok = tok < T;
      const int64_t tk = ok ? tok : 0;
      const int nb = ok ? 16 : 0;
      cp_async16(xb + (r * VPR + v) * 16, x + tk * nC + k0 + v * EPV, nb);
      cp_async16(zb + (r * VPR + v) * 16, dz + tk * C + c0 + v * EPV, nb);
      if (dx_add) cp_async16(ab + (r * VPR + v) * 16, dx_add + tk * nC + k0 + v * EPV, nb);
    }
    const int64_t dm_total = T * FD, dm0 = t0 * FD;
    for (int e = tid; e < Pc::DMB / 16; e += 256) {
      const int64_t left = dm_total - (dm0 + 4 * e);
      const int nb = left >= 4 ? 16 : (left > 0 ? (int)left * 4 : 0);
      cp_async16(db + e * 16, dm_ws + (nb ? dm0 + 4 * e : 0), nb);
    }
    for (int e = tid; e < TT / 4; e += 256) {
      const int64_t left = T - (t0 + 4 * e);
      const int nb = left >= 4 ? 16 : (left > 0 ? (int)left * 4 : 0);
      cp_async16(ib + e * 16, inv_rms + (nb ? t0 + 4 * e : 0), nb);
      cp_async16(rb + e * 16, rowb_ws + (nb ? t0 + 4 * e : 0), nb);
    }
    const int64_t g_total = T * N, g0 = t0 * N;
    for (int e = tid; e < Pc::GB / 16; e += 256) {
      const int64_t left = g_total - (g0 + 4 * e);
      const int nb = left >= 4 ? 16 : (left > 0 ? (int)left * 4 : 0);
      cp_async16(gb + e * 16, gate_ws + (nb ? g0 + 4 * e : 0), nb);
    }
    cp_async_commit();
  };

  if (tile_beg < tile_end) issue(tile_beg, 0);
  for (int e = tid; e < KC * FD; e += blockDim.x) {
    const int r = e / FD, j = e - r * FD;
    psT[j * KC + r] = load_dyn(phi, pdt, (k0 + r) * FD + j);
  }
  __syncthreads();
  constexpr bool PREG = FD <= 32;
  // packed fp32 pairs (fma.rn.f32x2, two FMAs per instruction) where the
  // widths allow: dx's dm . phi over j pairs for two adjacent columns per
  // thread, dphi over projection-column pairs
  constexpr bool PAIR = Pc::PAIR;
  using sm100::f2_fma;
  using sm100::f2_pack;
  using sm100::f2_unpack;
  float pcol[(PREG && !PAIR) ? FD : 1];
  if constexpr (PREG && !PAIR) {
#pragma unroll
    for (int j = 0; j < FD; ++j) pcol[j] = psT[j * KC + kk];
  }
  // phi of columns 2*lane (A) and 2*lane + 1 (B) as (j, j+1) pairs
  uint64_t pcA[PAIR ? FD / 2 : 1], pcB[PAIR ? FD / 2 : 1];
  if constexpr (PAIR) {
#pragma unroll
    for (int j = 0; j < FD / 2; ++j) {
      pcA[j] = f2_pack(psT[(2 * j) * KC + 2 * lane], psT[(2 * j + 1) * KC + 2 * lane]);
      pcB[j] = f2_pack(psT[(2 * j) * KC + 2 * lane + 1], psT[(2 * j + 1) * KC + 2 * lane + 1]);
    }
  }
  float acc[2 * JR];
#pragma unroll
  for (int q = 0; q < 2 * JR; ++q) acc[q] = 0.f;
  uint64_t acc2[PAIR ? JR : 1];  // [column][q/2]: projection columns q, q+1 of column 2*lane + column
#pragma unroll
  for (int q = 0; q < (PAIR ? JR : 1); ++q) acc2[q] = f2_pack(0.f, 0.f);

  int b = 0;
  for (int64_t tile = tile_beg; tile < tile_end; ++tile, b ^= 1) {
    __syncthreads();  // every thread is done with stage b ^ 1 (the previous tile)
    if (tile + 1 < tile_end) {
      issue(tile + 1, b ^ 1);
      cp_async_wait<1>();  // this tile's group has landed (the next may be in flight)
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint8_t *st = stage(b);
    const Tx *xs = reinterpret_cast<const Tx *>(st);
    const Tx *zs = reinterpret_cast<const Tx *>(st + Pc::XB);
    const Tx *as = reinterpret_cast<const Tx *>(st + 2 * Pc::XB);
    const float *dms = reinterpret_cast<const float *>(st + 3 * Pc::XB);
    const float *tinv = reinterpret_cast<const float *>(st + 3 * Pc::XB + Pc::DMB);
    const float *trow = tinv + TT;
    const float *tgate = trow + TT;
    const int64_t t0 = tile * TT;
    if constexpr (PAIR) {
      // dx for columns 2*lane, 2*lane + 1 and rows warp + 8r: one broadcast of
      // the row's dm serves both columns; even and odd j accumulate in the two
      // halves of two packed accumulators per column
#pragma unroll 2
      for (int r = 0; r < TT / 8; ++r) {
        const int row = warp + 8 * r;
        const int64_t tok = t0 + row;
        if (tok >= T) continue;
        uint64_t sa0 = f2_pack(0.f, 0.f), sa1 = sa0, sb0 = sa0, sb1 = sa0;
#pragma unroll
        for (int j = 0; j < FD; j += 4) {
          const float4 d4 = *reinterpret_cast<const float4 *>(dms + row * FD + j);  // one row: broadcast
          const uint64_t p01 = f2_pack(d4.x, d4.y), p23 = f2_pack(d4.z, d4.w);
          sa0 = f2_fma(p01, pcA[j / 2], sa0);
          sa1 = f2_fma(p23, pcA[j / 2 + 1], sa1);
          sb0 = f2_fma(p01, pcB[j / 2], sb0);
          sb1 = f2_fma(p23, pcB[j / 2 + 1], sb1);
        }
        float u0, u1, u2, u3;
        f2_unpack(sa0, u0, u1);
        f2_unpack(sa1, u2, u3);
        const float aA = (u0 + u1) + (u2 + u3);
        f2_unpack(sb0, u0, u1);
        f2_unpack(sb1, u2, u3);
        const float aB = (u0 + u1) + (u2 + u3);
        const float2 x2 = ld2f(xs + row * KC + 2 * lane);
        const float2 z2 = ld2f(zs + row * KC + 2 * lane);
        const float iv = tinv[row], rb = trow[row], gw = tgate[row * N + stream_i];
        float vA = iv * aA - rb * x2.x;
        float vB = iv * aB - rb * x2.y;
        vA = fmaf(gw, z2.x, vA);
        vB = fmaf(gw, z2.y, vB);
        if (dx_add) {
          const float2 a2 = ld2f(as + row * KC + 2 * lane);
          vA += a2.x;
          vB += a2.y;
        }
        st2(dx + tok * nC + k0 + 2 * lane, vA, vB);
      }
    }
    // dx for rows jgrp + JGRP*r, column kk
#pragma unroll 2
    for (int r = 0; r < (PAIR ? 0 : RR); ++r) {
      const int row = jgrp + JGRP * r;
      const int64_t tok = t0 + row;
      if (tok >= T) continue;
      float a = 0.f;
      if constexpr (!PREG) {
#pragma unroll 8
        for (int j = 0; j < FD; ++j) a = fmaf(dms[row * FD + j], psT[j * KC + kk], a);
      } else if constexpr (FD % 4 == 0) {
#pragma unroll
        for (int j = 0; j < FD; j += 4) {
          const float4 d4 = *reinterpret_cast<const float4 *>(dms + row * FD + j);  // one row: broadcast
          a = fmaf(d4.x, pcol[j], a);
          a = fmaf(d4.y, pcol[j + 1], a);
          a = fmaf(d4.z, pcol[j + 2], a);
          a = fmaf(d4.w, pcol[j + 3], a);
        }
      } else {
#pragma unroll
        for (int j = 0; j < FD; ++j) a = fmaf(dms[row * FD + j], pcol[j], a);
      }
      float v = tinv[row] * a - trow[row] * to_f(xs[row * KC + kk]);
      v = fmaf(tgate[row * N + stream_i], to_f(zs[row * KC + kk]), v);
      if (dx_add) v += to_f(as[row * KC + kk]);
      dx[tok * nC + kglob] = from_f<Tx>(v);
    }
    // dphi[k, j] += sum_t (x * inv)[t, k] dm[t, j]: 2 columns x JR projection
    // columns per thread, the tile's tokens split over TG warp groups
#pragma unroll 2
    for (int u = 0; u < TT / TG; ++u) {
      const int t = tg + TG * u;
      float2 x2 = ld2f(xs + t * KC + 2 * lane);
      const float iv = tinv[t];
      x2.x *= iv;
      x2.y *= iv;
      const float *drow = dms + t * FD + jh * JR;
      if constexpr (PAIR) {
        const uint64_t xa = f2_pack(x2.x, x2.x), xb = f2_pack(x2.y, x2.y);
#pragma unroll
        for (int q = 0; q < JR; q += 4) {
          const float4 d4 = *reinterpret_cast<const float4 *>(drow + q);
          const uint64_t p0 = f2_pack(d4.x, d4.y), p1 = f2_pack(d4.z, d4.w);
          acc2[q / 2] = f2_fma(xa, p0, acc2[q / 2]);
          acc2[q / 2 + 1] = f2_fma(xa, p1, acc2[q / 2 + 1]);
          acc2[JR / 2 + q / 2] = f2_fma(xb, p0, acc2[JR / 2 + q / 2]);
          acc2[JR / 2 + q / 2 + 1] = f2_fma(xb, p1, acc2[JR / 2 + q / 2 + 1]);
        }
      } else if constexpr (JR % 4 == 0 && FD % 4 == 0) {
#pragma unroll
        for (int q = 0; q < JR; q += 4) {
          const float4 d4 = *reinterpret_cast<const float4 *>(drow + q);
          acc[q] = fmaf(x2.x, d4.x, acc[q]);
          acc[q + 1] = fmaf(x2.x, d4.y, acc[q + 1]);
          acc[q + 2] = fmaf(x2.x, d4.z, acc[q + 2]);
          acc[q + 3] = fmaf(x2.x, d4.w, acc[q + 3]);
          acc[JR + q] = fmaf(x2.y, d4.x, acc[JR + q]);
          acc[JR + q + 1] = fmaf(x2.y, d4.y, acc[JR + q + 1]);
          acc[JR + q + 2] = fmaf(x2.y, d4.z, acc[JR + q + 2]);
          acc[JR + q + 3] = fmaf(x2.y, d4.w, acc[JR + q + 3]);
        }
      } else if constexpr (JR % 2 == 0 && FD % 2 == 0) {
#pragma unroll
        for (int q = 0; q < JR; q += 2) {
          const float2 d2 = *reinterpret_cast<const float2 *>(drow + q);
          acc[q] = fmaf(x2.x, d2.x, acc[q]);
          acc[q + 1] = fmaf(x2.x, d2.y, acc[q + 1]);
          acc[JR + q] = fmaf(x2.y, d2.x, acc[JR + q]);
          acc[JR + q + 1] = fmaf(x2.y, d2.y, acc[JR + q + 1]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < JR; ++q) {
          if (jh * JR + q < FD) {
            const float d = drow[q];
            acc[q] = fmaf(x2.x, d, acc[q]);
            acc[JR + q] = fmaf(x2.y, d, acc[JR + q]);
          }
        }
      }
    }
  }
  if constexpr (PAIR) {
#pragma unroll
    for (int q = 0; q < JR; q += 2) {
      f2_unpack(acc2[q / 2], acc[q], acc[q + 1]);
      f2_unpack(acc2[JR / 2 + q / 2], acc[JR + q], acc[JR + q + 1]);
    }
  }
  // the token groups' partials, summed in a fixed order (deterministic)
  __syncthreads();
  constexpr int FDP = Cf::FDP;
  float *red = reinterpret_cast<float *>(sm);  // [TG][KC][FDP]
#pragma unroll
  for (int q = 0; q < JR; ++q) {
    const int j = jh * JR + q;
    if (j < FD) {
      red[(tg * KC + 2 * lane) * FDP + j] = acc[q];
      red[(tg * KC + 2 * lane + 1) * FDP + j] = acc[JR + q];
    }
  }
  __syncthreads();
  for (int e = tid; e < KC * FD; e += blockDim.x) {
    const int col = e / FD, j = e - col * FD;
    float v = red[col * FDP + j];
#pragma unroll
    for (int g = 1; g < TG; ++g) v += red[(g * KC + col) * FDP + j];
    dphi_part[((int64_t)blockIdx.y * nC + k0) * FD + e] = v;
  }
}

// ---------------------------------------------------------------------------
// K3
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
reduce_dphi_kernel(const float *__restrict__ part, int splits, int64_t elems, void *dphi, int pdt) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < elems;
       e += (int64_t)gridDim.x * blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < splits; ++s) a += part[(int64_t)s * elems + e];
    store_dyn(dphi, pdt, e, a);
  }
}

// one warp per coefficient-gradient slot; lane-strided fixed-order sums then a
// fixed butterfly
__global__ void __launch_bounds__(256)
reduce_coef_kernel(const float *__restrict__ part, int blocks, int ng, int n, int mode, int pdt,
                   void *da_pre, void *db_pre, void *da_post, void *db_post, void *da_res,
                   void *db_res) {
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (g >= ng) return;
  float a = 0.f;
  for (int b = lane; b < blocks; b += 32) a += part[(int64_t)b * ng + g];
  a = warp_sum(a);
  if (lane != 0) return;
  if (g == 0) { if (da_pre) store_dyn(da_pre, pdt, 0, a); return; }
  if (g == 1) { if (da_post && mode != HEAD) store_dyn(da_post, pdt, 0, a); return; }
  if (g == 2) { if (da_res && mode == FULL) store_dyn(da_res, pdt, 0, a); return; }
  const int j = g - 3;
  if (j < n) { if (db_pre) store_dyn(db_pre, pdt, j, a); return; }
  if (mode == HEAD) return;
  if (j < 2 * n) { if (db_post) store_dyn(db_post, pdt, j - n, a); return; }
  if (mode == FULL && db_res) store_dyn(db_res, pdt, j - 2 * n, a);
}

cudaError_t launch_pre_bwd(int mode, int n, int x_dtype, const void *x, int64_t T, int C,
                           const void *phi, const CoefParams &p, const float *inv_rms,
                           const float *mixes, const void *dz, const void *dh_pre,
                           const void *dh_post, const void *dh_res, int coef_dtype,
                           const void *dx_add, void *dx, void *dphi, void *dalpha_pre,
                           void *dbias_pre, void *dalpha_post, void *dbias_post,
                           void *dalpha_res, void *dbias_res, void *workspace,
                           const PreBwdPlan &plan, bool use_tc, cudaStream_t stream) {
  char *ws = reinterpret_cast<char *>(workspace);
  float *dm_ws = reinterpret_cast<float *>(ws + plan.off_dm);
  float *rowb_ws = reinterpret_cast<float *>(ws + plan.off_rowb);
  float *gate_ws = reinterpret_cast<float *>(ws + plan.off_gate);
  float *dphi_part = reinterpret_cast<float *>(ws + plan.off_dphi_part);
  float *coef_part = reinterpret_cast<float *>(ws + plan.off_coef_part);
  const int64_t nC = (int64_t)n * C;
  const int sms = device_sm_count();
  // token splits whose dphi partials K3 sums
  const int splits = use_tc ? pre_bwd_tc_splits(n, C, T, sms, plan.k2_tsplits) : plan.k2_tsplits;
  return with_mode(mode, [&](auto md) {
    constexpr int MODE = decltype(md)::value;
    return with_n(n, [&](auto nn) {
      constexpr int N = decltype(nn)::value;
      return with_dtype(x_dtype, [&](auto tag) -> cudaError_t {
        using Tx = decltype(tag);
        constexpr int FD = Dims<N, MODE>::FD;
        constexpr int NG = 3 + FD;
        constexpr int VEC = 16 / sizeof(Tx);
        if (T > 0) {
          // K1
          const int TB = plan.k1_tokens;
          const size_t traj =
              (MODE == FULL && p.apply_sinkhorn) ? (size_t)sk_ckpt_count(N, p.sk_iters) * N * N * TB : 0;
          const size_t smem1 = ((size_t)(3 + 2 * N + N * N) + (size_t)TB * N + (size_t)TB * NG + traj) * 4;
          const bool vecok = C % VEC == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)dz & 15) == 0;
          // K1a: the dot products, a streaming pass with every SM busy
          float *dots = reinterpret_cast<float *>(ws + plan.off_dots);
          const int64_t dblocks_need = (T + 7) / 8;
          const int64_t dblocks_cap = (int64_t)(sms > 0 ? sms : 148) * 16;
          coef_dots_kernel<N, Tx><<<(unsigned)(dblocks_need < dblocks_cap ? dblocks_need : dblocks_cap), 256, 0,
                                    stream>>>((const Tx *)x, (const Tx *)dz, T, C, dots, vecok);
          cudaError_t e = cudaGetLastError();
          if (e != cudaSuccess) return e;
          // K1: one thread per token (TB tokens per block, one warp)
          auto k1 = coef_bwd_kernel<N, MODE, Tx>;
          e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
          if (e != cudaSuccess) return e;
          k1<<<plan.k1_blocks, 32, smem1, stream>>>((const Tx *)x, T, C, p, inv_rms, mixes,
                                                    (const Tx *)dz, dh_pre, dh_post, dh_res,
                                                    coef_dtype, TB, dm_ws, rowb_ws, gate_ws, coef_part,
                                                    vecok, dots);
          if ((e = cudaGetLastError()) != cudaSuccess) return e;
          // K2
          if (use_tc) {
            e = launch_pre_bwd_tc(mode, n, x, T, C, phi, p.param_dtype, inv_rms, dm_ws, rowb_ws, gate_ws, dz,
                                  dx_add, dx, dphi_part, splits, stream);
            if (e != cudaSuccess) return e;
          } else {
            dim3 grid2(plan.k2_kblocks, plan.k2_tsplits);
            bool done = false;
            if constexpr (DxDphiCfg<N, MODE>::RT) {
              const bool pipe = C % 64 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)dz & 15) == 0 &&
                                ((uintptr_t)dx_add & 15) == 0 && ((uintptr_t)inv_rms & 15) == 0 &&
                                ((uintptr_t)dx & 15) == 0;
              if (pipe) {
                const size_t smemp = (size_t)PipeCfg<N, MODE, Tx>::BYTES;
                auto kp = dx_dphi_pipe_kernel<N, MODE, Tx>;
                e = cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smemp);
                if (e != cudaSuccess) return e;
                kp<<<grid2, 256, smemp, stream>>>((const Tx *)x, T, C, phi, p.param_dtype, inv_rms, dm_ws,
                                                  rowb_ws, gate_ws, (const Tx *)dz, (const Tx *)dx_add, (Tx *)dx,
                                                  dphi_part, plan.k2_tsplits);
                if ((e = cudaGetLastError()) != cudaSuccess) return e;
                done = true;
              }
            }
            if (!done) {
              const size_t smem2 = (size_t)DxDphiCfg<N, MODE>::SMEM_FLOATS * 4;
              const bool xvec = sizeof(Tx) == 4 && nC % 4 == 0 && ((uintptr_t)x & 15) == 0;
              auto k2 = dx_dphi_kernel<N, MODE, Tx>;
              e = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
              if (e != cudaSuccess) return e;
              k2<<<grid2, 256, smem2, stream>>>((const Tx *)x, T, C, phi, p.param_dtype, inv_rms, dm_ws,
                                                rowb_ws, gate_ws, (const Tx *)dz, (const Tx *)dx_add,
                                                (Tx *)dx, dphi_part, plan.k2_tsplits, xvec);
              if ((e = cudaGetLastError()) != cudaSuccess) return e;
            }
          }
        }
        // K3
        const int64_t elems = nC * FD;
        if (dphi) {
          if (T > 0) {
            reduce_dphi_kernel<<<grid_for(elems, 256, sms, 4), 256, 0, stream>>>(
                dphi_part, splits, elems, dphi, p.param_dtype);
          } else {
            reduce_dphi_kernel<<<grid_for(elems, 256, sms, 4), 256, 0, stream>>>(
                dphi_part, 0, elems, dphi, p.param_dtype);
          }
        }
        reduce_coef_kernel<<<(NG + 7) / 8, 256, 0, stream>>>(
            coef_part, T > 0 ? plan.k1_blocks : 0, NG, N, MODE, p.param_dtype, dalpha_pre,
            dbias_pre, dalpha_post, dbias_post, dalpha_res, dbias_res);
        return cudaGetLastError();
      });
    });
  });
}

}  // namespace mhc
