// Single-read fused coefficient + pre-aggregate kernel for bf16 activations
// on sm_100a: x is read from HBM exactly once.
//
// The coefficients of a token depend on its whole n*C row (RMS statistics and
// the n*C x FD projection) and the sublayer input z = sum_i w_i x_i needs
// them, so every x element is needed twice: once before the token's weights
// exist and once after.  Here the second use reads an on-chip copy instead of
// HBM or L2.
//
// One persistent kernel per call, launched as clusters of S = C / 128 CTAs
// (4 <= S <= 8; one CTA per SM).  CTA r of a cluster owns columns
// [128 r, 128 r + 128) of every stream: its K slice of the projection is those
// n x 128 columns, and it computes z for the same 128 columns, so everything
// it needs for z is in its own slice.  A cluster walks a sequence of
// 128-token tiles; a tile's slice is 2n chunks of 128 rows x 64 columns (16
// KB, 128-byte swizzle), block-major (the n streams of column block 0, then of
// block 1).
//
//   warp 0      TMA producer: x chunks into an 8-slot shared-memory ring.
//   warp 1      tcgen05 MMA issuer: D[128 tok, NB] += x_chunk . phi_chunk^T
//               (M = 128, K = 16 per instruction, fp32 accumulators in TMEM,
//               two buffers).  phi's slice is split once per launch into bf16
//               hi | lo halves held in shared memory (projection accurate to
//               ~2^-17).
//   warps 2-5   ingest (thread = token row = TMEM lane): each landed chunk row
//               is read from shared memory once, its squares are summed for the
//               RMS statistics, and it is stored into a TMEM retention slot
//               (12 slots of 32 columns); the ring slot is then free.  At the
//               end of a tile the warps read the projection partial from TMEM
//               and push (FD partials, sum of squares) with st.async into the
//               inbox of the row's owner CTA (row r -> CTA r mod S).
//   warp 6      coefficient warp (owner of rows r = rank + S l): sums the S
//               slices in a fixed order (deterministic), applies 1/rms, the
//               sigmoid gates and the H_res affine map, pushes the fp32
//               aggregation weights to every CTA of the cluster with st.async
//               and writes the per-token outputs.
//   warps 7-8   Sinkhorn warps (alternate tiles): H_res of the owned rows, one
//               token per lane, the matrix in registers.
//   warps 9-12  z warps (thread = token row): once the tile's weights are in,
//               the retained chunks are read back from TMEM, z is accumulated
//               in fp32 packed pairs, written to a per-warp shared-memory
//               staging block and stored with a TMA store; the retention slots
//               are then free.
//
// x in flight or on chip per CTA: 8 ring chunks (128 KB of shared memory) plus
// 12 retained chunks (192 KB of TMEM) -- about 2.5 tiles, which covers the
// cluster round trip of a tile's partial rows and weights while the next
// tiles stream in.
//
// All hand-offs are mbarriers and every wait is bounded (mhc_sm100.cuh): a
// wait that runs out records an error code (device word and registered host
// flag), the CTA drains its asynchronous work, overwrites the outputs it owns
// with NaN, frees TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "mhc_device.cuh"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"
#include "mhc_sm100.cuh"

namespace mhc {

__device__ int g_sr_error = 0;  // first error code recorded by the single-read kernel

namespace sr {

using namespace sm100;

constexpr int TM = 128;                    // tokens per tile (UMMA M, TMEM lanes)
constexpr int COLS = 128;                  // columns of every stream owned by a CTA
constexpr int CHUNK = TM * 128;            // 128 rows x 64 bf16 (128-byte swizzle)
constexpr int RING = 8;                    // shared-memory x chunk slots
constexpr int RET = 12;                    // TMEM retention slots (32 columns each)
constexpr int ACC_COLS = 64;               // one projection accumulator (NB <= 64)
constexpr int RET_COL0 = 2 * ACC_COLS;     // first retention column
constexpr int TMEM_COLS = 512;
static_assert(RET_COL0 + RET * 32 <= TMEM_COLS, "TMEM budget");
constexpr int HB = 2;                      // aggregation-weight buffers
constexpr int HBL = 4;                     // H_res logit buffers (two per Sinkhorn warp)
constexpr int NRT = 4;                     // "tile retained" barriers: more than the tiles RET slots can hold
constexpr int HPN = 4;                     // weights per token row (n <= 4, padded)
constexpr int W_PROD = 0, W_MMA = 1, W_ING = 2, W_COEF = 6, W_SK = 7, W_Z = 9;
constexpr int NWARPS = 13, NTHREADS = NWARPS * 32;
constexpr int W_CONV = 2, NCONV = NWARPS - W_CONV;  // warps that convert phi in the prologue
constexpr int ZST = 32 * 128;              // per-z-warp staging block: 32 rows x 64 bf16

enum ErrCode { ERR_PROD = 21, ERR_MMA = 22, ERR_ING = 23, ERR_COEF = 24, ERR_SK = 25, ERR_Z = 26 };

template <int N, int MODE>
struct Cfg {
  static constexpr int FD = Dims<N, MODE>::FD;
  static constexpr int NB = ((2 * FD + 15) / 16) * 16;   // hi | lo projection columns
  static constexpr int IBS = ((FD + 1 + 3) / 4) * 4;     // inbox row: FD partials + sum of squares
  static constexpr int NPAR = 3 + 2 * N + N * N;
  static constexpr int CH = 2 * N;                       // chunks per tile
  static_assert(NB <= ACC_COLS, "projection accumulator");
  static_assert(N <= HPN, "weights row");
};

// barrier slots
constexpr int B_FULL = 0, B_EMPTY = RING, B_ACCF = 2 * RING, B_ACCE = B_ACCF + 2, B_RFREE = B_ACCE + 2,
              B_RT = B_RFREE + RET, B_INF = B_RT + NRT, B_INE = B_INF + 1, B_HPF = B_INE + 1, B_HPE = B_HPF + HB,
              B_ZD = B_HPE + HB, B_LGF = B_ZD + HB, B_LGE = B_LGF + HBL, B_DRAIN = B_LGE + HBL,
              B_PHI = B_DRAIN + 1, NBARS = B_PHI + 1;

struct Layout {
  uint32_t ring, phi, zst, inbox, hp, lg, par, bar, tmem, abort, total;
};

__host__ __device__ inline int owned_max(int S) { return (TM + S - 1) / S; }

__host__ __device__ inline Layout make_layout(int S, int CH, int NB, int IBS, int NPAR) {
  Layout L;
  uint32_t o = 0;
  L.ring = o;  o += (uint32_t)RING * CHUNK;
  L.phi = o;   o += (uint32_t)CH * NB * 128;
  L.zst = o;   o += 4u * ZST;
  L.inbox = o; o += (uint32_t)S * owned_max(S) * IBS * 4;
  L.hp = o;    o += (uint32_t)HB * TM * HPN * 4;
  L.lg = o;    o += (uint32_t)HBL * owned_max(S) * 16 * 4;
  L.par = o;   o += ((NPAR * 4 + 15) / 16) * 16;
  L.bar = o;   o += NBARS * 8;
  L.tmem = o;  o += 4;
  L.abort = o; o += 4;
  L.total = o;
  return L;
}

struct Args {
  int64_t T;
  int C, nC, S;
  const void *phi;
  CoefParams p;
  __nv_bfloat16 *z;
  void *h_pre, *h_post, *h_res;
  int coef_dtype;
  float *inv_rms, *mixes;
  int *err_flag;  // pinned host error word (mhc_set_error_flag) or null
};

// byte offset of element (row j, column kk < 64) inside one phi chunk block:
// 128-byte swizzled K-major rows (granule index XOR row-in-atom)
__device__ __forceinline__ uint32_t phi_off(int j, int kk) {
  return (uint32_t)(j >> 3) * 1024 + (j & 7) * 128 + ((((kk >> 3) ^ (j & 7))) << 4) + ((kk & 7) << 1);
}

__device__ __forceinline__ void record_error(int code, volatile int *abort_flag, int *err_flag) {
  *abort_flag = 1;
  report_give_up(&g_sr_error, err_flag, code);
}

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

// After a wait gave up, the CTA overwrites its share of every tile of its
// cluster with NaN: z columns [128 rank, 128 rank + 128) of the tile's rows and
// every per-token output of the rows it owns.
template <int N, int MODE>
__device__ void poison_share(const Args &a, int cid, int ncl, int rank, int ntiles, int tid, int nthreads) {
  constexpr int FD = Dims<N, MODE>::FD;
  const float qnan = __int_as_float(0x7fc00000);
  const __nv_bfloat16 bnan = __float2bfloat16_rn(qnan);
  const int c0 = rank * COLS;
  for (int tile = cid; tile < ntiles; tile += ncl) {
    const int64_t t0 = (int64_t)tile * TM;
    const int rows = a.T - t0 < TM ? (int)(a.T - t0) : TM;
    for (int e = tid; e < rows * COLS; e += nthreads) {
      const int r = e / COLS, c = e - r * COLS;
      a.z[(t0 + r) * a.C + c0 + c] = bnan;
    }
    for (int r = rank + tid * a.S; r < rows; r += nthreads * a.S) {
      const int64_t tok = t0 + r;
      a.inv_rms[tok] = qnan;
      for (int j = 0; j < FD; ++j) a.mixes[tok * FD + j] = qnan;
      if constexpr (MODE != HEAD) {
        for (int i = 0; i < N; ++i) {
          if (a.h_pre) store_dyn(a.h_pre, a.coef_dtype, tok * N + i, qnan);
          store_dyn(a.h_post, a.coef_dtype, tok * N + i, qnan);
        }
      }
      if constexpr (MODE == FULL) {
        if (a.h_res)
          for (int k = 0; k < N * N; ++k) store_dyn(a.h_res, a.coef_dtype, tok * N * N + k, qnan);
      }
    }
  }
}

template <int N, int MODE>
__global__ void __launch_bounds__(NTHREADS, 1)
pre_sr_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap zmap, Args a) {
  using Cf = Cfg<N, MODE>;
  constexpr int FD = Cf::FD, NB = Cf::NB, IBS = Cf::IBS, NPAR = Cf::NPAR, CH = Cf::CH;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t *base = smem_raw + (base_u32 - raw_u32);
  const int S = a.S;
  const int OWN = owned_max(S);
  const Layout L = make_layout(S, CH, NB, IBS, NPAR);
  float *inbox = reinterpret_cast<float *>(base + L.inbox);
  float *hp = reinterpret_cast<float *>(base + L.hp);
  float *lg = reinterpret_cast<float *>(base + L.lg);
  float *par = reinterpret_cast<float *>(base + L.par);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(base + L.abort);
  const uint32_t bar0 = base_u32 + L.bar;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
// warp-uniform bounded wait: every lane waits (and so acquires), the warp
// agrees on the outcome so it always leaves a loop together
#define WAIT_WARP(CL, bar, ph) (__all_sync(0xffffffffu, wait_parity<CL>((bar), (ph), abort_flag)))

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank(), cid = cluster_id_x(), ncl = ncluster_x();
  const int ntiles = (int)((a.T + TM - 1) / TM);
  const int cnt = (TM - (int)rank + S - 1) / S;  // rows this CTA owns in every tile
  const uint32_t inbox_tx = (uint32_t)S * cnt * IBS * 4;
  constexpr uint32_t HP_TX = (uint32_t)TM * HPN * 4;

  // ---------------- prologue ----------------
  if (tid == 0) {
    *abort_flag = 0;
    for (int i = 0; i < RING; ++i) {
      mbar_init(BAR(B_FULL + i), 1);
      mbar_init(BAR(B_EMPTY + i), 1 + 4);  // MMA commit + the 4 ingest warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(B_ACCF + b), 1);
      mbar_init(BAR(B_ACCE + b), 4);
    }
    for (int b = 0; b < NRT; ++b) mbar_init(BAR(B_RT + b), 4);  // ingest warps: the tile's chunks are in TMEM
    for (int i = 0; i < RET; ++i) mbar_init(BAR(B_RFREE + i), 4);  // z warps done with the slot
    mbar_init(BAR(B_INF), 1);              // armed by the coefficient warp; st.async bytes complete it
    mbar_init(BAR(B_INE), S);              // one per owner CTA (its inbox drained)
    for (int b = 0; b < HB; ++b) {
      mbar_init(BAR(B_HPF + b), 1);        // armed by a z warp; st.async bytes complete it
      mbar_init(BAR(B_HPE + b), S);        // one per CTA (its z warps are done with the buffer)
      mbar_init(BAR(B_ZD + b), 4);         // local: z warps done reading the buffer
    }
    for (int b = 0; b < HBL; ++b) {
      mbar_init(BAR(B_LGF + b), 1);
      mbar_init(BAR(B_LGE + b), 1);
    }
    mbar_init(BAR(B_DRAIN), 1);
    mbar_init(BAR(B_PHI), NCONV);
    fence_mbar_init_cluster();
  }
  if (warp == W_MMA) {
    tmem_alloc(base_u32 + L.tmem, TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  cluster_sync_all();  // every CTA's barriers exist before any remote arrive or st.async
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(base + L.tmem);
  // set-up above overlaps the previous kernel of the stream (programmatic
  // dependent launch); every input read comes after this wait
  grid_dep_launch();
  grid_dep_wait();
  if (warp >= W_CONV) {
    // this CTA's phi slice -> bf16 hi | lo, K-major, 128-byte swizzle, chunk by
    // chunk in the order the x chunks arrive
    const int ctid = tid - W_CONV * 32, nconv = NCONV * 32;
    const int KS = CH * 64, total = KS * FD;
    for (int e0 = ctid; e0 < total; e0 += 4 * nconv) {
      float v[4];
      int kk4[4], j4[4], ch4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = e0 + u * nconv;
        v[u] = 0.f;
        if (e < total) {
          const int kl = e / FD, j = e - kl * FD;
          const int ch = kl >> 6, kk = kl & 63;
          const int i = ch % N, b = ch / N;
          const int64_t k = (int64_t)i * a.C + (int64_t)rank * COLS + 64 * b + kk;
          v[u] = load_dyn(a.phi, a.p.param_dtype, k * FD + j);
          kk4[u] = kk;
          j4[u] = j;
          ch4[u] = ch;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (e0 + u * nconv < total) {
          uint8_t *blk = base + L.phi + (uint32_t)ch4[u] * NB * 128;
          const __nv_bfloat16 hi = __float2bfloat16_rn(v[u]);
          const __nv_bfloat16 lo = __float2bfloat16_rn(v[u] - __bfloat162float(hi));
          *reinterpret_cast<__nv_bfloat16 *>(blk + phi_off(j4[u], kk4[u])) = hi;
          *reinterpret_cast<__nv_bfloat16 *>(blk + phi_off(j4[u] + FD, kk4[u])) = lo;
        }
      }
    }
    constexpr int PADR = NB - 2 * FD;
    if constexpr (PADR > 0) {
      for (int e = ctid; e < KS * PADR; e += nconv) {
        const int kl = e / PADR, j = 2 * FD + (e - kl * PADR);
        uint8_t *blk = base + L.phi + (uint32_t)(kl >> 6) * NB * 128;
        *reinterpret_cast<__nv_bfloat16 *>(blk + phi_off(j, kl & 63)) = __float2bfloat16_rn(0.f);
      }
    }
    load_params<N, MODE>(par, a.p, ctid, nconv);
    fence_proxy_async_smem();  // generic phi writes -> tensor-core (async proxy) reads
    __syncwarp();
    if (lane == 0) mbar_arrive(BAR(B_PHI));
  }

  if (warp == W_PROD) {
    // ---------------- x chunk producer ----------------
    if (lane == 0) {
      uint32_t q = 0;
      bool ok = true;
      for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl) {
        for (int ch = 0; ch < CH; ++ch, ++q) {
          const uint32_t slot = q % RING, ph = (q / RING) & 1u;
          if (!wait_parity<false>(BAR(B_EMPTY + slot), ph ^ 1u, abort_flag)) { ok = false; break; }
          const int i = ch % N, b = ch / N;
          mbar_arrive_expect_tx(BAR(B_FULL + slot), CHUNK);
          tma_load_2d(base_u32 + L.ring + slot * CHUNK, &xmap, i * a.C + (int)rank * COLS + 64 * b, tile * TM,
                      BAR(B_FULL + slot));
        }
      }
      if (!ok) record_error(ERR_PROD, abort_flag, a.err_flag);
      // copies in flight must land before the CTA can exit
      const uint32_t q0 = q > (uint32_t)RING ? q - RING : 0u;
      for (uint32_t p = q0; p < q; ++p) wait_parity<false>(BAR(B_FULL + p % RING), (p / RING) & 1u, nullptr);
    }
    __syncwarp();
  } else if (warp == W_MMA) {
    // ---------------- tcgen05 MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(128, NB);
      uint32_t q = 0;
      int lt = 0;
      bool ok = wait_parity<false>(BAR(B_PHI), 0u, abort_flag);  // phi slice converted
      for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
        const int buf = lt & 1;
        if (!wait_parity<false>(BAR(B_ACCE + buf), ((uint32_t)(lt >> 1) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem_base + (uint32_t)buf * ACC_COLS;
        for (int ch = 0; ch < CH; ++ch, ++q) {
          const uint32_t slot = q % RING, ph = (q / RING) & 1u;
          if (!wait_parity<false>(BAR(B_FULL + slot), ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = base_u32 + L.ring + slot * CHUNK;
          const uint32_t b0 = base_u32 + L.phi + (uint32_t)ch * NB * 128u;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(dcol, umma_desc_sw128(a0 + k * 32), umma_desc_sw128(b0 + k * 32), idesc,
                      (ch | k) != 0 ? 1u : 0u);
          umma_commit(BAR(B_EMPTY + slot));
        }
        if (!ok) break;
        umma_commit(BAR(B_ACCF + buf));
      }
      if (!ok) record_error(ERR_MMA, abort_flag, a.err_flag);
      // every issued MMA completes before TMEM is released
      umma_commit(BAR(B_DRAIN));
      wait_parity<false>(BAR(B_DRAIN), 0u, nullptr);
    }
    __syncwarp();
  } else if (warp >= W_ING && warp < W_ING + 4) {
    // ---------------- ingest warps ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // token row of the tile = TMEM lane
    const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16);
    const uint32_t owner = (uint32_t)(row % S);
    const int oidx = row / S;
    uint32_t q = 0;
    int lt = 0;
    bool ok = true;
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      uint64_t ss2 = f2_pack(0.f, 0.f);  // sum of squares, two fp32 partial sums
      for (int ch = 0; ch < CH; ++ch, ++q) {
        const uint32_t slot = q % RING, ph = (q / RING) & 1u;
        const uint32_t rs = q % RET, rph = (q / RET) & 1u;
        if (!WAIT_WARP(false, BAR(B_FULL + slot), ph)) { ok = false; break; }
        if (!WAIT_WARP(false, BAR(B_RFREE + rs), rph ^ 1u)) { ok = false; break; }
        tc_fence_after();
        const uint8_t *rowp = base + L.ring + slot * CHUNK + row * 128;
        uint32_t w[32];
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const uint4 v = *reinterpret_cast<const uint4 *>(rowp + ((g ^ (row & 7)) << 4));
          w[4 * g] = v.x; w[4 * g + 1] = v.y; w[4 * g + 2] = v.z; w[4 * g + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const uint64_t xv = bf16x2_to_f2(w[j]);
          ss2 = f2_fma(xv, xv, ss2);
        }
        tmem_st32(lane_base + (uint32_t)(RET_COL0 + rs * 32), w);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_EMPTY + slot));
      }
      if (!ok) break;
      if (lane == 0) mbar_arrive(BAR(B_RT + lt % NRT));  // the tile's chunks are retained
      // the slice's projection partial of this row
      const int buf = lt & 1;
      if (!WAIT_WARP(false, BAR(B_ACCF + buf), (uint32_t)(lt >> 1) & 1u)) { ok = false; break; }
      tc_fence_after();
      float d[NB];
#pragma unroll
      for (int c16 = 0; c16 < NB / 16; ++c16) {
        float t16[16];
        tmem_ld16(lane_base + (uint32_t)(buf * ACC_COLS + c16 * 16), t16);
#pragma unroll
        for (int i = 0; i < 16; ++i) d[c16 * 16 + i] = t16[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_ACCE + buf));
      float vals[IBS];
#pragma unroll
      for (int j = 0; j < IBS; ++j) vals[j] = 0.f;
#pragma unroll
      for (int j = 0; j < FD; ++j) vals[j] = d[j] + d[FD + j];
      {
        float s0, s1;
        f2_unpack(ss2, s0, s1);
        vals[FD] = s0 + s1;
      }
      // every owner's inbox must have been drained of the previous tile
      if (!WAIT_WARP(true, BAR(B_INE), ((uint32_t)lt & 1u) ^ 1u)) { ok = false; break; }
      const uint32_t dst = mapa(base_u32 + L.inbox + (uint32_t)(((int)rank * OWN + oidx) * IBS * 4), owner);
      const uint32_t dbar = mapa(BAR(B_INF), owner);
#pragma unroll
      for (int v = 0; v < IBS / 4; ++v)
        st_async_v4(dst + v * 16, vals[4 * v], vals[4 * v + 1], vals[4 * v + 2], vals[4 * v + 3], dbar);
    }
    if (!ok) record_error(ERR_ING, abort_flag, a.err_flag);
  } else if (warp == W_COEF) {
    // ---------------- coefficient warp: rows rank + S l ----------------
    int lt = 0;
    bool ok = WAIT_WARP(false, BAR(B_PHI), 0u);  // gate parameters loaded
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const int hb = lt % HB, lb = lt % HBL;
      if (lane == 0) mbar_arrive_expect_tx(BAR(B_INF), inbox_tx);  // arm: S slices' rows
      if (!WAIT_WARP(true, BAR(B_INF), (uint32_t)lt & 1u)) { ok = false; break; }
      float acc[IBS];
#pragma unroll
      for (int j = 0; j < IBS; ++j) acc[j] = 0.f;
      if (lane < cnt) {
        for (int s = 0; s < S; ++s) {  // fixed order over the K slices: deterministic
          const float4 *src = reinterpret_cast<const float4 *>(inbox + (s * OWN + lane) * IBS);
#pragma unroll
          for (int v = 0; v < IBS / 4; ++v) {
            const float4 q4 = src[v];
            acc[4 * v] += q4.x; acc[4 * v + 1] += q4.y; acc[4 * v + 2] += q4.z; acc[4 * v + 3] += q4.w;
          }
        }
      }
      __syncwarp();
      if (lane < S) mbar_arrive_remote(mapa(BAR(B_INE), (uint32_t)lane));  // inbox free again
      const int t = (int)rank + lane * S;  // token row of the tile
      const int64_t tok = (int64_t)tile * TM + t;
      const bool live = lane < cnt && tok < a.T;
      float w[HPN], m[FD], ho[N];
      float inv = 0.f;
#pragma unroll
      for (int i = 0; i < HPN; ++i) w[i] = 0.f;
      // the weights buffer must be free in every CTA (tile lt-HB done everywhere)
      if (!WAIT_WARP(true, BAR(B_HPE + hb), ((uint32_t)(lt / HB) & 1u) ^ 1u)) { ok = false; break; }
      if constexpr (MODE == FULL) {
        if (!WAIT_WARP(false, BAR(B_LGE + lb), ((uint32_t)(lt / HBL) & 1u) ^ 1u)) { ok = false; break; }
      }
      if (lane < cnt) {
        inv = rsqrtf(acc[FD] / (float)a.nC + a.p.rms_eps);
#pragma unroll
        for (int j = 0; j < FD; ++j) m[j] = acc[j] * inv;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          w[i] = sigmoidf_(__fadd_rn(__fmul_rn(m[i], par[0]), par[3 + i])) + a.p.pre_eps;
          if constexpr (MODE != HEAD)
            ho[i] = sigmoidf_(__fadd_rn(__fmul_rn(m[N + i], par[1]), par[3 + N + i])) * a.p.post_mult;
        }
        if constexpr (MODE == FULL) {
          float *lrow = lg + (lb * OWN + lane) * 16;
#pragma unroll
          for (int k = 0; k < N * N; ++k) lrow[k] = __fadd_rn(__fmul_rn(m[2 * N + k], par[2]), par[3 + 2 * N + k]);
        }
        // publish the aggregation weights to every CTA of the cluster
        const uint32_t loc = base_u32 + L.hp + (uint32_t)((hb * TM + t) * HPN * 4);
#pragma unroll 1
        for (int dcta = 0; dcta < S; ++dcta) {
          const uint32_t dst = mapa(loc, (uint32_t)dcta);
          const uint32_t dbar = mapa(BAR(B_HPF + hb), (uint32_t)dcta);
          st_async_v4(dst, w[0], w[1], w[2], w[3], dbar);
        }
      }
      if constexpr (MODE == FULL) {
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_LGF + lb));  // logits ready for the Sinkhorn warp
      }
      // per-token outputs
      if (live) {
        a.inv_rms[tok] = inv;
#pragma unroll
        for (int j = 0; j < FD; ++j) a.mixes[tok * FD + j] = m[j];
        if constexpr (MODE != HEAD) {
#pragma unroll
          for (int i = 0; i < N; ++i) {
            if (a.h_pre) store_dyn(a.h_pre, a.coef_dtype, tok * N + i, w[i]);
            store_dyn(a.h_post, a.coef_dtype, tok * N + i, ho[i]);
          }
        }
      }
    }
    if (!ok) record_error(ERR_COEF, abort_flag, a.err_flag);
  } else if (warp == W_SK || warp == W_SK + 1) {
    // ---------------- Sinkhorn warps: H_res of the owned rows ----------------
    // warp W_SK + s takes the local tiles lt = s (mod 2), whose logits sit in
    // buffers s and s + 2 (each buffer is used by one warp, phases in order)
    if constexpr (MODE == FULL) {
      const int s = warp - W_SK;
      int lt = s;
      bool ok = true;
      for (int tile = (int)cid + s * (int)ncl; tile < ntiles && ok; tile += 2 * (int)ncl, lt += 2) {
        const int lb = lt % HBL;
        if (!WAIT_WARP(false, BAR(B_LGF + lb), (uint32_t)(lt / HBL) & 1u)) { ok = false; break; }
        const int64_t tok = (int64_t)tile * TM + (int)rank + lane * S;
        if (lane < cnt && tok < a.T) {
          float hm[N * N];
#pragma unroll
          for (int k = 0; k < N * N; ++k) hm[k] = lg[(lb * OWN + lane) * 16 + k];
          if (a.p.apply_sinkhorn) sinkhorn_fwd<N>(hm, a.p.sk_iters, a.p.sk_eps);
          if (a.h_res) {
#pragma unroll
            for (int k = 0; k < N * N; ++k) store_dyn(a.h_res, a.coef_dtype, tok * N * N + k, hm[k]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_LGE + lb));  // logits buffer free
      }
      if (!ok) record_error(ERR_SK, abort_flag, a.err_flag);
    }
  } else if (warp >= W_Z && warp < W_Z + 4) {
    // ---------------- z warps ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16);
    const uint32_t stage = base_u32 + L.zst + (uint32_t)(warp - W_Z) * ZST;
    uint8_t *stage_p = base + L.zst + (warp - W_Z) * ZST;
    const int c0 = (int)rank * COLS;
    int lt = 0;
    bool ok = true;
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const int hb = lt % HB;
      const uint32_t hph = (uint32_t)(lt / HB) & 1u;
      if (warp == W_Z && lane == 0) mbar_arrive_expect_tx(BAR(B_HPF + hb), HP_TX);  // arm: S owners' weights
      if (!WAIT_WARP(true, BAR(B_HPF + hb), hph)) { ok = false; break; }
      if (!WAIT_WARP(false, BAR(B_RT + lt % NRT), (uint32_t)(lt / NRT) & 1u)) { ok = false; break; }
      tc_fence_after();
      const float4 w4 = *reinterpret_cast<const float4 *>(hp + (hb * TM + row) * HPN);
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
      const uint32_t q0 = (uint32_t)lt * CH;
      const int64_t row0 = (int64_t)tile * TM + quad * 32;
#pragma unroll 1
      for (int b = 0; b < 2; ++b) {
        // the staging block must have been read by this warp's previous store
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int piece = 0; piece < 2; ++piece) {
          uint32_t xr[N][16];
#pragma unroll
          for (int i = 0; i < N; ++i) {
            const uint32_t rs = (q0 + (uint32_t)(b * N + i)) % RET;
            tmem_ld16u(lane_base + (uint32_t)(RET_COL0 + rs * 32 + piece * 16), xr[i]);
          }
          uint32_t out[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            uint64_t acc = f2_fma(f2_pack(wv[0], wv[0]), bf16x2_to_f2(xr[0][j]), f2_pack(0.f, 0.f));
#pragma unroll
            for (int i = 1; i < N; ++i) acc = f2_fma(f2_pack(wv[i], wv[i]), bf16x2_to_f2(xr[i][j]), acc);
            float lo, hi;
            f2_unpack(acc, lo, hi);
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
            out[j] = *reinterpret_cast<const uint32_t *>(&h2);
          }
          // 16 words = granules 4 piece .. 4 piece + 3 of this row (128-byte swizzle)
          uint8_t *rp = stage_p + lane * 128;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int gg = piece * 4 + g;
            *reinterpret_cast<uint4 *>(rp + ((gg ^ (lane & 7)) << 4)) =
                make_uint4(out[4 * g], out[4 * g + 1], out[4 * g + 2], out[4 * g + 3]);
          }
        }
        fence_proxy_async_smem();  // generic staging writes -> TMA store reads
        __syncwarp();
        if (lane == 0 && row0 < a.T) {
          tma_store_2d(&zmap, stage, c0 + 64 * b, (int)row0);
          bulk_commit();
        }
      }
      // the tile's retention slots and weights are no longer needed here
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        for (int ch = 0; ch < CH; ++ch) mbar_arrive(BAR(B_RFREE + (q0 + (uint32_t)ch) % RET));
        mbar_arrive(BAR(B_ZD + hb));
      }
      if (warp == W_Z) {
        int good = 1;
        if (lane == 0) {
          good = wait_parity<false>(BAR(B_ZD + hb), hph, abort_flag) ? 1 : 0;
          if (good)
            for (int s = 0; s < S; ++s) mbar_arrive_remote(mapa(BAR(B_HPE + hb), (uint32_t)s));
        }
        if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
      }
    }
    if (!ok) record_error(ERR_Z, abort_flag, a.err_flag);
    if (lane == 0) bulk_wait_all();  // the z stores are complete before the CTA exits
    __syncwarp();
  }

  // ---------------- teardown ----------------
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (*abort_flag) poison_share<N, MODE>(a, (int)cid, (int)ncl, (int)rank, ntiles, tid, NTHREADS);
  cluster_sync_all();  // no CTA leaves while a peer may still touch its shared memory
#undef WAIT_WARP
#undef BAR
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

constexpr size_t SMEM_LIMIT = 232448;  // opt-in dynamic shared memory per block on sm_100

template <int N, int MODE>
static size_t smem_bytes(int S) {
  using Cf = Cfg<N, MODE>;
  return (size_t)make_layout(S, Cf::CH, Cf::NB, Cf::IBS, Cf::NPAR).total + 1024;
}

// 2-D bf16 map over a (rows x cols) row-major matrix with the given box and a
// 128-byte swizzle
static bool encode_2d(CUtensorMap &m, const void *p, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(p), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per kernel instantiation, device and cluster size: the dynamic shared
// memory already granted and the number of co-resident clusters.
struct KernEntry {
  const void *kern;
  int dev, S;
  int clusters;
};
static std::mutex g_mu;
static KernEntry g_kerns[64];
static int g_kerns_n = 0;

template <int N, int MODE>
static cudaError_t launch_impl(const void *x, Args a, cudaStream_t stream) {
  const size_t smem = smem_bytes<N, MODE>(a.S);
  if (smem > SMEM_LIMIT) return cudaErrorNotSupported;
  auto kern = pre_sr_kernel<N, MODE>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // cluster shape only for the occupancy query
  cfg.blockDim = dim3(NTHREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;

  int max_clusters = 0;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    KernEntry *ke = nullptr;
    for (int i = 0; i < g_kerns_n; ++i)
      if (g_kerns[i].kern == (const void *)kern && g_kerns[i].dev == dev && g_kerns[i].S == a.S) ke = &g_kerns[i];
    if (!ke) {
      if (g_kerns_n == 64) return cudaErrorNotSupported;
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT);
      if (e != cudaSuccess) return e;
      cfg.gridDim = dim3((unsigned)(a.S * 32), 1, 1);
      int v = 0;
      e = cudaOccupancyMaxActiveClusters(&v, (void *)kern, &cfg);
      if (e != cudaSuccess) return e;
      if (v <= 0) return cudaErrorNotSupported;
      ke = &g_kerns[g_kerns_n++];
      *ke = KernEntry{(const void *)kern, dev, a.S, v};
    }
    max_clusters = ke->clusters;
  }

  CUtensorMap xmap, zmap;
  if (!encode_2d(xmap, x, a.T, a.nC, 64, TM)) return cudaErrorNotSupported;
  if (!encode_2d(zmap, a.z, a.T, a.C, 64, 32)) return cudaErrorNotSupported;
  const int64_t ntiles = (a.T + TM - 1) / TM;
  const int clusters = (int)(ntiles < max_clusters ? ntiles : max_clusters);
  cfg.gridDim = dim3((unsigned)(clusters * a.S), 1, 1);
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, xmap, zmap, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace sr

bool pre_sr_eligible(int mode, int n, int x_dtype, const void *x, const void *z, int64_t T, int C) {
  if (x_dtype != MHC_BF16 || T < 1) return false;
  if (n != 2 && n != 4) return false;
  if (mode == HEAD && n < 2) return false;
  if (C % sr::COLS != 0) return false;
  const int S = C / sr::COLS;
  if (S < 4 || S > 8) return false;
  if (((uintptr_t)x & 15) != 0 || ((uintptr_t)z & 15) != 0) return false;
  return true;
}

cudaError_t launch_pre_sr(int mode, int n, const void *x, int64_t T, int C, const void *phi, const CoefParams &p,
                          void *z, void *h_pre, void *h_post, void *h_res, int coef_dtype, float *inv_rms,
                          float *mixes, cudaStream_t stream) {
  sr::Args a;
  a.T = T;
  a.C = C;
  a.nC = n * C;
  a.S = C / sr::COLS;
  a.phi = phi;
  a.p = p;
  a.z = reinterpret_cast<__nv_bfloat16 *>(z);
  a.h_pre = h_pre;
  a.h_post = h_post;
  a.h_res = h_res;
  a.coef_dtype = coef_dtype;
  a.inv_rms = inv_rms;
  a.mixes = mixes;
  a.err_flag = host_error_flag();
  return with_mode(mode, [&](auto md) -> cudaError_t {
    constexpr int MODE = decltype(md)::value;
    switch (n) {
      case 2: return sr::launch_impl<2, MODE>(x, a, stream);
      case 4: return sr::launch_impl<4, MODE>(x, a, stream);
      default: break;
    }
    return cudaErrorNotSupported;
  });
}

int read_sr_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_sr_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_sr_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace mhc
