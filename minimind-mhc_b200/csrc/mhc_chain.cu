// Fused merge of one sublayer and coefficient pass of the next (post(l) +
// pre(l+1)) for bf16 streams on sm_100a, with the next sublayer's input
// RMSNorm optionally applied to its pre-aggregate.
//
//   x'[t, i*C+c] = sum_j H_res[t,i,j] x[t, j*C+c] + H_post[t,i] f[t,c]      (merge of sublayer l)
//   coefficients, Sinkhorn and z[t,c] = sum_i h_pre[t,i] x'[t, i*C+c]      (pre of sublayer l+1)
//   y[t,c] = z[t,c] / sqrt(mean_c z[t,:]^2 + eps) * w[c]                   (optional input RMSNorm)
//
// x is read from HBM once, f once, x' and z (and y) written once: per token
// 2nC + 2C elements instead of the 3nC + 2C of the merge kernel followed by
// the coefficient kernel.  Without a merge (f == NULL) the kernel is a plain
// coefficient pass over x with the optional RMSNorm.
//
// One persistent kernel, clusters of S = C/128 CTAs (one per SM).  CTA r owns
// columns [128r, 128r+128) of every stream, so everything the merge of a
// column needs (all n streams and f at that column) is in the CTA, and so is
// everything the pre-aggregate of those columns needs.  A tile is 128 tokens;
// the CTA's columns are streamed in quarters of 32.
//
//   warp 0      TMA producer: per tile and quarter (32 columns), the n x
//               chunks (and the f chunk) of 128 x 32 bf16 into a ring
//               (64-byte swizzle, 8 KB per slot; about 3.5 quarters fit, so
//               loads run well ahead of the merge).
//   warp 1      tcgen05 MMA issuer: D[128 tok, NB] += x'_chunk . phi_chunk^T
//               with phi split into bf16 hi | lo halves (held in shared memory
//               for the launch); without a merge also the Gram block x . x^T
//               whose diagonal is each row's sum of squares (with a merge the
//               merge warps sum the squares).  Double-buffered accumulator.
//   warps 2-5   row warps (thread = token row = TMEM lane): partial projection
//               and sum of squares pushed with st.async to the token's owner.
//   warp 6      coefficient warp: the owner of TPC = ceil(128/S) tokens of
//               every tile sums the S partial rows in a fixed order, applies
//               1/rms, the gates and the H_res affine map, publishes the
//               aggregation weights to every CTA and writes per-token outputs.
//   warp 7      Sinkhorn warp (full mHC): H_res of the owner's tokens.
//   warps 8-15  pre-aggregate: z for the CTA's 128 columns from x' (or x),
//               read back from L2 once the weights are in; with the RMSNorm,
//               per-row partial sums of z^2 are exchanged across the cluster
//               and y is written from the z values still in registers.
//   warps 16-19 merge warps (merge only; thread = token row): x' formed in
//               place in the ring from the x and f chunks (same swizzled
//               offset in every chunk, packed fp32 pair FMAs in the merge
//               kernel's order) and handed to the MMA issuer, which also
//               TMA-stores the x' chunks (L2 evict-last: the pre-aggregate
//               reads them back) and frees the slots once the stores have
//               read them.
//
// fp32 streams (XF; coefficient pass only, no merge or norm): the residual
// stream of the reference's bf16-autocast trainers.  A ring slot holds 128
// tokens x 32 fp32 columns (128-byte rows, 128-byte swizzle, 16 KB); warps
// 16-19 (thread = token row) read their row, sum its squares in fp32 and
// write it back over itself as [bf16 hi (32) | bf16 lo (32)], hi = rn(x),
// lo = rn(x - hi): the same 128 bytes of the same row, so no other thread's
// data is touched.  The MMA then reads the row as 64 bf16 K values, the hi
// half and the lo half each against the 32 phi rows of the chunk:
// (x_hi + x_lo) . (phi_hi + phi_lo), x to 2^-17 like phi.  z is accumulated
// in fp32 from the fp32 x read back from L2 and written as fp32.
//
// Every hand-off is an mbarrier and every wait is bounded (mhc_sm100.cuh): a
// wait that gives up sets the device error word, poisons the CTA's share of
// the outputs with NaN and exits after draining its asynchronous work.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "mhc_device.cuh"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"
#include "mhc_sm100.cuh"

namespace mhc {

__device__ int g_ch_error = 0;  // first error code recorded by the post + pre kernel

namespace ch {

using namespace sm100;

#ifndef MHC_CH_STORE_HINT
#define MHC_CH_STORE_HINT 1
#endif
constexpr int TM = 128;              // tokens per tile (UMMA M)
constexpr int COLS = 128;            // columns of every stream owned by a CTA
constexpr int QC = 32;               // columns per chunk (a quarter of the CTA's 128)
constexpr int NQ = COLS / QC;        // quarters per tile
constexpr int CHUNK = TM * QC * 2;   // one ring slot: 128 rows x 32 bf16, 64-byte swizzle
constexpr int CHUNK_F = TM * QC * 4; // fp32 streams: 128 rows x 32 fp32, 128-byte swizzle
constexpr int RING_MAX = 24;
constexpr int S_MIN = 4, S_MAX = 8;  // cluster sizes (C = 128 S)
constexpr int NZW = 8, NMW = 4;      // pre-aggregate warps, merge warps
constexpr int W_PROD = 0, W_MMA = 1, W_ROW = 2, W_COEF = 6, W_SK = 7, W_Z = 8, W_MRG = 16;
constexpr int W_CONV = 2;            // first warp that converts phi in the prologue
constexpr int HB = 2;                // aggregation-weight buffers
constexpr int HBL = 3;               // H_res logit buffers
constexpr int XSB = 4;               // "x' of tile stored" barriers
constexpr int MGB = 6;               // "merged quarter ready" barriers
constexpr int ACC_STRIDE = 256, TMEM_COLS = 512, GRAM = 64;

// warps 16-19 exist with a merge (merge warps) and for fp32 streams (convert warps)
template <bool CONV>
struct Warps {
  static constexpr int NWARPS = CONV ? W_MRG + NMW : W_MRG;
  static constexpr int NTHREADS = NWARPS * 32;
};

enum ErrCode { ERR_PROD = 31, ERR_MMA = 32, ERR_ROW = 33, ERR_COEF = 34, ERR_Z = 35, ERR_SK = 36, ERR_MRG = 37 };

template <int N, int MODE>
struct Cfg {
  static constexpr int FD = Dims<N, MODE>::FD;
  static constexpr int NB = ((2 * FD + 15) / 16) * 16;   // hi | lo projection columns
  static constexpr int IBS = ((FD + 1 + 3) / 4) * 4;     // inbox row: FD partials + sum of squares
  static constexpr int NPAR = 3 + 2 * N + N * N;
  static constexpr int HPN = N < 4 ? 4 : N;              // weights row (16-byte multiple)
  static constexpr int CH = NQ * N;                      // 32-column chunks of the CTA's slice
};

// barrier slots
constexpr int B_FULL = 0, B_EMPTY = RING_MAX, B_ACCF = 2 * RING_MAX, B_ACCE = B_ACCF + 2, B_INF = B_ACCE + 2,
              B_INE = B_INF + 1, B_HPF = B_INE + 1, B_HPE = B_HPF + HB, B_ZD = B_HPE + HB, B_ZGO = B_ZD + HB,
              B_LGF = B_ZGO + HB, B_LGE = B_LGF + HBL, B_MRG = B_LGE + HBL, B_XSF = B_MRG + MGB,
              B_XSE = B_XSF + XSB, B_ZSF = B_XSE + XSB, B_SSF = B_ZSF + HB, B_SSE = B_SSF + 2,
              B_DRAIN = B_SSE + 2, B_PHI = B_DRAIN + 1, NBARS = B_PHI + 1;

struct Layout {
  uint32_t ring, phi, inbox, hp, lg, zss, nw, ssb, par, bar, tmem, abort, total;
};

__host__ __device__ inline Layout make_layout(int RING, int SLOT, int CH, int NB, int IBS, int HPN, int NPAR, int S,
                                              int TPC, int norm) {
  Layout L;
  uint32_t o = 0;
  L.ring = o;  o += (uint32_t)RING * SLOT;
  L.phi = o;   o += (uint32_t)CH * NB * 64;
  L.inbox = o; o += (uint32_t)S * TPC * IBS * 4;
  L.hp = o;    o += (uint32_t)HB * TM * HPN * 4;
  L.lg = o;    o += (uint32_t)HBL * TPC * 16 * 4;       // H_res logits of the owner's tokens (n <= 4)
  L.zss = o;   o += norm ? (uint32_t)HB * S * TM * 4 : 0u;  // partial sums of z^2 from every CTA
  L.nw = o;    o += norm ? (uint32_t)COLS * 4 : 0u;          // RMSNorm weight of the CTA's columns
  L.ssb = o;   o += 2u * TM * 4;                             // merged rows' sums of squares (2 tiles)
  L.par = o;   o += ((NPAR * 4 + 15) / 16) * 16;
  L.bar = o;   o += NBARS * 8;
  L.tmem = o;  o += 4;
  L.abort = o; o += 4;
  L.total = o;
  return L;
}

struct Args {
  int64_t T;
  int C, nC, S, TPC, RING;
  const void *phi;
  CoefParams p;
  const void *xz;            // what the pre-aggregate reads: x' (merge) or x (bf16, or fp32 for XF)
  __nv_bfloat16 *x_out;      // x' (merge), for poisoning
  const void *hres_prev;     // merge coefficients of the previous sublayer (NULL: H_res = I)
  const void *hpost_prev;
  int prev_dtype;
  void *z;                   // pre-aggregate (x's dtype)
  __nv_bfloat16 *y;          // its RMSNorm (may be NULL)
  const void *norm_w;
  int norm_dtype;
  float norm_eps;
  void *h_pre, *h_post, *h_res;
  int coef_dtype;
  float *inv_rms, *mixes;
  int *err_flag;
};

// byte offset of element (row j, column kk < 32) inside one phi chunk block:
// 64-byte swizzled K-major rows (8-row atoms of 512 B; 16-byte granule index
// XOR bits 1-2 of the row)
__device__ __forceinline__ uint32_t phi_off(int j, int kk) {
  return (uint32_t)(j >> 3) * 512 + (j & 7) * 64 + ((((kk >> 3) ^ ((j >> 1) & 3))) << 4) + ((kk & 7) << 1);
}

__device__ __forceinline__ void record_error(int code, volatile int *abort_flag, int *err_flag) {
  *abort_flag = 1;
  report_give_up(&g_ch_error, err_flag, code);
}

// 2-D tiled store with an L2 eviction-priority hint (x' is read again from L2
// by the pre-aggregate of the same tile).
__device__ __forceinline__ void tma_store_2d_hint(const void *tmap, uint32_t src, int x, int y, uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;"
               ::"l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(src), "l"(policy)
               : "memory");
}
// completed async-proxy (TMA store) writes before generic reads of them
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// After a wait gave up the CTA overwrites its share of every tile of its
// cluster with NaN: its 128 columns of z, y and x' and the per-token outputs
// of the tokens it owns.
template <int N, int MODE, bool XF>
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
      if (XF) reinterpret_cast<float *>(a.z)[(t0 + r) * a.C + c0 + c] = qnan;
      else reinterpret_cast<__nv_bfloat16 *>(a.z)[(t0 + r) * a.C + c0 + c] = bnan;
      if (a.y) a.y[(t0 + r) * a.C + c0 + c] = bnan;
      if (a.x_out)
        for (int i = 0; i < N; ++i) a.x_out[(t0 + r) * a.nC + i * a.C + c0 + c] = bnan;
    }
    const int cnt = min(a.TPC, TM - rank * a.TPC);
    for (int e = tid; e < cnt; e += nthreads) {
      const int64_t tok = t0 + rank * a.TPC + e;
      if (tok >= a.T) continue;
      a.inv_rms[tok] = qnan;
      for (int j = 0; j < FD; ++j) a.mixes[tok * FD + j] = qnan;
      for (int i = 0; i < N; ++i) {
        if (a.h_pre) store_dyn(a.h_pre, a.coef_dtype, tok * N + i, qnan);
        store_dyn(a.h_post, a.coef_dtype, tok * N + i, qnan);
      }
      if constexpr (MODE == FULL) {
        if (a.h_res)
          for (int k = 0; k < N * N; ++k) store_dyn(a.h_res, a.coef_dtype, tok * N * N + k, qnan);
      }
    }
  }
}

template <int N, int MODE>
__device__ __forceinline__ void load_params(float *par, const CoefParams &p, int tid, int nthreads) {
  constexpr int NPAR = 3 + 2 * N + N * N;
  for (int i = tid; i < NPAR; i += nthreads) {
    float v = 0.f;
    const int dt = p.param_dtype;
    if (i == 0) v = load_dyn(p.alpha_pre, dt, 0);
    else if (i == 1) v = load_dyn(p.alpha_post, dt, 0);
    else if (i == 2) { if (MODE == FULL) v = load_dyn(p.alpha_res, dt, 0); }
    else if (i < 3 + N) v = load_dyn(p.bias_pre, dt, i - 3);
    else if (i < 3 + 2 * N) v = load_dyn(p.bias_post, dt, i - 3 - N);
    else { if (MODE == FULL) v = load_dyn(p.bias_res, dt, i - 3 - 2 * N); }
    par[i] = v;
  }
}

template <int N, int MODE, bool MERGE, bool NORM, bool XF>
__global__ void __launch_bounds__(Warps<MERGE || XF>::NTHREADS, 1)
post_pre_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmf,
                const __grid_constant__ CUtensorMap tmo, Args a) {
  static_assert(!(XF && (MERGE || NORM)), "fp32 streams: coefficient pass only");
  using Cf = Cfg<N, MODE>;
  constexpr int FD = Cf::FD, NB = Cf::NB, IBS = Cf::IBS, NPAR = Cf::NPAR, HPN = Cf::HPN, CH = Cf::CH;
  constexpr bool CONV = MERGE || XF;     // warps 16-19 rewrite the ring slots before the MMA
  constexpr int NTHREADS = Warps<CONV>::NTHREADS, NWARPS = Warps<CONV>::NWARPS;
  constexpr int NCONV = NWARPS - W_CONV;
  constexpr int NL = MERGE ? N + 1 : N;  // ring slots per quarter (x chunks, then f)
  constexpr uint32_t SLOT = XF ? CHUNK_F : CHUNK;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t *base = smem_raw + (base_u32 - raw_u32);
  const int S = a.S, TPC = a.TPC, RING = a.RING;
  const Layout L = make_layout(RING, SLOT, CH, NB, IBS, HPN, NPAR, S, TPC, NORM ? 1 : 0);
  float *inbox = reinterpret_cast<float *>(base + L.inbox);
  float *hp = reinterpret_cast<float *>(base + L.hp);
  float *lg = reinterpret_cast<float *>(base + L.lg);
  float *zss = reinterpret_cast<float *>(base + L.zss);
  float *nw = reinterpret_cast<float *>(base + L.nw);
  float *ssb = reinterpret_cast<float *>(base + L.ssb);
  float *par = reinterpret_cast<float *>(base + L.par);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(base + L.abort);
  const uint32_t bar0 = base_u32 + L.bar;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
#define WAIT_WARP(CL, bar, par) (__all_sync(0xffffffffu, wait_parity<CL>((bar), (par), abort_flag)))

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank(), cid = cluster_id_x(), ncl = ncluster_x();
  const int ntiles = (int)((a.T + TM - 1) / TM);
  const int c0 = (int)rank * COLS;                                   // first owned column of every stream
  const int cnt = min(TPC, TM - (int)rank * TPC);                    // tokens of a tile this CTA owns
  const uint32_t inbox_tx = (uint32_t)(S * cnt * IBS * 4);           // partial rows landing per tile
  constexpr uint32_t HP_TX = (uint32_t)TM * HPN * 4;                 // weights landing per tile

  // ---------------- prologue ----------------
  if (tid == 0) {
    *abort_flag = 0;
    for (int i = 0; i < RING; ++i) {
      mbar_init(BAR(B_FULL + i), 1);
      // merge: x' slots are freed by the MMA commit and by the end of the x'
      // store's shared-memory reads, f slots by the MMA issuer (two arrivals)
      mbar_init(BAR(B_EMPTY + i), MERGE ? 2 : 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(B_ACCF + b), 1);
      mbar_init(BAR(B_ACCE + b), 4);
    }
    mbar_init(BAR(B_INF), 1);              // armed by the coefficient warp; st.async bytes complete it
    mbar_init(BAR(B_INE), S);              // one per owner CTA (inbox rows consumed)
    for (int b = 0; b < HB; ++b) {
      mbar_init(BAR(B_HPF + b), 1);        // armed by a pre-aggregate warp; st.async bytes complete it
      mbar_init(BAR(B_HPE + b), S);        // one per CTA (its pre-aggregate of the tile is done)
      mbar_init(BAR(B_ZD + b), NZW);       // local: pre-aggregate warps done
      mbar_init(BAR(B_ZGO + b), 1);        // local: the tile's source is in L2
      mbar_init(BAR(B_ZSF + b), 1);        // armed by a pre-aggregate warp; st.async bytes complete it
    }
    for (int b = 0; b < HBL; ++b) {
      mbar_init(BAR(B_LGF + b), 1);
      mbar_init(BAR(B_LGE + b), 1);
    }
    for (int b = 0; b < MGB; ++b) mbar_init(BAR(B_MRG + b), NMW);  // one per merge / convert warp
    for (int b = 0; b < XSB; ++b) {
      mbar_init(BAR(B_XSF + b), 1);        // x' of the tile complete in global memory
      mbar_init(BAR(B_XSE + b), 1);        // coefficient warp saw it
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(B_SSF + b), NMW);      // merge / convert warps wrote the tile's sums of squares
      mbar_init(BAR(B_SSE + b), 4);        // row warps read them
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
  cluster_sync_all();        // every CTA's barriers exist before any remote arrive or st.async
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(base + L.tmem);
  grid_dep_launch();
  grid_dep_wait();
  if (warp >= W_CONV) {
    // phi rows of the CTA's slice -> bf16 hi | lo, K-major, 64-byte swizzle.
    // Local K index k: chunk k/32 = (stream i = chunk/NQ, quarter chunk%NQ),
    // global phi row i*C + 128 rank + 32 quarter + k%32.
    const int ctid = tid - W_CONV * 32, nconv = NCONV * 32;
    auto grow = [&](int k) -> int64_t {
      const int c = k >> 5;
      return (int64_t)(c / NQ) * a.C + c0 + (c % NQ) * QC + (k & 31);
    };
    auto put = [&](int k, int j, float v) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
      uint8_t *blk = base + L.phi + (uint32_t)(k >> 5) * NB * 64;
      *reinterpret_cast<__nv_bfloat16 *>(blk + phi_off(j, k & 31)) = hi;
      *reinterpret_cast<__nv_bfloat16 *>(blk + phi_off(j + FD, k & 31)) = lo;
    };
    constexpr int KS = CH * QC;
    for (int e0 = ctid; e0 < KS * FD; e0 += 8 * nconv) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * nconv;
        if (e < KS * FD) {
          const int k = e / FD, j = e - k * FD;
          v[u] = load_dyn(a.phi, a.p.param_dtype, grow(k) * FD + j);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * nconv;
        if (e < KS * FD) {
          const int k = e / FD, j = e - k * FD;
          put(k, j, v[u]);
        }
      }
    }
    constexpr int PADR = NB - 2 * FD;
    if constexpr (PADR > 0) {
      for (int e = ctid; e < KS * PADR; e += nconv) {
        const int k = e / PADR, j = 2 * FD + (e - k * PADR);
        *reinterpret_cast<__nv_bfloat16 *>(base + L.phi + (uint32_t)(k >> 5) * NB * 64 + phi_off(j, k & 31)) =
            __float2bfloat16_rn(0.f);
      }
    }
    load_params<N, MODE>(par, a.p, ctid, nconv);
    if constexpr (NORM) {
      for (int c = ctid; c < COLS; c += nconv) nw[c] = load_dyn(a.norm_w, a.norm_dtype, c0 + c);
    }
    fence_proxy_async_smem();  // generic phi writes -> tensor-core (async proxy) reads
    __syncwarp();
    if (lane == 0) mbar_arrive(BAR(B_PHI));
  }

  if (warp == W_PROD) {
    if (lane == 0) {
      // ---------------- chunk producer ----------------
      // x is re-read from L2 by the pre-aggregate when there is no merge;
      // with a merge it is read once (x' is what is re-read)
      const uint64_t xpol = MERGE ? l2_policy_evict_first() : l2_policy_evict_last();
      const uint64_t fpol = l2_policy_evict_first();
      uint32_t q = 0;
      bool ok = true;
      for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl) {
        for (int qq = 0; qq < NQ && ok; ++qq) {
          for (int i = 0; i < NL; ++i, ++q) {
            const uint32_t slot = q % RING, ph = (q / RING) & 1u;
            if (!wait_parity<false>(BAR(B_EMPTY + slot), ph ^ 1u, abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(BAR(B_FULL + slot), SLOT);
            const uint32_t dst = base_u32 + L.ring + slot * SLOT;
            if (i < N) tma_load_2d_hint(dst, &tmx, i * a.C + c0 + qq * QC, tile * TM, BAR(B_FULL + slot), xpol);
            else tma_load_2d_hint(dst, &tmf, c0 + qq * QC, tile * TM, BAR(B_FULL + slot), fpol);
          }
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
      constexpr uint32_t gdesc = umma_idesc_bf16_f32(128, 128);
      const uint64_t opol = l2_policy_evict_last();
      uint32_t q = 0, hq = 0;
      int lt = 0;
      bool ok = wait_parity<false>(BAR(B_PHI), 0u, abort_flag);  // phi slice converted
      for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
        const int buf = lt & 1;
        const uint32_t aph = (uint32_t)(lt >> 1) & 1u;
        if (!wait_parity<false>(BAR(B_ACCE + buf), aph ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + (uint32_t)buf * ACC_STRIDE;
        for (int qq = 0; qq < NQ && ok; ++qq, ++hq) {
          if (CONV) {
            // the merge warps formed this quarter's x' chunks in place (fp32
            // streams: the convert warps split them into bf16 hi | lo)
            if (!wait_parity<false>(BAR(B_MRG + hq % MGB), (hq / MGB) & 1u, abort_flag)) { ok = false; break; }
            tc_fence_after();
          }
          for (int i = 0; i < NL; ++i, ++q) {
            const uint32_t slot = q % RING, ph = (q / RING) & 1u;
            if (i == N) continue;  // the f chunk: the store warp frees it
            if (!CONV) {
              if (!wait_parity<false>(BAR(B_FULL + slot), ph, abort_flag)) { ok = false; break; }
              tc_fence_after();
            }
            const uint32_t a0 = base_u32 + L.ring + slot * SLOT;
            const uint32_t b0 = base_u32 + L.phi + (uint32_t)(i * NQ + qq) * NB * 64u;
            if constexpr (XF) {
              // 128-byte rows [hi k0..31 | lo k0..31]: K steps 0-1 the hi
              // half, 2-3 the lo half, each against phi rows k0..31
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_bf16(dcol, umma_desc_sw128(a0 + k * 32), umma_desc_sw64(b0 + (k & 1) * 32), idesc,
                          (qq | i | k) != 0 ? 1u : 0u);
            } else {
#pragma unroll
              for (int k = 0; k < 2; ++k) {
                const uint64_t ad = umma_desc_sw64(a0 + k * 32);
                const uint32_t accum = (qq | i | k) != 0 ? 1u : 0u;
                umma_bf16(dcol, ad, umma_desc_sw64(b0 + k * 32), idesc, accum);
                // sum of squares of each row = diagonal of x . x^T
                if (!MERGE) umma_bf16(dcol + GRAM, ad, ad, gdesc, accum);
              }
            }
            umma_commit(BAR(B_EMPTY + slot));
          }
          if (MERGE && ok) {
            // x' of the quarter to global memory; its slots (and the f slot,
            // which the merge has read) are free once the stores have read them
            const uint32_t q0 = q - NL;
#pragma unroll
            for (int i = 0; i < N; ++i) {
#if MHC_CH_STORE_HINT
              tma_store_2d_hint(&tmo, base_u32 + L.ring + ((q0 + i) % RING) * SLOT, i * a.C + c0 + qq * QC,
                                tile * TM, opol);
#else
              tma_store_2d(&tmo, base_u32 + L.ring + ((q0 + i) % RING) * SLOT, i * a.C + c0 + qq * QC, tile * TM);
#endif
            }
            bulk_commit();
            mbar_arrive(BAR(B_EMPTY + (q0 + N) % RING));
            mbar_arrive(BAR(B_EMPTY + (q0 + N) % RING));
            bulk_wait_read_all();
#pragma unroll
            for (int i = 0; i < N; ++i) mbar_arrive(BAR(B_EMPTY + (q0 + i) % RING));
          }
        }
        if (!ok) break;
        umma_commit(BAR(B_ACCF + buf));
        if (MERGE) {
          // the tile's x' is complete in global memory before the
          // pre-aggregate reads it back (the coefficient warp passes it on,
          // at most XSB tiles behind)
          bulk_wait_all();
          fence_proxy_async_global();
          const int xsb = lt % XSB;
          if (!wait_parity<false>(BAR(B_XSE + xsb), ((uint32_t)(lt / XSB) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive(BAR(B_XSF + xsb));
        }
      }
      if (!ok) record_error(ERR_MMA, abort_flag, a.err_flag);
      if (MERGE) bulk_wait_all();  // no store may still read shared memory at exit
      // every issued MMA completes before TMEM is released
      umma_commit(BAR(B_DRAIN));
      wait_parity<false>(BAR(B_DRAIN), 0u, nullptr);
    }
    __syncwarp();
  }
  else if (warp >= W_ROW && warp < W_ROW + 4) {
    // ---------------- row warps ----------------
    const int quad = warp & 3;            // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;     // token row of the tile = TMEM lane
    const int owner = row / TPC;
    int lt = 0;
    bool ok = true;
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const int buf = lt & 1;
      const uint32_t aph = (uint32_t)(lt >> 1) & 1u;
      if (!WAIT_WARP(false, BAR(B_ACCF + buf), aph)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)buf * ACC_STRIDE;
      float d[NB];
#pragma unroll
      for (int c16 = 0; c16 < NB / 16; ++c16) {
        float t16[16];
        tmem_ld16(tb + (uint32_t)c16 * 16u, t16);
#pragma unroll
        for (int i = 0; i < 16; ++i) d[c16 * 16 + i] = t16[i];
      }
      float ss = 0.f;
      if constexpr (!CONV) {
        // Gram diagonal: this lane's row is column quad*32 + lane of the block
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float t16[16];
          tmem_ld16(tb + GRAM + (uint32_t)(quad * 32 + h * 16), t16);
#pragma unroll
          for (int i = 0; i < 16; ++i) ss = (lane == h * 16 + i) ? t16[i] : ss;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_ACCE + buf));
      if constexpr (CONV) {
        // the merge / convert warps' sum of squares of the row
        if (!WAIT_WARP(false, BAR(B_SSF + buf), aph)) { ok = false; break; }
        ss = ssb[buf * TM + row];
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_SSE + buf));
      }
      float vals[IBS];
#pragma unroll
      for (int j = 0; j < IBS; ++j) vals[j] = 0.f;
#pragma unroll
      for (int j = 0; j < FD; ++j) vals[j] = d[j] + d[FD + j];
      vals[FD] = ss;
      // the owners' inbox must have been drained (previous tile)
      if (!WAIT_WARP(true, BAR(B_INE), ((uint32_t)lt & 1u) ^ 1u)) { ok = false; break; }
      const uint32_t dst =
          mapa(base_u32 + L.inbox + (uint32_t)(((int)rank * TPC + (row - owner * TPC)) * IBS * 4), (uint32_t)owner);
      const uint32_t dbar = mapa(BAR(B_INF), (uint32_t)owner);
#pragma unroll
      for (int v = 0; v < IBS / 4; ++v)
        st_async_v4(dst + v * 16, vals[4 * v], vals[4 * v + 1], vals[4 * v + 2], vals[4 * v + 3], dbar);
    }
    if (!ok) record_error(ERR_ROW, abort_flag, a.err_flag);
  } else if (warp == W_COEF) {
    // ---------------- coefficient warp ----------------
    int lt = 0;
    bool ok = WAIT_WARP(false, BAR(B_PHI), 0u);  // gate parameters loaded
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const int hb = lt % HB;
      const uint32_t iph = (uint32_t)lt & 1u, hph = (uint32_t)(lt / HB) & 1u;
      if (lane == 0) mbar_arrive_expect_tx(BAR(B_INF), inbox_tx);  // arm: S slices' rows of the owned tokens
      if (!WAIT_WARP(true, BAR(B_INF), iph)) { ok = false; break; }
      float acc[IBS];
#pragma unroll
      for (int j = 0; j < IBS; ++j) acc[j] = 0.f;
      if (lane < cnt) {
#pragma unroll 2
        for (int s = 0; s < S; ++s) {  // fixed order over the column slices: deterministic
          const float4 *src = reinterpret_cast<const float4 *>(inbox + (s * TPC + lane) * IBS);
#pragma unroll
          for (int v = 0; v < IBS / 4; ++v) {
            const float4 q4 = src[v];
            acc[4 * v] += q4.x; acc[4 * v + 1] += q4.y; acc[4 * v + 2] += q4.z; acc[4 * v + 3] += q4.w;
          }
        }
      }
      __syncwarp();
      if (lane < S) mbar_arrive_remote(mapa(BAR(B_INE), (uint32_t)lane));  // inbox rows free again
      const int t = (int)rank * TPC + lane;  // token row of the tile
      const int64_t tok = (int64_t)tile * TM + t;
      const bool live = lane < cnt && tok < a.T;
      float w[HPN], m[FD], ho[N];
      float inv = 0.f;
#pragma unroll
      for (int i = 0; i < HPN; ++i) w[i] = 0.f;
      // the weights buffer `hb` must be free in every CTA (tile lt-HB done everywhere)
      if (!WAIT_WARP(true, BAR(B_HPE + hb), hph ^ 1u)) { ok = false; break; }
      if constexpr (MERGE) {
        // this CTA's x' columns of the tile are stored and visible
        const int xb = lt % XSB;
        if (!WAIT_WARP(false, BAR(B_XSF + xb), (uint32_t)(lt / XSB) & 1u)) { ok = false; break; }
        if (lane == 0) mbar_arrive(BAR(B_XSE + xb));
      }
      // the tile's source (x, or x') is in L2: the pre-aggregate may load it
      if (lane == 0) mbar_arrive(BAR(B_ZGO + hb));
      const int lb = lt % HBL;
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
          ho[i] = sigmoidf_(__fadd_rn(__fmul_rn(m[N + i], par[1]), par[3 + N + i])) * a.p.post_mult;
        }
        if constexpr (MODE == FULL) {
          float *lrow = lg + (lb * TPC + lane) * 16;
#pragma unroll
          for (int k = 0; k < N * N; ++k) lrow[k] = __fadd_rn(__fmul_rn(m[2 * N + k], par[2]), par[3 + 2 * N + k]);
        }
        // publish the aggregation weights to every CTA of the cluster
        const uint32_t loc = base_u32 + L.hp + (uint32_t)((hb * TM + t) * HPN * 4);
#pragma unroll 1
        for (int dcta = 0; dcta < S; ++dcta) {
          const uint32_t dst = mapa(loc, (uint32_t)dcta);
          const uint32_t dbar = mapa(BAR(B_HPF + hb), (uint32_t)dcta);
#pragma unroll
          for (int v = 0; v < HPN / 4; ++v)
            st_async_v4(dst + v * 16, w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3], dbar);
        }
      }
      if constexpr (MODE == FULL) {
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_LGF + lb));  // logits ready for the Sinkhorn warp
      }
      if (live) {
        a.inv_rms[tok] = inv;
#pragma unroll
        for (int j = 0; j < FD; ++j) a.mixes[tok * FD + j] = m[j];
#pragma unroll
        for (int i = 0; i < N; ++i) {
          if (a.h_pre) store_dyn(a.h_pre, a.coef_dtype, tok * N + i, w[i]);
          store_dyn(a.h_post, a.coef_dtype, tok * N + i, ho[i]);
        }
      }
    }
    if (!ok) record_error(ERR_COEF, abort_flag, a.err_flag);
  } else if (warp == W_SK) {
    // ---------------- Sinkhorn warp: H_res of the owned tokens ----------------
    if constexpr (MODE == FULL) {
      int lt = 0;
      bool ok = true;
      for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
        const int lb = lt % HBL;
        if (!WAIT_WARP(false, BAR(B_LGF + lb), (uint32_t)(lt / HBL) & 1u)) { ok = false; break; }
        const int64_t tok = (int64_t)tile * TM + (int)rank * TPC + lane;
        if (lane < cnt && tok < a.T) {
          float hm[N * N];
#pragma unroll
          for (int k = 0; k < N * N; ++k) hm[k] = lg[(lb * TPC + lane) * 16 + k];
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
  }
  else if (warp >= W_Z && warp < W_Z + NZW) {
    // ---------------- pre-aggregate warps ----------------
    // thread = (vector v of 8 columns, rows r0 + 16u, u < 8): 128 rows x 16
    // vectors over 256 threads; a row's 16 vectors are one half-warp.
    // (fp32 streams: an item is 8 fp32 columns, two 16-byte vectors per stream)
    constexpr int IPT = 8, IPB = (NORM || XF) ? 2 : 4;  // items per thread, items per batch of loads
    constexpr int XV = XF ? 2 : 1;                      // 16-byte vectors per stream and item
    const int ztid = tid - W_Z * 32;
    const int v = ztid & 15, r0 = ztid >> 4;
    int lt = 0;
    bool ok = true;
    if constexpr (NORM) ok = WAIT_WARP(false, BAR(B_PHI), 0u);  // RMSNorm weight staged
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const int hb = lt % HB;
      const uint32_t hph = (uint32_t)(lt / HB) & 1u;
      if (warp == W_Z && lane == 0) {
        mbar_arrive_expect_tx(BAR(B_HPF + hb), HP_TX);  // arm: every owner's weights
        if (NORM) mbar_arrive_expect_tx(BAR(B_ZSF + hb), (uint32_t)(S * TM * 4));  // every CTA's z^2 sums
      }
      if (!WAIT_WARP(false, BAR(B_ZGO + hb), hph)) { ok = false; break; }
      const int64_t t0 = (int64_t)tile * TM;
      const int rows = a.T - t0 < TM ? (int)(a.T - t0) : TM;
      constexpr int ES = XF ? 4 : 2;  // element bytes of x and z
      const uint8_t *xb = reinterpret_cast<const uint8_t *>(a.xz) + (t0 * a.nC + c0 + v * 8) * ES;
      uint8_t *zb = reinterpret_cast<uint8_t *>(a.z) + (t0 * a.C + c0 + v * 8) * ES;
      const float *hps = hp + hb * TM * HPN;
      uint4 zk[NORM ? IPT : 1];
      float ss[NORM ? IPT : 1];
#pragma unroll
      for (int b = 0; b < IPT / IPB; ++b) {
        uint4 xv[IPB][N][XV];
#pragma unroll
        for (int u = 0; u < IPB; ++u) {
          const int r = r0 + 16 * (b * IPB + u);
          if (r < rows) {
#pragma unroll
            for (int st = 0; st < N; ++st)
#pragma unroll
              for (int h = 0; h < XV; ++h)
                xv[u][st][h] = __ldcs(
                    reinterpret_cast<const uint4 *>(xb + ((int64_t)r * a.nC + st * a.C) * ES + h * 16));
          }
        }
        if (b == 0) {
          if (!WAIT_WARP(true, BAR(B_HPF + hb), hph)) { ok = false; break; }
        }
#pragma unroll
        for (int u = 0; u < IPB; ++u) {
          const int r = r0 + 16 * (b * IPB + u);
          uint4 out = make_uint4(0u, 0u, 0u, 0u);
          if (r < rows) {
            float wv[HPN];
#pragma unroll
            for (int v4 = 0; v4 < HPN / 4; ++v4) {
              const float4 q4 = *reinterpret_cast<const float4 *>(hps + r * HPN + 4 * v4);
              wv[4 * v4] = q4.x; wv[4 * v4 + 1] = q4.y; wv[4 * v4 + 2] = q4.z; wv[4 * v4 + 3] = q4.w;
            }
            // fp32 accumulation in packed pairs: acc[j] holds columns 2j, 2j+1
            uint64_t acc[4];
#pragma unroll
            for (int st = 0; st < N; ++st) {
              const uint64_t w2 = f2_pack(wv[st], wv[st]);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint64_t xp;
                if constexpr (XF) {
                  const uint4 q4 = xv[u][st][j >> 1];
                  xp = (j & 1) ? f2_pack(__uint_as_float(q4.z), __uint_as_float(q4.w))
                               : f2_pack(__uint_as_float(q4.x), __uint_as_float(q4.y));
                } else {
                  const uint32_t xw[4] = {xv[u][st][0].x, xv[u][st][0].y, xv[u][st][0].z, xv[u][st][0].w};
                  xp = bf16x2_to_f2(xw[j]);
                }
                acc[j] = st == 0 ? f2_fma(w2, xp, f2_pack(0.f, 0.f)) : f2_fma(w2, xp, acc[j]);
              }
            }
            uint8_t *zr = zb + (int64_t)r * a.C * ES;
            if constexpr (XF) {
              float o[8];
#pragma unroll
              for (int j = 0; j < 4; ++j) f2_unpack(acc[j], o[2 * j], o[2 * j + 1]);
              reinterpret_cast<float4 *>(zr)[0] = make_float4(o[0], o[1], o[2], o[3]);
              reinterpret_cast<float4 *>(zr)[1] = make_float4(o[4], o[5], o[6], o[7]);
            } else {
              uint32_t ow[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float lo, hi;
                f2_unpack(acc[j], lo, hi);
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
                ow[j] = *reinterpret_cast<const uint32_t *>(&h2);
              }
              out = make_uint4(ow[0], ow[1], ow[2], ow[3]);
              *reinterpret_cast<uint4 *>(zr) = out;
            }
          }
          if constexpr (NORM) {
            // the row's sum of squares over this vector, of the bf16 z values
            // (as a norm applied to z sees them)
            zk[b * IPB + u] = out;
            const uint32_t zw[4] = {out.x, out.y, out.z, out.w};
            float sq = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&zw[j]));
              sq = fmaf(f2.x, f2.x, sq);
              sq = fmaf(f2.y, f2.y, sq);
            }
            ss[b * IPB + u] = sq;
          }
        }
      }
      if (!ok) break;
      if constexpr (NORM) {
        // partial sum of squares of each row's 128 columns, reduced over the
        // row's half-warp and sent to every CTA of the cluster
#pragma unroll
        for (int u = 0; u < IPT; ++u)
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
        if (v == 0) {
#pragma unroll 1
          for (int d = 0; d < S; ++d) {
            const uint32_t dbar = mapa(BAR(B_ZSF + hb), (uint32_t)d);
            const uint32_t dst = mapa(base_u32 + L.zss + (uint32_t)(((hb * S + (int)rank) * TM) * 4), (uint32_t)d);
#pragma unroll
            for (int u = 0; u < IPT; ++u) st_async_f32(dst + (uint32_t)(r0 + 16 * u) * 4u, ss[u], dbar);
          }
        }
        if (!WAIT_WARP(true, BAR(B_ZSF + hb), hph)) { ok = false; break; }
        __nv_bfloat16 *yb = a.y + t0 * a.C + c0 + v * 8;
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
          const int r = r0 + 16 * u;
          if (r >= rows) continue;
          float tot = 0.f;
          for (int s = 0; s < S; ++s) tot += zss[(hb * S + s) * TM + r];  // fixed order: deterministic
          const float rr = rsqrtf(tot / (float)a.C + a.norm_eps);
          const uint32_t zw[4] = {zk[u].x, zk[u].y, zk[u].z, zk[u].w};
          uint32_t ow[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&zw[j]));
            const float2 w2 = *reinterpret_cast<const float2 *>(nw + v * 8 + 2 * j);
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(f2.x * rr * w2.x, f2.y * rr * w2.y);
            ow[j] = *reinterpret_cast<const uint32_t *>(&h2);
          }
          *reinterpret_cast<uint4 *>(yb + (int64_t)r * a.C) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      }
      // this CTA is done with the weights (and z^2 sums) of `hb`: tell every CTA
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_ZD + hb));
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
  } else if (MERGE && warp >= W_MRG && warp < W_MRG + NMW) {
    // ---------------- merge warps ----------------
    const int row = tid - W_MRG * 32;                 // token row of the tile
    const uint32_t rsw = (uint32_t)((row >> 1) & 3);  // 64-byte swizzle of the row
    const bool has_res = a.hres_prev != nullptr;
    uint32_t q = 0, hq = 0;
    bool ok = true;
    int lt = 0;
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const int64_t tok = (int64_t)tile * TM + row;
      const bool live = tok < a.T;
      uint64_t ss2 = f2_pack(0.f, 0.f);  // sum of squares of the row's bf16 x' (column pairs)
      float H[N * N], Hp[N];
#pragma unroll
      for (int k = 0; k < N * N; ++k) H[k] = (has_res && live) ? load_dyn(a.hres_prev, a.prev_dtype, tok * N * N + k) : 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) Hp[i] = live ? load_dyn(a.hpost_prev, a.prev_dtype, tok * N + i) : 0.f;
      for (int qq = 0; qq < NQ; ++qq, ++hq, q += NL) {
        uint32_t sl[NL];
#pragma unroll
        for (int i = 0; i < NL; ++i) {
          sl[i] = (q + i) % RING;
          if (!WAIT_WARP(false, BAR(B_FULL + sl[i]), ((q + i) / RING) & 1u)) { ok = false; break; }
        }
        if (!ok) break;
        // x'_i = sum_j H_res[i,j] x_j + H_post[i] f at the same swizzled
        // offset of every chunk, written back over x_i: fp32 FMAs on column
        // pairs, in the merge kernel's order (bit-identical x')
#pragma unroll
        for (int g = 0; g < QC / 8; ++g) {
          const uint32_t off = (uint32_t)row * (QC * 2) + ((((uint32_t)g) ^ rsw) << 4);
          uint4 xv[N], fv;
#pragma unroll
          for (int j = 0; j < N; ++j) xv[j] = *reinterpret_cast<const uint4 *>(base + L.ring + sl[j] * CHUNK + off);
          fv = *reinterpret_cast<const uint4 *>(base + L.ring + sl[N] * CHUNK + off);
          const uint32_t fw[4] = {fv.x, fv.y, fv.z, fv.w};
#pragma unroll
          for (int i = 0; i < N; ++i) {
            const uint64_t hp2 = f2_pack(Hp[i], Hp[i]);
            uint32_t ow[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              uint64_t acc;
              if (has_res) {
                acc = f2_pack(0.f, 0.f);
#pragma unroll
                for (int j = 0; j < N; ++j) {
                  const uint32_t xw[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
                  acc = f2_fma(f2_pack(H[i * N + j], H[i * N + j]), bf16x2_to_f2(xw[p]), acc);
                }
              } else {
                const uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
                acc = bf16x2_to_f2(xw[p]);
              }
              acc = f2_fma(hp2, bf16x2_to_f2(fw[p]), acc);
              float lo, hi;
              f2_unpack(acc, lo, hi);
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
              ow[p] = *reinterpret_cast<const uint32_t *>(&h2);
              const uint64_t r2 = bf16x2_to_f2(ow[p]);
              ss2 = f2_fma(r2, r2, ss2);
            }
            *reinterpret_cast<uint4 *>(base + L.ring + sl[i] * CHUNK + off) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
          }
        }
        fence_proxy_async_smem();  // generic x' writes -> MMA and TMA-store (async proxy) reads
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_MRG + hq % MGB));
      }
      if (!ok) break;
      // the row's sum of squares for the row warps (buffer free once they
      // read the tile two back)
      const int sb = lt & 1;
      if (!WAIT_WARP(false, BAR(B_SSE + sb), ((uint32_t)(lt >> 1) & 1u) ^ 1u)) { ok = false; break; }
      float slo, shi;
      f2_unpack(ss2, slo, shi);
      ssb[sb * TM + row] = slo + shi;
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_SSF + sb));
    }
    if (!ok) record_error(ERR_MRG, abort_flag, a.err_flag);
  } else if (XF && warp >= W_MRG && warp < W_MRG + NMW) {
    // ---------------- convert warps (fp32 streams) ----------------
    // Row `row` of a slot is 128 bytes: 32 fp32 in 16-byte granules g at
    // granule position g ^ (row & 7).  It is rewritten as 64 bf16, hi of the
    // 32 values in granules 0-3 and lo in granules 4-7 (same swizzle), which
    // the MMA reads as one 128-byte K-major row.
    const int row = tid - W_MRG * 32;
    const uint32_t r7 = (uint32_t)(row & 7);
    uint32_t q = 0, hq = 0;
    bool ok = true;
    int lt = 0;
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      uint64_t ss2 = f2_pack(0.f, 0.f);  // sum of squares of the row (column pairs)
      for (int qq = 0; qq < NQ; ++qq, ++hq) {
#pragma unroll 1
        for (int i = 0; i < N; ++i, ++q) {
          const uint32_t sl = q % RING;
          if (!WAIT_WARP(false, BAR(B_FULL + sl), (q / RING) & 1u)) { ok = false; break; }
          uint8_t *rp = base + L.ring + sl * SLOT + (uint32_t)row * 128u;
          float4 xv[8];
#pragma unroll
          for (int g = 0; g < 8; ++g) xv[g] = *reinterpret_cast<const float4 *>(rp + ((((uint32_t)g) ^ r7) << 4));
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float e[8] = {xv[2 * h].x, xv[2 * h].y, xv[2 * h].z, xv[2 * h].w,
                                xv[2 * h + 1].x, xv[2 * h + 1].y, xv[2 * h + 1].z, xv[2 * h + 1].w};
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const __nv_bfloat162 hi2 = __floats2bfloat162_rn(e[2 * p], e[2 * p + 1]);
              const float2 hf = __bfloat1622float2(hi2);
              const __nv_bfloat162 lo2 = __floats2bfloat162_rn(e[2 * p] - hf.x, e[2 * p + 1] - hf.y);
              hw[p] = *reinterpret_cast<const uint32_t *>(&hi2);
              lw[p] = *reinterpret_cast<const uint32_t *>(&lo2);
              const uint64_t x2 = f2_pack(e[2 * p], e[2 * p + 1]);
              ss2 = f2_fma(x2, x2, ss2);
            }
            *reinterpret_cast<uint4 *>(rp + ((((uint32_t)h) ^ r7) << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(rp + ((((uint32_t)(4 + h)) ^ r7) << 4)) =
                make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
        }
        if (!ok) break;
        fence_proxy_async_smem();  // generic hi | lo writes -> MMA (async proxy) reads
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_MRG + hq % MGB));
      }
      if (!ok) break;
      // the row's sum of squares for the row warps (buffer free once they
      // read the tile two back)
      const int sb = lt & 1;
      if (!WAIT_WARP(false, BAR(B_SSE + sb), ((uint32_t)(lt >> 1) & 1u) ^ 1u)) { ok = false; break; }
      float slo, shi;
      f2_unpack(ss2, slo, shi);
      ssb[sb * TM + row] = slo + shi;
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_SSF + sb));
    }
    if (!ok) record_error(ERR_MRG, abort_flag, a.err_flag);
  }

  // ---------------- teardown ----------------
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (*abort_flag) poison_share<N, MODE, XF>(a, (int)cid, (int)ncl, (int)rank, ntiles, tid, NTHREADS);
  cluster_sync_all();  // no CTA leaves while a peer may still touch its shared memory
#undef WAIT_WARP
#undef BAR
}

}  // namespace ch
}  // namespace mhc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace mhc {
namespace ch {

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

// The longest ring that fits the shared-memory budget, at least `need` slots
// (merge: one column half = n + 1 chunks; at most MGB halves so that a
// "merged half" barrier is never two phases ahead of its waiters).
template <int N, int MODE, bool MERGE, bool NORM, bool XF>
static int pick_ring(int S, int TPC) {
  using Cf = Cfg<N, MODE>;
  const int slot = XF ? CHUNK_F : CHUNK;
  const int need = MERGE ? N + 1 : (XF ? N : 3);
  // merge / convert: the warps 16-19 run at most RING / quarter ahead of the
  // MMA issuer, which must stay under MGB quarters
  const int cap = MERGE ? (MGB * (N + 1) < RING_MAX ? MGB * (N + 1) : RING_MAX)
                        : (XF ? ((MGB - 1) * N < RING_MAX ? (MGB - 1) * N : RING_MAX) : RING_MAX);
  for (int r = cap; r >= need; --r)
    if ((size_t)make_layout(r, slot, Cf::CH, Cf::NB, Cf::IBS, Cf::HPN, Cf::NPAR, S, TPC, NORM ? 1 : 0).total + 1024 <=
        SMEM_LIMIT)
      return r;
  return 0;
}

// a (rows x cols) row-major matrix in 128-row x 32-column boxes: bf16 with a
// 64-byte swizzle (the MMA's K-major operand layout for 64-byte rows), fp32
// with a 128-byte swizzle (128-byte rows)
static bool encode_2d(CUtensorMap &m, const void *p, int64_t rows, int64_t cols, bool f32 = false) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * (f32 ? 4 : 2)};
  const cuuint32_t box[2] = {(cuuint32_t)QC, (cuuint32_t)TM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(p),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per kernel instantiation, device and cluster size: the number of
// co-resident clusters (the dynamic shared memory limit is raised once).
struct KernEntry {
  const void *kern;
  int dev, S;
  int clusters;
};
static std::mutex g_mu;
static KernEntry g_kerns[64];
static int g_kerns_n = 0;

template <int N, int MODE, bool MERGE, bool NORM, bool XF = false>
static cudaError_t launch_impl(const void *x, const void *f, Args a, cudaStream_t stream) {
  using Cf = Cfg<N, MODE>;
  a.RING = pick_ring<N, MODE, MERGE, NORM, XF>(a.S, a.TPC);
  if (a.RING == 0) return cudaErrorNotSupported;
  const size_t smem = (size_t)make_layout(a.RING, XF ? CHUNK_F : CHUNK, Cf::CH, Cf::NB, Cf::IBS, Cf::HPN, Cf::NPAR,
                                          a.S, a.TPC, NORM ? 1 : 0).total +
                      1024;
  auto kern = post_pre_kernel<N, MODE, MERGE, NORM, XF>;
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
  cfg.blockDim = dim3(Warps<MERGE || XF>::NTHREADS, 1, 1);
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

  CUtensorMap tmx, tmf, tmo;
  if (!encode_2d(tmx, x, a.T, a.nC, XF)) return cudaErrorNotSupported;
  if (MERGE) {
    if (!encode_2d(tmf, f, a.T, a.C)) return cudaErrorNotSupported;
    if (!encode_2d(tmo, a.x_out, a.T, a.nC)) return cudaErrorNotSupported;
  } else {
    tmf = tmx;  // unused
    tmo = tmx;  // unused
  }
  const int64_t ntiles = (a.T + TM - 1) / TM;
  const int clusters = (int)(ntiles < max_clusters ? ntiles : max_clusters);
  cfg.gridDim = dim3((unsigned)(clusters * a.S), 1, 1);
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, tmx, tmf, tmo, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace ch

bool post_pre_eligible(int mode, int n, int x_dtype, const void *x, const void *f, const void *x_out,
                       const void *z, const void *y, int64_t T, int C) {
  if (x_dtype != MHC_BF16 || T < 1) return false;
  if (mode != FULL && mode != NOHRES) return false;
  if (n != 2 && n != 4) return false;
  if (C % ch::COLS != 0) return false;
  const int S = C / ch::COLS;
  if (S < ch::S_MIN || S > ch::S_MAX) return false;
  for (const void *p : {x, f, x_out, z, y})
    if (((uintptr_t)p & 15) != 0) return false;
  return true;
}

cudaError_t launch_post_pre(int mode, int n, const void *x, const void *f, const void *h_res_prev,
                            const void *h_post_prev, int prev_dtype, void *x_out, int64_t T, int C,
                            const void *phi, const CoefParams &p, void *z, void *h_pre, void *h_post,
                            void *h_res, int coef_dtype, float *inv_rms, float *mixes, const void *norm_w,
                            int norm_dtype, float norm_eps, void *y, cudaStream_t stream) {
  ch::Args a;
  a.T = T;
  a.C = C;
  a.nC = n * C;
  a.S = C / ch::COLS;
  a.TPC = (ch::TM + a.S - 1) / a.S;
  a.RING = 0;
  a.phi = phi;
  a.p = p;
  const bool merge = f != nullptr;
  const bool norm = norm_w != nullptr;
  a.xz = merge ? x_out : x;
  a.x_out = merge ? reinterpret_cast<__nv_bfloat16 *>(x_out) : nullptr;
  a.hres_prev = h_res_prev;
  a.hpost_prev = h_post_prev;
  a.prev_dtype = prev_dtype;
  a.z = z;
  a.y = norm ? reinterpret_cast<__nv_bfloat16 *>(y) : nullptr;
  a.norm_w = norm_w;
  a.norm_dtype = norm_dtype;
  a.norm_eps = norm_eps;
  a.h_pre = h_pre;
  a.h_post = h_post;
  a.h_res = h_res;
  a.coef_dtype = coef_dtype;
  a.inv_rms = inv_rms;
  a.mixes = mixes;
  a.err_flag = host_error_flag();
  return with_mode(mode, [&](auto md) -> cudaError_t {
    constexpr int MODE = decltype(md)::value;
    if constexpr (MODE == FULL || MODE == NOHRES) {
      auto go = [&](auto nn) -> cudaError_t {
        constexpr int NN = decltype(nn)::value;
        if (merge) {
          return norm ? ch::launch_impl<NN, MODE, true, true>(x, f, a, stream)
                      : ch::launch_impl<NN, MODE, true, false>(x, f, a, stream);
        }
        return norm ? ch::launch_impl<NN, MODE, false, true>(x, f, a, stream)
                    : ch::launch_impl<NN, MODE, false, false>(x, f, a, stream);
      };
      if (n == 2) return go(std::integral_constant<int, 2>{});
      if (n == 4) return go(std::integral_constant<int, 4>{});
    }
    return cudaErrorNotSupported;
  });
}

bool pre_xf_eligible(int mode, int n, int x_dtype, const void *x, const void *z, int64_t T, int C) {
  if (x_dtype != MHC_F32 || T < 1) return false;
  if (mode != FULL && mode != NOHRES) return false;
  if (n != 2 && n != 4) return false;
  if (C % ch::COLS != 0) return false;
  const int S = C / ch::COLS;
  if (S < ch::S_MIN || S > ch::S_MAX) return false;
  return ((uintptr_t)x & 15) == 0 && ((uintptr_t)z & 15) == 0;
}

cudaError_t launch_pre_xf(int mode, int n, const void *x, int64_t T, int C, const void *phi, const CoefParams &p,
                          void *z, void *h_pre, void *h_post, void *h_res, int coef_dtype, float *inv_rms,
                          float *mixes, cudaStream_t stream) {
  ch::Args a = {};
  a.T = T;
  a.C = C;
  a.nC = n * C;
  a.S = C / ch::COLS;
  a.TPC = (ch::TM + a.S - 1) / a.S;
  a.phi = phi;
  a.p = p;
  a.xz = x;
  a.z = z;
  a.h_pre = h_pre;
  a.h_post = h_post;
  a.h_res = h_res;
  a.coef_dtype = coef_dtype;
  a.inv_rms = inv_rms;
  a.mixes = mixes;
  a.err_flag = host_error_flag();
  return with_mode(mode, [&](auto md) -> cudaError_t {
    constexpr int MODE = decltype(md)::value;
    if constexpr (MODE == FULL || MODE == NOHRES) {
      if (n == 2) return ch::launch_impl<2, MODE, false, false, true>(x, nullptr, a, stream);
      if (n == 4) return ch::launch_impl<4, MODE, false, false, true>(x, nullptr, a, stream);
    }
    return cudaErrorNotSupported;
  });
}

int read_ch_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ch_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_ch_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace mhc
