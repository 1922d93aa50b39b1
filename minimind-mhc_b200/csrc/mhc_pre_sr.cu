// Single-read fused coefficient + pre-aggregate kernel for bf16 activations
// on sm_100a: x is read from HBM exactly once.
//
// The coefficients of a token depend on its whole n*C row (RMS statistics and
// the n*C x FD projection) and the sublayer input z = sum_i w_i x_i needs
// them, so every x element is needed twice: once before the token's weights
// exist and once after.  Here the second use reads an on-chip copy (TMEM)
// instead of HBM or L2.
//
// One persistent kernel per call, launched as clusters of S = C / 128 CTAs
// (4 <= S <= 8; one CTA per SM).  CTA r of a cluster owns columns
// [128 r, 128 r + 128) of every stream: its K slice of the projection is those
// n x 128 columns, and it computes z for the same 128 columns, so everything
// it needs for z is in its own slice.  A cluster walks a sequence of
// 128-token tiles; a tile's slice is n chunks of 128 rows x 128 columns (32
// KB, one per stream, each one 3-D TMA box of two 128-row x 64-column blocks
// with a 128-byte swizzle).  Chunks are large because every tensor-pipe
// operation on a chunk (copy, MMA, commit) costs a fixed time besides its bytes.
//
//   warp 0       TMA producer: x chunks into a shared-memory ring.
//   warp 1       tcgen05 MMA issuer: D[128 tok, NB] += x_chunk . phi_chunk^T
//                (M = 128, K = 16 per instruction, fp32 accumulator in TMEM).
//                phi's slice is split once per launch into bf16 hi | lo halves
//                held in shared memory (projection accurate to ~2^-17).
//   warp 2       copier: tcgen05.cp of each landed chunk from the ring into a
//                TMEM retention slot (7 slots of 64 columns).  The ring slot
//                is free once both the MMA issuer's and the copier's commits
//                have arrived; no other thread touches the ring.
//   warps 3-6    row warps (thread = token row = TMEM lane): once a tile is
//                retained and projected, each reads its row's retained chunks
//                from TMEM for the sum of squares, reads the slice's
//                projection partial, and pushes, with st.async, the H_pre
//                partials and the sum of squares of its row to every CTA of
//                the cluster and the remaining partials (H_post, H_res) to the
//                row's owner CTA (row r -> CTA r mod S).  One barrier wait per
//                tile instead of per chunk.
//   warp 7       coefficient warp (owner of rows r = rank + S l): sums the S
//                slices in a fixed order (deterministic), applies 1/rms, the
//                sigmoid gates and the H_res affine map and writes the
//                per-token outputs.
//   warps 8-9    Sinkhorn warps (alternate tiles): H_res of the owned rows, one
//                token per lane, the matrix in registers.
//   warps 10-13  z warps (thread = token row, one TMEM lane quadrant each):
//                each computes its row's aggregation weights
//                from the S pushed partials (the same operations, in the same
//                order, as the owner), reads its block's n retained chunks back
//                from TMEM, accumulates z in fp32 packed pairs and stores its
//                row's 128 z columns; the retention slots are then free.
//
// The weights therefore need a single DSMEM hop after a tile's last chunk.
// x on chip per CTA: the ring's landing slots plus 7 retained chunks (224 KB
// of TMEM), which covers the hop and the z pass while the next tiles stream.
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
constexpr int SUB = TM * 128;              // one block: 128 rows x 64 bf16 (128-byte swizzle)
constexpr int CHUNK = 2 * SUB;             // a stream's 128 columns of a tile
constexpr int RING_MAX = 5;                // shared-memory x chunk slots (runtime count <= this)
constexpr int ACC_COLS = 64;               // the projection accumulator (NB <= 64)
constexpr int RET = 7;                     // TMEM retention slots (64 columns each)
constexpr int TMEM_COLS = 512;
static_assert(ACC_COLS + RET * 64 <= TMEM_COLS, "TMEM budget");
constexpr int HBL = 4;                     // H_res logit buffers (two per Sinkhorn warp)
constexpr int NRT = 4;                     // "tile retained" barriers: more than the tiles RET slots hold
constexpr int W_PROD = 0, W_MMA = 1, W_CP = 2, W_ROW = 3, W_COEF = 7, W_SK = 8, W_Z = 10;
constexpr int NZ = 4;                      // z warps: one per TMEM lane quadrant
constexpr int NWARPS = W_Z + NZ, NTHREADS = NWARPS * 32;
constexpr int W_CONV = 2, NCONV = NWARPS - W_CONV;  // warps that convert phi in the prologue
constexpr int NPRE_USERS = NZ + 1;         // readers of the pushed H_pre partials: z warps + coefficient warp
constexpr int ZST = 32 * 128;              // z staging block of one z warp (128-byte swizzle)

enum ErrCode { ERR_PROD = 21, ERR_MMA = 22, ERR_ROW = 23, ERR_COEF = 24, ERR_SK = 25, ERR_Z = 26, ERR_CONV = 27,
               ERR_CP = 28 };

struct Args;
template <int FD>
__device__ __forceinline__ bool phi_bulk_ok(const Args &a);

template <int N, int MODE>
struct Cfg {
  static constexpr int FD = Dims<N, MODE>::FD;
  static constexpr int NB = ((2 * FD + 15) / 16) * 16;   // hi | lo projection columns
  static constexpr int RS = ((FD - N + 3) / 4) * 4;      // owner-inbox row: H_post and H_res partials
  static constexpr int NPAR = 3 + 2 * N + N * N;
  static constexpr int CH = N;                           // chunks per tile (one per stream)
  static_assert(NB <= ACC_COLS, "projection accumulator");
  static_assert(N <= 4, "one 16-byte H_pre push per row");
};

// barrier slots
constexpr int B_FULL = 0, B_EMPTY = RING_MAX, B_ACCF = 2 * RING_MAX, B_ACCE = B_ACCF + 1, B_RFREE = B_ACCE + 1,
              B_RT = B_RFREE + RET, B_PF = B_RT + NRT, B_PD = B_PF + 1, B_PE = B_PD + 1, B_OF = B_PE + 1,
              B_OE = B_OF + 1, B_LGF = B_OE + 1, B_LGE = B_LGF + HBL, B_DRAIN = B_LGE + HBL, B_PHI = B_DRAIN + 1,
              B_PHL = B_PHI + 1, B_DRAIN2 = B_PHL + 1, B_CPD = B_DRAIN2 + 1, NBARS = B_CPD + RET;

struct Layout {
  uint32_t ring, phi, zst, pre, ss, own, lg, par, bar, tmem, abort, total;
};

__host__ __device__ inline int owned_max(int S) { return (TM + S - 1) / S; }

__host__ __device__ inline Layout make_layout(int S, int ring, int CH, int NB, int RS, int NPAR) {
  Layout L;
  uint32_t o = 0;
  L.ring = o;  o += (uint32_t)ring * CHUNK;
  L.phi = o;   o += (uint32_t)2 * CH * NB * 128;            // one phi block per 64 columns
  L.zst = o;   o += (uint32_t)NZ * 2 * ZST;                 // per-z-warp staging: 32 rows x 2 blocks of 64 z
  L.pre = o;   o += (uint32_t)S * TM * 16;                 // [S][TM] H_pre partials (4 floats)
  L.ss = o;    o += (uint32_t)S * TM * 4;                  // [S][TM] sums of squares
  L.own = o;   o += (uint32_t)S * owned_max(S) * RS * 4;   // [S][OWN][RS] the owner's other partials
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
  int C, nC, S, RING;
  const void *phi;
  CoefParams p;
  __nv_bfloat16 *z;
  void *h_pre, *h_post, *h_res;
  int coef_dtype;
  float *inv_rms, *mixes;
  int *err_flag;  // pinned host error word (mhc_set_error_flag) or null
};

// The prologue bulk-copies the fp32 phi slice when its row blocks are whole
// 16-byte units: FD a multiple of 4, fp32 parameters, a 16-byte aligned phi.
template <int FD>
__device__ __forceinline__ bool phi_bulk_ok(const Args &a) {
  return (FD % 4 == 0) && a.p.param_dtype == MHC_F32 && ((uintptr_t)a.phi & 15) == 0;
}

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

// 1/rms and the H_pre projection of row `row` from the S pushed slices, summed
// in slice order.  The owner and every z warp call this same function, so the
// weights used for z are bit-identical to the h_pre the owner writes.
template <int N>
__device__ __forceinline__ void pre_sums(const float *pre, const float *ss, int S, int row, float nC, float eps,
                                         float &inv, float (&m)[N]) {
  // every slice's values are loaded before the first add (S <= 8), then summed
  // in slice order
  float4 v[8];
  float q[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    if (s < S) {
      v[s] = *reinterpret_cast<const float4 *>(pre + (s * TM + row) * 4);
      q[s] = ss[s * TM + row];
    }
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float sq = 0.f;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    if (s < S) {
      acc[0] += v[s].x; acc[1] += v[s].y; acc[2] += v[s].z; acc[3] += v[s].w;
      sq += q[s];
    }
  }
  inv = rsqrtf(sq / nC + eps);
#pragma unroll
  for (int i = 0; i < N; ++i) m[i] = acc[i] * inv;
}

__device__ __forceinline__ float pre_gate(float m, float alpha, float bias, float pre_eps) {
  return sigmoidf_(__fadd_rn(__fmul_rn(m, alpha), bias)) + pre_eps;
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
  constexpr int FD = Cf::FD, NB = Cf::NB, RS = Cf::RS, NPAR = Cf::NPAR, CH = Cf::CH;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t *base = smem_raw + (base_u32 - raw_u32);
  const int S = a.S, RING = a.RING;
  const int OWN = owned_max(S);
  const Layout L = make_layout(S, RING, CH, NB, RS, NPAR);
  float *pre = reinterpret_cast<float *>(base + L.pre);
  float *ssq = reinterpret_cast<float *>(base + L.ss);
  float *own = reinterpret_cast<float *>(base + L.own);
  float *lg = reinterpret_cast<float *>(base + L.lg);
  float *par = reinterpret_cast<float *>(base + L.par);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(base + L.abort);
  const uint32_t bar0 = base_u32 + L.bar;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
// warp-uniform bounded wait: every lane waits (and so acquires), the warp
// agrees on the outcome so it always leaves a loop together
#define WAIT_WARP(CL, bar, ph) (__all_sync(0xffffffffu, wait_parity_fast<CL>((bar), (ph), abort_flag)))

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank(), cid = cluster_id_x(), ncl = ncluster_x();
  const int ntiles = (int)((a.T + TM - 1) / TM);
  const int cnt = (TM - (int)rank + S - 1) / S;  // rows this CTA owns in every tile
  const uint32_t pre_tx = (uint32_t)S * TM * (16 + 4);
  const uint32_t own_tx = (uint32_t)S * cnt * RS * 4;
  const float nCf = (float)a.nC;
  // the per-token outputs take 16-byte stores when every output row starts on
  // a 16-byte boundary (the output pointers are 16-byte aligned)
  const bool vec_out = ((reinterpret_cast<uintptr_t>(a.mixes) | reinterpret_cast<uintptr_t>(a.h_pre) |
                         reinterpret_cast<uintptr_t>(a.h_post) | reinterpret_cast<uintptr_t>(a.h_res)) & 15) == 0;

  // ---------------- prologue ----------------
  if (tid == 0) {
    *abort_flag = 0;
    for (int i = 0; i < RING; ++i) {
      mbar_init(BAR(B_FULL + i), 1);
      mbar_init(BAR(B_EMPTY + i), 2);      // the MMA issuer's and the copier's commits
    }
    mbar_init(BAR(B_ACCF), 1);
    mbar_init(BAR(B_ACCE), 4);             // the 4 row warps have read the partial
    for (int i = 0; i < RET; ++i) mbar_init(BAR(B_RFREE + i), NZ);  // every z warp has read the chunk
    for (int b = 0; b < NRT; ++b) mbar_init(BAR(B_RT + b), 1);     // copier's commit: the tile is in TMEM
    for (int i = 0; i < RET; ++i) mbar_init(BAR(B_CPD + i), 1);    // copier's commit: the slot's chunk is in TMEM
    mbar_init(BAR(B_PF), 1);               // armed by a z warp; st.async bytes of every CTA complete it
    mbar_init(BAR(B_PD), NPRE_USERS);      // local: the pushed H_pre partials have been read
    mbar_init(BAR(B_PE), S);               // one per CTA: its readers are done with the tile
    mbar_init(BAR(B_OF), 1);               // armed by the coefficient warp; st.async bytes complete it
    mbar_init(BAR(B_OE), S);               // one per owner CTA (its inbox drained)
    for (int b = 0; b < HBL; ++b) {
      mbar_init(BAR(B_LGF + b), 1);
      mbar_init(BAR(B_LGE + b), 1);
    }
    mbar_init(BAR(B_DRAIN), 1);
    mbar_init(BAR(B_DRAIN2), 1);
    mbar_init(BAR(B_PHI), NCONV);
    mbar_init(BAR(B_PHL), 1);              // the fp32 phi slice has landed in the (still idle) ring
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
    const int KS = CH * COLS, total = KS * FD;
    auto put = [&](int kl, int j, float v) {
      uint8_t *blk = base + L.phi + (uint32_t)(kl >> 6) * NB * 128;
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
      *reinterpret_cast<__nv_bfloat16 *>(blk + phi_off(j, kl & 63)) = hi;
      *reinterpret_cast<__nv_bfloat16 *>(blk + phi_off(j + FD, kl & 63)) = lo;
    };
    // fp32 phi: the slice's rows of chunk ch are 64 consecutive rows of FD
    // floats in global memory; they were bulk-copied into the ring (idle until
    // the producer starts) and are converted from there
    const bool vec = phi_bulk_ok<FD>(a);
    if (vec) {
      if (!WAIT_WARP(false, BAR(B_PHL), 0u)) record_error(ERR_CONV, abort_flag, a.err_flag);
      const float *stg = reinterpret_cast<const float *>(base + L.ring);
      for (int e = ctid; e < total; e += nconv) put(e / FD, e % FD, stg[e]);
    }
    for (int e0 = ctid; !vec && e0 < total; e0 += 4 * nconv) {
      float v[4];
      int kk4[4], j4[4], ch4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = e0 + u * nconv;
        v[u] = 0.f;
        kk4[u] = j4[u] = ch4[u] = 0;
        if (e < total) {
          const int kl = e / FD, j = e - kl * FD;
          const int ch = kl >> 6, kk = kl & 63;
          const int i = ch >> 1, b = ch & 1;  // phi block ch: stream i, 64-column block b
          const int64_t k = (int64_t)i * a.C + (int64_t)rank * COLS + 64 * b + kk;
          v[u] = load_dyn(a.phi, a.p.param_dtype, k * FD + j);
          kk4[u] = kk;
          j4[u] = j;
          ch4[u] = ch;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (e0 + u * nconv < total) put(ch4[u] * 64 + kk4[u], j4[u], v[u]);
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
      if (phi_bulk_ok<FD>(a)) {
        // the fp32 phi slice into the ring, then the ring is x's once converted
        const uint32_t blk_bytes = 64u * FD * 4u;
        mbar_arrive_expect_tx(BAR(B_PHL), (uint32_t)(2 * CH) * blk_bytes);
        for (int ch = 0; ch < 2 * CH; ++ch) {
          const int i = ch >> 1, b = ch & 1;
          const int64_t k0 = (int64_t)i * a.C + (int64_t)rank * COLS + 64 * b;
          bulk_load(base_u32 + L.ring + (uint32_t)ch * blk_bytes, reinterpret_cast<const float *>(a.phi) + k0 * FD,
                    blk_bytes, BAR(B_PHL));
        }
        ok = wait_parity<false>(BAR(B_PHI), 0u, abort_flag);
      }
      for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl) {
        for (int ch = 0; ch < CH; ++ch, ++q) {
          const uint32_t slot = q % RING, ph = (q / RING) & 1u;
          if (!wait_parity<false>(BAR(B_EMPTY + slot), ph ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(BAR(B_FULL + slot), CHUNK);
          tma_load_3d(base_u32 + L.ring + slot * CHUNK, &xmap, 0, tile * TM, (ch * a.C + (int)rank * COLS) / 64,
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
        // the ingest warps have read the previous tile's partial
        if (!wait_parity<false>(BAR(B_ACCE), ((uint32_t)lt & 1u) ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int ch = 0; ch < CH; ++ch, ++q) {
          const uint32_t slot = q % RING, ph = (q / RING) & 1u;
          if (!wait_parity<false>(BAR(B_FULL + slot), ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int sb = 0; sb < 2; ++sb) {
            const uint32_t a0 = base_u32 + L.ring + slot * CHUNK + sb * SUB;
            const uint32_t b0 = base_u32 + L.phi + (uint32_t)(2 * ch + sb) * NB * 128u;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_bf16(tmem_base, umma_desc_sw128(a0 + k * 32), umma_desc_sw128(b0 + k * 32), idesc,
                        (ch | sb | k) != 0 ? 1u : 0u);
          }
          umma_commit(BAR(B_EMPTY + slot));
        }
        if (!ok) break;
        umma_commit(BAR(B_ACCF));
      }
      if (!ok) record_error(ERR_MMA, abort_flag, a.err_flag);
      // every issued MMA completes before TMEM is released
      umma_commit(BAR(B_DRAIN));
      wait_parity<false>(BAR(B_DRAIN), 0u, nullptr);
    }
    __syncwarp();
  } else if (warp == W_CP) {
    // ---------------- copier: ring chunk -> TMEM retention slot ----------------
    if (lane == 0) {
      uint32_t q = 0;
      int lt = 0;
      bool ok = true;
      for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
        for (int ch = 0; ch < CH; ++ch, ++q) {
          const uint32_t slot = q % RING, ph = (q / RING) & 1u;
          const uint32_t rs = q % RET, rph = (q / RET) & 1u;
          if (!wait_parity_fast<false>(BAR(B_FULL + slot), ph, abort_flag)) { ok = false; break; }
          // the retention slot's previous chunk has been read by its z warps
          if (!wait_parity_fast<false>(BAR(B_RFREE + rs), rph ^ 1u, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = base_u32 + L.ring + slot * CHUNK;
          const uint32_t t0 = tmem_base + (uint32_t)(ACC_COLS + rs * 64);
#pragma unroll
          for (int k = 0; k < 8; ++k)  // 32-byte column groups 0-3 of block 0, then of block 1
            tmem_cp_128x256b(t0 + (uint32_t)(k * 8), umma_desc_sw128(a0 + (k >> 2) * SUB + (k & 3) * 32));
          umma_commit(BAR(B_EMPTY + slot));
          umma_commit(BAR(B_CPD + rs));  // the row warps may read this chunk
        }
        if (!ok) break;
        umma_commit(BAR(B_RT + lt % NRT));  // the tile's chunks are retained
      }
      if (!ok) record_error(ERR_CP, abort_flag, a.err_flag);
      // every issued copy completes before TMEM is released
      umma_commit(BAR(B_DRAIN2));
      wait_parity<false>(BAR(B_DRAIN2), 0u, nullptr);
    }
    __syncwarp();
  } else if (warp >= W_ROW && warp < W_ROW + 4) {
    // ---------------- row warps ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // token row of the tile = TMEM lane
    const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16);
    const uint32_t owner = (uint32_t)(row % S);
    const int oidx = row / S;
    int lt = 0;
    bool ok = true;
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      // sum of squares of the row's slice, chunk by chunk as the copies land:
      // four chains of two fp32 partial sums
      uint64_t ss2[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) ss2[k] = f2_pack(0.f, 0.f);
      const uint32_t q0 = (uint32_t)lt * CH;
#pragma unroll 1
      for (int c = 0; c < CH; ++c) {
        const uint32_t q = q0 + (uint32_t)c;
        if (!WAIT_WARP(false, BAR(B_CPD + q % RET), (q / RET) & 1u)) { ok = false; break; }
        tc_fence_after();
        uint32_t w[2][32];
        const uint32_t col = lane_base + (uint32_t)(ACC_COLS + (q % RET) * 64);
        tmem_ld32x2u(col, col + 32u, w);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const uint64_t xv = bf16x2_to_f2(w[h][j]);
            ss2[j & 3] = f2_fma(xv, xv, ss2[j & 3]);
          }
      }
      if (!ok) break;
      if (!WAIT_WARP(false, BAR(B_ACCF), (uint32_t)lt & 1u)) { ok = false; break; }
      tc_fence_after();
      // the slice's projection partial of this row
      float d[NB];
#pragma unroll
      for (int c16 = 0; c16 < NB / 16; ++c16) {
        float t16[16];
        tmem_ld16(lane_base + (uint32_t)(c16 * 16), t16);
#pragma unroll
        for (int i = 0; i < 16; ++i) d[c16 * 16 + i] = t16[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_ACCE));
      float vals[FD];
#pragma unroll
      for (int j = 0; j < FD; ++j) vals[j] = d[j] + d[FD + j];
      float ssum = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float s0, s1;
        f2_unpack(ss2[k], s0, s1);
        ssum += s0 + s1;
      }
      float p4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < N; ++i) p4[i] = vals[i];
      // H_pre partials and the sum of squares to every CTA: their readers must
      // be done with the previous tile
      if (!WAIT_WARP(true, BAR(B_PE), ((uint32_t)lt & 1u) ^ 1u)) { ok = false; break; }
      const uint32_t pre_loc = base_u32 + L.pre + (uint32_t)(((int)rank * TM + row) * 16);
      const uint32_t ss_loc = base_u32 + L.ss + (uint32_t)(((int)rank * TM + row) * 4);
#pragma unroll 1
      for (int dcta = 0; dcta < S; ++dcta) {
        const uint32_t dbar = mapa(BAR(B_PF), (uint32_t)dcta);
        st_async_v4(mapa(pre_loc, (uint32_t)dcta), p4[0], p4[1], p4[2], p4[3], dbar);
        st_async_f32(mapa(ss_loc, (uint32_t)dcta), ssum, dbar);
      }
      if constexpr (RS > 0) {
        // the other partials to the row's owner, once it drained the previous tile
        float r4[RS];
#pragma unroll
        for (int j = 0; j < RS; ++j) r4[j] = (N + j < FD) ? vals[N + j] : 0.f;
        if (!WAIT_WARP(true, BAR(B_OE), ((uint32_t)lt & 1u) ^ 1u)) { ok = false; break; }
        const uint32_t dst = mapa(base_u32 + L.own + (uint32_t)(((int)rank * OWN + oidx) * RS * 4), owner);
        const uint32_t dbar = mapa(BAR(B_OF), owner);
#pragma unroll
        for (int v = 0; v < RS / 4; ++v)
          st_async_v4(dst + v * 16, r4[4 * v], r4[4 * v + 1], r4[4 * v + 2], r4[4 * v + 3], dbar);
      }
    }
    if (!ok) record_error(ERR_ROW, abort_flag, a.err_flag);
  } else if (warp == W_COEF) {
    // ---------------- coefficient warp: rows rank + S l ----------------
    int lt = 0;
    bool ok = WAIT_WARP(false, BAR(B_PHI), 0u);  // gate parameters loaded
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const int lb = lt % HBL;
      const uint32_t tph = (uint32_t)lt & 1u;
      const int t = (int)rank + lane * S;  // token row of the tile
      const int64_t tok = (int64_t)tile * TM + t;
      const bool mine = lane < cnt;
      const bool live = mine && tok < a.T;
      float m[FD], ho[N], w[N];
      float inv = 0.f;
#pragma unroll
      for (int j = 0; j < FD; ++j) m[j] = 0.f;
      // the H_pre partials and sums of squares of every slice
      if (!WAIT_WARP(true, BAR(B_PF), tph)) { ok = false; break; }
      {
        float mp[N];
        pre_sums<N>(pre, ssq, S, mine ? t : 0, nCf, a.p.rms_eps, inv, mp);
#pragma unroll
        for (int i = 0; i < N; ++i) m[i] = mp[i];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_PD));
      // once every local reader (z warps and this warp) is done, tell every CTA
      // that its next pushes may land: one remote arrive per lane, in parallel
      if (!WAIT_WARP(false, BAR(B_PD), tph)) { ok = false; break; }
      if (lane < S) mbar_arrive_remote(mapa(BAR(B_PE), (uint32_t)lane));
      if constexpr (RS > 0) {
        if (lane == 0) mbar_arrive_expect_tx(BAR(B_OF), own_tx);  // arm: S slices' other partials
        if (!WAIT_WARP(true, BAR(B_OF), tph)) { ok = false; break; }
        float acc[RS];
#pragma unroll
        for (int j = 0; j < RS; ++j) acc[j] = 0.f;
        if (mine) {
          // per 16-byte group: every slice's value loaded first, then summed in
          // slice order (fixed order: deterministic)
#pragma unroll
          for (int v = 0; v < RS / 4; ++v) {
            float4 q4[8];
#pragma unroll
            for (int s = 0; s < 8; ++s)
              if (s < S) q4[s] = reinterpret_cast<const float4 *>(own + (s * OWN + lane) * RS)[v];
#pragma unroll
            for (int s = 0; s < 8; ++s)
              if (s < S) {
                acc[4 * v] += q4[s].x; acc[4 * v + 1] += q4[s].y; acc[4 * v + 2] += q4[s].z; acc[4 * v + 3] += q4[s].w;
              }
          }
        }
        __syncwarp();
        if (lane < S) mbar_arrive_remote(mapa(BAR(B_OE), (uint32_t)lane));  // inbox free again
#pragma unroll
        for (int j = N; j < FD; ++j) m[j] = acc[j - N] * inv;
      }
      if constexpr (MODE == FULL) {
        if (!WAIT_WARP(false, BAR(B_LGE + lb), ((uint32_t)(lt / HBL) & 1u) ^ 1u)) { ok = false; break; }
      }
      if (mine) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
          w[i] = pre_gate(m[i], par[0], par[3 + i], a.p.pre_eps);
          if constexpr (MODE != HEAD)
            ho[i] = sigmoidf_(__fadd_rn(__fmul_rn(m[N + i], par[1]), par[3 + N + i])) * a.p.post_mult;
        }
        if constexpr (MODE == FULL) {
          float *lrow = lg + (lb * OWN + lane) * 16;
#pragma unroll
          for (int k = 0; k < N * N; ++k) lrow[k] = __fadd_rn(__fmul_rn(m[2 * N + k], par[2]), par[3 + 2 * N + k]);
        }
      }
      if constexpr (MODE == FULL) {
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_LGF + lb));  // logits ready for the Sinkhorn warp
      }
      // per-token outputs: 16-byte stores where the rows allow (each lane's
      // token is a different row, so every store is a separate transaction)
      if (live) {
        a.inv_rms[tok] = inv;
        if (FD % 4 == 0 && vec_out) {
          float4 *mrow = reinterpret_cast<float4 *>(a.mixes + tok * FD);
#pragma unroll
          for (int v = 0; v < FD / 4; ++v) mrow[v] = make_float4(m[4 * v], m[4 * v + 1], m[4 * v + 2], m[4 * v + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < FD; ++j) a.mixes[tok * FD + j] = m[j];
        }
        if constexpr (MODE != HEAD) {
          if (N == 4 && a.coef_dtype == MHC_F32 && vec_out) {
            if (a.h_pre) reinterpret_cast<float4 *>(a.h_pre)[tok] = make_float4(w[0], w[1 % N], w[2 % N], w[3 % N]);
            reinterpret_cast<float4 *>(a.h_post)[tok] = make_float4(ho[0], ho[1 % N], ho[2 % N], ho[3 % N]);
          } else {
#pragma unroll
            for (int i = 0; i < N; ++i) {
              if (a.h_pre) store_dyn(a.h_pre, a.coef_dtype, tok * N + i, w[i]);
              store_dyn(a.h_post, a.coef_dtype, tok * N + i, ho[i]);
            }
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
            if (N == 4 && a.coef_dtype == MHC_F32 && vec_out) {
              float4 *hrow = reinterpret_cast<float4 *>(a.h_res) + tok * 4;
#pragma unroll
              for (int v = 0; v < 4; ++v)
                hrow[v] = make_float4(hm[(4 * v) % (N * N)], hm[(4 * v + 1) % (N * N)], hm[(4 * v + 2) % (N * N)],
                                      hm[(4 * v + 3) % (N * N)]);
            } else {
#pragma unroll
              for (int k = 0; k < N * N; ++k) store_dyn(a.h_res, a.coef_dtype, tok * N * N + k, hm[k]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_LGE + lb));  // logits buffer free
      }
      if (!ok) record_error(ERR_SK, abort_flag, a.err_flag);
    }
  } else if (warp >= W_Z && warp < W_Z + NZ) {
    // ---------------- z warps ----------------
    const int zw = warp - W_Z;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16);
    const uint32_t stage = base_u32 + L.zst + (uint32_t)zw * 2 * ZST;
    uint8_t *stage_rows = base + L.zst + zw * 2 * ZST + lane * 128;
    int lt = 0;
    bool ok = WAIT_WARP(false, BAR(B_PHI), 0u);  // gate parameters loaded
    for (int tile = (int)cid; tile < ntiles && ok; tile += (int)ncl, ++lt) {
      const uint32_t tph = (uint32_t)lt & 1u;
      if (zw == 0 && lane == 0) mbar_arrive_expect_tx(BAR(B_PF), pre_tx);  // arm: every slice's pushes
      if (!WAIT_WARP(true, BAR(B_PF), tph)) { ok = false; break; }
      float inv, m[N], wv[N];
      pre_sums<N>(pre, ssq, S, row, nCf, a.p.rms_eps, inv, m);
#pragma unroll
      for (int i = 0; i < N; ++i) wv[i] = pre_gate(m[i], par[0], par[3 + i], a.p.pre_eps);
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_PD));
      if (!WAIT_WARP(false, BAR(B_RT + lt % NRT), (uint32_t)(lt / NRT) & 1u)) { ok = false; break; }
      tc_fence_after();
      const uint32_t q0 = (uint32_t)lt * CH;  // the tile's first chunk (stream 0)
      const int64_t row0 = (int64_t)tile * TM + quad * 32;
      // the staging blocks must have been read by this warp's previous stores
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll 1
      for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
        for (int piece = 0; piece < 2; ++piece) {
          uint32_t xr[4][16];
          uint32_t ad[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            ad[i] = lane_base +
                    (uint32_t)(ACC_COLS + ((q0 + (uint32_t)(i < N ? i : 0)) % RET) * 64 + blk * 32 + piece * 16);
          tmem_ld16x4u(ad[0], ad[1], ad[2], ad[3], xr);
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
          uint8_t *rp = stage_rows + blk * ZST;
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
          tma_store_2d(&zmap, stage + (uint32_t)blk * ZST, (int)rank * COLS + 64 * blk, (int)row0);
          bulk_commit();  // rows past T are not written
        }
      }
      // this warp is done with the block's retention slots
      tc_fence_before();
      __syncwarp();
      if (lane == 0)
        for (int i = 0; i < N; ++i) mbar_arrive(BAR(B_RFREE + (q0 + (uint32_t)i) % RET));  // all z warps
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

// the longest ring (up to RING_MAX, at least 3) that fits the budget; 0 if none
template <int N, int MODE>
static int pick_ring(int S) {
  using Cf = Cfg<N, MODE>;
  for (int r = RING_MAX; r >= 3; --r)
    if ((size_t)make_layout(S, r, Cf::CH, Cf::NB, Cf::RS, Cf::NPAR).total + 1024 <= SMEM_LIMIT) return r;
  return 0;
}

// a (rows x cols) row-major bf16 matrix in boxes of box_rows x 64 columns,
// 128-byte swizzle (x: 128-row boxes; z: 32-row boxes)
static bool encode_2d(CUtensorMap &m, const void *p, int64_t rows, int64_t cols, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(p), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// x as a 3-D tensor (64 columns, T rows, nC / 64 column blocks): a box of 2
// blocks x 128 rows lands as two consecutive 128-row x 64-column blocks, each
// with a 128-byte swizzle (the MMA's K-major operand layout)
static bool encode_x3(CUtensorMap &m, const void *p, int64_t rows, int64_t cols) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)cols / 64};
  const cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
  const cuuint32_t box[3] = {64, (cuuint32_t)TM, 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(p), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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

template <int N, int MODE>
static cudaError_t launch_impl(const void *x, Args a, cudaStream_t stream) {
  using Cf = Cfg<N, MODE>;
  a.RING = pick_ring<N, MODE>(a.S);
  if (a.RING == 0) return cudaErrorNotSupported;
  const size_t smem = (size_t)make_layout(a.S, a.RING, Cf::CH, Cf::NB, Cf::RS, Cf::NPAR).total + 1024;
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
  if (!encode_x3(xmap, x, a.T, a.nC)) return cudaErrorNotSupported;
  if (!encode_2d(zmap, a.z, a.T, a.C, 32)) return cudaErrorNotSupported;
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
  a.RING = 0;
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
