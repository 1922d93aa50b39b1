// Tensor-core dx / dphi stage of the coefficient backward (sm_100a, bf16 x).
//
// Replaces the CUDA-core dx_dphi_kernel for bf16 activations.  After K1 has
// produced per token dm = dL/dmixes, rowb = inv^2 <dm, m> / nC and the
// aggregation weights, this kernel computes
//
//   dx[t, k]    = inv[t] * (dm[t,:] . phi[k,:]) - rowb[t] x[t,k]
//                 + w[t, k / C] dz[t, k % C] + dx_add[t, k]
//   dphi[k, j] += sum_t x[t,k] (inv[t] dm[t,j])
//
// One CTA per SM owns 128 consecutive columns k of n*C (inside one stream)
// and a contiguous range of 128-token tiles.  Both products run on tcgen05
// with fp32 accumulators in TMEM:
//
//   * dx product, M = 128 tokens, N = 128 columns, K = 3*FD (padded to 16):
//     A = [dm_hi | dm_lo | dm_hi] built per tile by the prep warps, B =
//     [phi_hi | phi_hi | phi_lo] built once -- three bf16 products give the
//     fp32 result to ~2^-16.
//   * dphi product, M = 128 columns, N = 2*FD (padded to 16), K = 128 tokens,
//     accumulated in TMEM over all tiles of the CTA: A = x^T read straight
//     from the TMA-staged x tile as an MN-major operand (the tile's 128-byte
//     rows are tokens, i.e. K), B = [inv*dm hi ; lo] with tokens along K.
//
// Warp roles: 0 TMA producer of the x tiles (3 stages), 1 MMA issuer, 2 TMA
// producer of the dx_add tiles (2 buffers, which then receive dx), 3-10 the dx
// epilogue (thread = token row = TMEM lane, two warps per lane quadrant, 64
// columns each; dz and the per-token scalars are loaded one tile ahead; an x
// stage is released after the arithmetic, a dx buffer after its coalesced
// write-back), 11-14 prep warps (thread = token row; their operand buffers are
// single or double, whichever fits).  All hand-offs are
// mbarriers; every wait is bounded and a timeout sets the device error word.
// The per-CTA dphi partials go to workspace and are summed in a fixed order
// by the reduction kernel, so the result is deterministic.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "mhc_device.cuh"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"
#include "mhc_sm100.cuh"

namespace mhc {

__device__ int g_tcb_error = 0;  // first error code recorded by the backward tensor-core kernel

namespace tcb {

using namespace sm100;

constexpr int TM = 128;                 // tokens per tile
constexpr int KCOL = 128;               // columns of n*C per CTA
constexpr int XS = 3;                   // x tile stages
constexpr int AS = 2;                   // dx_add / dx tile buffers
constexpr int NEPI = 8, NPREP = 4;
constexpr int W_PROD = 0, W_MMA = 1, W_APROD = 2, W_EPI = 3, W_PREP = W_EPI + NEPI;
constexpr int NWARPS = W_PREP + NPREP, NTHREADS = NWARPS * 32;
constexpr int CHUNK = TM * 128;         // 128 rows x 64 bf16 columns (128-byte swizzle)
constexpr int XSTAGE = 2 * CHUNK;       // the CTA's 128 columns of one tile (x, or dx_add then dx)
constexpr int DB = 2;                   // dx accumulators in TMEM (one tile each; 3 measured no faster)
constexpr int D2COL = DB * 128;         // the dphi accumulator follows them
constexpr int TMEM_COLS = 512;          // D1 x DB at columns 0, 128, ..., then D2 (N <= 128)

enum ErrCode { ERR_PROD = 11, ERR_MMA = 12, ERR_EPI = 13, ERR_PREP = 14 };

// A of the dx product: 8-row groups are padded by one 16-byte granule so the
// prep threads' row writes do not collide on shared-memory banks
__host__ __device__ constexpr uint32_t a1_sbo(int K1) { return (uint32_t)(K1 / 8) * 128u + 16u; }

constexpr size_t SMEM_LIMIT = 232448;  // opt-in dynamic shared memory per block on sm_100

__host__ __device__ constexpr uint32_t blayout_bytes(int K1, int NB2, int PB) {
  return (uint32_t)(XS + AS) * XSTAGE + (uint32_t)KCOL * K1 * 2 + (uint32_t)PB * (TM / 8) * a1_sbo(K1) +
         (uint32_t)PB * NB2 * TM * 2 + 512u;
}

template <int N, int MODE>
struct BCfg {
  static constexpr int FD = Dims<N, MODE>::FD;
  static constexpr int K1 = ((3 * FD + 15) / 16) * 16;   // dx product K
  static constexpr int NB2 = ((2 * FD + 15) / 16) * 16;  // dphi product N
  // prep operand buffers: two when they fit beside the x / dx rings, else one
  static constexpr int PB = blayout_bytes(K1, NB2, 2) + 1024 <= SMEM_LIMIT ? 2 : 1;
  static_assert(NB2 <= TMEM_COLS - D2COL, "dphi accumulator must fit after the dx accumulators");
};

// barrier slots
constexpr int B_XF = 0, B_XE = XS, B_AF = 2 * XS, B_AE = B_AF + AS, B_PF = B_AE + AS, B_PE = B_PF + 2,
              B_DF = B_PE + 2, B_DE = B_DF + DB, B_DRAIN = B_DE + DB, NBARS = B_DRAIN + 1;

struct BLayout {
  uint32_t xs, as, b1, a1, b2, bar, tmem, abort, total;
};

__host__ __device__ inline BLayout make_blayout(int K1, int NB2, int PB) {
  BLayout L;
  uint32_t o = 0;
  L.xs = o;    o += XS * XSTAGE;
  L.as = o;    o += AS * XSTAGE;
  L.b1 = o;    o += (uint32_t)KCOL * K1 * 2;
  L.a1 = o;    o += (uint32_t)PB * (TM / 8) * a1_sbo(K1);
  L.b2 = o;    o += (uint32_t)PB * NB2 * TM * 2;
  L.bar = o;   o += NBARS * 8;
  L.tmem = o;  o += 4;
  L.abort = o; o += 4;
  L.total = o;
  return L;
}

struct BArgs {
  int64_t T;
  int C, nC, TS;
  const void *phi;
  int pdt;
  const float *inv_rms, *dm, *rowb, *gate;
  const __nv_bfloat16 *dz, *dx_add;
  __nv_bfloat16 *dx;
  float *dphi_part;  // [TS][nC][FD]
  int *err_flag;     // pinned host error word (mhc_set_error_flag) or null
};

// byte offset of (row r, column k) of a no-swizzle K-major operand built from
// 8-row x 16-byte core matrices (8-row groups `sbo` bytes apart, the core
// matrices of a group contiguous along K)
__device__ __forceinline__ uint32_t cm_off(int r, int k, uint32_t sbo) {
  return (uint32_t)(r >> 3) * sbo + (uint32_t)(k >> 3) * 128u + (uint32_t)(r & 7) * 16u + (uint32_t)(k & 7) * 2u;
}
// byte offset of (MN index n, K index k) of a no-swizzle MN-major operand:
// one 16-byte granule holds 8 consecutive n of one k; the 8 k of a group are
// consecutive granules (K groups 128 B apart), MN blocks of 8 `sbo` bytes apart
__device__ __forceinline__ uint32_t mn_off(int n, int k, uint32_t sbo) {
  return (uint32_t)(n >> 3) * sbo + (uint32_t)(k >> 3) * 128u + (uint32_t)(k & 7) * 16u + (uint32_t)(n & 7) * 2u;
}

__device__ __forceinline__ void record_error(int code, volatile int *abort_flag, int *err_flag) {
  *abort_flag = 1;
  report_give_up(&g_tcb_error, err_flag, code);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <int N, int MODE>
__global__ void __launch_bounds__(NTHREADS, 1)
pre_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap amap,
                  BArgs a) {
  using Cf = BCfg<N, MODE>;
  constexpr int FD = Cf::FD, K1 = Cf::K1, NB2 = Cf::NB2, PB = Cf::PB;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t *base = smem_raw + (base_u32 - raw_u32);
  const BLayout L = make_blayout(K1, NB2, PB);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(base + L.abort);
  const uint32_t bar0 = base_u32 + L.bar;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
#define WAIT_WARP(bar, par) (__all_sync(0xffffffffu, wait_parity<false>((bar), (par), abort_flag)))

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nslices = a.nC / KCOL;
  const int slice = (int)blockIdx.x % nslices, split = (int)blockIdx.x / nslices;
  const int col0 = slice * KCOL;
  const int stream_i = col0 / a.C, c_in = col0 - stream_i * a.C;
  const int64_t tiles = (a.T + TM - 1) / TM;
  const int64_t tile_beg = tiles * split / a.TS, tile_end = tiles * (split + 1) / a.TS;
  const int ntile = (int)(tile_end - tile_beg);
  const int64_t tok_end = tile_end * TM < a.T ? tile_end * TM : a.T;

  // ---------------- prologue ----------------
  if (tid == 0) {
    *abort_flag = 0;
    for (int i = 0; i < XS; ++i) {
      mbar_init(BAR(B_XF + i), 1);
      mbar_init(BAR(B_XE + i), 1 + NEPI);  // MMA commit + every epilogue warp has read the x tile
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(BAR(B_AF + i), 1);
      mbar_init(BAR(B_AE + i), NEPI);      // every epilogue warp has written its dx block back
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(B_PF + b), NPREP);
      mbar_init(BAR(B_PE + b), 1);
    }
    for (int b = 0; b < DB; ++b) {
      mbar_init(BAR(B_DF + b), 1);
      mbar_init(BAR(B_DE + b), NEPI);
    }
    mbar_init(BAR(B_DRAIN), 1);
    fence_mbar_init_cluster();
  }
  if (warp == W_MMA) {
    tmem_alloc(base_u32 + L.tmem, TMEM_COLS);
    tmem_relinquish();
  }
  grid_dep_launch();
  grid_dep_wait();
  {
    // B of the dx product: [phi_hi | phi_hi | phi_lo | 0] for the CTA's columns
    uint8_t *b1 = base + L.b1;
    for (int e = tid; e < KCOL * K1; e += NTHREADS) {
      const int r = e / K1, k = e - r * K1;
      float v = 0.f;
      if (k < 3 * FD) {
        const int j = k < FD ? k : (k < 2 * FD ? k - FD : k - 2 * FD);
        const float f = load_dyn(a.phi, a.pdt, (int64_t)(col0 + r) * FD + j);
        const float hi = __bfloat162float(__float2bfloat16_rn(f));
        v = k < 2 * FD ? hi : f - hi;
      }
      *reinterpret_cast<__nv_bfloat16 *>(b1 + cm_off(r, k, (K1 / 8) * 128u)) = __float2bfloat16_rn(v);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(base + L.tmem);

  if (warp == W_PROD || warp == W_APROD) {
    // x tiles (warp W_PROD) and dx_add tiles (warp W_APROD) stream through
    // rings of their own depth, one issuing thread each
    if (lane == 0) {
      const bool is_x = warp == W_PROD;
      const int NS = is_x ? XS : AS;
      const int bf = is_x ? B_XF : B_AF, be = is_x ? B_XE : B_AE;
      const uint32_t ring = base_u32 + (is_x ? L.xs : L.as);
      const CUtensorMap *map = is_x ? &tmap : &amap;
      const bool load = is_x || a.dx_add != nullptr;
      bool ok = true;
      int lt = 0;
      for (; lt < ntile && ok; ++lt) {
        const int s = lt % NS;
        if (!wait_parity<false>(BAR(be + s), ((uint32_t)(lt / NS) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
        if (!load) {
          mbar_arrive(BAR(bf + s));  // no dx_add: the buffer only receives dx
          continue;
        }
        mbar_arrive_expect_tx(BAR(bf + s), XSTAGE);
        const int t0 = (int)((tile_beg + lt) * TM);
        tma_load_2d(ring + s * XSTAGE, map, col0, t0, BAR(bf + s));
        tma_load_2d(ring + s * XSTAGE + CHUNK, map, col0 + 64, t0, BAR(bf + s));
      }
      if (!ok) record_error(ERR_PROD, abort_flag, a.err_flag);
      const int l0 = lt > NS ? lt - NS : 0;
      for (int p = l0; p < lt; ++p) wait_parity<false>(BAR(bf + p % NS), (uint32_t)(p / NS) & 1u, nullptr);
    }
    __syncwarp();
  } else if (warp == W_MMA) {
    if (lane == 0) {
      constexpr uint32_t idesc1 = umma_idesc_bf16_f32_major(128, 128, 0, 0);
      constexpr uint32_t idesc2 = umma_idesc_bf16_f32_major(128, NB2, 1, 1);
      const uint32_t sbo1 = (uint32_t)(K1 / 8) * 128u;
      bool ok = true;
      for (int lt = 0; lt < ntile && ok; ++lt) {
        const int b = lt % DB, s = lt % XS, pb = lt % PB;
        const uint32_t bph = (uint32_t)(lt / DB) & 1u;
        if (!wait_parity<false>(BAR(B_PF + pb), (uint32_t)(lt / PB) & 1u, abort_flag)) { ok = false; break; }
        if (!wait_parity<false>(BAR(B_XF + s), (uint32_t)(lt / XS) & 1u, abort_flag)) { ok = false; break; }
        if (!wait_parity<false>(BAR(B_DE + b), bph ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        // dx product into D1[b]
        const uint32_t a1 = base_u32 + L.a1 + (uint32_t)pb * (TM / 8) * a1_sbo(K1);
        const uint32_t b1 = base_u32 + L.b1;
#pragma unroll
        for (int ks = 0; ks < K1 / 16; ++ks)
          umma_bf16(tmem_base + (uint32_t)b * 128u, umma_desc(a1 + ks * 256, 128, a1_sbo(K1), 0),
                    umma_desc(b1 + ks * 256, 128, sbo1, 0), idesc1, ks > 0 ? 1u : 0u);
        // dphi product, accumulated over every tile: A = x^T (MN-major, the
        // two 64-column chunks 16 KB apart), B = inv*dm (MN-major, 8-feature
        // blocks TM*16 bytes apart), tokens along K for both
        const uint32_t xa = base_u32 + L.xs + s * XSTAGE;
        const uint32_t b2 = base_u32 + L.b2 + (uint32_t)pb * NB2 * TM * 2;
#pragma unroll
        for (int ks = 0; ks < TM / 16; ++ks)
          umma_bf16(tmem_base + (uint32_t)D2COL, umma_desc(xa + ks * 2048, CHUNK, 1024, 2),
                    umma_desc(b2 + ks * 256, 128, TM * 16, 0), idesc2, (lt | ks) != 0 ? 1u : 0u);
        umma_commit(BAR(B_DF + b));
        umma_commit(BAR(B_PE + pb));
        umma_commit(BAR(B_XE + s));
      }
      if (!ok) record_error(ERR_MMA, abort_flag, a.err_flag);
      umma_commit(BAR(B_DRAIN));
    }
    __syncwarp();
  } else if (warp >= W_PREP) {
    // ---------------- prep warps: thread = token row of the tile ----------------
    const int row = tid - W_PREP * 32;
    bool ok = true;
    // dm and 1/rms of the next tile are loaded while this tile's operands are
    // built (the buffer wait would otherwise expose the load latency)
    auto load_dm = [&](int lt_, float (&dst)[FD], float &inv_) {
      const int64_t tk = (tile_beg + lt_) * TM + row;
#pragma unroll
      for (int j = 0; j < FD; ++j) dst[j] = 0.f;
      inv_ = 0.f;
      if (lt_ < ntile && tk < tok_end) {
        inv_ = a.inv_rms[tk];
        if constexpr (FD % 4 == 0) {
          const float4 *src = reinterpret_cast<const float4 *>(a.dm + tk * FD);
#pragma unroll
          for (int q = 0; q < FD / 4; ++q) {
            const float4 v = src[q];
            dst[4 * q] = v.x; dst[4 * q + 1] = v.y; dst[4 * q + 2] = v.z; dst[4 * q + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < FD; ++j) dst[j] = a.dm[tk * FD + j];
        }
      }
    };
    float dm[FD], inv;
    load_dm(0, dm, inv);
    for (int lt = 0; lt < ntile && ok; ++lt) {
      const int b = lt % PB;
      float dmn[FD], invn;
      load_dm(lt + 1, dmn, invn);
      if (!WAIT_WARP(BAR(B_PE + b), ((uint32_t)(lt / PB) & 1u) ^ 1u)) { ok = false; break; }
      // A of the dx product: row `row` = [dm_hi | dm_lo | dm_hi | 0], 16-byte granules
      uint8_t *a1 = base + L.a1 + (uint32_t)b * (TM / 8) * a1_sbo(K1);
#pragma unroll
      for (int g = 0; g < K1 / 8; ++g) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int k = g * 8 + e;
          float val = 0.f;
          if (k < 3 * FD) {
            const int j = k < FD ? k : (k < 2 * FD ? k - FD : k - 2 * FD);
            const float hi = __bfloat162float(__float2bfloat16_rn(dm[j]));
            val = (k >= FD && k < 2 * FD) ? dm[j] - hi : hi;
          }
          v[e] = val;
        }
        *reinterpret_cast<uint4 *>(a1 + cm_off(row, g * 8, a1_sbo(K1))) =
            make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
      }
      // B of the dphi product (MN-major): token `row` holds [inv*dm hi | lo | 0],
      // written as 16-byte granules of 8 features
      uint8_t *b2 = base + L.b2 + (uint32_t)b * NB2 * TM * 2;
#pragma unroll
      for (int g = 0; g < NB2 / 8; ++g) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = g * 8 + e;
          float val = 0.f;
          if (j < 2 * FD) {
            const float di = dm[j < FD ? j : j - FD] * inv;
            const float hi = __bfloat162float(__float2bfloat16_rn(di));
            val = j < FD ? hi : di - hi;
          }
          v[e] = val;
        }
        *reinterpret_cast<uint4 *>(b2 + mn_off(g * 8, row, TM * 16)) =
            make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
      }
      fence_proxy_async_smem();  // generic writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_PF + b));
#pragma unroll
      for (int j = 0; j < FD; ++j) dm[j] = dmn[j];
      inv = invn;
    }
    if (!ok) record_error(ERR_PREP, abort_flag, a.err_flag);
  } else {
    // ---------------- dx epilogue ----------------
    const int e = warp - W_EPI;
    const int quad = warp & 3;           // TMEM lane quadrant
    const int half = e >> 2;             // columns [64*half, 64*half + 64)
    const int row = quad * 32 + lane;    // token row of the tile = TMEM lane
    bool ok = true;
    // dz row and per-token scalars of the next tile are loaded while the
    // current tile is finished
    uint4 dzv[8];
    float inv = 0.f, rowb = 0.f, wgt = 0.f;
    auto load_next = [&](int lt_, uint4 (&dst)[8], float &inv_, float &rowb_, float &wgt_) {
      const int64_t tk = (tile_beg + lt_) * TM + row;
      if (lt_ < ntile && tk < tok_end) {
        const uint4 *dzp = reinterpret_cast<const uint4 *>(a.dz + tk * a.C + c_in + half * 64);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = __ldcs(dzp + q);
        inv_ = a.inv_rms[tk];
        rowb_ = a.rowb[tk];
        wgt_ = a.gate[tk * N + stream_i];
      }
    };
    load_next(0, dzv, inv, rowb, wgt);
    for (int lt = 0; lt < ntile && ok; ++lt) {
      const int b = lt % DB, s = lt % XS, sa = lt % AS;
      const int64_t tok = (tile_beg + lt) * TM + row;
      const bool valid = tok < tok_end;
      uint4 dzn[8];
      float inv_n = 0.f, rowb_n = 0.f, wgt_n = 0.f;
      load_next(lt + 1, dzn, inv_n, rowb_n, wgt_n);
      if (!WAIT_WARP(BAR(B_DF + b), (uint32_t)(lt / DB) & 1u)) { ok = false; break; }
      if (!WAIT_WARP(BAR(B_XF + s), (uint32_t)(lt / XS) & 1u)) { ok = false; break; }
      if (!WAIT_WARP(BAR(B_AF + sa), (uint32_t)(lt / AS) & 1u)) { ok = false; break; }
      tc_fence_after();
      const uint8_t *xrow = base + L.xs + s * XSTAGE + half * CHUNK + row * 128;
      uint8_t *arow = base + L.as + sa * XSTAGE + half * CHUNK + row * 128;  // dx_add tile; dx goes back here
      // 32 accumulator columns per TMEM load (one wait each), used by two
      // 16-column groups
      uint32_t d1r[32];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        if ((g & 1) == 0) {
          tmem_ld32_nowait(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)b * 128u + (uint32_t)(half * 64 + g * 16),
                           d1r);
          tmem_wait_ld();
        }
        float d1[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) d1[i] = __uint_as_float(d1r[(g & 1) * 16 + i]);
        if (valid) {
          uint32_t o[8];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int q = 2 * g + h;  // 16-byte granule of the 64-column half
            const uint32_t goff = (uint32_t)((q ^ (row & 7)) << 4);
            const uint4 xr = *reinterpret_cast<const uint4 *>(xrow + goff);
            uint4 ar = make_uint4(0u, 0u, 0u, 0u);
            if (a.dx_add) ar = *reinterpret_cast<const uint4 *>(arow + goff);
            const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
            const uint32_t zw[4] = {dzv[q].x, dzv[q].y, dzv[q].z, dzv[q].w};
            const uint32_t aw[4] = {ar.x, ar.y, ar.z, ar.w};
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const float xv[2] = {__uint_as_float(xw[p] << 16), __uint_as_float(xw[p] & 0xffff0000u)};
              const float zv[2] = {__uint_as_float(zw[p] << 16), __uint_as_float(zw[p] & 0xffff0000u)};
              const float av[2] = {__uint_as_float(aw[p] << 16), __uint_as_float(aw[p] & 0xffff0000u)};
              float r[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                float v = inv * d1[h * 8 + 2 * p + u] - rowb * xv[u];
                v = fmaf(wgt, zv[u], v);
                r[u] = v + av[u];
              }
              o[h * 4 + p] = pack_bf16(r[0], r[1]);
            }
            // dx replaces the dx_add granule it was computed from (same thread)
            *reinterpret_cast<uint4 *>(arow + goff) = make_uint4(o[h * 4], o[h * 4 + 1], o[h * 4 + 2], o[h * 4 + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();  // the warp's 32 x 64 dx block is complete in shared memory
      if (lane == 0) {
        mbar_arrive(BAR(B_DE + b));
        mbar_arrive(BAR(B_XE + s));  // the x tile was read by the arithmetic above
      }
      // coalesced write-back of the warp's own block: an instruction stores
      // 4 whole 128-byte row segments (lane -> row k*4 + lane/8, granule lane%8)
      {
        const int gq = lane & 7;
        const uint8_t *blk = base + L.as + sa * XSTAGE + half * CHUNK;
        __nv_bfloat16 *dxb = a.dx + col0 + half * 64 + gq * 8;
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = quad * 32 + k * 4 + (lane >> 3);
          v[k] = *reinterpret_cast<const uint4 *>(blk + r * 128 + ((gq ^ (r & 7)) << 4));
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = quad * 32 + k * 4 + (lane >> 3);
          const int64_t tk = (tile_beg + lt) * TM + r;
          if (tk < tok_end) __stcs(reinterpret_cast<uint4 *>(dxb + tk * a.nC), v[k]);
        }
        // the loads above have returned (the stores consumed them): only now
        // may the producer refill the stage
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(B_AE + sa));
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) dzv[q] = dzn[q];
      inv = inv_n;
      rowb = rowb_n;
      wgt = wgt_n;
    }
    if (!ok) record_error(ERR_EPI, abort_flag, a.err_flag);
    // dphi partial of this CTA: D2 lanes are its columns
    if (half == 0) {
      const bool drained = WAIT_WARP(BAR(B_DRAIN), 0u);
      if (drained && ok) {
        tc_fence_after();
        float d2[NB2];
#pragma unroll
        for (int c16 = 0; c16 < NB2 / 16; ++c16) {
          float t16[16];
          tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)D2COL + (uint32_t)c16 * 16u, t16);
#pragma unroll
          for (int i = 0; i < 16; ++i) d2[c16 * 16 + i] = t16[i];
        }
        float *dst = a.dphi_part + ((int64_t)split * a.nC + col0 + row) * FD;
#pragma unroll
        for (int j = 0; j < FD; ++j) dst[j] = d2[j] + d2[FD + j];
      }
    }
  }

  // ---------------- teardown ----------------
  __syncthreads();
  if (warp == W_MMA) {
    // every issued MMA has completed before TMEM is released
    wait_parity<false>(BAR(B_DRAIN), 0u, nullptr);
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (*abort_flag) {
    // a wait gave up: the CTA's whole share (dx of its 128 columns over its
    // token range, its dphi partial) becomes NaN instead of partly written
    const float qnan = __int_as_float(0x7fc00000);
    const __nv_bfloat16 bnan = __float2bfloat16_rn(qnan);
    const int64_t t_beg = tile_beg * TM;
    for (int64_t e = tid; e < (tok_end - t_beg) * KCOL; e += NTHREADS) {
      const int64_t r = e / KCOL;
      a.dx[(t_beg + r) * a.nC + col0 + (int)(e - r * KCOL)] = bnan;
    }
    float *dst = a.dphi_part + ((int64_t)split * a.nC + col0) * FD;
    for (int e = tid; e < KCOL * FD; e += NTHREADS) dst[e] = qnan;
  }
#undef WAIT_WARP
#undef BAR
}

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

template <int N, int MODE>
static cudaError_t launch_impl(const void *x, BArgs a, int sms, cudaStream_t stream) {
  using Cf = BCfg<N, MODE>;
  const BLayout L = make_blayout(Cf::K1, Cf::NB2, Cf::PB);
  const size_t smem = (size_t)L.total + 1024;
  if (smem > SMEM_LIMIT) return cudaErrorNotSupported;
  auto kern = pre_bwd_tc_kernel<N, MODE>;
  static std::mutex mu;
  static size_t smem_set[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (smem_set[dev & 63] < smem) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      smem_set[dev & 63] = smem;
    }
  }
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  // x and dx_add as (T rows) x (nC columns): 128-row x 64-column boxes, 128-byte swizzle
  CUtensorMap tmap, amap;
  const cuuint64_t dims[2] = {(cuuint64_t)a.nC, (cuuint64_t)a.T};
  const cuuint64_t strides[1] = {(cuuint64_t)a.nC * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)TM};
  const cuuint32_t estr[2] = {1, 1};
  const void *srcs[2] = {x, a.dx_add ? (const void *)a.dx_add : x};
  CUtensorMap *maps[2] = {&tmap, &amap};
  for (int m = 0; m < 2; ++m)
    if (enc(maps[m], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(srcs[m]), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorNotSupported;
  const int nslices = a.nC / KCOL;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)(nslices * a.TS), 1, 1);
  cfg.blockDim = dim3(NTHREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  (void)sms;
  e = cudaLaunchKernelEx(&cfg, kern, tmap, amap, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace tcb

int pre_bwd_tc_splits(int n, int C, int64_t T, int sm_count, int max_splits) {
  const int64_t nC = (int64_t)n * C;
  const int nslices = (int)(nC / tcb::KCOL);
  if (nslices <= 0) return 0;
  int ts = (sm_count > 0 ? sm_count : 148) / nslices;
  const int64_t tiles = (T + tcb::TM - 1) / tcb::TM;
  if (ts > tiles) ts = (int)tiles;
  if (ts > max_splits) ts = max_splits;
  return ts < 1 ? 1 : ts;
}

bool pre_bwd_tc_eligible(int mode, int n, int x_dtype, int64_t T, int C, const void *x, const void *dz,
                         const void *dx_add, const void *dx) {
  if (x_dtype != MHC_BF16 || T < 1) return false;
  if (mode == FULL && n > 4) return false;
  if (n > 8) return false;
  if (C % tcb::KCOL != 0) return false;  // a CTA's 128 columns lie inside one stream
  const uintptr_t m = (uintptr_t)x | (uintptr_t)dz | (uintptr_t)dx | (uintptr_t)dx_add;
  if ((m & 15) != 0) return false;
  return true;
}

cudaError_t launch_pre_bwd_tc(int mode, int n, const void *x, int64_t T, int C, const void *phi, int pdt,
                              const float *inv_rms, const float *dm, const float *rowb, const float *gate,
                              const void *dz, const void *dx_add, void *dx, float *dphi_part, int splits,
                              cudaStream_t stream) {
  tcb::BArgs a;
  a.T = T;
  a.C = C;
  a.nC = n * C;
  a.TS = splits;
  a.phi = phi;
  a.pdt = pdt;
  a.inv_rms = inv_rms;
  a.dm = dm;
  a.rowb = rowb;
  a.gate = gate;
  a.dz = reinterpret_cast<const __nv_bfloat16 *>(dz);
  a.dx_add = reinterpret_cast<const __nv_bfloat16 *>(dx_add);
  a.dx = reinterpret_cast<__nv_bfloat16 *>(dx);
  a.dphi_part = dphi_part;
  a.err_flag = host_error_flag();
  const int sms = device_sm_count();
  return with_mode(mode, [&](auto md) -> cudaError_t {
    constexpr int MODE = decltype(md)::value;
    switch (n) {
      case 1: return tcb::launch_impl<1, MODE>(x, a, sms, stream);
      case 2: return tcb::launch_impl<2, MODE>(x, a, sms, stream);
      case 4: return tcb::launch_impl<4, MODE>(x, a, sms, stream);
      case 8: if constexpr (MODE != FULL) return tcb::launch_impl<8, MODE>(x, a, sms, stream); break;
      default: break;
    }
    return cudaErrorNotSupported;
  });
}

int read_tcb_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tcb_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_tcb_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace mhc
