// sm_100a building blocks in inline PTX: mbarriers (local and cluster-remote),
// cluster rank / DSMEM addressing, TMA tiled loads, and the tcgen05 tensor-core
// path (TMEM allocation, UMMA shared-memory descriptors, MMA, commit, loads).
//
// Every wait is bounded: `wait_parity` gives up after MHC_WAIT_CYCLES clock
// cycles (about one second) and returns false so the caller can record an
// error, drain its own work and exit instead of hanging the GPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifndef MHC_WAIT_CYCLES
#define MHC_WAIT_CYCLES (2000000000LL)
#endif

namespace mhc {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init_cluster() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Arrive on a barrier of any CTA of the cluster (address from mapa), with
// release semantics at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
// Arrive on a barrier of any CTA of the cluster with the default (CTA-scope
// release) semantics: for "buffer free again" signals that publish no data.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Wait that acquires at cluster scope (for phases completed by remote arrives).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Non-blocking probes of the same (no suspension): the fast path of a wait
// whose phase has usually completed already.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_test_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false after `limit` clock cycles or as soon as
// *abort (if given) becomes non-zero.
template <bool CLUSTER>
__device__ __forceinline__ bool wait_parity_limit(uint32_t bar, uint32_t parity, const volatile int *abort,
                                                  long long limit) {
  const long long t0 = clock64();
  while (true) {
    const bool ok = CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
    if (ok) return true;
    if (abort != nullptr && *abort) return false;
    if (clock64() - t0 > limit) return false;
  }
}

// The wait every kernel uses: bounded by MHC_WAIT_CYCLES (about one second).
template <bool CLUSTER>
__device__ __forceinline__ bool wait_parity(uint32_t bar, uint32_t parity, const volatile int *abort) {
  return wait_parity_limit<CLUSTER>(bar, parity, abort, MHC_WAIT_CYCLES);
}

// The same with a non-blocking probe first, for waits that are mostly
// satisfied already when they are reached.
template <bool CLUSTER>
__device__ __forceinline__ bool wait_parity_fast(uint32_t bar, uint32_t parity, const volatile int *abort) {
  if (CLUSTER ? mbar_test_wait_cluster(bar, parity) : mbar_test_wait(bar, parity)) return true;
  return wait_parity_limit<CLUSTER>(bar, parity, abort, MHC_WAIT_CYCLES);
}

// What a kernel does when one of its bounded waits gives up: the first error
// code wins in the kernel's device error word and, if the caller registered
// one (mhc_set_error_flag), in a pinned host word that the host can read
// without synchronising.  The kernel then poisons (NaN) the outputs it owns
// and exits normally.
__device__ __forceinline__ void report_give_up(int *dev_word, int *host_flag, int code) {
  atomicCAS(dev_word, 0, code);
  if (host_flag != nullptr) {
    atomicCAS_system(host_flag, 0, code);
    __threadfence_system();
  }
}

// ---- cluster ----------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t ncluster_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of `local_addr` in the CTA of rank `rank`.
__device__ __forceinline__ uint32_t mapa(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
// Asynchronous store of 16 bytes into another CTA's shared memory that, once
// the data has landed, completes 16 bytes of the transaction count of the
// destination CTA's mbarrier (both addresses from mapa).  The consumer arms the
// barrier with mbarrier.arrive.expect_tx and waits on it; no fence is needed.
__device__ __forceinline__ void st_async_v4(uint32_t addr, float a, float b, float c, float d, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
               ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
               : "memory");
}
// The same for one 4-byte word.
__device__ __forceinline__ void st_async_f32(uint32_t addr, float a, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(addr), "f"(a),
               "r"(bar)
               : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- packed fp32 pairs (f32x2: two floats in a 64-bit register pair) ---------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// the two bf16 halves of a 32-bit word as an f32 pair (exact)
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t w) {
  return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// ---- TMA ----------------------------------------------------------------------
// 2-D tiled load of one box into this CTA's shared memory, completing `bar`'s
// transaction count (this CTA's shared memory only).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte
// aligned) from global memory into this CTA's shared memory, completing
// `bar`'s transaction count.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// 3-D tiled load of one box into this CTA's shared memory, completing `bar`'s
// transaction count.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void *tmap, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// L2 eviction-priority policies for the cache_hint forms below.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2-D tiled load with an L2 eviction-priority hint.
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const void *tmap, int x, int y, uint32_t bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// ---- tcgen05 --------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor for a K-major operand in the 128-byte swizzle
// layout: rows of 128 B, 8-row groups 1024 B apart (SBO), leading offset 16 B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);       // start address
  d |= (uint64_t)1 << 16;                              // leading byte offset (16 B)
  d |= (uint64_t)(1024 >> 4) << 32;                    // stride byte offset (1024 B)
  d |= (uint64_t)1 << 46;                              // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                              // 128-byte swizzle
  return d;
}

// The same for the 64-byte swizzle layout: rows of 64 B, 8-row groups 512 B
// apart (SBO); the layout the TMA's 64-byte swizzle writes for a 32-column
// bf16 box.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);       // start address
  d |= (uint64_t)1 << 16;                              // leading byte offset (16 B)
  d |= (uint64_t)(512 >> 4) << 32;                     // stride byte offset (512 B)
  d |= (uint64_t)1 << 46;                              // descriptor version (sm_100)
  d |= (uint64_t)4 << 61;                              // 64-byte swizzle
  return d;
}

// UMMA shared-memory descriptor, general form: leading / stride byte offsets
// and the layout type (0 = no swizzle, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor with the operand majors given: D fp32, A/B bf16;
// a_mn / b_mn = 1 for an MN-major operand.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32_major(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor: D fp32, A/B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int M, int N) {
  return (1u << 4)                       // D format fp32
         | (1u << 7)                     // A format bf16
         | (1u << 10)                    // B format bf16
         | ((uint32_t)(N >> 3) << 17)    // N
         | ((uint32_t)(M >> 4) << 24);   // M
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05 op of this thread is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; thread i receives lane (base+i).
// The wait for the load is part of the same asm statement so no register is
// read before the asynchronous load has landed.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 columns of this warp's 32 TMEM lanes without waiting: the registers are
// valid only after tmem_wait_ld (several loads can share one wait)
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 16 columns of this warp's 32 TMEM lanes as raw 32-bit words, waiting for
// the load inside the same asm statement
__device__ __forceinline__ void tmem_ld16u(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Four loads of 16 columns each (column addresses a0..a3) and their wait in
// one asm statement, so no register is read before the data has landed.
__device__ __forceinline__ void tmem_ld16x4u(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t (&r)[4][16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%65];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47}, [%66];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%67];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]), "=r"(r[0][5]), "=r"(r[0][6]),
        "=r"(r[0][7]), "=r"(r[0][8]), "=r"(r[0][9]), "=r"(r[0][10]), "=r"(r[0][11]), "=r"(r[0][12]),
        "=r"(r[0][13]), "=r"(r[0][14]), "=r"(r[0][15]),
        "=r"(r[1][0]), "=r"(r[1][1]), "=r"(r[1][2]), "=r"(r[1][3]), "=r"(r[1][4]), "=r"(r[1][5]), "=r"(r[1][6]),
        "=r"(r[1][7]), "=r"(r[1][8]), "=r"(r[1][9]), "=r"(r[1][10]), "=r"(r[1][11]), "=r"(r[1][12]),
        "=r"(r[1][13]), "=r"(r[1][14]), "=r"(r[1][15]),
        "=r"(r[2][0]), "=r"(r[2][1]), "=r"(r[2][2]), "=r"(r[2][3]), "=r"(r[2][4]), "=r"(r[2][5]), "=r"(r[2][6]),
        "=r"(r[2][7]), "=r"(r[2][8]), "=r"(r[2][9]), "=r"(r[2][10]), "=r"(r[2][11]), "=r"(r[2][12]),
        "=r"(r[2][13]), "=r"(r[2][14]), "=r"(r[2][15]),
        "=r"(r[3][0]), "=r"(r[3][1]), "=r"(r[3][2]), "=r"(r[3][3]), "=r"(r[3][4]), "=r"(r[3][5]), "=r"(r[3][6]),
        "=r"(r[3][7]), "=r"(r[3][8]), "=r"(r[3][9]), "=r"(r[3][10]), "=r"(r[3][11]), "=r"(r[3][12]),
        "=r"(r[3][13]), "=r"(r[3][14]), "=r"(r[3][15])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3));
}

// Two loads of 32 columns each (column addresses a0, a1) and their wait in one
// asm statement.
__device__ __forceinline__ void tmem_ld32x2u(uint32_t a0, uint32_t a1, uint32_t (&r)[2][32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]), "=r"(r[0][5]), "=r"(r[0][6]), "=r"(r[0][7]), "=r"(r[0][8]), "=r"(r[0][9]), "=r"(r[0][10]), "=r"(r[0][11]), "=r"(r[0][12]), "=r"(r[0][13]), "=r"(r[0][14]), "=r"(r[0][15]), "=r"(r[0][16]), "=r"(r[0][17]), "=r"(r[0][18]), "=r"(r[0][19]), "=r"(r[0][20]), "=r"(r[0][21]), "=r"(r[0][22]), "=r"(r[0][23]), "=r"(r[0][24]), "=r"(r[0][25]), "=r"(r[0][26]), "=r"(r[0][27]), "=r"(r[0][28]), "=r"(r[0][29]), "=r"(r[0][30]), "=r"(r[0][31]), "=r"(r[1][0]), "=r"(r[1][1]), "=r"(r[1][2]), "=r"(r[1][3]), "=r"(r[1][4]), "=r"(r[1][5]), "=r"(r[1][6]), "=r"(r[1][7]), "=r"(r[1][8]), "=r"(r[1][9]), "=r"(r[1][10]), "=r"(r[1][11]), "=r"(r[1][12]), "=r"(r[1][13]), "=r"(r[1][14]), "=r"(r[1][15]), "=r"(r[1][16]), "=r"(r[1][17]), "=r"(r[1][18]), "=r"(r[1][19]), "=r"(r[1][20]), "=r"(r[1][21]), "=r"(r[1][22]), "=r"(r[1][23]), "=r"(r[1][24]), "=r"(r[1][25]), "=r"(r[1][26]), "=r"(r[1][27]), "=r"(r[1][28]), "=r"(r[1][29]), "=r"(r[1][30]), "=r"(r[1][31])
      : "r"(a0), "r"(a1));
}

// Asynchronous copy of a 128-row x 32-byte block of a shared-memory matrix
// (described by a UMMA descriptor, swizzle included) into TMEM lanes 0-127,
// 8 columns from taddr.  Ordered with the issuing thread's later tcgen05.mma
// and tracked by its tcgen05.commit.
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers:
// thread i writes lane (base + i).  Complete once tmem_wait_st returns.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---- TMA stores (bulk async-groups) -------------------------------------------
// 2-D tiled store of one box from this CTA's shared memory; rows or columns
// outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const void *tmap, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// all but the newest committed group of this thread are complete
__device__ __forceinline__ void bulk_wait_all_but_one() { asm volatile("cp.async.bulk.wait_group 1;" ::: "memory"); }
// every committed store of this thread has finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every committed store of this thread is complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace sm100
}  // namespace mhc
