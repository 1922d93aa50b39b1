// C ABI entry points (include/mhc_b200.h): argument validation, workspace
// carving and dispatch to the kernel launchers.  No entry point allocates,
// synchronises or launches anything when its arguments are rejected.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "mhc_b200.h"
#include "mhc_dispatch.cuh"
#include "mhc_kernels.h"

namespace mhc {

static thread_local char g_err[512] = "";

static int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static int cuda_status(cudaError_t e, const char *where) {
  if (e == cudaSuccess) return MHC_OK;
  return fail(MHC_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

int device_sm_count() {
  static int cache[128] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return -1;
  if (dev < 128 && cache[dev] > 0) return cache[dev];
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  if (dev < 128) cache[dev] = v;
  return v;
}

static bool dtype_ok(int d) { return d == MHC_F32 || d == MHC_BF16 || d == MHC_F16; }
static bool n_ok(int n) { return n == 1 || n == 2 || n == 4 || n == 8 || n == 16; }
static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
static bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
static size_t esize(int d) { return d == MHC_F32 ? 4 : 2; }

static int check_shape(int64_t T, int n, int C) {
  if (T < 0) return fail(MHC_ERR_SHAPE, "T must be >= 0 (got %lld)", (long long)T);
  if (!n_ok(n)) return fail(MHC_ERR_SHAPE, "n must be one of 1,2,4,8,16 (got %d)", n);
  if (C < 1) return fail(MHC_ERR_SHAPE, "C must be >= 1 (got %d)", C);
  if ((int64_t)n * C > (int64_t)1 << 30) return fail(MHC_ERR_SHAPE, "n*C too large");
  return MHC_OK;
}

static int g_policy = MHC_PATH_AUTO;
// kernel family of the last pre-stage call in the process (the autograd
// engine runs backward on its own thread, so this is not thread-local)
static std::atomic<int> g_last_path{0};

// Pinned host word the fused kernels also write their give-up code into
// (mhc_set_error_flag); null until a caller registers one.
static std::atomic<int *> g_host_flag{nullptr};
int *host_error_flag() { return g_host_flag.load(std::memory_order_acquire); }

// Which fused forward kernel MHC_PATH_AUTO runs, from B200 measurements
// (µs per call, two-read / single-read): full layer C=768 at 4K tokens
// 30.8 / 26.6, 16K 54.3 / 51.6, 32K 83.7 / 84.7, 64K 144 / 151, 256K 512 /
// 550; no-H_res at 32K tokens C=768 75.9 / 71.2, C=1024 93.5 / 89.3.  The
// single-read kernel wins when the tile sequence per cluster is short (its
// per-tile latency chain is hidden less) and for the narrow projections of the
// no-H_res and head layers; the two-read kernel for long full-layer batches.
static bool use_single_read(int mode, int n, int x_dtype, const void *x, const void *z, int64_t T, int C) {
  if (g_policy == MHC_PATH_SINGLE_READ) return pre_sr_eligible(mode, n, x_dtype, x, z, T, C);
  const bool automatic = g_policy == MHC_PATH_AUTO || g_policy == MHC_PATH_FUSED_POST_PRE;
  if (!automatic || !pre_sr_eligible(mode, n, x_dtype, x, z, T, C)) return false;
  if (!pre_tc_eligible(mode, n, x_dtype, x, z, T, C)) return true;
  return mode != 0 || T < 32768;
}

static int check_elem_align(const void *p, int dtype, const char *name) {
  if (p && !aligned(p, esize(dtype))) return fail(MHC_ERR_ALIGN, "%s is not %zu-byte aligned", name, esize(dtype));
  return MHC_OK;
}

}  // namespace mhc

using namespace mhc;

#define MHC_TRY(expr)           \
  do {                          \
    const int _s = (expr);      \
    if (_s != MHC_OK) return _s; \
  } while (0)

extern "C" {

int mhc_abi_version(void) { return 1; }

const char *mhc_last_error(void) { return g_err; }

int mhc_device_sm_count(void) { return device_sm_count(); }

int mhc_set_path_policy(int policy) {
  const int prev = g_policy;
  if (policy == MHC_PATH_AUTO || policy == MHC_PATH_GENERIC || policy == MHC_PATH_TWO_READ ||
      policy == MHC_PATH_SINGLE_READ || policy == MHC_PATH_FUSED_POST_PRE)
    g_policy = policy;
  return prev;
}

int mhc_last_path(void) { return g_last_path.load(); }

int mhc_device_error(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  const int words[5] = {read_sr_error(clear != 0), read_tc_error(clear != 0), read_tcb_error(clear != 0),
                        read_ch_error(clear != 0), read_selftest_error(clear != 0)};
  for (int w : words)
    if (w < 0) return -1;
  for (int w : words)
    if (w != 0) return w;
  return 0;
}

int mhc_set_error_flag(int *host_flag) {
  g_err[0] = 0;
  if (host_flag) {
    if (!aligned(host_flag, 4)) return fail(MHC_ERR_ALIGN, "mhc_set_error_flag: flag is not 4-byte aligned");
    cudaPointerAttributes at;
    const cudaError_t e = cudaPointerGetAttributes(&at, host_flag);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return cuda_status(e, "mhc_set_error_flag: cudaPointerGetAttributes");
    }
    // pinned (page-locked) host memory is addressable by every device at the
    // same pointer under unified addressing; pageable memory is not
    if (at.type != cudaMemoryTypeHost || at.devicePointer != static_cast<void *>(host_flag))
      return fail(MHC_ERR_UNSUPPORTED, "mhc_set_error_flag: the flag must be pinned host memory "
                                       "(cudaHostAlloc / cudaMallocHost / torch pin_memory)");
  }
  g_host_flag.store(host_flag, std::memory_order_release);
  return MHC_OK;
}

size_t mhc_pre_fwd_workspace(int64_t T, int n, int C, int with_res) {
  (void)C;
  (void)with_res;
  if (T <= 0 || n <= 0) return 256;
  return align256((size_t)T * n * 4);
}

int mhc_pre_fwd(const void *x, int x_dtype, int64_t T, int n, int C, const void *phi,
                const void *alpha_pre, const void *bias_pre, const void *alpha_post,
                const void *bias_post, const void *alpha_res, const void *bias_res, int param_dtype,
                int with_res, int apply_sinkhorn, int sinkhorn_iters, float post_mult,
                float pre_eps, float rms_eps, float sinkhorn_eps, void *z, void *h_pre,
                void *h_post, void *h_res, int coef_dtype, float *inv_rms, float *mixes,
                void *workspace, size_t workspace_bytes, void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(x_dtype) || !dtype_ok(param_dtype) || !dtype_ok(coef_dtype))
    return fail(MHC_ERR_DTYPE, "mhc_pre_fwd: bad dtype code (x=%d param=%d coef=%d)", x_dtype,
                param_dtype, coef_dtype);
  if (with_res != 0 && with_res != 1) return fail(MHC_ERR_SHAPE, "with_res must be 0 or 1");
  if (sinkhorn_iters < 0 || sinkhorn_iters > 100000) return fail(MHC_ERR_SHAPE, "bad sinkhorn_iters %d", sinkhorn_iters);
  if (T == 0) return MHC_OK;
  if (!x || !phi || !alpha_pre || !bias_pre || !alpha_post || !bias_post || !z || !inv_rms || !mixes)
    return fail(MHC_ERR_NULL, "mhc_pre_fwd: required pointer is NULL");
  if (with_res && (!alpha_res || !bias_res)) return fail(MHC_ERR_NULL, "mhc_pre_fwd: alpha_res/bias_res NULL");
  const size_t need = mhc_pre_fwd_workspace(T, n, C, with_res);
  if (!workspace || workspace_bytes < need)
    return fail(MHC_ERR_WORKSPACE, "mhc_pre_fwd: workspace %zu < %zu bytes", workspace_bytes, need);
  if (!aligned(workspace, 16) || !aligned(inv_rms, 4) || !aligned(mixes, 4))
    return fail(MHC_ERR_ALIGN, "mhc_pre_fwd: workspace/inv_rms/mixes misaligned");
  MHC_TRY(check_elem_align(x, x_dtype, "x"));
  MHC_TRY(check_elem_align(z, x_dtype, "z"));
  CoefParams p{alpha_pre, bias_pre, alpha_post, bias_post, alpha_res, bias_res, param_dtype,
               post_mult, pre_eps, rms_eps, sinkhorn_eps, apply_sinkhorn ? 1 : 0, sinkhorn_iters};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float *gate = reinterpret_cast<float *>(workspace);
  const int mode = with_res ? 0 : 1;
  g_last_path = 0;
  if (use_single_read(mode, n, x_dtype, x, z, T, C)) {
    cudaError_t e = launch_pre_sr(mode, n, x, T, C, phi, p, z, h_pre, h_post, with_res ? h_res : nullptr,
                                  coef_dtype, inv_rms, mixes, s);
    if (e == cudaSuccess) {
      g_last_path = 2;
      return MHC_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "mhc_pre_fwd single-read");
    cudaGetLastError();  // not supported on this device: the kernels below
  }
  if (g_policy != MHC_PATH_GENERIC && pre_tc_eligible(mode, n, x_dtype, x, z, T, C)) {
    cudaError_t e = launch_pre_tc(mode, n, x, T, C, phi, p, z, h_pre, h_post, with_res ? h_res : nullptr,
                                  coef_dtype, inv_rms, mixes, s);
    if (e == cudaSuccess) {
      g_last_path = 1;
      return MHC_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "mhc_pre_fwd fused");
    cudaGetLastError();  // not supported on this device: generic kernels below
  }
  if (g_policy != MHC_PATH_GENERIC && pre_xf_eligible(mode, n, x_dtype, x, z, T, C)) {
    cudaError_t e = launch_pre_xf(mode, n, x, T, C, phi, p, z, h_pre, h_post, with_res ? h_res : nullptr,
                                  coef_dtype, inv_rms, mixes, s);
    if (e == cudaSuccess) {
      g_last_path = 4;
      return MHC_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "mhc_pre_fwd fp32 stream");
    cudaGetLastError();  // not supported on this device: generic kernels below
  }
  MHC_TRY(cuda_status(launch_coef_fwd(mode, n, x_dtype, x, T, C, phi, p, h_pre, h_post,
                                      with_res ? h_res : nullptr, coef_dtype, inv_rms, mixes, gate,
                                      device_sm_count(), s),
                      "mhc_pre_fwd coef"));
  return cuda_status(launch_aggregate(n, x_dtype, x, gate, z, T, C, s), "mhc_pre_fwd aggregate");
}

size_t mhc_post_pre_fwd_workspace(int64_t T, int n, int C, int with_res) {
  return mhc_pre_fwd_workspace(T, n, C, with_res);
}

int mhc_post_pre_fwd(const void *x, int x_dtype, const void *h_res_prev, const void *h_post_prev,
                     int prev_coef_dtype, const void *f, int f_dtype, void *x_out, int64_t T, int n, int C,
                     const void *phi, const void *alpha_pre, const void *bias_pre, const void *alpha_post,
                     const void *bias_post, const void *alpha_res, const void *bias_res, int param_dtype,
                     int with_res, int apply_sinkhorn, int sinkhorn_iters, float post_mult, float pre_eps,
                     float rms_eps, float sinkhorn_eps, void *z, void *h_pre, void *h_post, void *h_res,
                     int coef_dtype, float *inv_rms, float *mixes, const void *norm_weight, int norm_dtype,
                     float norm_eps, void *y, void *workspace, size_t workspace_bytes, void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  const bool merge = f != nullptr, norm = norm_weight != nullptr;
  if (!dtype_ok(x_dtype) || !dtype_ok(param_dtype) || !dtype_ok(coef_dtype) ||
      (merge && (!dtype_ok(f_dtype) || !dtype_ok(prev_coef_dtype))) || (norm && !dtype_ok(norm_dtype)))
    return fail(MHC_ERR_DTYPE, "mhc_post_pre_fwd: bad dtype code");
  if (with_res != 0 && with_res != 1) return fail(MHC_ERR_SHAPE, "with_res must be 0 or 1");
  if (sinkhorn_iters < 0 || sinkhorn_iters > 100000) return fail(MHC_ERR_SHAPE, "bad sinkhorn_iters %d", sinkhorn_iters);
  if (!(norm_eps >= 0.f)) return fail(MHC_ERR_SHAPE, "mhc_post_pre_fwd: norm_eps must be >= 0");
  if (T == 0) return MHC_OK;
  if (!x || !phi || !alpha_pre || !bias_pre || !alpha_post || !bias_post || !z || !inv_rms || !mixes)
    return fail(MHC_ERR_NULL, "mhc_post_pre_fwd: required pointer is NULL");
  if (with_res && (!alpha_res || !bias_res)) return fail(MHC_ERR_NULL, "mhc_post_pre_fwd: alpha_res/bias_res NULL");
  if (merge && (!h_post_prev || !x_out)) return fail(MHC_ERR_NULL, "mhc_post_pre_fwd: h_post_prev/x_out NULL");
  if (merge && x_out == x) return fail(MHC_ERR_SHAPE, "mhc_post_pre_fwd: x_out must not alias x");
  if (norm && !y) return fail(MHC_ERR_NULL, "mhc_post_pre_fwd: y NULL with norm_weight");
  const size_t need = mhc_pre_fwd_workspace(T, n, C, with_res);
  if (!workspace || workspace_bytes < need)
    return fail(MHC_ERR_WORKSPACE, "mhc_post_pre_fwd: workspace %zu < %zu bytes", workspace_bytes, need);
  if (!aligned(workspace, 16) || !aligned(inv_rms, 4) || !aligned(mixes, 4))
    return fail(MHC_ERR_ALIGN, "mhc_post_pre_fwd: workspace/inv_rms/mixes misaligned");
  MHC_TRY(check_elem_align(x, x_dtype, "x"));
  MHC_TRY(check_elem_align(z, x_dtype, "z"));
  if (merge) {
    MHC_TRY(check_elem_align(x_out, x_dtype, "x_out"));
    MHC_TRY(check_elem_align(f, f_dtype, "f"));
  }
  if (norm) MHC_TRY(check_elem_align(y, x_dtype, "y"));
  CoefParams p{alpha_pre, bias_pre, alpha_post, bias_post, alpha_res, bias_res, param_dtype,
               post_mult, pre_eps, rms_eps, sinkhorn_eps, apply_sinkhorn ? 1 : 0, sinkhorn_iters};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int mode = with_res ? 0 : 1;
  // The fused kernel only under MHC_PATH_FUSED_POST_PRE: on B200 the merge
  // kernel followed by the coefficient kernel is measured faster (config 2,
  // 32768 tokens, n = 4, C = 768: 158 us for the two against 171 us fused;
  // with the input RMSNorm 214 us against 214 us).
  const bool fused = g_policy == MHC_PATH_FUSED_POST_PRE && (!merge || f_dtype == MHC_BF16) &&
                     post_pre_eligible(mode, n, x_dtype, x, f, x_out, z, y, T, C);
  if (fused) {
    cudaError_t e = launch_post_pre(mode, n, x, f, h_res_prev, h_post_prev, prev_coef_dtype, merge ? x_out : nullptr,
                                    T, C, phi, p, z, h_pre, h_post, with_res ? h_res : nullptr, coef_dtype, inv_rms,
                                    mixes, norm_weight, norm_dtype, norm_eps, norm ? y : nullptr, s);
    if (e == cudaSuccess) {
      g_last_path = 3;
      return MHC_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "mhc_post_pre_fwd fused");
    cudaGetLastError();  // not supported on this device: the separate kernels below
  }
  const void *src = x;
  if (merge) {
    MHC_TRY(cuda_status(launch_post_fwd(n, x_dtype, x, h_res_prev, prev_coef_dtype, h_post_prev, prev_coef_dtype, f,
                                        f_dtype, x_out, T, C, 0, 0, 0.f, nullptr, s),
                        "mhc_post_pre_fwd merge"));
    src = x_out;
  }
  MHC_TRY(mhc_pre_fwd(src, x_dtype, T, n, C, phi, alpha_pre, bias_pre, alpha_post, bias_post, alpha_res, bias_res,
                      param_dtype, with_res, apply_sinkhorn, sinkhorn_iters, post_mult, pre_eps, rms_eps,
                      sinkhorn_eps, z, h_pre, h_post, h_res, coef_dtype, inv_rms, mixes, workspace,
                      workspace_bytes, stream));
  if (norm)
    return cuda_status(launch_rmsnorm_rows(x_dtype, z, norm_weight, norm_dtype, norm_eps, y, T, C, s),
                       "mhc_post_pre_fwd norm");
  return MHC_OK;
}

int mhc_post_fwd(const void *x, int x_dtype, const void *h_res, int h_res_dtype, const void *h_post,
                 int h_post_dtype, const void *f, int f_dtype, void *out, int64_t T, int n, int C,
                 int res_is_logits, int sinkhorn_iters, float sinkhorn_eps, void *h_res_out,
                 void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(x_dtype) || !dtype_ok(h_post_dtype) || !dtype_ok(f_dtype) ||
      (h_res && !dtype_ok(h_res_dtype)))
    return fail(MHC_ERR_DTYPE, "mhc_post_fwd: bad dtype code");
  if (T == 0) return MHC_OK;
  if (!x || !h_post || !f || !out) return fail(MHC_ERR_NULL, "mhc_post_fwd: required pointer is NULL");
  if (res_is_logits && (sinkhorn_iters < 0 || sinkhorn_iters > 100000))
    return fail(MHC_ERR_SHAPE, "mhc_post_fwd: bad sinkhorn_iters %d", sinkhorn_iters);
  if (h_res_out && !(h_res && res_is_logits))
    return fail(MHC_ERR_NULL, "mhc_post_fwd: h_res_out needs h_res logits");
  MHC_TRY(check_elem_align(x, x_dtype, "x"));
  MHC_TRY(check_elem_align(out, x_dtype, "out"));
  MHC_TRY(check_elem_align(f, f_dtype, "f"));
  return cuda_status(launch_post_fwd(n, x_dtype, x, h_res, h_res_dtype, h_post, h_post_dtype, f,
                                     f_dtype, out, T, C, res_is_logits, sinkhorn_iters, sinkhorn_eps,
                                     h_res_out, reinterpret_cast<cudaStream_t>(stream)),
                     "mhc_post_fwd");
}

int mhc_post_bwd(const void *dout, const void *x, int x_dtype, const void *h_res, int h_res_dtype,
                 const void *h_post, int h_post_dtype, const void *f, int f_dtype, void *dx,
                 void *dh_res, void *dh_post, void *df, int64_t T, int n, int C, void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(x_dtype) || !dtype_ok(h_post_dtype) || !dtype_ok(f_dtype) ||
      (h_res && !dtype_ok(h_res_dtype)))
    return fail(MHC_ERR_DTYPE, "mhc_post_bwd: bad dtype code");
  if (!h_res && dh_res) return fail(MHC_ERR_NULL, "mhc_post_bwd: dh_res given without h_res");
  if (T == 0) return MHC_OK;
  if (!dout || !h_post || !f) return fail(MHC_ERR_NULL, "mhc_post_bwd: required pointer is NULL");
  if (h_res && !x) return fail(MHC_ERR_NULL, "mhc_post_bwd: x required with h_res");
  MHC_TRY(check_elem_align(dout, x_dtype, "dout"));
  MHC_TRY(check_elem_align(x, x_dtype, "x"));
  MHC_TRY(check_elem_align(dx, x_dtype, "dx"));
  MHC_TRY(check_elem_align(df, f_dtype, "df"));
  return cuda_status(launch_post_bwd(n, x_dtype, dout, x ? x : dout, h_res, h_res_dtype, h_post,
                                     h_post_dtype, f, f_dtype, dx, dh_res, dh_post, df, T, C,
                                     reinterpret_cast<cudaStream_t>(stream)),
                     "mhc_post_bwd");
}

size_t mhc_pre_bwd_workspace(int64_t T, int n, int C, int with_res, int apply_sinkhorn,
                             int sinkhorn_iters) {
  if (T < 0 || !n_ok(n) || C < 1) return 0;
  const int mode = with_res ? 0 : 1;
  return plan_pre_bwd(mode, n, T, C, apply_sinkhorn ? sinkhorn_iters : 0, device_sm_count()).total;
}

static int pre_bwd_common(int mode, const void *x, int x_dtype, int64_t T, int n, int C,
                          const void *phi, const CoefParams &p, const float *inv_rms,
                          const float *mixes, const void *dz, const void *dh_pre,
                          const void *dh_post, const void *dh_res, int coef_dtype,
                          const void *dx_add, void *dx, void *dphi, void *da_pre, void *db_pre,
                          void *da_post, void *db_post, void *da_res, void *db_res,
                          void *workspace, size_t workspace_bytes, void *stream, const char *who) {
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(x_dtype) || !dtype_ok(p.param_dtype) || !dtype_ok(coef_dtype))
    return fail(MHC_ERR_DTYPE, "%s: bad dtype code", who);
  if (p.sk_iters < 0 || p.sk_iters > 100000) return fail(MHC_ERR_SHAPE, "%s: bad sinkhorn_iters", who);
  const PreBwdPlan plan = plan_pre_bwd(mode, n, T, C, (mode == 0 && p.apply_sinkhorn) ? p.sk_iters : 0,
                                       device_sm_count());
  if (plan.k1_tokens <= 0)
    return fail(MHC_ERR_UNSUPPORTED, "%s: Sinkhorn trajectory of %d iterations does not fit in shared memory", who,
                p.sk_iters);
  if (T > 0) {
    if (!x || !phi || !inv_rms || !mixes || !dz || !dx)
      return fail(MHC_ERR_NULL, "%s: required pointer is NULL", who);
    MHC_TRY(check_elem_align(x, x_dtype, "x"));
    MHC_TRY(check_elem_align(dz, x_dtype, "dz"));
    MHC_TRY(check_elem_align(dx, x_dtype, "dx"));
    MHC_TRY(check_elem_align(dx_add, x_dtype, "dx_add"));
  }
  if (!workspace || workspace_bytes < plan.total)
    return fail(MHC_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, plan.total);
  if (!aligned(workspace, 256)) return fail(MHC_ERR_ALIGN, "%s: workspace must be 256-byte aligned", who);
  const bool use_tc = g_policy != MHC_PATH_GENERIC && pre_bwd_tc_eligible(mode, n, x_dtype, T, C, x, dz, dx_add, dx);
  g_last_path = use_tc ? 1 : 0;
  return cuda_status(launch_pre_bwd(mode, n, x_dtype, x, T, C, phi, p, inv_rms, mixes, dz, dh_pre,
                                    dh_post, dh_res, coef_dtype, dx_add, dx, dphi, da_pre, db_pre,
                                    da_post, db_post, da_res, db_res, workspace, plan, use_tc,
                                    reinterpret_cast<cudaStream_t>(stream)),
                     who);
}

int mhc_pre_bwd(const void *x, int x_dtype, int64_t T, int n, int C, const void *phi,
                const void *alpha_pre, const void *bias_pre, const void *alpha_post,
                const void *bias_post, const void *alpha_res, const void *bias_res, int param_dtype,
                int with_res, int apply_sinkhorn, int sinkhorn_iters, float post_mult,
                float pre_eps, float rms_eps, float sinkhorn_eps, const float *inv_rms,
                const float *mixes, const void *dz, const void *dh_pre, const void *dh_post,
                const void *dh_res, int coef_dtype, const void *dx_add, void *dx, void *dphi,
                void *dalpha_pre, void *dbias_pre, void *dalpha_post, void *dbias_post,
                void *dalpha_res, void *dbias_res, void *workspace, size_t workspace_bytes,
                void *stream) {
  g_err[0] = 0;
  if (with_res != 0 && with_res != 1) return fail(MHC_ERR_SHAPE, "with_res must be 0 or 1");
  if (T > 0 && (!alpha_pre || !bias_pre || !alpha_post || !bias_post))
    return fail(MHC_ERR_NULL, "mhc_pre_bwd: parameter pointer is NULL");
  if (with_res && T > 0 && (!alpha_res || !bias_res)) return fail(MHC_ERR_NULL, "mhc_pre_bwd: alpha_res/bias_res NULL");
  if (!with_res && (dh_res || dalpha_res || dbias_res))
    return fail(MHC_ERR_NULL, "mhc_pre_bwd: res gradients given with with_res = 0");
  CoefParams p{alpha_pre, bias_pre, alpha_post, bias_post, alpha_res, bias_res, param_dtype,
               post_mult, pre_eps, rms_eps, sinkhorn_eps, apply_sinkhorn ? 1 : 0, sinkhorn_iters};
  return pre_bwd_common(with_res ? 0 : 1, x, x_dtype, T, n, C, phi, p, inv_rms, mixes, dz, dh_pre,
                        dh_post, with_res ? dh_res : nullptr, coef_dtype, dx_add, dx, dphi,
                        dalpha_pre, dbias_pre, dalpha_post, dbias_post, dalpha_res, dbias_res,
                        workspace, workspace_bytes, stream, "mhc_pre_bwd");
}

int mhc_sinkhorn_fwd(const void *M, int m_dtype, void *Y, int y_dtype, int64_t batch, int n,
                     int iters, float eps, void *stream) {
  g_err[0] = 0;
  if (batch < 0 || !n_ok(n)) return fail(MHC_ERR_SHAPE, "mhc_sinkhorn_fwd: bad batch/n");
  if (!dtype_ok(m_dtype) || !dtype_ok(y_dtype)) return fail(MHC_ERR_DTYPE, "mhc_sinkhorn_fwd: bad dtype");
  if (iters < 0 || iters > 100000) return fail(MHC_ERR_SHAPE, "mhc_sinkhorn_fwd: bad iters");
  if (batch == 0) return MHC_OK;
  if (!M || !Y) return fail(MHC_ERR_NULL, "mhc_sinkhorn_fwd: NULL pointer");
  return cuda_status(launch_sinkhorn_fwd(n, M, m_dtype, Y, y_dtype, batch, iters, eps,
                                         reinterpret_cast<cudaStream_t>(stream)),
                     "mhc_sinkhorn_fwd");
}

int mhc_sinkhorn_bwd(const void *M, int m_dtype, const void *dY, int dy_dtype, void *dM,
                     int dm_dtype, int64_t batch, int n, int iters, float eps, void *stream) {
  g_err[0] = 0;
  if (batch < 0 || !n_ok(n)) return fail(MHC_ERR_SHAPE, "mhc_sinkhorn_bwd: bad batch/n");
  if (!dtype_ok(m_dtype) || !dtype_ok(dy_dtype) || !dtype_ok(dm_dtype))
    return fail(MHC_ERR_DTYPE, "mhc_sinkhorn_bwd: bad dtype");
  if (iters < 0 || iters > 100000) return fail(MHC_ERR_SHAPE, "mhc_sinkhorn_bwd: bad iters");
  if (sinkhorn_bwd_smem_per_item(n, iters) > 200 * 1024)
    return fail(MHC_ERR_UNSUPPORTED, "mhc_sinkhorn_bwd: trajectory too large for shared memory");
  if (batch == 0) return MHC_OK;
  if (!M || !dY || !dM) return fail(MHC_ERR_NULL, "mhc_sinkhorn_bwd: NULL pointer");
  return cuda_status(launch_sinkhorn_bwd(n, M, m_dtype, dY, dy_dtype, dM, dm_dtype, batch, iters, eps,
                                         reinterpret_cast<cudaStream_t>(stream)),
                     "mhc_sinkhorn_bwd");
}

size_t mhc_head_fwd_workspace(int64_t T, int n, int C) { return mhc_pre_fwd_workspace(T, n, C, 0); }

int mhc_head_fwd(const void *x, int x_dtype, int64_t T, int n, int C, const void *phi,
                 const void *alpha, const void *bias, int param_dtype, float pre_eps, float rms_eps,
                 void *out, float *inv_rms, float *mix_raw, void *workspace, size_t workspace_bytes,
                 void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(x_dtype) || !dtype_ok(param_dtype)) return fail(MHC_ERR_DTYPE, "mhc_head_fwd: bad dtype");
  if (T == 0) return MHC_OK;
  if (!x || !out || !inv_rms) return fail(MHC_ERR_NULL, "mhc_head_fwd: required pointer is NULL");
  MHC_TRY(check_elem_align(x, x_dtype, "x"));
  MHC_TRY(check_elem_align(out, x_dtype, "out"));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n == 1) return cuda_status(launch_head1_fwd(x_dtype, x, out, inv_rms, T, C, rms_eps, s), "mhc_head_fwd");
  if (!phi || !alpha || !bias || !mix_raw) return fail(MHC_ERR_NULL, "mhc_head_fwd: phi/alpha/bias/mix_raw NULL");
  const size_t need = mhc_head_fwd_workspace(T, n, C);
  if (!workspace || workspace_bytes < need)
    return fail(MHC_ERR_WORKSPACE, "mhc_head_fwd: workspace %zu < %zu bytes", workspace_bytes, need);
  CoefParams p{alpha, bias, nullptr, nullptr, nullptr, nullptr, param_dtype, 1.f, pre_eps, rms_eps, 0.f, 0, 0};
  float *gate = reinterpret_cast<float *>(workspace);
  g_last_path = 0;
  if (use_single_read(2, n, x_dtype, x, out, T, C)) {
    cudaError_t e = launch_pre_sr(2, n, x, T, C, phi, p, out, nullptr, nullptr, nullptr, MHC_F32, inv_rms,
                                  mix_raw, s);
    if (e == cudaSuccess) {
      g_last_path = 2;
      return MHC_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "mhc_head_fwd single-read");
    cudaGetLastError();
  }
  if (g_policy != MHC_PATH_GENERIC && pre_tc_eligible(2, n, x_dtype, x, out, T, C)) {
    cudaError_t e = launch_pre_tc(2, n, x, T, C, phi, p, out, nullptr, nullptr, nullptr, MHC_F32, inv_rms,
                                  mix_raw, s);
    if (e == cudaSuccess) {
      g_last_path = 1;
      return MHC_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "mhc_head_fwd fused");
    cudaGetLastError();
  }
  MHC_TRY(cuda_status(launch_coef_fwd(2, n, x_dtype, x, T, C, phi, p, nullptr, nullptr, nullptr,
                                      MHC_F32, inv_rms, mix_raw, gate, device_sm_count(), s),
                      "mhc_head_fwd coef"));
  return cuda_status(launch_aggregate(n, x_dtype, x, gate, out, T, C, s), "mhc_head_fwd aggregate");
}

size_t mhc_head_bwd_workspace(int64_t T, int n, int C) {
  if (T < 0 || !n_ok(n) || C < 1) return 0;
  if (n == 1) return 256;
  return plan_pre_bwd(2, n, T, C, 0, device_sm_count()).total;
}

int mhc_head_bwd(const void *x, int x_dtype, int64_t T, int n, int C, const void *phi,
                 const void *alpha, const void *bias, int param_dtype, float pre_eps, float rms_eps,
                 const float *inv_rms, const float *mix_raw, const void *dout, void *dx, void *dphi,
                 void *dalpha, void *dbias, void *workspace, size_t workspace_bytes, void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(x_dtype) || !dtype_ok(param_dtype)) return fail(MHC_ERR_DTYPE, "mhc_head_bwd: bad dtype");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n == 1) {
    if (T == 0) return MHC_OK;
    if (!x || !inv_rms || !dout || !dx) return fail(MHC_ERR_NULL, "mhc_head_bwd: required pointer is NULL");
    return cuda_status(launch_head1_bwd(x_dtype, x, inv_rms, dout, dx, T, C, s), "mhc_head_bwd");
  }
  if (T > 0 && (!alpha || !bias)) return fail(MHC_ERR_NULL, "mhc_head_bwd: alpha/bias NULL");
  CoefParams p{alpha, bias, nullptr, nullptr, nullptr, nullptr, param_dtype, 1.f, pre_eps, rms_eps, 0.f, 0, 0};
  return pre_bwd_common(2, x, x_dtype, T, n, C, phi, p, inv_rms, mix_raw, dout, nullptr, nullptr,
                        nullptr, MHC_F32, nullptr, dx, dphi, dalpha, dbias, nullptr, nullptr, nullptr,
                        nullptr, workspace, workspace_bytes, stream, "mhc_head_bwd");
}

int mhc_stream_expand_fwd(const void *x, void *out, int dtype, int64_t T, int n, int C, void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(dtype)) return fail(MHC_ERR_DTYPE, "mhc_stream_expand_fwd: bad dtype");
  if (T == 0) return MHC_OK;
  if (!x || !out) return fail(MHC_ERR_NULL, "mhc_stream_expand_fwd: NULL pointer");
  return cuda_status(launch_expand_fwd(dtype, x, out, T, n, C, reinterpret_cast<cudaStream_t>(stream)),
                     "mhc_stream_expand_fwd");
}

int mhc_stream_expand_bwd(const void *dout, void *dx, int dtype, int64_t T, int n, int C, void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  if (!dtype_ok(dtype)) return fail(MHC_ERR_DTYPE, "mhc_stream_expand_bwd: bad dtype");
  if (T == 0) return MHC_OK;
  if (!dout || !dx) return fail(MHC_ERR_NULL, "mhc_stream_expand_bwd: NULL pointer");
  return cuda_status(launch_expand_bwd(dtype, dout, dx, T, n, C, reinterpret_cast<cudaStream_t>(stream)),
                     "mhc_stream_expand_bwd");
}

/* ------------------------------------------------------------------------ */
/* mhc_pre_fwd without a caller workspace                                    */
/* ------------------------------------------------------------------------ */

}  // extern "C"

namespace mhc {
// Fixed device scratch of mhc_pre_fwd_noalloc: 16 MiB, enough for T*n <=
// 4,194,304 (the generic path's per-token fp32 gate weights).  Every word the
// kernels read from it is written earlier in the same call, so nothing in it
// has to start at zero.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static std::mutex g_noalloc_mu;
static void *g_noalloc_ptr[128] = {nullptr};

// Device address of the scratch on the current device, looked up once per
// device (the first call on a device does the lookup).  The cached address
// belongs to the device's current context: after cudaDeviceReset the module is
// loaded again and the array may sit elsewhere, so the entry point must not be
// used in a process after such a reset.
static int noalloc_scratch(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "mhc_pre_fwd_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 128) return fail(MHC_ERR_UNSUPPORTED, "mhc_pre_fwd_noalloc: device index %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "mhc_pre_fwd_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return MHC_OK;
}
}  // namespace mhc

extern "C" {

int mhc_pre_fwd_noalloc(const void *x, int x_dtype, int64_t T, int n, int C, const void *phi,
                        const void *alpha_pre, const void *bias_pre, const void *alpha_post,
                        const void *bias_post, const void *alpha_res, const void *bias_res,
                        int param_dtype, int with_res, int apply_sinkhorn, int sinkhorn_iters,
                        float post_mult, float pre_eps, float rms_eps, float sinkhorn_eps, void *z,
                        void *h_pre, void *h_post, void *h_res, int coef_dtype, float *inv_rms,
                        float *mixes, void *stream) {
  g_err[0] = 0;
  MHC_TRY(check_shape(T, n, C));
  const size_t need = mhc_pre_fwd_workspace(T, n, C, with_res);
  if (need > kNoAllocScratchBytes)
    return fail(MHC_ERR_WORKSPACE,
                "mhc_pre_fwd_noalloc: T=%lld x n=%d needs %zu bytes of scratch; the fixed device scratch "
                "holds %zu (T*n <= %zu); use mhc_pre_fwd with a workspace",
                (long long)T, n, need, kNoAllocScratchBytes, kNoAllocScratchBytes / 4);
  void *scratch = nullptr;
  if (T > 0) MHC_TRY(noalloc_scratch(&scratch));
  return mhc_pre_fwd(x, x_dtype, T, n, C, phi, alpha_pre, bias_pre, alpha_post, bias_post, alpha_res,
                     bias_res, param_dtype, with_res, apply_sinkhorn, sinkhorn_iters, post_mult, pre_eps,
                     rms_eps, sinkhorn_eps, z, h_pre, h_post, h_res, coef_dtype, inv_rms, mixes, scratch,
                     scratch ? kNoAllocScratchBytes : 0, stream);
}

}  // extern "C"
