/*
 * mhc_b200.h — C ABI of the B200 (sm_100a) mHC residual-path kernels.
 *
 * Drop-in boundary for the manifold-constrained hyper-connection (mHC) layer of
 * Tshirt-hfk/minimind-mhc.  Every entry point replaces one kernel launch (plus
 * the torch reductions around it) that the reference performs inside its
 * autograd Functions; the citation beside each declaration names the reference
 * lines it replaces (paths relative to the reference project root).
 *
 * Conventions
 *  - Plain device pointers, element counts and dtype codes; no framework types.
 *  - Activations are row-major: x is (T, n*C) with the n streams of a token
 *    stored one after the other (stream i at columns [i*C, (i+1)*C)), z and f
 *    are (T, C), per-token coefficient tensors are (T, n) and (T, n, n).
 *  - phi is (n*C, FD) row-major, exactly the layout of the reference's
 *    `phi_weight` parameter (model/mhc_fused.py:798).
 *  - `stream` is a cudaStream_t passed as void*.  Nothing here synchronises,
 *    allocates device memory or keeps per-call host state; scratch memory is
 *    the caller's `workspace` (size from the matching *_workspace() query).
 *  - Every call validates its arguments before launching and returns MHC_OK or
 *    a negative status; `mhc_last_error()` gives a message for the calling
 *    thread.  A call that returns an error launched nothing.
 *  - Kernels are reentrant: calls on different streams with disjoint buffers
 *    may run concurrently.
 */
#ifndef MHC_B200_H
#define MHC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define MHC_F32  0
#define MHC_BF16 1
#define MHC_F16  2

/* status codes */
#define MHC_OK               0
#define MHC_ERR_NULL        -1  /* a required pointer is NULL                  */
#define MHC_ERR_DTYPE       -2  /* unsupported dtype code                      */
#define MHC_ERR_SHAPE       -3  /* unsupported n, C, T, iteration count        */
#define MHC_ERR_ALIGN       -4  /* pointer misaligned for the required access  */
#define MHC_ERR_WORKSPACE   -5  /* workspace missing or too small              */
#define MHC_ERR_CUDA        -6  /* CUDA launch / runtime failure               */
#define MHC_ERR_UNSUPPORTED -7  /* combination not implemented                 */

/* Version of this ABI (bumped on any signature change). */
int mhc_abi_version(void);

/* Message describing the last failing call on the calling thread ("" if none). */
const char *mhc_last_error(void);

/* ------------------------------------------------------------------------ */
/* Forward: coefficients (+ Sinkhorn) and the pre-aggregate                 */
/* ------------------------------------------------------------------------ */

/* Bytes of scratch `mhc_pre_fwd` needs for T tokens. */
size_t mhc_pre_fwd_workspace(int64_t T, int n, int C, int with_res);

/*
 * Coefficient kernel + pre-aggregate of one mHC sublayer.
 *
 *   inv_rms[t] = 1/sqrt(mean_k x[t,k]^2 + rms_eps)            (fp32, required)
 *   mixes[t,:] = inv_rms[t] * (x[t,:] @ phi)                  (fp32, required, FD wide)
 *   h_pre      = sigmoid(alpha_pre*mixes[:, :n] + bias_pre) + pre_eps
 *   h_post     = sigmoid(alpha_post*mixes[:, n:2n] + bias_post) * post_mult
 *   h_res      = alpha_res*mixes[:, 2n:].view(n,n) + bias_res         (apply_sinkhorn == 0)
 *              = Sinkhorn(that, sinkhorn_iters, sinkhorn_eps)         (apply_sinkhorn != 0)
 *   z[t,c]     = sum_i h_pre[t,i] * x[t, i*C + c]
 *
 * with_res = 1: full mHC (FD = 2n + n^2);  with_res = 0: no-H_res variant
 * (FD = 2n; alpha_res, bias_res, h_res ignored and may be NULL).
 * h_pre, h_post, h_res are written in `coef_dtype` and may be NULL when not
 * wanted; z is written in x_dtype.  Parameters (phi, alphas, biases) are read
 * in `param_dtype` and converted to fp32; all coefficient math is fp32.
 *
 * Replaces: model/mhc_fused.py:615-625 (_pre_phase_full_fwd_kernel launch in
 * _PrePhaseFullFn.forward) and, with apply_sinkhorn, model/mhc_fused.py:120-123
 * (_sinkhorn_fwd_kernel launch in _SinkhornFn.forward); with with_res = 0,
 * model/mhc_fused_no_hres.py:440-449 (_pre_phase_fwd_kernel launch).
 */
int mhc_pre_fwd(const void *x, int x_dtype, int64_t T, int n, int C,
                const void *phi, const void *alpha_pre, const void *bias_pre,
                const void *alpha_post, const void *bias_post,
                const void *alpha_res, const void *bias_res, int param_dtype,
                int with_res, int apply_sinkhorn, int sinkhorn_iters,
                float post_mult, float pre_eps, float rms_eps, float sinkhorn_eps,
                void *z, void *h_pre, void *h_post, void *h_res, int coef_dtype,
                float *inv_rms, float *mixes,
                void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ */
/* Forward: merge of sublayer l fused with the coefficient pass of l+1       */
/* ------------------------------------------------------------------------ */

/* Bytes of scratch `mhc_post_pre_fwd` needs (same as mhc_pre_fwd). */
size_t mhc_post_pre_fwd_workspace(int64_t T, int n, int C, int with_res);

/*
 * One call for the step between two consecutive mHC sublayers, with the next
 * sublayer's input RMSNorm:
 *
 *   x_out = x merged with sublayer l's output f:                         (f != NULL)
 *           x_out[t, i*C+c] = sum_j h_res_prev[t,i,j] x[t, j*C+c] + h_post_prev[t,i] f[t,c]
 *           (h_res_prev == NULL: H_res = I), exactly as mhc_post_fwd
 *   z, h_pre, h_post, h_res, inv_rms, mixes = mhc_pre_fwd of sublayer l+1 on x_out
 *           (on x itself when f == NULL; x_out, h_*_prev are then ignored)
 *   y[t,c] = z[t,c] * rsqrt(mean_c z[t,:]^2 + norm_eps) * norm_weight[c]  (norm_weight != NULL)
 *           the mean taken over z as stored (x_dtype); y has x_dtype
 *
 * Arguments after x_out have mhc_pre_fwd's meaning.  x_out must not alias x.
 * For bf16 streams with n in {2, 4}, C a multiple of 128 with 4 <= C/128 <= 8
 * and 16-byte aligned tensors, under MHC_PATH_FUSED_POST_PRE, the whole step
 * is one sm_100a kernel (x read once, x_out and z written once: 2nC + 2C
 * elements per token instead of the 3nC + 2C of mhc_post_fwd followed by
 * mhc_pre_fwd; mhc_last_path() = 3); otherwise it runs mhc_post_fwd,
 * mhc_pre_fwd and a row RMSNorm kernel, which is faster on B200 at every
 * measured shape.
 *
 * Replaces the pair model/mhc_fused.py:828-832 (post phase of sublayer l) +
 * :818-826 (pre phase of sublayer l+1) at the call sites
 * model/model_minimind.py:338-339 (attention then MLP) and :392-400
 * (consecutive blocks), and the input norms model/model_minimind.py:313-314
 * (attn_in_norm / ffn_in_norm applied to z in the closures at :330, :336).
 */
int mhc_post_pre_fwd(const void *x, int x_dtype, const void *h_res_prev, const void *h_post_prev,
                     int prev_coef_dtype, const void *f, int f_dtype, void *x_out,
                     int64_t T, int n, int C,
                     const void *phi, const void *alpha_pre, const void *bias_pre,
                     const void *alpha_post, const void *bias_post,
                     const void *alpha_res, const void *bias_res, int param_dtype,
                     int with_res, int apply_sinkhorn, int sinkhorn_iters,
                     float post_mult, float pre_eps, float rms_eps, float sinkhorn_eps,
                     void *z, void *h_pre, void *h_post, void *h_res, int coef_dtype,
                     float *inv_rms, float *mixes,
                     const void *norm_weight, int norm_dtype, float norm_eps, void *y,
                     void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ */
/* Forward: post / res merge                                                 */
/* ------------------------------------------------------------------------ */

/*
 *   out[t, i*C + c] = sum_j h_res[t,i,j] * x[t, j*C + c] + h_post[t,i] * f[t,c]
 * h_res == NULL means H_res = I (no-H_res variant: out = x + h_post (x) f).
 * out has x_dtype.
 * res_is_logits != 0: h_res holds the raw H_res logits; each token's matrix is
 * first projected with Sinkhorn-Knopp (sinkhorn_iters, sinkhorn_eps, the same
 * steps as mhc_sinkhorn_fwd) and, when h_res_out is not NULL, the normalised
 * matrices are stored there (h_res_dtype) for the backward pass.
 *
 * Replaces: model/mhc_fused.py:736-739 (_post_phase_full_fwd_kernel launch),
 * with res_is_logits also model/mhc_fused.py:828-830 (sinkhorn_normalize of
 * h_res_raw), and model/mhc_fused_no_hres.py:547-550 (_post_phase_fwd_kernel).
 */
int mhc_post_fwd(const void *x, int x_dtype, const void *h_res, int h_res_dtype,
                 const void *h_post, int h_post_dtype, const void *f, int f_dtype,
                 void *out, int64_t T, int n, int C, int res_is_logits, int sinkhorn_iters,
                 float sinkhorn_eps, void *h_res_out, void *stream);

/*
 * Backward of mhc_post_fwd for upstream gradient dout (x_dtype):
 *   dx[t, j*C+c]  = sum_i h_res[t,i,j] * dout[t, i*C+c]     (= dout when h_res == NULL)
 *   dh_res[t,i,j] = sum_c dout[t, i*C+c] * x[t, j*C+c]      (h_res_dtype)
 *   dh_post[t,i]  = sum_c dout[t, i*C+c] * f[t,c]          (h_post_dtype)
 *   df[t,c]       = sum_i h_post[t,i] * dout[t, i*C+c]     (f_dtype)
 * Any output pointer may be NULL to skip it (dh_res must be NULL when h_res is).
 *
 * Replaces: model/mhc_fused.py:761-766 (_post_phase_full_bwd_kernel launch) and
 * model/mhc_fused_no_hres.py:572-576 (_post_phase_bwd_kernel launch).
 */
int mhc_post_bwd(const void *dout, const void *x, int x_dtype,
                 const void *h_res, int h_res_dtype, const void *h_post, int h_post_dtype,
                 const void *f, int f_dtype,
                 void *dx, void *dh_res, void *dh_post, void *df,
                 int64_t T, int n, int C, void *stream);

/* ------------------------------------------------------------------------ */
/* Backward: coefficients (+ Sinkhorn by recompute) and pre-aggregate        */
/* ------------------------------------------------------------------------ */

/* Bytes of scratch `mhc_pre_bwd` needs for T tokens with the same with_res /
 * apply_sinkhorn / sinkhorn_iters arguments.  The answer depends on the SM count
 * of the current device: query on the device the call will run on. */
size_t mhc_pre_bwd_workspace(int64_t T, int n, int C, int with_res, int apply_sinkhorn,
                             int sinkhorn_iters);

/*
 * Backward of mhc_pre_fwd.  Inputs: x, phi, parameters, the saved fp32
 * inv_rms (T) and mixes (T, FD), and the upstream gradients dz (x_dtype),
 * dh_pre / dh_post / dh_res (coef_dtype, each may be NULL = zero).
 * apply_sinkhorn != 0: dh_res is the gradient w.r.t. the Sinkhorn OUTPUT and the
 * Sinkhorn backward runs by recompute from mixes; otherwise dh_res is the
 * gradient w.r.t. the raw logits.  dx_add (x_dtype, may be NULL) is added into
 * dx (fuses the residual-gradient sum autograd would otherwise do in a separate
 * pass).  Outputs: dx (x_dtype), dphi (n*C, FD) and the alpha/bias gradients in
 * param_dtype (any may be NULL to skip; the res ones must be NULL when
 * with_res = 0).  Parameter gradients are reduced over tokens deterministically
 * (fixed-order two-pass reduction, no atomics).
 *
 * Replaces: model/mhc_fused.py:681-711 (_pre_phase_full_bwd_kernel launch, the
 * cuBLAS grad_W GEMM and the torch alpha/bias reductions), with apply_sinkhorn
 * also model/mhc_fused.py:131-137 (_SinkhornFn.backward), and
 * model/mhc_fused_no_hres.py:500-524 for with_res = 0.
 */
int mhc_pre_bwd(const void *x, int x_dtype, int64_t T, int n, int C,
                const void *phi, const void *alpha_pre, const void *bias_pre,
                const void *alpha_post, const void *bias_post,
                const void *alpha_res, const void *bias_res, int param_dtype,
                int with_res, int apply_sinkhorn, int sinkhorn_iters,
                float post_mult, float pre_eps, float rms_eps, float sinkhorn_eps,
                const float *inv_rms, const float *mixes,
                const void *dz, const void *dh_pre, const void *dh_post, const void *dh_res,
                int coef_dtype, const void *dx_add,
                void *dx, void *dphi, void *dalpha_pre, void *dbias_pre,
                void *dalpha_post, void *dbias_post, void *dalpha_res, void *dbias_res,
                void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ */
/* Stand-alone Sinkhorn-Knopp                                                */
/* ------------------------------------------------------------------------ */

/*
 * Y[b] = Sinkhorn(M[b]) for `batch` n x n matrices: row softmax + eps, one
 * column normalisation, then (iters-1) row/column normalisations, each
 * dividing by (sum + eps).  Math in fp32.
 * Replaces: model/mhc_fused.py:120-123 (_sinkhorn_fwd_kernel launch).
 */
int mhc_sinkhorn_fwd(const void *M, int m_dtype, void *Y, int y_dtype,
                     int64_t batch, int n, int iters, float eps, void *stream);

/*
 * dM = d Sinkhorn(M) / dM applied to dY, by recomputing the forward
 * trajectory.  Replaces: model/mhc_fused.py:131-137 (_SinkhornFn.backward).
 */
int mhc_sinkhorn_bwd(const void *M, int m_dtype, const void *dY, int dy_dtype,
                     void *dM, int dm_dtype, int64_t batch, int n, int iters, float eps,
                     void *stream);

/* ------------------------------------------------------------------------ */
/* Model exit (MHCHead) and entry (StreamExpand)                             */
/* ------------------------------------------------------------------------ */

/* Bytes of scratch `mhc_head_fwd` needs for T tokens. */
size_t mhc_head_fwd_workspace(int64_t T, int n, int C);

/*
 * MHCHead: out[t,c] = sum_i w[t,i] x[t, i*C+c], w = sigmoid(alpha*mix + bias) + pre_eps,
 * mix = inv_rms * (x @ phi) with phi (n*C, n).  n == 1: out = x * inv_rms
 * (plain unweighted RMSNorm, phi/alpha/bias unused, mix_raw may be NULL).
 * inv_rms (T) and mix_raw (T, n) are fp32 saved tensors.
 * Replaces: model/mhc_common.py:344-351 (_mhc_head_fwd_kernel launch) and the
 * n == 1 branch model/mhc_common.py:438-442.
 */
int mhc_head_fwd(const void *x, int x_dtype, int64_t T, int n, int C,
                 const void *phi, const void *alpha, const void *bias, int param_dtype,
                 float pre_eps, float rms_eps,
                 void *out, float *inv_rms, float *mix_raw,
                 void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of scratch `mhc_head_bwd` needs for T tokens (current device). */
size_t mhc_head_bwd_workspace(int64_t T, int n, int C);

/*
 * Backward of mhc_head_fwd: dx (x_dtype), dphi / dalpha / dbias (param_dtype,
 * may be NULL; unused for n == 1).
 * Replaces: model/mhc_common.py:377-395 (_mhc_head_bwd_kernel launch, cuBLAS
 * grad_W and the torch alpha/bias reductions).
 */
int mhc_head_bwd(const void *x, int x_dtype, int64_t T, int n, int C,
                 const void *phi, const void *alpha, const void *bias, int param_dtype,
                 float pre_eps, float rms_eps, const float *inv_rms, const float *mix_raw,
                 const void *dout, void *dx, void *dphi, void *dalpha, void *dbias,
                 void *workspace, size_t workspace_bytes, void *stream);

/*
 * StreamExpand: out[t, i*C + c] = x[t, c] for i < n.  Backward: dx[t,c] =
 * sum_i dout[t, i*C + c].  Replaces: model/mhc_common.py:115-119 (expand +
 * reshape copy) and its autograd.
 */
int mhc_stream_expand_fwd(const void *x, void *out, int dtype, int64_t T, int n, int C,
                          void *stream);
int mhc_stream_expand_bwd(const void *dout, void *dx, int dtype, int64_t T, int n, int C,
                          void *stream);

/* Number of SMs of the current device (cached per device); <0 on error. */
int mhc_device_sm_count(void);

/*
 * Kernel selection for mhc_pre_fwd / mhc_head_fwd.  Two sm_100a kernels
 * compute the forward coefficient stage for bf16 activations: the two-read
 * cluster kernel (n*C a multiple of 512, C a multiple of 64, n <= 4 for the
 * full layer, n <= 8 otherwise; x read from HBM, then again from L2) and the
 * single-read kernel (n in {2, 4}, C a multiple of 128 with 512 <= C <= 1024;
 * x read from HBM once and kept in TMEM).  MHC_PATH_AUTO (default) picks the
 * faster of the two for the call, as measured on B200: the single-read kernel
 * for the no-H_res and head layers and for full layers of fewer than 32,768
 * tokens, the two-read kernel for longer full-layer batches; then the generic
 * CUDA-core kernels.  MHC_PATH_SINGLE_READ prefers the single-read kernel;
 * MHC_PATH_TWO_READ never uses it; MHC_PATH_GENERIC forces the generic
 * kernels (forward and backward).  Process-wide; returns the previous policy.
 * No reference counterpart (the reference selected Triton kernels through
 * environment flags, model/mhc_common.py:25-29).
 */
#define MHC_PATH_AUTO        0
#define MHC_PATH_GENERIC     1
#define MHC_PATH_TWO_READ    2
#define MHC_PATH_SINGLE_READ 3
/* As AUTO, and mhc_post_pre_fwd runs its fused merge + coefficient sm_100a
 * kernel where it applies (under every other policy it runs the merge kernel,
 * mhc_pre_fwd and a row RMSNorm kernel, measured faster on B200). */
#define MHC_PATH_FUSED_POST_PRE 4
int mhc_set_path_policy(int policy);

/* Kernel the process's last mhc_pre_fwd / mhc_head_fwd / mhc_post_pre_fwd ran
 * (on any thread: autograd runs backward on a thread of its own): 4 the
 * fp32-stream sm_100a coefficient kernel (fp32 x, n in {2, 4}, full or
 * no-H_res, C a multiple of 128 with 4 <= C/128 <= 8, 16-byte aligned x and
 * z; every policy but MHC_PATH_GENERIC), 3 the fused
 * merge + coefficient sm_100a kernel, 2 the single-read sm_100a kernel, 1 the
 * two-read sm_100a kernel, 0 the generic kernels; after
 * mhc_pre_bwd / mhc_head_bwd: 1 if the tensor-core dx / dphi kernel ran, 0
 * for the generic kernels. */
int mhc_last_path(void);

/*
 * First error code recorded by a fused kernel on the current device (0 = none;
 * 1..6 = a bounded wait of the producer / MMA / row / coefficient /
 * pre-aggregate / Sinkhorn role of the two-read forward kernel ran out,
 * 21..26 = the producer / MMA / ingest / coefficient / Sinkhorn / z role of
 * the single-read forward kernel, 31..37 = the producer / MMA / row /
 * coefficient / pre-aggregate / Sinkhorn / merge role of the fused merge +
 * coefficient kernel, 11..14 = one of the producer / MMA /
 * epilogue / prep roles of the backward tensor-core kernel, 99 = the
 * self-test below).  A kernel whose wait runs out gives up
 * instead of hanging and overwrites the outputs it owns with NaN.
 * Synchronises the device.  clear != 0 resets the word.  No reference
 * counterpart.
 */
int mhc_device_error(int clear);

/*
 * Registers a pinned host int (cudaHostAlloc / cudaMallocHost / a pinned
 * torch tensor; pageable memory is rejected with MHC_ERR_UNSUPPORTED) that
 * every fused kernel whose bounded wait runs out also writes its error code
 * into (first code wins).  The host reads it without any synchronisation, so
 * a caller can check for a give-up on every call at no cost; the code shows
 * up once the failing kernel has run, i.e. at a later call.  The caller owns
 * the word and resets it to 0.  NULL unregisters.  Process-wide.  No
 * reference counterpart.
 */
int mhc_set_error_flag(int *host_flag);

/*
 * Self-test of the bounded wait every fused kernel uses: a one-block kernel
 * waits on an mbarrier that nothing arrives at, with a limit of limit_cycles
 * SM clock cycles (use_abort != 0: a second warp raises the kernel's abort
 * flag after ~2e5 cycles, which must end the wait early).  result[0] = 1 if
 * the wait gave up, result[1] = cycles it lasted.  On giving up the kernel
 * takes the fused kernels' give-up path: error code 99 in its device word
 * (mhc_device_error) and in the registered host flag (mhc_set_error_flag),
 * and NaN over poison[0 .. poison_n) (a device fp32 buffer, or NULL with
 * poison_n = 0).  The kernel then exits normally and the context stays
 * usable.  Synchronises the device; allocates 16 bytes of device memory for
 * the result.  limit_cycles in (0, 4e9].  No reference counterpart (the
 * reference has no device-side waits).
 */
int mhc_selftest_bounded_wait(long long limit_cycles, int use_abort, long long *result, float *poison,
                              long long poison_n);

/*
 * mhc_pre_fwd without a caller workspace: the same arguments and results as
 * mhc_pre_fwd minus (workspace, workspace_bytes).  Scratch is a fixed 16 MiB
 * device array inside the library (a file-scope __device__ variable; its
 * address is looked up once per device, on the first call on that device --
 * make that first call outside any stream capture; the looked-up address is not
 * valid after cudaDeviceReset of that device, so do not use this entry point
 * in a process after such a reset).  Limit: T*n <= 4,194,304;
 * larger batches are rejected with MHC_ERR_WORKSPACE before any CUDA call.
 * Nothing is allocated and nothing in the scratch needs to start at zero.
 * All calls on one device share the scratch: two calls that overlap in time
 * (different streams or threads) race on it.
 * No counterpart in the reference (its launches allocate through the PyTorch
 * caching allocator, model/mhc_fused.py:589-595).
 */
int mhc_pre_fwd_noalloc(const void *x, int x_dtype, int64_t T, int n, int C,
                        const void *phi, const void *alpha_pre, const void *bias_pre,
                        const void *alpha_post, const void *bias_post,
                        const void *alpha_res, const void *bias_res, int param_dtype,
                        int with_res, int apply_sinkhorn, int sinkhorn_iters,
                        float post_mult, float pre_eps, float rms_eps, float sinkhorn_eps,
                        void *z, void *h_pre, void *h_post, void *h_res, int coef_dtype,
                        float *inv_rms, float *mixes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MHC_B200_H */
