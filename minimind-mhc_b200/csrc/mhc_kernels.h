// Host-side launchers implemented by the kernel translation units and called by
// the C ABI layer (mhc_capi.cu).  Arguments are validated by the caller; these
// functions only pick the template instance and launch on `stream`.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mhc {

struct CoefParams {
  const void *alpha_pre, *bias_pre, *alpha_post, *bias_post, *alpha_res, *bias_res;
  int param_dtype;
  float post_mult, pre_eps, rms_eps, sk_eps;
  int apply_sinkhorn, sk_iters;
};

// ---- forward --------------------------------------------------------------
// mode: 0 FULL, 1 NOHRES, 2 HEAD.  `gate_ws` receives the fp32 aggregation
// weights (h_pre, or the head weights), T x n.
cudaError_t launch_coef_fwd(int mode, int n, int x_dtype, const void *x, int64_t T, int C,
                            const void *phi, const CoefParams &p, void *h_pre, void *h_post,
                            void *h_res, int coef_dtype, float *inv_rms, float *mixes,
                            float *gate_ws, int sm_count, cudaStream_t stream);

cudaError_t launch_aggregate(int n, int x_dtype, const void *x, const float *w, void *z,
                             int64_t T, int C, cudaStream_t stream);

cudaError_t launch_head1_fwd(int x_dtype, const void *x, void *out, float *inv_rms, int64_t T,
                             int C, float rms_eps, cudaStream_t stream);
cudaError_t launch_head1_bwd(int x_dtype, const void *x, const float *inv_rms, const void *dout,
                             void *dx, int64_t T, int C, cudaStream_t stream);

// res_is_logits: h_res holds H_res logits; the kernel applies Sinkhorn-Knopp
// (sk_iters, sk_eps) per token before the merge and, if h_res_out is given,
// stores the normalised matrices there (h_res_dtype).
cudaError_t launch_post_fwd(int n, int x_dtype, const void *x, const void *h_res, int h_res_dtype,
                            const void *h_post, int h_post_dtype, const void *f, int f_dtype,
                            void *out, int64_t T, int C, int res_is_logits, int sk_iters,
                            float sk_eps, void *h_res_out, cudaStream_t stream);

// ---- fused sm_100a coefficient + pre-aggregate (bf16 activations) -----------
bool pre_tc_eligible(int mode, int n, int x_dtype, const void *x, const void *z, int64_t T, int C);
cudaError_t launch_pre_tc(int mode, int n, const void *x, int64_t T, int C, const void *phi,
                          const CoefParams &p, void *z, void *h_pre, void *h_post, void *h_res,
                          int coef_dtype, float *inv_rms, float *mixes, cudaStream_t stream);
int read_tc_error(bool clear);

// ---- single-read sm_100a coefficient + pre-aggregate (bf16 activations) ----
// n in {2, 4}, C a multiple of 128 with 4 <= C / 128 <= 8
bool pre_sr_eligible(int mode, int n, int x_dtype, const void *x, const void *z, int64_t T, int C);
cudaError_t launch_pre_sr(int mode, int n, const void *x, int64_t T, int C, const void *phi,
                          const CoefParams &p, void *z, void *h_pre, void *h_post, void *h_res,
                          int coef_dtype, float *inv_rms, float *mixes, cudaStream_t stream);
int read_sr_error(bool clear);

// ---- merge of sublayer l fused with the coefficient pass of l+1 (bf16) ----
// n in {2, 4}, full or no-H_res, C a multiple of 128 with 4 <= C / 128 <= 8.
// f == NULL: no merge (coefficient pass over x); norm_w == NULL: no RMSNorm.
bool post_pre_eligible(int mode, int n, int x_dtype, const void *x, const void *f, const void *x_out,
                       const void *z, const void *y, int64_t T, int C);
cudaError_t launch_post_pre(int mode, int n, const void *x, const void *f, const void *h_res_prev,
                            const void *h_post_prev, int prev_dtype, void *x_out, int64_t T, int C,
                            const void *phi, const CoefParams &p, void *z, void *h_pre, void *h_post,
                            void *h_res, int coef_dtype, float *inv_rms, float *mixes, const void *norm_w,
                            int norm_dtype, float norm_eps, void *y, cudaStream_t stream);
// the same kernel's coefficient pass for fp32 activations (z fp32): x split
// into bf16 hi | lo in shared memory for the tensor-core projection
bool pre_xf_eligible(int mode, int n, int x_dtype, const void *x, const void *z, int64_t T, int C);
cudaError_t launch_pre_xf(int mode, int n, const void *x, int64_t T, int C, const void *phi, const CoefParams &p,
                          void *z, void *h_pre, void *h_post, void *h_res, int coef_dtype, float *inv_rms,
                          float *mixes, cudaStream_t stream);
int read_ch_error(bool clear);
cudaError_t launch_rmsnorm_rows(int z_dtype, const void *z, const void *w, int w_dtype, float eps, void *y,
                                int64_t T, int C, cudaStream_t stream);

cudaError_t launch_post_bwd(int n, int x_dtype, const void *dout, const void *x, const void *h_res,
                            int h_res_dtype, const void *h_post, int h_post_dtype, const void *f,
                            int f_dtype, void *dx, void *dh_res, void *dh_post, void *df,
                            int64_t T, int C, cudaStream_t stream);

// ---- backward of the coefficient / aggregate stage --------------------------
struct PreBwdPlan {
  int fd;            // projection width
  int k1_tokens;     // tokens per block of the coefficient-backward kernel
  int k1_blocks;     // blocks of that kernel
  int k2_kc;         // k columns per block of the dx / dphi kernel
  int k2_kblocks;    // ceil(nC / kc)
  int k2_tsplits;    // token splits (one dphi partial per split)
  size_t off_dm, off_rowb, off_gate, off_dphi_part, off_coef_part, off_dots, total;
};

PreBwdPlan plan_pre_bwd(int mode, int n, int64_t T, int C, int sk_iters, int sm_count);

cudaError_t launch_pre_bwd(int mode, int n, int x_dtype, const void *x, int64_t T, int C,
                           const void *phi, const CoefParams &p, const float *inv_rms,
                           const float *mixes, const void *dz, const void *dh_pre,
                           const void *dh_post, const void *dh_res, int coef_dtype,
                           const void *dx_add, void *dx, void *dphi, void *dalpha_pre,
                           void *dbias_pre, void *dalpha_post, void *dbias_post,
                           void *dalpha_res, void *dbias_res, void *workspace,
                           const PreBwdPlan &plan, bool use_tc, cudaStream_t stream);

// Tensor-core dx / dphi stage (bf16 x, sm_100a): replaces the CUDA-core one
// where eligible; `splits` token ranges, one dphi partial each.
bool pre_bwd_tc_eligible(int mode, int n, int x_dtype, int64_t T, int C, const void *x, const void *dz,
                         const void *dx_add, const void *dx);
int pre_bwd_tc_splits(int n, int C, int64_t T, int sm_count, int max_splits);
cudaError_t launch_pre_bwd_tc(int mode, int n, const void *x, int64_t T, int C, const void *phi, int pdt,
                              const float *inv_rms, const float *dm, const float *rowb, const float *gate,
                              const void *dz, const void *dx_add, void *dx, float *dphi_part, int splits,
                              cudaStream_t stream);
int read_tcb_error(bool clear);

// Pinned host word registered with mhc_set_error_flag (null when none): the
// fused kernels' give-up path writes its error code there as well as into
// their device error words.
int *host_error_flag();
int read_selftest_error(bool clear);

// ---- stand-alone pieces -----------------------------------------------------
cudaError_t launch_sinkhorn_fwd(int n, const void *M, int m_dtype, void *Y, int y_dtype,
                                int64_t batch, int iters, float eps, cudaStream_t stream);
cudaError_t launch_sinkhorn_bwd(int n, const void *M, int m_dtype, const void *dY, int dy_dtype,
                                void *dM, int dm_dtype, int64_t batch, int iters, float eps,
                                cudaStream_t stream);
size_t sinkhorn_bwd_smem_per_item(int n, int iters);

cudaError_t launch_expand_fwd(int dtype, const void *x, void *out, int64_t T, int n, int C,
                              cudaStream_t stream);
cudaError_t launch_expand_bwd(int dtype, const void *dout, void *dx, int64_t T, int n, int C,
                              cudaStream_t stream);

}  // namespace mhc
