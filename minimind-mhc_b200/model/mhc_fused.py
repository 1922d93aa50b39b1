"""Full mHC sublayer connection (H_pre, H_post, H_res) on B200.

Drop-in for the reference's ``model/mhc_fused.py``: ``MHCConnection_Fused``
(same constructor, parameters and ``forward(x_flat, sublayer_fn)``),
``sinkhorn_normalize``, and the autograd Functions ``_SinkhornFn``,
``_PrePhaseFullFn`` and ``_PostPhaseFullFn`` with the reference's ``apply``
argument orders.  All math runs in the sm_100a kernels of ``libmhc_b200.so``;
CUDA tensors only, no CPU path and no Triton.

Per sublayer the module launches: the coefficient kernel (RMS statistics, the
n*C x (2n+n^2) projection, sigmoid gates and the per-token Sinkhorn-Knopp
projection of H_res, fused) and the pre-aggregate (``mhc_pre_fwd``), the
caller's ``sublayer_fn``, then the res/post merge (``mhc_post_fwd``).  In
backward, the post-merge kernel hands its residual gradient to the
coefficient-backward kernel, which adds it while writing dx (one pass instead
of autograd's separate sum), and Sinkhorn is differentiated by recomputing its
trajectory from the saved projection.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _native as nat


def _is_pow2(n: int) -> bool:
    return n >= 1 and (n & (n - 1)) == 0


# ---------------------------------------------------------------------------
# Sinkhorn-Knopp
# ---------------------------------------------------------------------------

class _SinkhornFn(torch.autograd.Function):
    """Sinkhorn-Knopp on (..., n, n): kernel forward, backward by recompute.

    Reference: ``model/mhc_fused.py:96-137``.
    """

    @staticmethod
    def forward(ctx, M, iters, eps):
        nat.require_cuda(M)
        n = M.shape[-1]
        assert M.shape[-2] == n, f"last two dims must match, got {tuple(M.shape)}"
        mc = M.contiguous()
        y = torch.empty_like(mc)
        batch = mc.numel() // (n * n) if n else 0
        code = nat.dtype_code(M.dtype)
        nat.call("mhc_sinkhorn_fwd", nat.ptr(mc), code, nat.ptr(y), code, batch, n, int(iters),
                 float(eps), nat.stream_of(M))
        ctx.save_for_backward(mc)
        ctx.iters, ctx.eps = int(iters), float(eps)
        return y

    @staticmethod
    def backward(ctx, dy):
        (mc,) = ctx.saved_tensors
        n = mc.shape[-1]
        dyc = dy.contiguous()
        dm = torch.empty_like(mc)
        nat.call("mhc_sinkhorn_bwd", nat.ptr(mc), nat.dtype_code(mc.dtype), nat.ptr(dyc),
                 nat.dtype_code(dy.dtype), nat.ptr(dm), nat.dtype_code(mc.dtype),
                 mc.numel() // (n * n), n, ctx.iters, ctx.eps, nat.stream_of(mc))
        return dm, None, None


@torch.amp.autocast("cuda", enabled=False)
def sinkhorn_normalize(M: torch.Tensor, iters: int = 10, eps: float = 1e-6) -> torch.Tensor:
    """(..., n, n) logits -> doubly-stochastic matrices (``model/mhc_fused.py:140-154``).

    softmax(-1) + eps, one column normalisation, then iters-1 alternating
    row / column normalisations, each dividing by (sum + eps); fp32 math.
    """
    return _SinkhornFn.apply(M, iters, eps)


# ---------------------------------------------------------------------------
# shared host helpers
# ---------------------------------------------------------------------------

def _params(phi, *rest):
    """Parameters in phi's dtype, contiguous (the kernels read one param dtype)."""
    pdt = phi.dtype
    return [phi.contiguous()] + [r.detach().to(pdt).contiguous() if r.dtype != pdt else r.contiguous()
                                 for r in rest]


def _grads_like(tensors):
    return [torch.empty_like(t) for t in tensors]


def _pre_fwd(x2d, ps, with_res, apply_sk, iters, post_mult, pre_eps, rms_eps, sk_eps, n, c,
             coef_dtype, want_h_pre):
    t = x2d.shape[0]
    dev = x2d.device
    fd = 2 * n + (n * n if with_res else 0)
    z = torch.empty(t, c, dtype=x2d.dtype, device=dev)
    h_pre = torch.empty(t, n, dtype=coef_dtype, device=dev) if want_h_pre else None
    h_post = torch.empty(t, n, dtype=coef_dtype, device=dev)
    h_res = torch.empty(t, n, n, dtype=coef_dtype, device=dev) if with_res else None
    inv_rms = torch.empty(t, dtype=torch.float32, device=dev)
    mixes = torch.empty(t, fd, dtype=torch.float32, device=dev)
    ws = nat.workspace(nat.lib().mhc_pre_fwd_workspace(t, n, c, with_res), dev)
    phi, a_pre, b_pre, a_post, b_post = ps[:5]
    a_res, b_res = (ps[5], ps[6]) if with_res else (None, None)
    nat.call("mhc_pre_fwd", nat.ptr(x2d), nat.dtype_code(x2d.dtype), t, n, c, nat.ptr(phi),
             nat.ptr(a_pre), nat.ptr(b_pre), nat.ptr(a_post), nat.ptr(b_post), nat.ptr(a_res),
             nat.ptr(b_res), nat.dtype_code(phi.dtype), int(with_res), int(apply_sk), int(iters),
             float(post_mult), float(pre_eps), float(rms_eps), float(sk_eps), nat.ptr(z),
             nat.ptr(h_pre), nat.ptr(h_post), nat.ptr(h_res), nat.dtype_code(coef_dtype),
             nat.ptr(inv_rms), nat.ptr(mixes), nat.ptr(ws), ws.numel(), nat.stream_of(x2d))
    return z, h_pre, h_post, h_res, inv_rms, mixes


def _pre_bwd(x2d, ps, with_res, apply_sk, iters, post_mult, pre_eps, rms_eps, sk_eps, n, c,
             inv_rms, mixes, dz, dh_pre, dh_post, dh_res, coef_dtype, dx_add):
    t = x2d.shape[0]
    dev = x2d.device
    dx = torch.empty_like(x2d)
    gps = _grads_like(ps)
    phi = ps[0]
    a_res, b_res = (ps[5], ps[6]) if with_res else (None, None)
    g_res = (gps[5], gps[6]) if with_res else (None, None)
    ws = nat.workspace(nat.lib().mhc_pre_bwd_workspace(t, n, c, int(with_res), int(apply_sk), int(iters)), dev)
    nat.call("mhc_pre_bwd", nat.ptr(x2d), nat.dtype_code(x2d.dtype), t, n, c, nat.ptr(phi),
             nat.ptr(ps[1]), nat.ptr(ps[2]), nat.ptr(ps[3]), nat.ptr(ps[4]), nat.ptr(a_res),
             nat.ptr(b_res), nat.dtype_code(phi.dtype), int(with_res), int(apply_sk), int(iters),
             float(post_mult), float(pre_eps), float(rms_eps), float(sk_eps), nat.ptr(inv_rms),
             nat.ptr(mixes), nat.ptr(dz), nat.ptr(dh_pre), nat.ptr(dh_post), nat.ptr(dh_res),
             nat.dtype_code(coef_dtype), nat.ptr(dx_add), nat.ptr(dx), nat.ptr(gps[0]),
             nat.ptr(gps[1]), nat.ptr(gps[2]), nat.ptr(gps[3]), nat.ptr(gps[4]),
             nat.ptr(g_res[0]), nat.ptr(g_res[1]), nat.ptr(ws), ws.numel(), nat.stream_of(x2d))
    return dx, gps


def _contig_or_none(g, shape, dtype):
    if g is None:
        return None
    return g.contiguous().view(*shape).to(dtype)


# ---------------------------------------------------------------------------
# Reference-API autograd Functions
# ---------------------------------------------------------------------------

class _PrePhaseFullFn(torch.autograd.Function):
    """PRE phase: (sublayer_in, h_pre, h_post, h_res_raw), all in x dtype.

    Same ``apply`` arguments as ``model/mhc_fused.py:571-717``:
    (x_flat, w_phi, alpha_pre, bias_pre, alpha_post, bias_post, alpha_res,
    bias_res, post_mult, pre_eps, rms_eps, n, c).  h_res_raw is the affine
    H_res logit (Sinkhorn is applied separately by ``sinkhorn_normalize``).
    """

    @staticmethod
    def forward(ctx, x_flat, w_phi, alpha_pre, bias_pre, alpha_post, bias_post,
                alpha_res, bias_res, post_mult, pre_eps, rms_eps, n, c):
        nat.require_cuda(x_flat, w_phi)
        b, l, nc = x_flat.shape
        fd = 2 * n + n * n
        assert nc == n * c and w_phi.shape == (nc, fd)
        x2d = x_flat.contiguous().view(b * l, nc)
        ps = _params(w_phi, alpha_pre, bias_pre, alpha_post, bias_post, alpha_res, bias_res)
        z, h_pre, h_post, h_res_raw, inv_rms, mixes = _pre_fwd(
            x2d, ps, True, False, 0, post_mult, pre_eps, rms_eps, 0.0, n, c, x_flat.dtype, True)
        ctx.save_for_backward(x2d, *ps, inv_rms, mixes)
        ctx.meta = (b, l, n, c, float(post_mult), float(pre_eps), float(rms_eps))
        ctx.pdtypes = [p.dtype for p in (w_phi, alpha_pre, bias_pre, alpha_post, bias_post, alpha_res, bias_res)]
        return (z.view(b, l, c), h_pre.view(b, l, n), h_post.view(b, l, n), h_res_raw.view(b, l, n, n))

    @staticmethod
    def backward(ctx, g_sub, g_h_pre, g_h_post, g_h_res_raw):
        saved = ctx.saved_tensors
        x2d, ps, inv_rms, mixes = saved[0], list(saved[1:8]), saved[8], saved[9]
        b, l, n, c, post_mult, pre_eps, rms_eps = ctx.meta
        t = b * l
        dt = x2d.dtype
        dz = _contig_or_none(g_sub, (t, c), dt)
        if dz is None:
            dz = torch.zeros(t, c, dtype=dt, device=x2d.device)
        dx, gps = _pre_bwd(x2d, ps, True, False, 0, post_mult, pre_eps, rms_eps, 0.0, n, c,
                           inv_rms, mixes, dz, _contig_or_none(g_h_pre, (t, n), dt),
                           _contig_or_none(g_h_post, (t, n), dt),
                           _contig_or_none(g_h_res_raw, (t, n * n), dt), dt, None)
        gps = [g.to(pd) for g, pd in zip(gps, ctx.pdtypes)]
        return (dx.view(b, l, n * c), *gps, None, None, None, None, None)


class _PostPhaseFullFn(torch.autograd.Function):
    """POST phase: out = H_res x + H_post (x) f (``model/mhc_fused.py:720-772``).

    ``apply`` arguments: (x_flat, h_res, h_post, f_out, n, c).
    """

    @staticmethod
    def forward(ctx, x_flat, h_res, h_post, f_out, n, c):
        nat.require_cuda(x_flat, h_res, h_post, f_out)
        b, l, nc = x_flat.shape
        t = b * l
        xc = x_flat.contiguous().view(t, nc)
        hr = h_res.contiguous().view(t, n, n)
        hp = h_post.contiguous().view(t, n)
        fc = f_out.contiguous().view(t, c)
        out = torch.empty_like(xc)
        nat.call("mhc_post_fwd", nat.ptr(xc), nat.dtype_code(xc.dtype), nat.ptr(hr),
                 nat.dtype_code(hr.dtype), nat.ptr(hp), nat.dtype_code(hp.dtype), nat.ptr(fc),
                 nat.dtype_code(fc.dtype), nat.ptr(out), t, n, c, 0, 0, 0.0, None, nat.stream_of(xc))
        ctx.save_for_backward(xc, hr, hp, fc)
        ctx.meta = (b, l, n, c)
        return out.view(b, l, nc)

    @staticmethod
    def backward(ctx, g):
        xc, hr, hp, fc = ctx.saved_tensors
        b, l, n, c = ctx.meta
        t = b * l
        gc = g.contiguous().view(t, n * c)
        dx = torch.empty_like(xc)
        dhr = torch.empty_like(hr)
        dhp = torch.empty_like(hp)
        df = torch.empty_like(fc)
        nat.call("mhc_post_bwd", nat.ptr(gc), nat.ptr(xc), nat.dtype_code(xc.dtype), nat.ptr(hr),
                 nat.dtype_code(hr.dtype), nat.ptr(hp), nat.dtype_code(hp.dtype), nat.ptr(fc),
                 nat.dtype_code(fc.dtype), nat.ptr(dx), nat.ptr(dhr), nat.ptr(dhp), nat.ptr(df),
                 t, n, c, nat.stream_of(xc))
        return (dx.view(b, l, n * c), dhr.view(b, l, n, n), dhp.view(b, l, n), df.view(b, l, c),
                None, None)


# ---------------------------------------------------------------------------
# Module-internal fused pair (coefficients + Sinkhorn in one kernel; the
# residual gradient of the merge is summed inside the pre backward)
# ---------------------------------------------------------------------------

class _GradLink:
    """Carries the merge kernel's residual gradient to the pre backward."""
    __slots__ = ("dx_post",)

    def __init__(self):
        self.dx_post = None


class _MHCPreFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_flat, w_phi, alpha_pre, bias_pre, alpha_post, bias_post, alpha_res, bias_res,
                link, with_res, iters, post_mult, pre_eps, rms_eps, sk_eps, n, c):
        nat.require_cuda(x_flat, w_phi)
        b, l, nc = x_flat.shape
        assert nc == n * c
        x2d = x_flat.contiguous().view(b * l, nc)
        raw = [w_phi, alpha_pre, bias_pre, alpha_post, bias_post] + ([alpha_res, bias_res] if with_res else [])
        ps = _params(*raw)
        # the coefficient kernel applies Sinkhorn-Knopp itself (fp32 H_res out);
        # backward differentiates it by recompute
        z, _, h_post, h_res, inv_rms, mixes = _pre_fwd(
            x2d, ps, with_res, with_res, iters, post_mult, pre_eps, rms_eps, sk_eps, n, c,
            torch.float32, False)
        ctx.save_for_backward(x2d, inv_rms, mixes, *ps)
        ctx.meta = (b, l, n, c, bool(with_res), int(iters), float(post_mult), float(pre_eps),
                    float(rms_eps), float(sk_eps))
        ctx.link = link
        ctx.pdtypes = [p.dtype for p in raw]
        if with_res:
            return z.view(b, l, c), h_post, h_res
        return z.view(b, l, c), h_post, h_post.new_empty(0)

    @staticmethod
    def backward(ctx, g_z, g_h_post, g_h_res):
        saved = ctx.saved_tensors
        x2d, inv_rms, mixes, ps = saved[0], saved[1], saved[2], list(saved[3:])
        b, l, n, c, with_res, iters, post_mult, pre_eps, rms_eps, sk_eps = ctx.meta
        t = b * l
        dz = g_z.contiguous().view(t, c) if g_z is not None else torch.zeros(t, c, dtype=x2d.dtype, device=x2d.device)
        if dz.dtype != x2d.dtype:
            dz = dz.to(x2d.dtype)
        dh_post = g_h_post.contiguous() if g_h_post is not None else None
        dh_res = g_h_res.contiguous() if (with_res and g_h_res is not None) else None
        dx_add = ctx.link.dx_post
        ctx.link.dx_post = None
        dx, gps = _pre_bwd(x2d, ps, with_res, with_res, iters, post_mult, pre_eps, rms_eps, sk_eps,
                           n, c, inv_rms, mixes, dz, None, dh_post, dh_res, torch.float32, dx_add)
        gps = [g.to(pd) for g, pd in zip(gps, ctx.pdtypes)]
        if not with_res:
            gps += [None, None]
        return (dx.view(b, l, n * c), *gps, None, None, None, None, None, None, None, None, None)


class _MHCPostFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_flat, h_res, h_post, f_out, link, with_res, iters, sk_eps, n, c):
        nat.require_cuda(x_flat, h_post, f_out)
        b, l, nc = x_flat.shape
        t = b * l
        xc = x_flat.contiguous().view(t, nc)
        fc = f_out.contiguous().view(t, c)
        out = torch.empty_like(xc)
        hr = h_res if with_res else None
        nat.call("mhc_post_fwd", nat.ptr(xc), nat.dtype_code(xc.dtype), nat.ptr(hr), nat.F32,
                 nat.ptr(h_post), nat.F32, nat.ptr(fc), nat.dtype_code(fc.dtype), nat.ptr(out),
                 t, n, c, 0, 0, 0.0, None, nat.stream_of(xc))
        ctx.save_for_backward(xc, h_res if with_res else h_post.new_empty(0), h_post, fc)
        ctx.meta = (b, l, n, c, bool(with_res))
        ctx.link = link
        return out.view(b, l, nc)

    @staticmethod
    def backward(ctx, g):
        xc, hr, hp, fc = ctx.saved_tensors
        b, l, n, c, with_res = ctx.meta
        t = b * l
        gc = g.contiguous().view(t, n * c)
        if gc.dtype != xc.dtype:
            gc = gc.to(xc.dtype)
        dhp = torch.empty_like(hp)
        df = torch.empty_like(fc)
        if with_res:
            dx = torch.empty_like(xc)
            dhr = torch.empty_like(hr)
            nat.call("mhc_post_bwd", nat.ptr(gc), nat.ptr(xc), nat.dtype_code(xc.dtype), nat.ptr(hr),
                     nat.F32, nat.ptr(hp), nat.F32, nat.ptr(fc), nat.dtype_code(fc.dtype), nat.ptr(dx),
                     nat.ptr(dhr), nat.ptr(dhp), nat.ptr(df), t, n, c, nat.stream_of(xc))
            ctx.link.dx_post = dx
        else:
            dhr = None
            nat.call("mhc_post_bwd", nat.ptr(gc), nat.ptr(xc), nat.dtype_code(xc.dtype), None,
                     nat.F32, nat.ptr(hp), nat.F32, nat.ptr(fc), nat.dtype_code(fc.dtype), None,
                     None, nat.ptr(dhp), nat.ptr(df), t, n, c, nat.stream_of(xc))
            ctx.link.dx_post = gc  # H_res = I: the residual gradient is g itself
        return None, dhr, dhp, df.view(b, l, c), None, None, None, None, None, None


def raise_no_cpu_path(cls_name: str):
    raise RuntimeError(
        f"{cls_name}._forward_ref: this B200 build has no CPU path (all math runs in the sm_100a "
        f"kernels).  Load the state_dict into the reference module for a CPU run; the parameter "
        f"names, shapes and dtypes are identical.")


def mhc_connection(x_flat, sublayer_fn, phi, alpha_pre, bias_pre, alpha_post, bias_post,
                   alpha_res, bias_res, *, n, c, sinkhorn_iters, post_mult, eps, pre_eps,
                   sinkhorn_eps, with_res=True):
    """One mHC sublayer update x' = H_res x + H_post (x) F(H_pre x) on the kernels."""
    link = _GradLink()
    z, h_post, h_res = _MHCPreFn.apply(x_flat, phi, alpha_pre, bias_pre, alpha_post, bias_post,
                                        alpha_res, bias_res, link, with_res, sinkhorn_iters,
                                        post_mult, pre_eps, eps, sinkhorn_eps, n, c)
    f_out = sublayer_fn(z)
    return _MHCPostFn.apply(x_flat, h_res, h_post, f_out, link, with_res, sinkhorn_iters,
                            sinkhorn_eps, n, c)


class MHCConnection_Fused(nn.Module):
    """Full mHC wrapper of one sublayer (H_pre, H_post, H_res all dynamic).

    Reference: ``model/mhc_fused.py:775-864`` — same constructor, parameters
    (``phi_weight`` (n*dim, 2n+n^2) Kaiming-uniform, ``alpha_pre/post/res``
    0-dim = alpha_init, ``bias_pre/post`` zeros, ``bias_res`` = I) and
    ``forward(x_flat, sublayer_fn)``.
    """

    def __init__(self, n: int, dim: int, alpha_init: float = 0.01,
                 sinkhorn_iters: int = 10, post_mult_value: float = 2.0,
                 eps: float = 1e-6, pre_eps: float = 1e-6, sinkhorn_eps: float = 1e-6):
        super().__init__()
        assert _is_pow2(n) and n <= 16, f"n must be in {{1,2,4,8,16}}, got {n}"
        assert post_mult_value > 1.0
        self.n = n
        self.dim = dim
        self.nC = n * dim
        self.N2 = n * n
        self.fused_dim = 2 * n + self.N2
        self.sinkhorn_iters = sinkhorn_iters
        self.post_mult_value = post_mult_value
        self.pre_eps = pre_eps
        self.sinkhorn_eps = sinkhorn_eps
        self.eps = eps
        self.phi_weight = nn.Parameter(torch.empty(self.nC, self.fused_dim))
        nn.init.kaiming_uniform_(self.phi_weight, a=math.sqrt(5))
        self.alpha_pre = nn.Parameter(torch.tensor(alpha_init))
        self.bias_pre = nn.Parameter(torch.zeros(n))
        self.alpha_post = nn.Parameter(torch.tensor(alpha_init))
        self.bias_post = nn.Parameter(torch.zeros(n))
        self.alpha_res = nn.Parameter(torch.tensor(alpha_init))
        self.bias_res = nn.Parameter(torch.eye(n))

    def extra_repr(self) -> str:
        return (f"n={self.n}, dim={self.dim}, fused_dim={self.fused_dim}, "
                f"sinkhorn_iters={self.sinkhorn_iters}, post_mult_value={self.post_mult_value}, "
                f"backend=sm_100a")

    def forward(self, x_flat: torch.Tensor, sublayer_fn) -> torch.Tensor:
        return mhc_connection(x_flat, sublayer_fn, self.phi_weight, self.alpha_pre, self.bias_pre,
                              self.alpha_post, self.bias_post, self.alpha_res, self.bias_res,
                              n=self.n, c=self.dim, sinkhorn_iters=self.sinkhorn_iters,
                              post_mult=self.post_mult_value, eps=self.eps, pre_eps=self.pre_eps,
                              sinkhorn_eps=self.sinkhorn_eps, with_res=True)

    def _forward_ref(self, x_flat: torch.Tensor, sublayer_fn) -> torch.Tensor:
        """The reference's pure-PyTorch path (``model/mhc_fused.py:836-864``)
        is not part of this build, which has no CPU path: the name is kept so
        that callers get this explanation instead of an AttributeError.  For a
        CPU run, load the same state_dict into the reference module."""
        raise_no_cpu_path(type(self).__name__)
