"""mHC sublayer connection with H_res fixed to the identity, on B200.

Drop-in for the reference's ``model/mhc_fused_no_hres.py``:
``MHCConnection_FusedNoHres`` (same constructor, parameters and
``forward(x_flat, sublayer_fn)``) and the autograd Functions ``_PrePhaseFn``
and ``_PostPhaseFn`` with the reference's ``apply`` argument orders.  The
kernels are the full layer's with the H_res segment compiled out
(projection width 2n, no Sinkhorn, merge x' = x + H_post (x) F).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _native as nat
from .mhc_fused import _contig_or_none, _params, _pre_bwd, _pre_fwd, mhc_connection, raise_no_cpu_path


def _is_pow2(n: int) -> bool:
    return n >= 1 and (n & (n - 1)) == 0


class _PrePhaseFn(torch.autograd.Function):
    """PRE phase -> (sublayer_in, h_pre, h_post) in x dtype.

    ``apply`` arguments as ``model/mhc_fused_no_hres.py:397-529``:
    (x_flat, w_phi, alpha_pre, bias_pre, alpha_post, bias_post, post_mult,
    pre_eps, rms_eps, n, c).
    """

    @staticmethod
    def forward(ctx, x_flat, w_phi, alpha_pre, bias_pre, alpha_post, bias_post,
                post_mult, pre_eps, rms_eps, n, c):
        nat.require_cuda(x_flat, w_phi)
        assert x_flat.dim() == 3
        b, l, nc = x_flat.shape
        assert nc == n * c and w_phi.shape == (nc, 2 * n)
        x2d = x_flat.contiguous().view(b * l, nc)
        ps = _params(w_phi, alpha_pre, bias_pre, alpha_post, bias_post)
        z, h_pre, h_post, _, inv_rms, mixes = _pre_fwd(
            x2d, ps, False, False, 0, post_mult, pre_eps, rms_eps, 0.0, n, c, x_flat.dtype, True)
        ctx.save_for_backward(x2d, *ps, inv_rms, mixes)
        ctx.meta = (b, l, n, c, float(post_mult), float(pre_eps), float(rms_eps))
        ctx.pdtypes = [p.dtype for p in (w_phi, alpha_pre, bias_pre, alpha_post, bias_post)]
        return z.view(b, l, c), h_pre.view(b, l, n), h_post.view(b, l, n)

    @staticmethod
    def backward(ctx, g_sub, g_h_pre, g_h_post):
        saved = ctx.saved_tensors
        x2d, ps, inv_rms, mixes = saved[0], list(saved[1:6]), saved[6], saved[7]
        b, l, n, c, post_mult, pre_eps, rms_eps = ctx.meta
        t = b * l
        dt = x2d.dtype
        dz = _contig_or_none(g_sub, (t, c), dt)
        if dz is None:
            dz = torch.zeros(t, c, dtype=dt, device=x2d.device)
        dx, gps = _pre_bwd(x2d, ps, False, False, 0, post_mult, pre_eps, rms_eps, 0.0, n, c,
                           inv_rms, mixes, dz, _contig_or_none(g_h_pre, (t, n), dt),
                           _contig_or_none(g_h_post, (t, n), dt), None, dt, None)
        gps = [g.to(pd) for g, pd in zip(gps, ctx.pdtypes)]
        return (dx.view(b, l, n * c), *gps, None, None, None, None, None)


class _PostPhaseFn(torch.autograd.Function):
    """POST phase: out = x + H_post (x) f (``model/mhc_fused_no_hres.py:532-581``).

    ``apply`` arguments: (x_flat, h_post, f_out, n, c).
    """

    @staticmethod
    def forward(ctx, x_flat, h_post, f_out, n, c):
        nat.require_cuda(x_flat, h_post, f_out)
        b, l, nc = x_flat.shape
        t = b * l
        xc = x_flat.contiguous().view(t, nc)
        hp = h_post.contiguous().view(t, n)
        fc = f_out.contiguous().view(t, c)
        out = torch.empty_like(xc)
        nat.call("mhc_post_fwd", nat.ptr(xc), nat.dtype_code(xc.dtype), None, nat.F32, nat.ptr(hp),
                 nat.dtype_code(hp.dtype), nat.ptr(fc), nat.dtype_code(fc.dtype), nat.ptr(out),
                 t, n, c, 0, 0, 0.0, None, nat.stream_of(xc))
        ctx.save_for_backward(hp, fc)
        ctx.meta = (b, l, n, c, xc.dtype)
        return out.view(b, l, nc)

    @staticmethod
    def backward(ctx, g):
        hp, fc = ctx.saved_tensors
        b, l, n, c, xdt = ctx.meta
        t = b * l
        gc = g.contiguous().view(t, n * c)
        dx = torch.empty_like(gc)
        dhp = torch.empty_like(hp)
        df = torch.empty_like(fc)
        nat.call("mhc_post_bwd", nat.ptr(gc), None, nat.dtype_code(gc.dtype), None, nat.F32,
                 nat.ptr(hp), nat.dtype_code(hp.dtype), nat.ptr(fc), nat.dtype_code(fc.dtype),
                 nat.ptr(dx), None, nat.ptr(dhp), nat.ptr(df), t, n, c, nat.stream_of(gc))
        return dx.view(b, l, n * c), dhp.view(b, l, n), df.view(b, l, c), None, None


class MHCConnection_FusedNoHres(nn.Module):
    """mHC wrapper of one sublayer with H_res = I_n (not learned).

    Reference: ``model/mhc_fused_no_hres.py:584-659`` — same constructor,
    parameters (``phi_weight`` (n*dim, 2n) Kaiming-uniform, ``alpha_pre/post``
    0-dim, ``bias_pre/post`` zeros) and ``forward(x_flat, sublayer_fn)``.
    """

    def __init__(self, n: int, dim: int, alpha_init: float = 0.01,
                 post_mult_value: float = 2.0, eps: float = 1e-6,
                 pre_eps: float = 1e-6):
        super().__init__()
        assert n >= 1 and isinstance(n, int)
        assert _is_pow2(n) and n <= 16, f"n must be in {{1,2,4,8,16}}, got {n}"
        assert post_mult_value > 1.0
        self.n = n
        self.dim = dim
        self.nC = n * dim
        self.fused_dim = 2 * n
        self.post_mult_value = post_mult_value
        self.pre_eps = pre_eps
        self.eps = eps
        self.phi_weight = nn.Parameter(torch.empty(self.nC, self.fused_dim))
        nn.init.kaiming_uniform_(self.phi_weight, a=math.sqrt(5))
        self.alpha_pre = nn.Parameter(torch.tensor(alpha_init))
        self.bias_pre = nn.Parameter(torch.zeros(n))
        self.alpha_post = nn.Parameter(torch.tensor(alpha_init))
        self.bias_post = nn.Parameter(torch.zeros(n))

    def extra_repr(self) -> str:
        return (f"n={self.n}, dim={self.dim}, fused_dim={self.fused_dim}, "
                f"post_mult_value={self.post_mult_value}, backend=sm_100a")

    def forward(self, x_flat: torch.Tensor, sublayer_fn) -> torch.Tensor:
        return mhc_connection(x_flat, sublayer_fn, self.phi_weight, self.alpha_pre, self.bias_pre,
                              self.alpha_post, self.bias_post, None, None, n=self.n, c=self.dim,
                              sinkhorn_iters=0, post_mult=self.post_mult_value, eps=self.eps,
                              pre_eps=self.pre_eps, sinkhorn_eps=0.0, with_res=False)

    def _forward_ref(self, x_flat: torch.Tensor, sublayer_fn) -> torch.Tensor:
        """The reference's pure-PyTorch path (``model/mhc_fused_no_hres.py:635-659``)
        is not part of this build, which has no CPU path: the name is kept so
        that callers get this explanation instead of an AttributeError."""
        raise_no_cpu_path(type(self).__name__)
