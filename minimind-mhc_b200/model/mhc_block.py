"""Block-level API: consecutive mHC sublayers with the merge of each sublayer
fused into the coefficient pass of the next, and each sublayer's input
RMSNorm fused into its pre-aggregate.

    x = mhc_chain(x_flat, [(conn_0, fn_0, norm_0), (conn_1, fn_1, norm_1), ...])

computes what the reference's blocks compute one sublayer at a time
(``model/model_minimind.py:330-339`` inside a block, ``:392-400`` across
blocks)::

    for conn, fn, norm in steps:
        x = conn(x, lambda z: fn(norm(z)))      # norm may be None: fn(z)

``conn`` is an :class:`MHCConnection_Fused` or :class:`MHCConnection_FusedNoHres`
(every step of one chain the same kind, n and dim), ``fn`` the sublayer and
``norm`` an ``nn.RMSNorm`` over ``dim`` (the reference's ``attn_in_norm`` /
``ffn_in_norm``) or ``None``.  The drop-in modules stay as they are; this is
an additional entry point for callers that own the loop over sublayers.

Forward per chain of L sublayers: one coefficient pass (with the norm) for
sublayer 0, then L-1 calls of ``mhc_post_pre_fwd`` (the merge of sublayer l
and the coefficient pass + norm of sublayer l+1 in one sm_100a kernel), then
the merge of the last sublayer.  Backward runs the same kernels as the
drop-in modules (coefficient backward by recompute, merge backward); the
RMSNorm backward recomputes torch's rms_norm on z under autograd.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import _native as nat
from .mhc_fused import MHCConnection_Fused, _GradLink, _MHCPostFn, _params, _pre_bwd
from .mhc_fused_no_hres import MHCConnection_FusedNoHres


def _meta(conn):
    """(n, c, with_res, sinkhorn_iters, post_mult, pre_eps, rms_eps, sinkhorn_eps)"""
    if isinstance(conn, MHCConnection_Fused):
        return (conn.n, conn.dim, True, int(conn.sinkhorn_iters), float(conn.post_mult_value),
                float(conn.pre_eps), float(conn.eps), float(conn.sinkhorn_eps))
    if isinstance(conn, MHCConnection_FusedNoHres):
        return (conn.n, conn.dim, False, 0, float(conn.post_mult_value), float(conn.pre_eps),
                float(conn.eps), 0.0)
    raise TypeError(f"mhc_chain: expected MHCConnection_Fused / MHCConnection_FusedNoHres, got {type(conn)}")


def _raw_params(conn, with_res):
    raw = [conn.phi_weight, conn.alpha_pre, conn.bias_pre, conn.alpha_post, conn.bias_post]
    if with_res:
        raw += [conn.alpha_res, conn.bias_res]
    else:
        raw += [None, None]
    return raw


def _norm_args(norm, c, dtype, device):
    """(weight, eps) of an nn.RMSNorm over c, or (None, 0.0)."""
    if norm is None:
        return None, 0.0
    if not isinstance(norm, nn.RMSNorm):
        raise TypeError(f"mhc_chain: the input norm must be nn.RMSNorm or None, got {type(norm)}")
    if tuple(norm.normalized_shape) != (c,):
        raise ValueError(f"mhc_chain: the input norm is over {tuple(norm.normalized_shape)}, expected ({c},)")
    w = norm.weight if norm.weight is not None else torch.ones(c, device=device)
    eps = norm.eps if norm.eps is not None else torch.finfo(dtype).eps
    return w, float(eps)


def _post_pre_fwd(x2d, hr_prev, hp_prev, f2d, ps, meta, norm_w, norm_eps):
    """One mhc_post_pre_fwd call (no merge when f2d is None)."""
    n, c, with_res, iters, post_mult, pre_eps, rms_eps, sk_eps = meta
    t = x2d.shape[0]
    dev = x2d.device
    fd = 2 * n + (n * n if with_res else 0)
    x_out = torch.empty_like(x2d) if f2d is not None else None
    z = torch.empty(t, c, dtype=x2d.dtype, device=dev)
    y = torch.empty_like(z) if norm_w is not None else None
    h_post = torch.empty(t, n, dtype=torch.float32, device=dev)
    h_res = torch.empty(t, n, n, dtype=torch.float32, device=dev) if with_res else None
    inv_rms = torch.empty(t, dtype=torch.float32, device=dev)
    mixes = torch.empty(t, fd, dtype=torch.float32, device=dev)
    ws = nat.workspace(nat.lib().mhc_post_pre_fwd_workspace(t, n, c, int(with_res)), dev)
    phi, a_pre, b_pre, a_post, b_post = ps[:5]
    a_res, b_res = (ps[5], ps[6]) if with_res else (None, None)
    fdt = nat.dtype_code(f2d.dtype) if f2d is not None else nat.BF16
    wdt = nat.dtype_code(norm_w.dtype) if norm_w is not None else nat.F32
    nat.call("mhc_post_pre_fwd", nat.ptr(x2d), nat.dtype_code(x2d.dtype), nat.ptr(hr_prev), nat.ptr(hp_prev),
             nat.F32, nat.ptr(f2d), fdt, nat.ptr(x_out), t, n, c, nat.ptr(phi), nat.ptr(a_pre), nat.ptr(b_pre),
             nat.ptr(a_post), nat.ptr(b_post), nat.ptr(a_res), nat.ptr(b_res), nat.dtype_code(phi.dtype),
             int(with_res), int(with_res), int(iters), float(post_mult), float(pre_eps), float(rms_eps),
             float(sk_eps), nat.ptr(z), None, nat.ptr(h_post), nat.ptr(h_res), nat.F32, nat.ptr(inv_rms),
             nat.ptr(mixes), nat.ptr(norm_w), wdt, float(norm_eps), nat.ptr(y), nat.ptr(ws), ws.numel(),
             nat.stream_of(x2d))
    return x_out, z, y, h_post, h_res, inv_rms, mixes


def _norm_bwd(g_y, z, w, eps):
    """Gradient of y = z * rsqrt(mean(z^2) + eps) * w w.r.t. z and w: torch's
    rms_norm recomputed under autograd (its fused kernels when z and w share a
    dtype), one forward and one backward pass over z."""
    with torch.enable_grad():
        zz = z.detach().requires_grad_(True)
        ww = w.detach().requires_grad_(True)
        yy = torch.nn.functional.rms_norm(zz, (z.shape[-1],), ww, eps)
        dz, dw = torch.autograd.grad(yy, (zz, ww), g_y.to(yy.dtype))
    return dz, dw


def _dz_total(ctx, g_z, g_y, z, t, c, dtype, device):
    dz = g_z.contiguous().view(t, c) if g_z is not None else None
    dw = None
    if ctx.norm and g_y is not None:
        dzn, dw = _norm_bwd(g_y.contiguous().view(t, c), z, ctx.norm_w, ctx.norm_eps)
        dz = dzn if dz is None else dz + dzn
    if dz is None:
        dz = torch.zeros(t, c, dtype=dtype, device=device)
    return dz.to(dtype), dw


def _pre_side_bwd(ctx, x2d, ps, inv_rms, mixes, dz, g_hpost, g_hres, dx_add):
    n, c, with_res, iters, post_mult, pre_eps, rms_eps, sk_eps = ctx.meta
    dh_post = g_hpost.contiguous() if g_hpost is not None else None
    dh_res = g_hres.contiguous() if (with_res and g_hres is not None) else None
    dx, gps = _pre_bwd(x2d, ps, with_res, with_res, iters, post_mult, pre_eps, rms_eps, sk_eps, n, c,
                       inv_rms, mixes, dz, None, dh_post, dh_res, torch.float32, dx_add)
    gps = [g.to(pd) for g, pd in zip(gps, ctx.pdtypes)]
    if not with_res:
        gps += [None, None]
    return dx, gps


class _ChainPreFn(torch.autograd.Function):
    """Coefficient pass (+ input norm) of the chain's first sublayer."""

    @staticmethod
    def forward(ctx, x_flat, norm_w, phi, a_pre, b_pre, a_post, b_post, a_res, b_res, link, meta, norm_eps):
        nat.require_cuda(x_flat, phi)
        n, c = meta[0], meta[1]
        b, l, nc = x_flat.shape
        assert nc == n * c
        x2d = x_flat.contiguous().view(b * l, nc)
        raw = [phi, a_pre, b_pre, a_post, b_post] + ([a_res, b_res] if meta[2] else [])
        ps = _params(*raw)
        nw = norm_w.detach().contiguous() if norm_w is not None else None
        _, z, y, h_post, h_res, inv_rms, mixes = _post_pre_fwd(x2d, None, None, None, ps, meta, nw, norm_eps)
        ctx.save_for_backward(x2d, z, inv_rms, mixes, *ps)
        ctx.meta, ctx.link, ctx.shape = meta, link, (b, l)
        ctx.norm, ctx.norm_w, ctx.norm_eps = nw is not None, nw, norm_eps
        ctx.norm_w_dtype = norm_w.dtype if norm_w is not None else None
        ctx.pdtypes = [p.dtype for p in raw]
        out_y = y.view(b, l, c) if y is not None else z.new_empty(0)
        return z.view(b, l, c), out_y, h_post, (h_res if h_res is not None else h_post.new_empty(0))

    @staticmethod
    def backward(ctx, g_z, g_y, g_hpost, g_hres):
        saved = ctx.saved_tensors
        x2d, z, inv_rms, mixes, ps = saved[0], saved[1], saved[2], saved[3], list(saved[4:])
        b, l = ctx.shape
        t, c = b * l, ctx.meta[1]
        dz, dw = _dz_total(ctx, g_z, g_y, z, t, c, x2d.dtype, x2d.device)
        dx_add = ctx.link.dx_post
        ctx.link.dx_post = None
        dx, gps = _pre_side_bwd(ctx, x2d, ps, inv_rms, mixes, dz, g_hpost, g_hres, dx_add)
        dnw = dw.to(ctx.norm_w_dtype) if dw is not None else None
        return (dx.view(b, l, -1), dnw, *gps, None, None, None)


class _PostPreFn(torch.autograd.Function):
    """Merge of sublayer l-1 + coefficient pass (+ input norm) of sublayer l."""

    @staticmethod
    def forward(ctx, x_flat, h_res_prev, h_post_prev, f_prev, norm_w, phi, a_pre, b_pre, a_post, b_post,
                a_res, b_res, link_in, link_out, meta, prev_res, norm_eps):
        nat.require_cuda(x_flat, h_post_prev, f_prev, phi)
        n, c = meta[0], meta[1]
        b, l, nc = x_flat.shape
        t = b * l
        x2d = x_flat.contiguous().view(t, nc)
        f2d = f_prev.contiguous().view(t, c)
        hr = h_res_prev.contiguous() if prev_res else None
        hp = h_post_prev.contiguous()
        raw = [phi, a_pre, b_pre, a_post, b_post] + ([a_res, b_res] if meta[2] else [])
        ps = _params(*raw)
        nw = norm_w.detach().contiguous() if norm_w is not None else None
        x_out, z, y, h_post, h_res, inv_rms, mixes = _post_pre_fwd(x2d, hr, hp, f2d, ps, meta, nw, norm_eps)
        ctx.save_for_backward(x2d, hr if hr is not None else hp.new_empty(0), hp, f2d, x_out, z, inv_rms, mixes,
                              *ps)
        ctx.meta, ctx.prev_res, ctx.shape = meta, bool(prev_res), (b, l)
        ctx.link_in, ctx.link_out = link_in, link_out
        ctx.norm, ctx.norm_w, ctx.norm_eps = nw is not None, nw, norm_eps
        ctx.norm_w_dtype = norm_w.dtype if norm_w is not None else None
        ctx.pdtypes = [p.dtype for p in raw]
        out_y = y.view(b, l, c) if y is not None else z.new_empty(0)
        return (x_out.view(b, l, nc), z.view(b, l, c), out_y, h_post,
                h_res if h_res is not None else h_post.new_empty(0))

    @staticmethod
    def backward(ctx, g_xout, g_z, g_y, g_hpost, g_hres):
        saved = ctx.saved_tensors
        x2d, hr, hp, f2d, x_out, z, inv_rms, mixes = saved[:8]
        ps = list(saved[8:])
        b, l = ctx.shape
        n, c = ctx.meta[0], ctx.meta[1]
        t = b * l
        dz, dw = _dz_total(ctx, g_z, g_y, z, t, c, x2d.dtype, x2d.device)
        # gradient of x_out from the next merge (carried by the link), plus any
        # direct use of x_out by the caller
        dx_add = ctx.link_out.dx_post
        ctx.link_out.dx_post = None
        if g_xout is not None:
            g = g_xout.contiguous().view(t, n * c).to(x2d.dtype)
            dx_add = g if dx_add is None else dx_add + g
        dxo, gps = _pre_side_bwd(ctx, x_out, ps, inv_rms, mixes, dz, g_hpost, g_hres, dx_add)
        # backward of the merge that produced x_out
        dhp = torch.empty_like(hp)
        df = torch.empty_like(f2d)
        s = nat.stream_of(x2d)
        if ctx.prev_res:
            dx = torch.empty_like(x2d)
            dhr = torch.empty_like(hr)
            nat.call("mhc_post_bwd", nat.ptr(dxo), nat.ptr(x2d), nat.dtype_code(x2d.dtype), nat.ptr(hr), nat.F32,
                     nat.ptr(hp), nat.F32, nat.ptr(f2d), nat.dtype_code(f2d.dtype), nat.ptr(dx), nat.ptr(dhr),
                     nat.ptr(dhp), nat.ptr(df), t, n, c, s)
        else:
            dx, dhr = dxo, None
            nat.call("mhc_post_bwd", nat.ptr(dxo), nat.ptr(x2d), nat.dtype_code(x2d.dtype), None, nat.F32,
                     nat.ptr(hp), nat.F32, nat.ptr(f2d), nat.dtype_code(f2d.dtype), None, None, nat.ptr(dhp),
                     nat.ptr(df), t, n, c, s)
        ctx.link_in.dx_post = dx
        dnw = dw.to(ctx.norm_w_dtype) if dw is not None else None
        return (None, dhr, dhp, df.view(b, l, c), dnw, *gps, None, None, None, None, None)


def mhc_chain(x_flat: torch.Tensor, steps) -> torch.Tensor:
    """Runs ``x = conn(x, lambda z: fn(norm(z)))`` for every ``(conn, fn, norm)``
    of ``steps`` with the merge of each sublayer fused into the next one's
    coefficient pass and the norm fused into the pre-aggregate."""
    steps = list(steps)
    if not steps:
        return x_flat
    metas = [_meta(conn) for conn, _, _ in steps]
    if any(m[:3] != metas[0][:3] for m in metas):
        raise ValueError("mhc_chain: every step must have the same kind of connection, n and dim")
    n, c, with_res = metas[0][:3]
    iters, sk_eps = metas[0][3], metas[0][7]

    def norm_of(norm):
        return _norm_args(norm, c, x_flat.dtype, x_flat.device)

    link = _GradLink()
    conn, fn, norm = steps[0]
    nw, neps = norm_of(norm)
    z, y, h_post, h_res = _ChainPreFn.apply(x_flat, nw, *_raw_params(conn, with_res), link, metas[0], neps)
    f = fn(y if nw is not None else z)
    x = x_flat
    for (conn, fn, norm), meta in zip(steps[1:], metas[1:]):
        nw, neps = norm_of(norm)
        link_out = _GradLink()
        x, z, y, h_post, h_res = _PostPreFn.apply(x, h_res, h_post, f, nw, *_raw_params(conn, with_res), link,
                                                  link_out, meta, with_res, neps)
        link = link_out
        f = fn(y if nw is not None else z)
    last = metas[-1]
    return _MHCPostFn.apply(x, h_res, h_post, f, link, with_res, last[3], last[7], n, c)
