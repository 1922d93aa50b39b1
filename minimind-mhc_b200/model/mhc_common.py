"""mHC model entry / exit on B200: ``StreamExpand`` and ``MHCHead``.

Drop-in for the reference's ``model/mhc_common.py``: same class names,
constructor signatures, parameter names / shapes / initialisation and the same
``_MHCHeadFn.apply`` argument order, computed by the sm_100a kernels of
``libmhc_b200.so`` (C ABI ``mhc_head_fwd`` / ``mhc_head_bwd`` /
``mhc_stream_expand_*``).  CUDA tensors only; there is no CPU path.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _native as nat


def max_sram_bytes(device=None) -> int:
    """Opt-in shared memory per block of the device (bytes).

    Mirrors ``model/mhc_common.py:41-56`` of the reference, which used this to
    guard its Triton tiles; the B200 kernels tile any width, so it is
    informational only.
    """
    if not torch.cuda.is_available():
        return 192 * 1024
    props = torch.cuda.get_device_properties(device)
    return int(getattr(props, "shared_memory_per_block_optin", 227 * 1024))


class _StreamExpandFn(torch.autograd.Function):
    """(B, L, C) -> (B, L, n*C) copy; backward sums the n copies."""

    @staticmethod
    def forward(ctx, x, n):
        nat.require_cuda(x)
        b, l, c = x.shape
        xc = x.contiguous()
        out = torch.empty(b, l, n * c, dtype=x.dtype, device=x.device)
        nat.call("mhc_stream_expand_fwd", nat.ptr(xc), nat.ptr(out), nat.dtype_code(x.dtype),
                 b * l, n, c, nat.stream_of(x))
        ctx.n, ctx.shape = n, (b, l, c)
        return out

    @staticmethod
    def backward(ctx, g):
        b, l, c = ctx.shape
        gc = g.contiguous()
        dx = torch.empty(b, l, c, dtype=g.dtype, device=g.device)
        nat.call("mhc_stream_expand_bwd", nat.ptr(gc), nat.ptr(dx), nat.dtype_code(g.dtype),
                 b * l, ctx.n, c, nat.stream_of(g))
        return dx, None


class StreamExpand(nn.Module):
    """(B, L, D) -> (B, L, n*D): n symmetric copies of the stream (no parameters).

    Reference: ``model/mhc_common.py:104-119``.
    """

    def __init__(self, n: int, dim: int):
        super().__init__()
        self.n = n
        self.dim = dim

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.n == 1:
            return x
        return _StreamExpandFn.apply(x, self.n)


def _param_dtype(*ps):
    return ps[0].dtype


class _MHCHeadFn(torch.autograd.Function):
    """MHCHead forward / backward on the B200 kernels.

    Same ``apply`` arguments as the reference (``model/mhc_common.py:311-400``):
    (x_flat (B,L,n*c), w_phi (n*c, n), alpha (1,), bias (n,), pre_eps, rms_eps, n, c).
    """

    @staticmethod
    def forward(ctx, x_flat, w_phi, alpha, bias, pre_eps, rms_eps, n, c):
        nat.require_cuda(x_flat, w_phi, alpha, bias)
        b, l, nc = x_flat.shape
        assert nc == n * c and w_phi.shape == (nc, n)
        t = b * l
        pdt = w_phi.dtype
        xc = x_flat.contiguous()
        wc = w_phi.contiguous()
        a = alpha.to(pdt).contiguous()
        bb = bias.to(pdt).contiguous()
        out = torch.empty(b, l, c, dtype=x_flat.dtype, device=x_flat.device)
        inv_rms = torch.empty(t, dtype=torch.float32, device=x_flat.device)
        mix_raw = torch.empty(t, n, dtype=torch.float32, device=x_flat.device)
        ws_bytes = nat.lib().mhc_head_fwd_workspace(t, n, c)
        ws = nat.workspace(ws_bytes, x_flat.device)
        nat.call("mhc_head_fwd", nat.ptr(xc), nat.dtype_code(x_flat.dtype), t, n, c, nat.ptr(wc),
                 nat.ptr(a), nat.ptr(bb), nat.dtype_code(pdt), float(pre_eps), float(rms_eps),
                 nat.ptr(out), nat.ptr(inv_rms), nat.ptr(mix_raw), nat.ptr(ws), ws.numel(),
                 nat.stream_of(x_flat))
        ctx.save_for_backward(xc, wc, a, bb, inv_rms, mix_raw)
        ctx.meta = (n, c, float(pre_eps), float(rms_eps), alpha.dtype, bias.dtype)
        return out

    @staticmethod
    def backward(ctx, g):
        xc, wc, a, bb, inv_rms, mix_raw = ctx.saved_tensors
        n, c, pre_eps, rms_eps, a_dt, b_dt = ctx.meta
        b, l, nc = xc.shape
        t = b * l
        gc = g.contiguous()
        dx = torch.empty_like(xc)
        dphi = torch.empty_like(wc)
        da = torch.empty_like(a)
        db = torch.empty_like(bb)
        ws = nat.workspace(nat.lib().mhc_head_bwd_workspace(t, n, c), xc.device)
        nat.call("mhc_head_bwd", nat.ptr(xc), nat.dtype_code(xc.dtype), t, n, c, nat.ptr(wc),
                 nat.ptr(a), nat.ptr(bb), nat.dtype_code(wc.dtype), pre_eps, rms_eps,
                 nat.ptr(inv_rms), nat.ptr(mix_raw), nat.ptr(gc), nat.ptr(dx), nat.ptr(dphi),
                 nat.ptr(da), nat.ptr(db), nat.ptr(ws), ws.numel(), nat.stream_of(xc))
        return dx, dphi, da.to(a_dt), db.to(b_dt), None, None, None, None


class _RMSNormHeadFn(torch.autograd.Function):
    """n == 1 head: unweighted RMSNorm of the single stream (``model/mhc_common.py:438-442``)."""

    @staticmethod
    def forward(ctx, x_flat, rms_eps):
        nat.require_cuda(x_flat)
        b, l, c = x_flat.shape
        xc = x_flat.contiguous()
        out = torch.empty_like(xc)
        inv_rms = torch.empty(b * l, dtype=torch.float32, device=x_flat.device)
        nat.call("mhc_head_fwd", nat.ptr(xc), nat.dtype_code(x_flat.dtype), b * l, 1, c, None, None,
                 None, nat.dtype_code(x_flat.dtype), 0.0, float(rms_eps), nat.ptr(out),
                 nat.ptr(inv_rms), None, None, 0, nat.stream_of(x_flat))
        ctx.save_for_backward(xc, inv_rms)
        return out

    @staticmethod
    def backward(ctx, g):
        xc, inv_rms = ctx.saved_tensors
        b, l, c = xc.shape
        gc = g.contiguous()
        dx = torch.empty_like(xc)
        ws = nat.workspace(256, xc.device)
        nat.call("mhc_head_bwd", nat.ptr(xc), nat.dtype_code(xc.dtype), b * l, 1, c, None, None, None,
                 nat.dtype_code(xc.dtype), 0.0, 0.0, nat.ptr(inv_rms), None, nat.ptr(gc),
                 nat.ptr(dx), None, None, None, nat.ptr(ws), ws.numel(), nat.stream_of(xc))
        return dx, None


class MHCHead(nn.Module):
    """(B, L, n*D) -> (B, L, D): learned sigmoid-weighted reduction of the n streams.

        x_norm = RMSNorm(vec(x))                 (unweighted)
        out    = sum_i (sigmoid(alpha * (x_norm @ phi) + bias) + eps)_i * x_i

    Reference: ``model/mhc_common.py:403-450`` (same parameters: ``phi_weight``
    (n*D, n) Kaiming-uniform, ``bias`` (n,) zeros, ``alpha`` (1,) = alpha_init).
    """

    def __init__(self, n: int, dim: int, alpha_init: float = 0.01,
                 eps: float = 1e-6, pre_eps: float = 1e-6):
        super().__init__()
        assert n >= 1 and (n & (n - 1)) == 0 and n <= 16, f"n must be in {{1,2,4,8,16}}, got {n}"
        self.n = n
        self.dim = dim
        self.nC = n * dim
        self.eps = eps
        self.pre_eps = pre_eps
        self.phi_weight = nn.Parameter(torch.empty(self.nC, n))
        nn.init.kaiming_uniform_(self.phi_weight, a=math.sqrt(5))
        self.bias = nn.Parameter(torch.zeros(n))
        self.alpha = nn.Parameter(torch.full((1,), alpha_init))

    def extra_repr(self) -> str:
        return f"n={self.n}, dim={self.dim}, backend=sm_100a"

    def forward(self, x_flat: torch.Tensor) -> torch.Tensor:
        if self.n == 1:
            return _RMSNormHeadFn.apply(x_flat, self.eps)
        return _MHCHeadFn.apply(x_flat, self.phi_weight, self.alpha, self.bias,
                                self.pre_eps, self.eps, self.n, self.dim)
