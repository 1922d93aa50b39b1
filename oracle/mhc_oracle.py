"""CPU oracle for the mHC (manifold-constrained hyper-connection) residual path.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The
product package (``minimind-mhc_b200/model``) never imports it and has no CPU
fallback.

It restates, with plain PyTorch CPU ops, the reference's pure-PyTorch path of
Tshirt-hfk/minimind-mhc.  Each function cites the reference lines it follows
(paths relative to the reference project root).  The rounding points of the
reference are kept on purpose (``x_norm`` is cast back to the activation dtype
before the projection, the Sinkhorn input is upcast to fp32, ``h_res`` is cast
back to the activation dtype), so running the oracle on bf16 tensors reproduces
the reference's bf16 behaviour and running it on fp32 tensors (or on bf16 values
upcast to fp32) gives the fp32 coefficient semantics the CUDA kernels target.

Backward passes are obtained with ``torch.autograd`` through these functions,
which is the same way the reference pins its own fused kernels
(``model/mhc_fused.py:927-943``).

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch


# ---------------------------------------------------------------------------
# Sinkhorn-Knopp projection onto the Birkhoff polytope
# ---------------------------------------------------------------------------

def sinkhorn(logits: torch.Tensor, iters: int, eps: float) -> torch.Tensor:
    """Doubly-stochastic projection of (..., n, n) logits.

    Follows ``model/mhc_fused.py:47-56`` (``_sinkhorn_ref``): a row softmax plus
    ``eps``, one column normalisation, then ``iters - 1`` alternating row and
    column normalisations, each dividing by (sum + eps).
    """
    p = torch.softmax(logits, dim=-1) + eps
    p = p / (p.sum(dim=-2, keepdim=True) + eps)
    for _ in range(iters - 1):
        p = p / (p.sum(dim=-1, keepdim=True) + eps)
        p = p / (p.sum(dim=-2, keepdim=True) + eps)
    return p


# ---------------------------------------------------------------------------
# Shared pieces: unweighted RMSNorm over n*C and the skinny projection
# ---------------------------------------------------------------------------

def rms_project(x_flat: torch.Tensor, phi: torch.Tensor, rms_eps: float):
    """Returns (inv_rms fp32 (..., 1), x_norm in x dtype, mixes = x_norm @ phi).

    ``model/mhc_fused.py:538-541`` / ``:843-846``: RMS statistics in fp32, the
    normalised activations rounded back to the activation dtype, then the
    projection in that dtype.
    """
    xf = x_flat.float()
    inv_rms = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + rms_eps)
    x_norm = (xf * inv_rms).to(x_flat.dtype)
    return inv_rms, x_norm, x_norm @ phi


def _gates(pre_seg, post_seg, a_pre, b_pre, a_post, b_post, post_mult, pre_eps):
    """``model/mhc_fused.py:549-552``: sigmoid gates for H_pre and H_post."""
    h_pre = torch.sigmoid(pre_seg * a_pre + b_pre) + pre_eps
    h_post = torch.sigmoid(post_seg * a_post + b_post) * post_mult
    return h_pre, h_post


def aggregate(x_flat: torch.Tensor, h_pre: torch.Tensor, n: int, c: int) -> torch.Tensor:
    """Sublayer input z = sum_i H_pre[i] * x_i (``model/mhc_fused.py:556-557``)."""
    lead = x_flat.shape[:-1]
    x = x_flat.view(*lead, n, c)
    return (h_pre.unsqueeze(-1) * x).sum(dim=-2)


# ---------------------------------------------------------------------------
# Full mHC layer (H_pre, H_post, H_res)
# ---------------------------------------------------------------------------

def pre_phase_full(x_flat, w_phi, a_pre, b_pre, a_post, b_post, a_res, b_res,
                   post_mult, pre_eps, rms_eps, n, c):
    """PRE phase with the H_res segment, before Sinkhorn.

    Follows ``model/mhc_fused.py:533-559`` (``_pre_phase_full_ref``).  Returns
    (z, h_pre, h_post, h_res_raw, inv_rms fp32 (...,), mixes fp32 (..., FD)).
    """
    assert x_flat.shape[-1] == n * c
    inv_rms, _, mixes = rms_project(x_flat, w_phi, rms_eps)
    assert mixes.shape[-1] == 2 * n + n * n
    h_pre, h_post = _gates(mixes[..., :n], mixes[..., n:2 * n],
                           a_pre, b_pre, a_post, b_post, post_mult, pre_eps)
    res = mixes[..., 2 * n:].reshape(*mixes.shape[:-1], n, n)
    h_res_raw = res * a_res + b_res
    z = aggregate(x_flat, h_pre, n, c)
    return z, h_pre, h_post, h_res_raw, inv_rms.squeeze(-1).float(), mixes.float()


def post_phase_full(x_flat, h_res, h_post, f_out, n, c):
    """x'_i = sum_j H_res[i,j] x_j + H_post[i] f (``model/mhc_fused.py:562-568``)."""
    lead = x_flat.shape[:-1]
    x = x_flat.view(*lead, n, c)
    mixed = torch.einsum('...ij,...jc->...ic', h_res, x)
    out = mixed + h_post.unsqueeze(-1) * f_out.unsqueeze(-2)
    return out.reshape(*lead, n * c)


@dataclass
class FullParams:
    """Parameters of one ``MHCConnection_Fused`` (``model/mhc_fused.py:798-809``)."""
    phi_weight: torch.Tensor   # (n*C, 2n+n^2)
    alpha_pre: torch.Tensor    # 0-dim
    bias_pre: torch.Tensor     # (n,)
    alpha_post: torch.Tensor   # 0-dim
    bias_post: torch.Tensor    # (n,)
    alpha_res: torch.Tensor    # 0-dim
    bias_res: torch.Tensor     # (n, n)

    def tensors(self):
        return [self.phi_weight, self.alpha_pre, self.bias_pre, self.alpha_post,
                self.bias_post, self.alpha_res, self.bias_res]

    NAMES = ("phi_weight", "alpha_pre", "bias_pre", "alpha_post", "bias_post",
             "alpha_res", "bias_res")


def full_forward(x_flat, p: FullParams, sublayer_fn: Callable, n: int, c: int,
                 sinkhorn_iters: int = 10, post_mult: float = 2.0, eps: float = 1e-6,
                 pre_eps: float = 1e-6, sinkhorn_eps: float = 1e-6):
    """The whole full-mHC sublayer update.

    Follows ``MHCConnection_Fused._forward_ref`` (``model/mhc_fused.py:836-864``):
    coefficients from the RMS-normalised streams, Sinkhorn in fp32 on the raw
    H_res logits, sublayer on z, then the res/post merge.
    """
    _, x_norm_unused, mixes = rms_project(x_flat, p.phi_weight, eps)
    del x_norm_unused
    h_pre, h_post = _gates(mixes[..., :n], mixes[..., n:2 * n], p.alpha_pre, p.bias_pre,
                           p.alpha_post, p.bias_post, post_mult, pre_eps)
    res = mixes[..., 2 * n:2 * n + n * n].reshape(*mixes.shape[:-1], n, n)
    h_res_raw = res * p.alpha_res + p.bias_res
    h_res = sinkhorn(h_res_raw.float(), sinkhorn_iters, sinkhorn_eps).to(x_flat.dtype)
    z = aggregate(x_flat, h_pre, n, c)
    f_out = sublayer_fn(z)
    return post_phase_full(x_flat, h_res, h_post, f_out, n, c)


# ---------------------------------------------------------------------------
# mHC without H_res (H_res fixed to the identity)
# ---------------------------------------------------------------------------

def pre_phase_no_hres(x_flat, w_phi, a_pre, b_pre, a_post, b_post,
                      post_mult, pre_eps, rms_eps, n, c):
    """``model/mhc_fused_no_hres.py:364-386`` (``_pre_phase_ref``).

    Returns (z, h_pre, h_post, inv_rms fp32, mixes fp32).
    """
    assert x_flat.shape[-1] == n * c
    inv_rms, _, mixes = rms_project(x_flat, w_phi, rms_eps)
    assert mixes.shape[-1] == 2 * n
    h_pre, h_post = _gates(mixes[..., :n], mixes[..., n:2 * n],
                           a_pre, b_pre, a_post, b_post, post_mult, pre_eps)
    z = aggregate(x_flat, h_pre, n, c)
    return z, h_pre, h_post, inv_rms.squeeze(-1).float(), mixes.float()


def post_phase_no_hres(x_flat, h_post, f_out, n, c):
    """x'_i = x_i + H_post[i] f (``model/mhc_fused_no_hres.py:389-394``)."""
    lead = x_flat.shape[:-1]
    x = x_flat.view(*lead, n, c)
    return (x + h_post.unsqueeze(-1) * f_out.unsqueeze(-2)).reshape(*lead, n * c)


@dataclass
class NoHresParams:
    """Parameters of one ``MHCConnection_FusedNoHres`` (``model/mhc_fused_no_hres.py:606-613``)."""
    phi_weight: torch.Tensor   # (n*C, 2n)
    alpha_pre: torch.Tensor
    bias_pre: torch.Tensor
    alpha_post: torch.Tensor
    bias_post: torch.Tensor

    def tensors(self):
        return [self.phi_weight, self.alpha_pre, self.bias_pre, self.alpha_post, self.bias_post]

    NAMES = ("phi_weight", "alpha_pre", "bias_pre", "alpha_post", "bias_post")


def no_hres_forward(x_flat, p: NoHresParams, sublayer_fn: Callable, n: int, c: int,
                    post_mult: float = 2.0, eps: float = 1e-6, pre_eps: float = 1e-6):
    """``MHCConnection_FusedNoHres._forward_ref`` (``model/mhc_fused_no_hres.py:635-659``)."""
    z, _, h_post, _, _ = pre_phase_no_hres(x_flat, p.phi_weight, p.alpha_pre, p.bias_pre,
                                           p.alpha_post, p.bias_post, post_mult, pre_eps,
                                           eps, n, c)
    return post_phase_no_hres(x_flat, h_post, sublayer_fn(z), n, c)


# ---------------------------------------------------------------------------
# Model entry / exit: StreamExpand and MHCHead
# ---------------------------------------------------------------------------

def stream_expand(x: torch.Tensor, n: int) -> torch.Tensor:
    """(B, L, C) -> (B, L, n*C) by copying the stream n times (``model/mhc_common.py:115-119``)."""
    if n == 1:
        return x
    b, l, d = x.shape
    return x.unsqueeze(-2).expand(b, l, n, d).reshape(b, l, n * d)


def mhc_head(x_flat, w_phi, alpha, bias, pre_eps, rms_eps, n, c):
    """Exit reduction out = sum_i (sigmoid(alpha * x_norm @ phi + bias) + eps)_i x_i.

    ``model/mhc_common.py:298-308`` (``_mhc_head_ref``); for n == 1 the head is a
    plain unweighted RMSNorm (``model/mhc_common.py:438-442``).
    """
    lead = x_flat.shape[:-1]
    if n == 1:
        xf = x_flat.float()
        inv_rms = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + rms_eps)
        return (xf * inv_rms).to(x_flat.dtype).view(*lead, c)
    _, _, mix_raw = rms_project(x_flat, w_phi, rms_eps)
    mix = torch.sigmoid(mix_raw * alpha + bias) + pre_eps
    return aggregate(x_flat, mix, n, c)


# ---------------------------------------------------------------------------
# Seeded synthetic inputs (the shapes and draws of the benchmark configs)
# ---------------------------------------------------------------------------

def make_full_params(n: int, c: int, *, init: str = "bench", dtype=torch.float32,
                     generator: Optional[torch.Generator] = None) -> FullParams:
    """Parameters for a full mHC layer.

    ``init="bench"``: phi ~ N(0, 0.02), all alpha = 0.01, all biases 0 (the
    draws the benchmark configs name).  ``init="module"``: the module's own
    constructor defaults (Kaiming-uniform phi, bias_res = I;
    ``model/mhc_fused.py:798-809``).
    """
    fd = 2 * n + n * n
    if init == "bench":
        phi = torch.randn(n * c, fd, generator=generator) * 0.02
        b_res = torch.zeros(n, n)
    elif init == "module":
        phi = torch.empty(n * c, fd)
        bound = 1.0 / math.sqrt(fd)  # kaiming_uniform_(a=sqrt(5)) on (nC, FD): fan_in = FD
        phi.uniform_(-bound, bound, generator=generator)
        b_res = torch.eye(n)
    else:
        raise ValueError(init)
    p = FullParams(phi, torch.tensor(0.01), torch.zeros(n), torch.tensor(0.01), torch.zeros(n),
                   torch.tensor(0.01), b_res)
    return FullParams(*[t.to(dtype) for t in p.tensors()])


def make_no_hres_params(n: int, c: int, *, dtype=torch.float32,
                        generator: Optional[torch.Generator] = None) -> NoHresParams:
    phi = torch.randn(n * c, 2 * n, generator=generator) * 0.02
    p = NoHresParams(phi, torch.tensor(0.01), torch.zeros(n), torch.tensor(0.01), torch.zeros(n))
    return NoHresParams(*[t.to(dtype) for t in p.tensors()])


def grads(outputs, inputs, grad_outputs):
    """Autograd helper: gradients of sum(outputs * grad_outputs) w.r.t. inputs."""
    outs = [o for o in outputs]
    gos = [g for g in grad_outputs]
    return torch.autograd.grad(outs, inputs, gos, allow_unused=True)
