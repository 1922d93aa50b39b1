"""The merge of sublayer l fused with the coefficient pass of sublayer l+1
(``mhc_post_pre_fwd``) and the block-level ``mhc_chain`` API.

* The fused kernel's x_out is bit-identical to the merge kernel's output (same
  fp32 operations in the same order, one bf16 rounding); its coefficients
  match the generic kernels run on that x_out to the tolerance of the other
  fused kernels (projection with phi split into bf16 hi + lo, ~2^-17), and
  the oracle (fp32 on the bf16 inputs) to 1e-4.
* y, the sublayer's input RMSNorm of z, matches ``nn.RMSNorm`` applied to the
  z the kernel wrote to one bf16 rounding (the kernel takes the mean of the
  squares over the bf16 z values, as the norm does).
* ``mhc_chain`` over a list of sublayers gives the same output and gradients
  as the drop-in modules called one after the other with the norms in the
  closures (the reference block's structure): to 1e-4 in fp32, and in bf16
  within the modules' own bf16 error against the fp32 result.
"""

import pytest
import torch
import torch.nn as nn

from conftest import max_rel
from oracle import mhc_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
AUTO, GENERIC, FUSED = 0, 1, 4
RAN_POST_PRE = 3


def _lib():
    from model import _native as nat
    return nat, nat.lib()


def _params(n, c, with_res, gen, scale=0.02):
    from model.mhc_fused import _params as prep
    fd = 2 * n + (n * n if with_res else 0)
    phi = torch.randn(n * c, fd, generator=gen) * scale
    ts = [phi, torch.tensor(0.3), torch.randn(n, generator=gen) * 0.1, torch.tensor(0.2),
          torch.randn(n, generator=gen) * 0.1]
    if with_res:
        ts += [torch.tensor(0.25), torch.eye(n) + torch.randn(n, n, generator=gen) * 0.1]
    return prep(*[t.to(DEV) for t in ts]), ts


def _meta(n, c, with_res):
    return (n, c, with_res, 20 if with_res else 0, 2.0, 1e-6, 1e-6, 1e-6 if with_res else 0.0)


def _prev_coefs(t, n, with_res, gen):
    """Merge coefficients of a previous sublayer: H_res doubly stochastic-ish, H_post in (0, 2)."""
    hp = (torch.rand(t, n, generator=gen) * 2.0).to(DEV)
    hr = None
    if with_res:
        hr = O.sinkhorn(torch.randn(t, n, n, generator=gen), 20, 1e-6).to(DEV)
    return hr, hp


def _post_pre(x, hr, hp, f, ps, meta, norm_w, policy):
    nat, L = _lib()
    from model.mhc_block import _post_pre_fwd
    prev = L.mhc_set_path_policy(policy)
    try:
        out = _post_pre_fwd(x, hr, hp, f, ps, meta, norm_w, 1e-5)
        path = L.mhc_last_path()
    finally:
        L.mhc_set_path_policy(prev)
    assert L.mhc_device_error(1) == 0, "the fused kernel reported a timed-out wait"
    return out, path


def _merge_kernel(x, hr, hp, f, n, c):
    nat, _ = _lib()
    out = torch.empty_like(x)
    nat.call("mhc_post_fwd", nat.ptr(x), nat.BF16, nat.ptr(hr), nat.F32, nat.ptr(hp), nat.F32, nat.ptr(f),
             nat.BF16, nat.ptr(out), x.shape[0], n, c, 0, 0, 0.0, None, torch.cuda.current_stream().cuda_stream)
    return out


CASES = [
    # (n, C, T, with_res, merge, norm)
    (4, 768, 4096, True, True, True),       # benchmark shape, reduced T
    (4, 768, 1, True, True, True),          # single token
    (4, 768, 129, False, True, True),       # one full tile + 1, no-H_res
    (4, 768, 4096, True, False, True),      # first sublayer of a chain: no merge
    (4, 768, 1000, True, True, False),      # merge without the norm
    (2, 512, 300, True, True, True),        # 4-CTA clusters, n = 2
    (4, 1024, 1000, False, True, True),     # config 3 width, 8-CTA clusters
    (4, 640, 300, True, True, True),        # 5-CTA clusters (uneven token owners)
    (4, 896, 257, False, True, True),       # 7-CTA clusters
    (2, 768, 515, False, True, False),
    (4, 768, 24 * 128 * 3 + 64, True, True, True),  # several tiles per cluster, a half tile
]


@pytest.mark.parametrize("n,c,t,with_res,merge,norm", CASES)
def test_post_pre_matches_separate_kernels_and_oracle(n, c, t, with_res, merge, norm):
    gen = torch.Generator().manual_seed(n * 1000 + t)
    ps, raw = _params(n, c, with_res, gen)
    meta = _meta(n, c, with_res)
    x = torch.randn(t, n * c, generator=gen).bfloat16().to(DEV)
    f = torch.randn(t, c, generator=gen).bfloat16().to(DEV) if merge else None
    hr, hp = _prev_coefs(t, n, with_res, gen) if merge else (None, None)
    nw = (1.0 + 0.1 * torch.randn(c, generator=gen)).to(DEV) if norm else None
    (xo, z, y, hpo, hro, inv, mix), path = _post_pre(x, hr, hp, f, ps, meta, nw, FUSED)
    assert path == RAN_POST_PRE, "the fused merge + coefficient kernel did not run"
    # the merge: bit-identical to the merge kernel
    src = x
    if merge:
        ref_xo = _merge_kernel(x, hr, hp, f, n, c)
        assert torch.equal(xo, ref_xo)
        src = ref_xo
    # the coefficient pass: the generic kernels on the same stream
    (_, zg, yg, hpg, hrg, invg, mixg), path_g = _post_pre(src, None, None, None, ps, meta, nw, GENERIC)
    assert path_g == 0
    assert max_rel(invg, inv) < 1e-5
    assert max_rel(mixg, mix) < 2e-5
    assert max_rel(hpg, hpo) < 2e-5
    if with_res:
        assert max_rel(hrg, hro) < 2e-5
    assert (zg.float() - z.float()).abs().max().item() <= 2 ** -7 * zg.float().abs().max().item()
    # and the oracle (fp32 on the bf16 stream)
    p = [r.float() for r in raw]
    oinv, _, omix = O.rms_project(src.float().cpu(), p[0], 1e-6)
    assert max_rel(omix, mix) < 1e-4
    assert max_rel(oinv.squeeze(-1), inv) < 1e-4
    if norm:
        # y = RMSNorm(z) as nn.RMSNorm computes it on the kernel's own z
        rms = nn.RMSNorm(c, eps=1e-5).to(DEV)
        with torch.no_grad():
            rms.weight.copy_(nw)
            y_ref = rms(z)
        assert y.dtype == z.dtype
        assert (y.float() - y_ref.float()).abs().max().item() <= 2 ** -7 * y_ref.float().abs().max().item()
        assert (yg.float() - y_ref.float()).abs().max().item() <= 2 ** -7 * y_ref.float().abs().max().item()


def test_post_pre_full_size_repeatable():
    """32768 tokens (the benchmark batch) twice: bit-identical outputs, no
    device error, sampled tokens against the separate kernels."""
    gen = torch.Generator().manual_seed(21)
    n, c, t = 4, 768, 16 * 2048
    ps, _ = _params(n, c, True, gen)
    meta = _meta(n, c, True)
    torch.manual_seed(5)
    x = torch.randn(t, n * c, device=DEV).bfloat16()
    f = torch.randn(t, c, device=DEV).bfloat16()
    hr, hp = _prev_coefs(t, n, True, gen)
    nw = torch.ones(c, device=DEV)
    a, pa = _post_pre(x, hr, hp, f, ps, meta, nw, FUSED)
    b, pb = _post_pre(x, hr, hp, f, ps, meta, nw, FUSED)
    assert pa == pb == RAN_POST_PRE
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    xo, z, y, _, hro, inv, mix = a
    assert torch.equal(xo, _merge_kernel(x, hr, hp, f, n, c))
    idx = torch.randperm(t, generator=gen)[:2048].to(DEV)
    (_, zg, _, _, hrg, invg, mixg), _ = _post_pre(xo[idx].contiguous(), None, None, None, ps, meta, nw, GENERIC)
    assert max_rel(mixg, mix[idx]) < 2e-5
    assert max_rel(hrg, hro[idx]) < 2e-5
    assert (zg.float() - z[idx].float()).abs().max().item() <= 2 ** -7 * zg.float().abs().max().item()


def _blocks(n, c, with_res, L, seed):
    from model.mhc_fused import MHCConnection_Fused
    from model.mhc_fused_no_hres import MHCConnection_FusedNoHres
    torch.manual_seed(seed)
    steps = []
    for _ in range(L):
        conn = (MHCConnection_Fused(n, c, sinkhorn_iters=20) if with_res else MHCConnection_FusedNoHres(n, c)).to(DEV)
        with torch.no_grad():
            conn.alpha_pre.fill_(0.3)
            conn.alpha_post.fill_(0.2)
            conn.phi_weight.mul_(0.5)
        lin = nn.Linear(c, c, bias=False).to(DEV).bfloat16()
        norm = nn.RMSNorm(c, eps=1e-6).to(DEV)
        with torch.no_grad():
            norm.weight.add_(0.1 * torch.randn(c, device=DEV))
        steps.append((conn, lin, norm))
    return steps


def _run_blocks(steps, x0, gref, chain):
    from model.mhc_block import mhc_chain
    x = x0.clone().requires_grad_(True)
    for conn, lin, norm in steps:
        for p in list(conn.parameters()) + list(lin.parameters()) + list(norm.parameters()):
            p.grad = None
    if chain:
        out = mhc_chain(x, steps)
    else:
        out = x
        for conn, lin, norm in steps:
            out = conn(out, lambda z, lin=lin, norm=norm: lin(norm(z)))
    (out.float() * gref).sum().backward()
    grads = [p.grad.detach().float().clone() for conn, lin, norm in steps
             for p in list(conn.parameters()) + list(lin.parameters()) + list(norm.parameters())]
    return out.detach().float(), x.grad.detach().float(), grads


@pytest.mark.parametrize("with_res", [True, False], ids=["full", "nohres"])
def test_chain_matches_modules_forward_and_backward(with_res):
    """Four sublayers (two blocks): mhc_chain vs the drop-in modules called in
    sequence with the norm inside the closure.

    fp32 (both on the generic kernels: the chain's autograd wiring): output,
    input gradient and every parameter gradient agree to 1e-4 relative.
    bf16 (the chain on the fused merge + coefficient kernel, policy
    MHC_PATH_FUSED_POST_PRE): against the fp32
    module run, the chain misses by no more than the bf16 modules do (2x their
    error plus 2e-3 of the largest mHC gradient: gradients that are small sums
    of large cancelling terms are bf16 noise in both)."""
    _, L = _lib()
    n, c, b, l = 4, 768, 2, 512
    steps = _blocks(n, c, with_res, 4, 3)
    torch.manual_seed(4)
    x0 = (torch.randn(b, l, n * c, device=DEV) * 0.5).bfloat16()
    torch.manual_seed(9)
    gref = torch.randn(b, l, n * c, device=DEV)
    prev = L.mhc_set_path_policy(FUSED)  # the chain on the fused merge + coefficient kernel
    try:
        c16 = _run_blocks(steps, x0, gref, True)
    finally:
        L.mhc_set_path_policy(prev)
    assert L.mhc_device_error(1) == 0
    m16 = _run_blocks(steps, x0, gref, False)
    for _, lin, _ in steps:
        lin.float()
    c32 = _run_blocks(steps, x0.float(), gref, True)
    m32 = _run_blocks(steps, x0.float(), gref, False)
    for _, lin, _ in steps:
        lin.bfloat16()
    assert max_rel(m32[0], c32[0]) < 1e-4
    assert max_rel(m32[1], c32[1]) < 1e-4
    for a, bb in zip(m32[2], c32[2]):
        assert (a - bb).abs().max().item() <= 1e-4 * a.abs().max().item() + 1e-6
    big = max(g.abs().max().item() for g in m32[2])
    for key in (0, 1):
        err_c = (c16[key] - m32[key]).abs().max().item()
        err_m = (m16[key] - m32[key]).abs().max().item()
        assert err_c <= 2 * err_m + 1e-3 * m32[key].abs().max().item()
    for gc, gm, gt in zip(c16[2], m16[2], m32[2]):
        err_c = (gc - gt).abs().max().item()
        err_m = (gm - gt).abs().max().item()
        assert err_c <= 2 * err_m + 2e-3 * big


def test_chain_kernel_follows_the_policy():
    """Under MHC_PATH_FUSED_POST_PRE the chain runs the fused kernel; under
    AUTO the merge kernel, the fastest coefficient kernel and the norm kernel
    (measured faster on B200), with the same result to bf16 rounding."""
    from model.mhc_block import mhc_chain
    nat, L = _lib()
    n, c = 4, 768
    steps = _blocks(n, c, True, 2, 5)
    x = torch.randn(1, 300, n * c, device=DEV).bfloat16()
    prev = L.mhc_set_path_policy(FUSED)
    try:
        with torch.no_grad():
            mhc_chain(x, steps[:1])
            assert L.mhc_last_path() == RAN_POST_PRE  # the first pass, no merge
            out_f = mhc_chain(x, steps)
            assert L.mhc_last_path() == RAN_POST_PRE
        L.mhc_set_path_policy(AUTO)
        with torch.no_grad():
            out_a = mhc_chain(x, steps)
            assert L.mhc_last_path() in (1, 2)
    finally:
        L.mhc_set_path_policy(prev)
    assert L.mhc_device_error(1) == 0
    assert (out_f.float() - out_a.float()).abs().max().item() <= 2e-2 * out_a.float().abs().max().item()
