"""GPU parity against the CPU oracle at benchmark shapes, odd shapes and full size.

Tolerances are the north-star bar, written here:
  * fp32 coefficient math (inv_rms, mixes, H_pre, H_post, H_res):  1e-4 relative
    (max|diff| / max|ref|) against the oracle run in fp32 on the same inputs
    (bf16 activations upcast to fp32);
  * Sinkhorn: every row and column sum of H_res within 1e-5 of 1 at the
    benchmark logits (alpha = 0.01, biases 0);
  * bf16 stream outputs (z, x'): within 1e-2 relative of the oracle, both of the
    fp32-upcast run and of the bf16 run (the reference's own rounding points).
The full-size case (16 x 2048 tokens, C = 768, n = 4) is checked on a random
sample of tokens: tokens are independent, so the oracle can recompute any
subset exactly.
"""

import pytest
import torch
import torch.nn.functional as F

from conftest import assert_close, max_rel
from oracle import mhc_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
COEF_RTOL = 1e-4
SK_TOL = 1e-5
STREAM_RTOL = 1e-2


def _bench_params(n, c, with_res, gen):
    if with_res:
        p = O.make_full_params(n, c, generator=gen)
    else:
        p = O.make_no_hres_params(n, c, generator=gen)
    return p


def _native_pre(x2d, p, with_res, iters, n, c, coef_dtype=torch.float32):
    from model.mhc_fused import _params, _pre_fwd
    raw = p.tensors()
    ps = _params(*[t.to(DEV) for t in raw])
    return _pre_fwd(x2d, ps, with_res, with_res, iters, 2.0, 1e-6, 1e-6, 1e-6, n, c, coef_dtype, True)


def _oracle_coefs(x2d_cpu, p, with_res, iters, n, c):
    xf = x2d_cpu.float()
    inv, _, mixes = O.rms_project(xf, p.phi_weight.float(), 1e-6)
    h_pre = torch.sigmoid(mixes[:, :n] * p.alpha_pre.float() + p.bias_pre.float()) + 1e-6
    h_post = torch.sigmoid(mixes[:, n:2 * n] * p.alpha_post.float() + p.bias_post.float()) * 2.0
    out = dict(inv_rms=inv.squeeze(-1), mixes=mixes, h_pre=h_pre, h_post=h_post)
    if with_res:
        raw = mixes[:, 2 * n:].reshape(-1, n, n) * p.alpha_res.float() + p.bias_res.float()
        out["h_res"] = O.sinkhorn(raw, iters, 1e-6)
    out["z"] = O.aggregate(xf, h_pre, n, c)
    return out


@pytest.mark.parametrize("with_res", [True, False])
def test_config2_shape_coefficients_and_streams(with_res):
    """C = 768, n = 4, bf16 activations, fp32 coefficients, 20 Sinkhorn iterations."""
    gen = torch.Generator().manual_seed(0)
    n, c, t = 4, 768, 4096
    x = torch.randn(t, n * c, generator=gen).bfloat16()
    p = _bench_params(n, c, with_res, gen)
    xd = x.to(DEV)
    z, h_pre, h_post, h_res, inv, mixes = _native_pre(xd, p, with_res, 20, n, c)
    ref = _oracle_coefs(x, p, with_res, 20, n, c)
    assert max_rel(ref["inv_rms"], inv) < COEF_RTOL
    assert max_rel(ref["mixes"], mixes) < COEF_RTOL
    assert max_rel(ref["h_pre"], h_pre) < COEF_RTOL
    assert max_rel(ref["h_post"], h_post) < COEF_RTOL
    if with_res:
        assert max_rel(ref["h_res"], h_res) < COEF_RTOL
        hr = h_res.double()
        assert (hr.sum(-1) - 1).abs().max().item() < SK_TOL
        assert (hr.sum(-2) - 1).abs().max().item() < SK_TOL
    assert max_rel(ref["z"], z) < STREAM_RTOL
    # the reference's bf16 rounding points
    pb = type(p)(*[tt.float() for tt in p.tensors()])
    if with_res:
        zb = O.pre_phase_full(x, pb.phi_weight.bfloat16(), *[tt for tt in pb.tensors()[1:]],
                              2.0, 1e-6, 1e-6, n, c)[0]
    else:
        zb = O.pre_phase_no_hres(x, pb.phi_weight.bfloat16(), *[tt for tt in pb.tensors()[1:]],
                                 2.0, 1e-6, 1e-6, n, c)[0]
    assert max_rel(zb, z) < STREAM_RTOL

    # post / res merge with an MLP-like f
    f = (torch.randn(t, c, generator=gen) * 0.5).bfloat16()
    from model import _native as nat
    out = torch.empty_like(xd)
    fd = f.to(DEV)
    nat.call("mhc_post_fwd", nat.ptr(xd), nat.BF16, nat.ptr(h_res) if with_res else None, nat.F32,
             nat.ptr(h_post), nat.F32, nat.ptr(fd), nat.BF16, nat.ptr(out), t, n, c, 0, 0, 0.0, None,
             torch.cuda.current_stream().cuda_stream)
    if with_res:
        ro = O.post_phase_full(x.float(), ref["h_res"], ref["h_post"], f.float(), n, c)
    else:
        ro = O.post_phase_no_hres(x.float(), ref["h_post"], f.float(), n, c)
    assert max_rel(ro, out) < STREAM_RTOL


SHAPES = [
    # (n, C, T, dtype, with_res)
    (1, 64, 37, torch.float32, True),
    (2, 96, 50, torch.bfloat16, True),
    (4, 100, 33, torch.float32, True),     # C not a multiple of the vector width
    (4, 7, 19, torch.float32, False),
    (4, 64, 1, torch.float16, True),
    (8, 32, 40, torch.float32, True),
    (8, 64, 24, torch.bfloat16, False),
    (16, 8, 12, torch.float32, True),
    (16, 16, 20, torch.float32, False),
    (4, 256, 300, torch.bfloat16, True),
    (4, 768, 257, torch.bfloat16, True),   # config-2 width: fused forward + tensor-core backward
    (4, 1024, 130, torch.bfloat16, False),  # config-3 width
    (2, 512, 129, torch.float16, True),
]


@pytest.mark.parametrize("n,c,t,dtype,with_res", SHAPES)
def test_module_fwd_bwd_vs_oracle(n, c, t, dtype, with_res):
    """Whole sublayer (fused module path, incl. the fused residual-gradient sum)
    against oracle autograd in fp32 on the same (dtype-rounded) inputs."""
    from model.mhc_fused import MHCConnection_Fused
    from model.mhc_fused_no_hres import MHCConnection_FusedNoHres
    torch.manual_seed(n * 1000 + c)
    gen = torch.Generator().manual_seed(n * 7 + c)
    iters = 20
    if with_res:
        mod = MHCConnection_Fused(n, c, sinkhorn_iters=iters)
    else:
        mod = MHCConnection_FusedNoHres(n, c)
    with torch.no_grad():
        for p in mod.parameters():
            p.add_(torch.randn(p.shape, generator=gen) * 0.05)
    w1 = torch.randn(2 * c, c, generator=gen) * (1.0 / c ** 0.5)
    w2 = torch.randn(c, 2 * c, generator=gen) * (1.0 / (2 * c) ** 0.5)
    x = torch.randn(1, t, n * c, generator=gen).to(dtype)
    gout = torch.randn(1, t, n * c, generator=gen).to(dtype)

    # oracle, fp32 on the same rounded inputs
    ps = [p.detach().float().clone().requires_grad_(True) for p in mod.parameters()]
    xo = x.float().clone().requires_grad_(True)
    fo = lambda z: F.silu(z @ w1.t()) @ w2.t()  # noqa: E731
    if with_res:
        yo = O.full_forward(xo, O.FullParams(*ps), fo, n, c, iters)
    else:
        yo = O.no_hres_forward(xo, O.NoHresParams(*ps), fo, n, c)
    go = torch.autograd.grad(yo, [xo] + ps, gout.float())

    # kernels
    modd = mod.to(DEV)
    xd = x.to(DEV).requires_grad_(True)
    w1d, w2d = w1.to(DEV).to(dtype), w2.to(DEV).to(dtype)
    yd = modd(xd, lambda z: F.silu(z @ w1d.t()) @ w2d.t())
    gd = torch.autograd.grad(yd, [xd] + list(modd.parameters()), gout.to(DEV))

    tol = 1e-4 if dtype == torch.float32 else 3e-2
    assert_close("out", yo, yd, tol, tol)
    names = ["x"] + [nm for nm, _ in mod.named_parameters()]
    for nm, a, b in zip(names, go, gd):
        assert_close("grad_" + nm, a, b, tol * 5, tol * 5)


def test_full_size_sampled_tokens():
    """Config 2 at full size (32768 tokens): sampled tokens vs the oracle, and
    the doubly-stochastic property on every token."""
    gen = torch.Generator().manual_seed(2)
    n, c, t = 4, 768, 16 * 2048
    torch.manual_seed(0)
    xd = torch.randn(t, n * c, device=DEV).bfloat16()
    p = _bench_params(n, c, True, gen)
    z, h_pre, h_post, h_res, inv, mixes = _native_pre(xd, p, True, 20, n, c)
    hr = h_res.double()
    assert (hr.sum(-1) - 1).abs().max().item() < SK_TOL
    assert (hr.sum(-2) - 1).abs().max().item() < SK_TOL
    idx = torch.randperm(t, generator=gen)[:512]
    xs = xd[idx.to(DEV)].cpu()
    ref = _oracle_coefs(xs, p, True, 20, n, c)
    sel = idx.to(DEV)
    assert max_rel(ref["h_pre"], h_pre[sel]) < COEF_RTOL
    assert max_rel(ref["h_post"], h_post[sel]) < COEF_RTOL
    assert max_rel(ref["h_res"], h_res[sel]) < COEF_RTOL
    assert max_rel(ref["mixes"], mixes[sel]) < COEF_RTOL
    assert max_rel(ref["z"], z[sel]) < STREAM_RTOL


def test_backward_is_deterministic():
    from model.mhc_fused import MHCConnection_Fused
    torch.manual_seed(3)
    n, c, t = 4, 768, 2048
    mod = MHCConnection_Fused(n, c, sinkhorn_iters=20).to(DEV)
    x = torch.randn(1, t, n * c, device=DEV, dtype=torch.bfloat16)
    g = torch.randn_like(x)
    outs = []
    for _ in range(2):
        xd = x.clone().requires_grad_(True)
        y = mod(xd, lambda z: z * 2.0)
        outs.append(torch.autograd.grad(y, [xd] + list(mod.parameters()), g))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_fused_module_matches_reference_api_composition():
    """The module's fused pair equals the reference-API composition
    _PrePhaseFullFn -> sinkhorn_normalize -> _PostPhaseFullFn (fp32)."""
    from model.mhc_fused import (MHCConnection_Fused, _PostPhaseFullFn, _PrePhaseFullFn,
                                 sinkhorn_normalize)
    torch.manual_seed(4)
    n, c = 4, 128
    mod = MHCConnection_Fused(n, c, sinkhorn_iters=20).to(DEV)
    x = torch.randn(2, 64, n * c, device=DEV, requires_grad=True)
    g = torch.randn_like(x)
    fn = lambda z: torch.tanh(z)  # noqa: E731
    y1 = mod(x, fn)
    g1 = torch.autograd.grad(y1, [x] + list(mod.parameters()), g)
    sub, _, hpost, hraw = _PrePhaseFullFn.apply(x, mod.phi_weight, mod.alpha_pre, mod.bias_pre,
                                                mod.alpha_post, mod.bias_post, mod.alpha_res,
                                                mod.bias_res, 2.0, 1e-6, 1e-6, n, c)
    hres = sinkhorn_normalize(hraw, 20, 1e-6)
    y2 = _PostPhaseFullFn.apply(x, hres, hpost, fn(sub), n, c)
    g2 = torch.autograd.grad(y2, [x] + list(mod.parameters()), g)
    assert_close("out", y2, y1, 1e-5, 1e-5)
    for a, b in zip(g2, g1):
        assert_close("grad", a, b, 1e-4, 1e-4)


def test_cpu_tensors_are_rejected():
    from model.mhc_fused import MHCConnection_Fused
    mod = MHCConnection_Fused(4, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        mod(torch.randn(1, 4, 256), lambda z: z)


@pytest.mark.parametrize("n", [2, 4, 8])
@pytest.mark.parametrize("iters", [1, 2, 3, 4, 5, 7, 10, 20, 21])
def test_sinkhorn_backward_checkpoint_segments(n, iters):
    """Sinkhorn-Knopp backward by recompute (states kept every 4th step for
    n <= 4, then recomputed segment by segment) against fp64 autograd of the
    oracle, at iteration counts that end on full and on partial segments."""
    from model.mhc_fused import sinkhorn_normalize
    gen = torch.Generator().manual_seed(n * 100 + iters)
    m = torch.randn(257, n, n, generator=gen) * 0.7
    dy = torch.randn(257, n, n, generator=gen)
    md = m.to(DEV).requires_grad_(True)
    y = sinkhorn_normalize(md, iters, 1e-6)
    (dm,) = torch.autograd.grad(y, md, dy.to(DEV))
    m64 = m.double().requires_grad_(True)
    y64 = O.sinkhorn(m64, iters, 1e-6)
    (dm64,) = torch.autograd.grad(y64, m64, dy.double())
    assert (y.double().cpu() - y64).abs().max().item() < 2e-6
    err = (dm.double().cpu() - dm64).abs().max().item()
    assert err < 1e-5 + 1e-4 * dm64.abs().max().item(), err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
def test_256k_tokens_sampled(dtype):
    """The top of the config-2 token sweep, T = 262,144 (x is 1.6 GB in bf16 and
    3.2 GB in fp32, so fp32 byte offsets pass 2^31).  bf16 takes the fused
    kernel, fp32 the generic kernels.  Sampled tokens, the last ones included,
    against the oracle; the doubly-stochastic property on every token."""
    gen = torch.Generator().manual_seed(5)
    n, c, t = 4, 768, 262144
    torch.manual_seed(1)
    xd = torch.randn(t, n * c, device=DEV, dtype=dtype)
    p = _bench_params(n, c, True, gen)
    z, h_pre, h_post, h_res, inv, mixes = _native_pre(xd, p, True, 20, n, c)
    hr = h_res.double()
    assert (hr.sum(-1) - 1).abs().max().item() < SK_TOL
    assert (hr.sum(-2) - 1).abs().max().item() < SK_TOL
    idx = torch.cat([torch.randperm(t, generator=gen)[:384], torch.arange(t - 16, t)])
    sel = idx.to(DEV)
    ref = _oracle_coefs(xd[sel].cpu(), p, True, 20, n, c)
    assert max_rel(ref["inv_rms"], inv[sel]) < COEF_RTOL
    assert max_rel(ref["h_pre"], h_pre[sel]) < COEF_RTOL
    assert max_rel(ref["h_post"], h_post[sel]) < COEF_RTOL
    assert max_rel(ref["h_res"], h_res[sel]) < COEF_RTOL
    assert max_rel(ref["mixes"], mixes[sel]) < COEF_RTOL
    assert max_rel(ref["z"], z[sel]) < (STREAM_RTOL if dtype == torch.bfloat16 else COEF_RTOL)


def test_autocast_fp32_stream_module_fwd_bwd():
    """The reference trainers' setting: fp32 weights under bf16 autocast
    (trainer/train_pretrain.py:129-130).  The residual stream stays fp32
    (embedding -> RMSNorm -> StreamExpand, model/model_minimind.py:365,
    384-385) and the sublayer's output is bf16, so the layer sees x fp32 and f
    bf16.  Forward and backward against fp32 oracle autograd, with the
    sublayer's bf16 rounding reproduced on the CPU."""
    from model.mhc_fused import MHCConnection_Fused
    torch.manual_seed(6)
    gen = torch.Generator().manual_seed(6)
    n, c, t = 4, 768, 384
    mod = MHCConnection_Fused(n, c, sinkhorn_iters=20)
    with torch.no_grad():
        for p in mod.parameters():
            p.add_(torch.randn(p.shape, generator=gen) * 0.05)
    w = torch.randn(c, c, generator=gen) / c ** 0.5
    x = torch.randn(1, t, n * c, generator=gen)
    gout = torch.randn(1, t, n * c, generator=gen)

    ps = [p.detach().clone().requires_grad_(True) for p in mod.parameters()]
    xo = x.clone().requires_grad_(True)
    fo = lambda z: F.linear(z.bfloat16(), w.bfloat16()).float()  # noqa: E731  (autocast's casts)
    yo = O.full_forward(xo, O.FullParams(*ps), fo, n, c, 20)
    go = torch.autograd.grad(yo, [xo] + ps, gout)

    modd = mod.to(DEV)
    lin = torch.nn.Linear(c, c, bias=False).to(DEV)
    with torch.no_grad():
        lin.weight.copy_(w)
    xd = x.to(DEV).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        seen = {}

        def fd(z):
            seen["z"] = z.dtype
            f = lin(z)
            seen["f"] = f.dtype
            return f
        yd = modd(xd, fd)
    assert seen == {"z": torch.float32, "f": torch.bfloat16} and yd.dtype == torch.float32
    gd = torch.autograd.grad(yd, [xd] + list(modd.parameters()), gout.to(DEV))
    assert_close("out", yo, yd, 1e-2, 1e-2)
    names = ["x"] + [nm for nm, _ in mod.named_parameters()]
    for nm, a, b in zip(names, go, gd):
        assert_close("grad_" + nm, a, b, 5e-2, 5e-2)
