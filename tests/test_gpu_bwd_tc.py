"""Tensor-core dx / dphi backward stage (sm_100a, bf16) vs the CUDA-core one.

mhc_pre_bwd runs K1 (per-token coefficient / Sinkhorn backward) and then
either the tensor-core dx / dphi kernel (policy AUTO, bf16, C a multiple of
128) or the CUDA-core one (policy GENERIC).  Both compute the same fp32 math:
the tensor-core kernel splits phi and inv*dm into bf16 hi + lo parts (products
accurate to ~2^-16), so dx agrees to one bf16 rounding and dphi to 1e-4
relative.  Every run also checks the backward kernel's device error word.
"""

import pytest
import torch

from conftest import max_rel

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run_bwd(n, c, t, with_res, policy, gen_seed):
    from model import _native as nat
    from model.mhc_fused import _params, _pre_bwd, _pre_fwd
    L = nat.lib()
    gen = torch.Generator().manual_seed(gen_seed)
    fd = 2 * n + (n * n if with_res else 0)
    raw = [torch.randn(n * c, fd, generator=gen) * 0.02, torch.tensor(0.3), torch.randn(n, generator=gen) * 0.1,
           torch.tensor(0.2), torch.randn(n, generator=gen) * 0.1]
    if with_res:
        raw += [torch.tensor(0.25), torch.eye(n) + torch.randn(n, n, generator=gen) * 0.1]
    ps = _params(*[r.to(DEV) for r in raw])
    x = torch.randn(t, n * c, generator=gen).bfloat16().to(DEV)
    dz = torch.randn(t, c, generator=gen).bfloat16().to(DEV)
    dh_post = torch.randn(t, n, generator=gen).to(DEV)
    dh_res = torch.randn(t, n * n, generator=gen).to(DEV) if with_res else None
    dx_add = torch.randn(t, n * c, generator=gen).bfloat16().to(DEV)
    _, _, _, _, inv, mixes = _pre_fwd(x, ps, with_res, with_res, 20, 2.0, 1e-6, 1e-6, 1e-6, n, c, torch.float32,
                                      False)
    prev = L.mhc_set_path_policy(policy)
    try:
        dx, gps = _pre_bwd(x, ps, with_res, with_res, 20, 2.0, 1e-6, 1e-6, 1e-6, n, c, inv, mixes, dz, None,
                           dh_post, dh_res, torch.float32, dx_add)
        path = L.mhc_last_path()
    finally:
        L.mhc_set_path_policy(prev)
    torch.cuda.synchronize()
    assert L.mhc_device_error(1) == 0, "backward kernel reported a timed-out wait"
    return dx, gps, path


CASES = [
    # (n, C, T, with_res)
    (4, 768, 1000, True),     # the benchmark shape, reduced T
    (4, 768, 1, True),
    (4, 768, 129, True),      # one tile + 1 token
    (4, 1024, 777, False),    # config 3, C = 1024
    (2, 512, 300, True),
    (8, 256, 260, False),
]


@pytest.mark.parametrize("n,c,t,with_res", CASES)
def test_tc_backward_matches_cuda_core(n, c, t, with_res):
    dx_t, g_t, p_t = _run_bwd(n, c, t, with_res, 0, 1000 + n * c + t)
    dx_g, g_g, p_g = _run_bwd(n, c, t, with_res, 1, 1000 + n * c + t)
    assert p_t == 1 and p_g == 0, "tensor-core backward did not run on an eligible shape"
    scale = dx_g.float().abs().max().item()
    assert (dx_t.float() - dx_g.float()).abs().max().item() <= 2 ** -7 * scale
    assert max_rel(g_g[0], g_t[0]) < 1e-4          # dphi
    for a, b in zip(g_g[1:], g_t[1:]):             # alpha / bias grads come from K1 in both paths
        assert torch.equal(a, b)


def test_tc_backward_full_size_repeatable():
    n, c, t = 4, 768, 16 * 2048
    dx1, g1, p1 = _run_bwd(n, c, t, True, 0, 5)
    dx2, g2, p2 = _run_bwd(n, c, t, True, 0, 5)
    assert p1 == 1 and p2 == 1
    assert torch.equal(dx1, dx2)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_tc_backward_full_size_vs_oracle_and_linear_in_tokens():
    """32,768 tokens at config 2 through the tensor-core backward.

    dx of a token depends only on that token's inputs, so 256 sampled tokens
    are checked against oracle autograd (fp32 on the same bf16 inputs,
    model/mhc_fused.py:533-559 with Sinkhorn, then the backward of
    <dz, z> + <dh_post, h_post> + <dh_res, H_res> plus dx_add).  dphi is a sum
    over tokens: the full batch's equals the sum over four 8,192-token chunks
    run separately, and every chunk's dx equals the full run's rows bit for bit.
    """
    from model import _native as nat
    from model.mhc_fused import _params, _pre_bwd, _pre_fwd
    from oracle import mhc_oracle as O
    L = nat.lib()
    n, c, t, iters = 4, 768, 16 * 2048, 20
    gen = torch.Generator().manual_seed(21)
    fd = 2 * n + n * n
    raw = [torch.randn(n * c, fd, generator=gen) * 0.02, torch.tensor(0.3), torch.randn(n, generator=gen) * 0.1,
           torch.tensor(0.2), torch.randn(n, generator=gen) * 0.1, torch.tensor(0.25),
           torch.eye(n) + torch.randn(n, n, generator=gen) * 0.1]
    ps = _params(*[r.to(DEV) for r in raw])
    torch.manual_seed(21)
    x = torch.randn(t, n * c, device=DEV).bfloat16()
    dz = torch.randn(t, c, device=DEV).bfloat16()
    dh_post = torch.randn(t, n, device=DEV)
    dh_res = torch.randn(t, n * n, device=DEV)
    dx_add = torch.randn(t, n * c, device=DEV).bfloat16()
    _, _, _, _, inv, mixes = _pre_fwd(x, ps, True, True, iters, 2.0, 1e-6, 1e-6, 1e-6, n, c, torch.float32, False)

    def bwd(sl):
        return _pre_bwd(x[sl], ps, True, True, iters, 2.0, 1e-6, 1e-6, 1e-6, n, c, inv[sl], mixes[sl], dz[sl], None,
                        dh_post[sl], dh_res[sl], torch.float32, dx_add[sl])

    prev = L.mhc_set_path_policy(0)
    try:
        dx, gps = bwd(slice(0, t))
        assert L.mhc_last_path() == 1, "the tensor-core backward did not run"
        chunk = t // 4
        dphi_sum = torch.zeros_like(gps[0])
        for k in range(4):
            sl = slice(k * chunk, (k + 1) * chunk)
            dxk, gk = bwd(sl)
            assert torch.equal(dxk, dx[sl])
            dphi_sum += gk[0]
    finally:
        L.mhc_set_path_policy(prev)
    torch.cuda.synchronize()
    assert L.mhc_device_error(1) == 0
    assert max_rel(gps[0], dphi_sum) < 1e-5

    idx = torch.randperm(t, generator=gen)[:256].to(DEV)
    p = [r.float() for r in raw]
    xo = x[idx].float().cpu().requires_grad_(True)
    z, _, h_post, h_res_raw, _, _ = O.pre_phase_full(xo, p[0], p[1], p[2], p[3], p[4], p[5], p[6], 2.0, 1e-6,
                                                     1e-6, n, c)
    h_res = O.sinkhorn(h_res_raw, iters, 1e-6)
    (gx,) = torch.autograd.grad([z, h_post, h_res], [xo],
                                [dz[idx].float().cpu(), dh_post[idx].cpu(), dh_res[idx].cpu().view(-1, n, n)])
    ref = gx + dx_add[idx].float().cpu()
    assert max_rel(ref, dx[idx]) < 2e-2
