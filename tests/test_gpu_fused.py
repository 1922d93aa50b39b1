"""The fused sm_100a coefficient kernels vs the generic CUDA-core kernels and
the oracle.

Two fused kernels compute the forward coefficient stage for bf16 activations:
the two-read kernel (x read from HBM, then from L2; policy AUTO where it
applies) and the single-read kernel (x read from HBM once, chunks retained in
TMEM; policy SINGLE_READ, and AUTO where the two-read kernel does not apply).  Both
compute the same fp32 coefficient math as the generic kernels; the projection
runs on the tensor cores with phi split into bf16 hi + lo halves (relative
error ~2^-17), so coefficients agree to 2e-5 relative and the bf16
pre-aggregate z to one bf16 rounding.  Every run also checks the device error
words (a bounded wait that ran out would set one).
"""

import pytest
import torch

from conftest import max_rel
from oracle import mhc_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
AUTO, GENERIC, TWO_READ, SINGLE_READ = 0, 1, 2, 3


def _lib():
    from model import _native as nat
    return nat, nat.lib()


def _sr_ok(n, c, mode="full"):
    return n in (2, 4) and c % 128 == 0 and 4 <= c // 128 <= 8


def _tc_ok(n, c, mode="full"):
    nc = n * c
    if nc % 512 or c % 64 or nc // 512 > 8 or c // 8 > 256:
        return False
    return n <= 4 if mode == "full" else n <= 8


def expected_path(n, c, policy, mode="full", t=32768):
    """The kernel family the C-ABI selects (2 single-read, 1 two-read, 0 generic)."""
    if policy == GENERIC:
        return 0
    if policy == SINGLE_READ and _sr_ok(n, c, mode):
        return 2
    if policy == AUTO and _sr_ok(n, c, mode) and (not _tc_ok(n, c, mode) or mode != "full" or t < 32768):
        return 2
    if _tc_ok(n, c, mode):
        return 1
    return 0


def _run_pre(x, ps, with_res, n, c, policy, apply_sk=False, iters=20):
    nat, L = _lib()
    from model.mhc_fused import _pre_fwd
    prev = L.mhc_set_path_policy(policy)
    try:
        out = _pre_fwd(x, ps, with_res, apply_sk, iters, 2.0, 1e-6, 1e-6, 1e-6, n, c, torch.float32, True)
        path = L.mhc_last_path()
    finally:
        L.mhc_set_path_policy(prev)
    assert L.mhc_device_error(1) == 0, "fused kernel reported a timed-out wait"
    return out, path


def _params(n, c, with_res, gen, scale=0.02):
    from model.mhc_fused import _params as prep
    fd = 2 * n + (n * n if with_res else 0)
    phi = torch.randn(n * c, fd, generator=gen) * scale
    ts = [phi, torch.tensor(0.3), torch.randn(n, generator=gen) * 0.1, torch.tensor(0.2),
          torch.randn(n, generator=gen) * 0.1]
    if with_res:
        ts += [torch.tensor(0.25), torch.eye(n) + torch.randn(n, n, generator=gen) * 0.1]
    return prep(*[t.to(DEV) for t in ts]), ts


CASES = [
    # (n, C, T, with_res)
    (4, 768, 4096, True),      # benchmark shape, reduced T
    (4, 768, 1, True),         # single token
    (4, 768, 129, True),       # one full tile + 1
    (4, 768, 127, False),
    (4, 1024, 1000, False),    # config 3, C = 1024
    (2, 512, 300, True),
    (4, 512, 777, True),
    (8, 512, 260, False),
    (2, 768, 515, False),
    (4, 768, 16 * 128 * 15 + 3, True),  # every cluster busy, a partial last tile
    (4, 640, 300, True),       # 5-CTA clusters in the single-read kernel
    (4, 896, 257, False),      # 7-CTA clusters
    (4, 768, 24 * 128 * 3 + 64, False),  # several tiles per cluster, a half tile
]


@pytest.mark.parametrize("policy", [SINGLE_READ, TWO_READ], ids=["single_read", "two_read"])
@pytest.mark.parametrize("n,c,t,with_res", CASES)
def test_fused_matches_generic_and_oracle(n, c, t, with_res, policy):
    mode = "full" if with_res else "nohres"
    want = expected_path(n, c, policy, mode, t)
    if want == 0 or (policy == SINGLE_READ and want != 2):
        pytest.skip("this kernel does not apply to the shape")
    gen = torch.Generator().manual_seed(n * 100 + t)
    ps, raw = _params(n, c, with_res, gen)
    x = torch.randn(t, n * c, generator=gen).bfloat16()
    xd = x.to(DEV)
    (zf, hpf, hof, hrf, invf, mixf), path_f = _run_pre(xd, ps, with_res, n, c, policy)
    (zg, hpg, hog, hrg, invg, mixg), path_g = _run_pre(xd, ps, with_res, n, c, GENERIC)
    assert path_f == want, "the expected fused sm_100a kernel did not run"
    assert path_g == 0
    assert max_rel(invg, invf) < 1e-5
    assert max_rel(mixg, mixf) < 2e-5
    assert max_rel(hpg, hpf) < 2e-5
    assert max_rel(hog, hof) < 2e-5
    if with_res:
        assert max_rel(hrg, hrf) < 2e-5
    # z: identical fp32 weights up to 2e-5, one bf16 rounding each
    assert (zg.float() - zf.float()).abs().max().item() <= 2 ** -7 * zg.float().abs().max().item()
    # and the oracle (fp32 on the bf16 inputs)
    p = [r.float() for r in raw]
    inv, _, mixes = O.rms_project(x.float(), p[0], 1e-6)
    assert max_rel(mixes, mixf) < 1e-4
    assert max_rel(inv.squeeze(-1), invf) < 1e-4


def test_fused_sinkhorn_matches_merge_kernel_sinkhorn():
    """Sinkhorn inside the fused coefficient kernel equals the oracle on the
    kernel's own logits, and the merge kernel's Sinkhorn-on-logits mode."""
    nat, L = _lib()
    gen = torch.Generator().manual_seed(7)
    n, c, t = 4, 768, 1024
    ps, _ = _params(n, c, True, gen)
    xd = torch.randn(t, n * c, generator=gen).bfloat16().to(DEV)
    (z, _, hpost, hres_norm, _, _), path = _run_pre(xd, ps, True, n, c, SINGLE_READ, apply_sk=True)
    assert path == 2
    (_, _, _, hres_logit, _, _), _ = _run_pre(xd, ps, True, n, c, SINGLE_READ, apply_sk=False)
    (_, _, _, hres_norm_tr, _, _), path_tr = _run_pre(xd, ps, True, n, c, TWO_READ, apply_sk=True)
    assert path_tr == 1
    assert max_rel(hres_norm_tr, hres_norm) < 1e-5
    ref = O.sinkhorn(hres_logit.cpu(), 20, 1e-6)
    assert max_rel(ref, hres_norm) < 1e-5
    f = torch.randn(t, c, generator=gen).bfloat16().to(DEV)
    out1 = torch.empty_like(xd)
    out2 = torch.empty_like(xd)
    hres_out = torch.empty_like(hres_logit)
    s = torch.cuda.current_stream().cuda_stream
    nat.call("mhc_post_fwd", nat.ptr(xd), nat.BF16, nat.ptr(hres_norm), nat.F32, nat.ptr(hpost), nat.F32,
             nat.ptr(f), nat.BF16, nat.ptr(out1), t, n, c, 0, 0, 0.0, None, s)
    nat.call("mhc_post_fwd", nat.ptr(xd), nat.BF16, nat.ptr(hres_logit), nat.F32, nat.ptr(hpost), nat.F32,
             nat.ptr(f), nat.BF16, nat.ptr(out2), t, n, c, 1, 20, 1e-6, nat.ptr(hres_out), s)
    # same steps, different summation trees (lane shuffles vs sequential sums)
    assert max_rel(hres_norm, hres_out) < 2e-6
    assert (out1.float() - out2.float()).abs().max().item() <= 2 ** -7 * out1.float().abs().max().item()


@pytest.mark.parametrize("policy", [SINGLE_READ, TWO_READ], ids=["single_read", "two_read"])
def test_fused_full_size_repeatable(policy):
    """32768 tokens (the benchmark batch) twice: bit-identical outputs, no
    device error, and sampled tokens against the generic path."""
    gen = torch.Generator().manual_seed(11)
    n, c, t = 4, 768, 16 * 2048
    ps, _ = _params(n, c, True, gen)
    torch.manual_seed(5)
    xd = torch.randn(t, n * c, device=DEV).bfloat16()
    (z1, _, ho1, hr1, inv1, mix1), p1 = _run_pre(xd, ps, True, n, c, policy)
    (z2, _, ho2, hr2, inv2, mix2), p2 = _run_pre(xd, ps, True, n, c, policy)
    assert p1 == p2 == expected_path(n, c, policy, "full", t)
    for a, b in [(z1, z2), (ho1, ho2), (hr1, hr2), (inv1, inv2), (mix1, mix2)]:
        assert torch.equal(a, b)
    idx = torch.randperm(t, generator=gen)[:2048].to(DEV)
    (zg, _, hog, hrg, invg, mixg), _ = _run_pre(xd[idx].contiguous(), ps, True, n, c, 1)
    assert max_rel(mixg, mix1[idx]) < 2e-5
    assert max_rel(hrg, hr1[idx]) < 2e-5
    assert (zg.float() - z1[idx].float()).abs().max().item() <= 2 ** -7 * zg.float().abs().max().item()


@pytest.mark.parametrize("policy", [SINGLE_READ, TWO_READ], ids=["single_read", "two_read"])
def test_fused_head_matches_generic(policy):
    nat, L = _lib()
    from model.mhc_common import MHCHead
    torch.manual_seed(3)
    n, c, t = 4, 768, 600
    head = MHCHead(n, c).to(DEV)
    x = torch.randn(1, t, n * c, device=DEV).bfloat16()
    prev = L.mhc_set_path_policy(policy)
    y_f = head(x)
    path = L.mhc_last_path()
    L.mhc_set_path_policy(GENERIC)
    y_g = head(x)
    L.mhc_set_path_policy(prev)
    assert path == expected_path(n, c, policy, "head", t)
    assert L.mhc_device_error(1) == 0
    assert (y_g.float() - y_f.float()).abs().max().item() <= 2 ** -7 * y_g.float().abs().max().item()


@pytest.mark.parametrize("n,c,t,with_res", [(4, 768, 4096, True), (4, 768, 32768, True), (4, 768, 2048, False),
                                            (4, 1024, 2048, False), (8, 512, 260, False), (4, 256, 300, True)])
def test_auto_policy_picks_the_measured_kernel(n, c, t, with_res):
    """AUTO runs the kernel the C-ABI's measured rule names for the shape."""
    gen = torch.Generator().manual_seed(t)
    ps, _ = _params(n, c, with_res, gen)
    xd = torch.randn(t, n * c, generator=gen).bfloat16().to(DEV)
    _, path = _run_pre(xd, ps, with_res, n, c, AUTO)
    assert path == expected_path(n, c, AUTO, "full" if with_res else "nohres", t)
