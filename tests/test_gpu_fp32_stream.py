"""The fp32-stream sm_100a coefficient kernel against the generic CUDA-core
kernels and the oracle.

The reference's trainers run the mHC residual stream in fp32 under bf16
autocast (trainer/train_pretrain.py:129-130, model/model_minimind.py:384-385),
so `mhc_pre_fwd` sees fp32 x.  For n in {2, 4}, the full and no-H_res layers
and C a multiple of 128 with 4 <= C/128 <= 8, it runs the column-owned cluster
kernel of csrc/mhc_chain.cu in its fp32 mode (`mhc_last_path() == 4`): x is
split into bf16 hi + lo in shared memory and projected on the tensor cores
against phi hi + lo, so the projection is accurate to ~2^-16 relative; the sum
of squares and z are fp32 arithmetic on the fp32 x.  Coefficients agree with
the generic kernels (fp32 FMAs) to 3e-5 relative and with the oracle to 1e-4
(the reference's own bar, model/mhc_fused.py:871-876); z to 1e-4 relative.
"""

import pytest
import torch

from conftest import max_rel
from oracle import mhc_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
AUTO, GENERIC = 0, 1
RAN_FP32_STREAM = 4


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


def _run_pre(x, ps, with_res, n, c, policy, apply_sk=True, iters=20):
    nat, L = _lib()
    from model.mhc_fused import _pre_fwd
    prev = L.mhc_set_path_policy(policy)
    try:
        out = _pre_fwd(x, ps, with_res, apply_sk, iters, 2.0, 1e-6, 1e-6, 1e-6, n, c, torch.float32, True)
        path = L.mhc_last_path()
    finally:
        L.mhc_set_path_policy(prev)
    assert L.mhc_device_error(1) == 0, "the kernel reported a timed-out wait"
    return out, path


CASES = [
    # (n, C, T, with_res)
    (4, 768, 4096, True),      # benchmark width, reduced T
    (4, 768, 1, True),         # single token
    (4, 768, 129, True),       # one tile + 1
    (4, 768, 127, False),
    (4, 1024, 1000, False),    # config 3, C = 1024 (8-CTA clusters)
    (2, 512, 300, True),       # 4-CTA clusters, n = 2
    (4, 512, 777, True),
    (2, 768, 515, False),
    (4, 640, 300, True),       # 5-CTA clusters: uneven token owners
    (4, 896, 257, False),      # 7-CTA clusters
    (4, 768, 22 * 128 * 3 + 64, False),  # several tiles per cluster, a half tile
]


@pytest.mark.parametrize("n,c,t,with_res", CASES)
def test_fp32_stream_kernel_matches_generic_and_oracle(n, c, t, with_res):
    gen = torch.Generator().manual_seed(n * 1000 + t)
    ps, raw = _params(n, c, with_res, gen)
    x = torch.randn(t, n * c, generator=gen)
    xd = x.to(DEV)
    (zf, hpf, hof, hrf, invf, mixf), path_f = _run_pre(xd, ps, with_res, n, c, AUTO)
    (zg, hpg, hog, hrg, invg, mixg), path_g = _run_pre(xd, ps, with_res, n, c, GENERIC)
    assert path_f == RAN_FP32_STREAM, "the fp32-stream sm_100a kernel did not run"
    assert path_g == 0
    assert zf.dtype == torch.float32
    assert max_rel(invg, invf) < 1e-5
    assert max_rel(mixg, mixf) < 3e-5
    assert max_rel(hpg, hpf) < 3e-5
    assert max_rel(hog, hof) < 3e-5
    if with_res:
        assert max_rel(hrg, hrf) < 3e-5
    assert max_rel(zg, zf) < 1e-4
    # the oracle: fp32 on the same inputs (model/mhc_fused.py:533-559)
    p = [r.float() for r in raw]
    if with_res:
        z_o, hp_o, ho_o, hr_raw, inv_o, mix_o = O.pre_phase_full(
            x, p[0], p[1], p[2], p[3], p[4], p[5], p[6], 2.0, 1e-6, 1e-6, n, c)
        assert max_rel(O.sinkhorn(hr_raw, 20, 1e-6), hrf) < 1e-4
    else:
        z_o, hp_o, ho_o, inv_o, mix_o = O.pre_phase_no_hres(x, p[0], p[1], p[2], p[3], p[4], 2.0, 1e-6, 1e-6, n, c)
    assert max_rel(inv_o, invf) < 1e-4
    assert max_rel(mix_o, mixf) < 1e-4
    assert max_rel(hp_o, hpf) < 1e-4
    assert max_rel(ho_o, hof) < 1e-4
    assert max_rel(z_o, zf) < 1e-4


def test_fp32_stream_kernel_full_size_repeatable():
    """32,768 tokens at config 2's width: bit-identical on a second run,
    sampled tokens against the generic kernels."""
    gen = torch.Generator().manual_seed(17)
    n, c, t = 4, 768, 32768
    ps, _ = _params(n, c, True, gen)
    torch.manual_seed(9)
    xd = torch.randn(t, n * c, device=DEV)
    (z1, hp1, ho1, hr1, inv1, mix1), p1 = _run_pre(xd, ps, True, n, c, AUTO)
    (z2, hp2, ho2, hr2, inv2, mix2), p2 = _run_pre(xd, ps, True, n, c, AUTO)
    assert p1 == p2 == RAN_FP32_STREAM
    for a, b in [(z1, z2), (hp1, hp2), (ho1, ho2), (hr1, hr2), (inv1, inv2), (mix1, mix2)]:
        assert torch.equal(a, b)
    idx = torch.randperm(t, generator=gen)[:2048].to(DEV)
    (zg, _, hog, hrg, invg, mixg), pg = _run_pre(xd[idx].contiguous(), ps, True, n, c, GENERIC)
    assert pg == 0
    assert max_rel(mixg, mix1[idx]) < 3e-5
    assert max_rel(hrg, hr1[idx]) < 3e-5
    assert max_rel(zg, z1[idx]) < 1e-4


def test_fp32_stream_shapes_outside_the_kernel_use_the_generic_path():
    """n = 8 or C not a multiple of 128 keep the generic kernels."""
    for n, c, t in [(8, 512, 64), (4, 200, 64), (4, 256, 64)]:
        gen = torch.Generator().manual_seed(c)
        ps, _ = _params(n, c, False, gen)
        xd = torch.randn(t, n * c, generator=gen).to(DEV)
        _, path = _run_pre(xd, ps, False, n, c, AUTO)
        assert path == 0
