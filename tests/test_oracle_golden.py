"""Pins the CPU oracle against golden vectors produced by the reference itself.

CPU only.  Each case in tests/golden/golden.pt was produced by running the
reference's own pure-PyTorch path (tests/golden/make_golden.py); the oracle must
reproduce it (same rounding points, same gradients through autograd).
"""

import torch
import torch.nn.functional as F

from conftest import assert_close, golden_sublayer
from oracle import mhc_oracle as O


def _mlp(w1, w2):
    return lambda z: F.silu(z @ w1.t()) @ w2.t()


def test_sinkhorn_matches_reference(golden):
    keys = [k for k in golden if k.startswith("sinkhorn_")]
    assert len(keys) >= 5
    for k in keys:
        g = golden[k]
        m = g["M"].clone().requires_grad_(True)
        y = O.sinkhorn(m, g["iters"], g["eps"])
        assert_close(k + ".Y", g["Y"], y, 1e-6, 1e-6)
        (dm,) = torch.autograd.grad(y, m, g["dY"])
        assert_close(k + ".dM", g["dM"], dm, 1e-5, 1e-5)


def test_sinkhorn_doubly_stochastic_at_config_logits(golden):
    # config-like logits (alpha*m + bias, small spread): both marginals within 1e-5 of 1
    g = golden["sinkhorn_n4_it20_s0.02"]
    y = O.sinkhorn(g["M"], 20, 1e-6)
    assert (y.sum(-1) - 1).abs().max() < 1e-5
    assert (y.sum(-2) - 1).abs().max() < 1e-5


def test_pre_phase_full_matches_reference(golden):
    for k in [k for k in golden if k.startswith("pre_full_")]:
        g = golden[k]
        tol = 1e-5 if g["x"].dtype == torch.float32 else 1e-2
        leaves = [g["x"].clone().requires_grad_(True)] + [p.clone().requires_grad_(True) for p in g["params"]]
        z, hp, ho, hr, inv, mixes = O.pre_phase_full(*leaves, 2.0, 1e-6, 1e-6, g["n"], g["C"])
        for name, a, b in [("z", g["z"], z), ("h_pre", g["h_pre"], hp), ("h_post", g["h_post"], ho),
                           ("h_res_raw", g["h_res_raw"], hr), ("inv_rms", g["inv_rms"], inv),
                           ("mixes", g["mixes"], mixes)]:
            assert_close(f"{k}.{name}", a, b, tol, tol)
        gr = torch.autograd.grad([z, ho, hr], leaves, [g["g_z"], g["g_h_post"], g["g_h_res_raw"]])
        for i, (a, b) in enumerate(zip(g["grads"], gr)):
            assert_close(f"{k}.grad{i}", a, b, tol, tol)


def test_post_phase_full_matches_reference(golden):
    for k in [k for k in golden if k.startswith("post_full_")]:
        g = golden[k]
        tol = 1e-6 if g["x"].dtype == torch.float32 else 1e-2
        leaves = [t.clone().requires_grad_(True) for t in (g["x"], g["h_res"], g["h_post"], g["f"])]
        o = O.post_phase_full(*leaves, g["n"], g["C"])
        assert_close(k + ".out", g["out"], o, tol, tol)
        gr = torch.autograd.grad(o, leaves, g["g_out"])
        for i, (a, b) in enumerate(zip(g["grads"], gr)):
            assert_close(f"{k}.grad{i}", a, b, tol, tol)


def _module_check(g, forward, params_cls, k):
    tol = 1e-5 if g["x"].dtype == torch.float32 else 2e-2
    x = g["x"].clone().requires_grad_(True)
    ps = [p.clone().requires_grad_(True) for p in g["params"]]
    assert tuple(g["param_names"]) == params_cls.NAMES
    fn = golden_sublayer(g)
    y = forward(x, params_cls(*ps), fn)
    assert_close(k + ".out", g["out"], y, tol, tol)
    loss = y.float().pow(2).mean()
    gr = torch.autograd.grad(loss, [x] + ps)
    for name, a, b in zip(("x",) + params_cls.NAMES, g["grads"], gr):
        assert_close(f"{k}.grad_{name}", a, b, tol * 5, tol * 5)


def test_full_module_matches_reference(golden):
    for k in [k for k in golden if k.startswith("module_full_")]:
        g = golden[k]
        _module_check(g, lambda x, p, fn: O.full_forward(x, p, fn, g["n"], g["C"], g["iters"]),
                      O.FullParams, k)


def test_no_hres_matches_reference(golden):
    for k in [k for k in golden if k.startswith("pre_nohres_")]:
        g = golden[k]
        tol = 1e-5 if g["x"].dtype == torch.float32 else 1e-2
        leaves = [g["x"].clone().requires_grad_(True)] + [p.clone().requires_grad_(True) for p in g["params"]]
        z, hp, ho, inv, mixes = O.pre_phase_no_hres(*leaves, 2.0, 1e-6, 1e-6, g["n"], g["C"])
        for name, a, b in [("z", g["z"], z), ("h_pre", g["h_pre"], hp), ("h_post", g["h_post"], ho),
                           ("inv_rms", g["inv_rms"], inv), ("mixes", g["mixes"], mixes)]:
            assert_close(f"{k}.{name}", a, b, tol, tol)
        gr = torch.autograd.grad([z, ho], leaves, [g["g_z"], g["g_h_post"]])
        for i, (a, b) in enumerate(zip(g["grads"], gr)):
            assert_close(f"{k}.grad{i}", a, b, tol, tol)
    for k in [k for k in golden if k.startswith("post_nohres_")]:
        g = golden[k]
        tol = 1e-6 if g["x"].dtype == torch.float32 else 1e-2
        leaves = [t.clone().requires_grad_(True) for t in (g["x"], g["h_post"], g["f"])]
        o = O.post_phase_no_hres(*leaves, g["n"], g["C"])
        assert_close(k + ".out", g["out"], o, tol, tol)
        gr = torch.autograd.grad(o, leaves, g["g_out"])
        for i, (a, b) in enumerate(zip(g["grads"], gr)):
            assert_close(f"{k}.grad{i}", a, b, tol, tol)
    for k in [k for k in golden if k.startswith("module_nohres_")]:
        g = golden[k]
        _module_check(g, lambda x, p, fn: O.no_hres_forward(x, p, fn, g["n"], g["C"]),
                      O.NoHresParams, k)


def test_head_and_expand_match_reference(golden):
    for k in [k for k in golden if k.startswith("head_")]:
        g = golden[k]
        tol = 1e-5 if g["x"].dtype == torch.float32 else 1e-2
        x = g["x"].clone().requires_grad_(True)
        ps = [p.clone().requires_grad_(True) for p in g["params"]]
        assert tuple(g["param_names"]) == ("phi_weight", "bias", "alpha")
        y = O.mhc_head(x, ps[0], ps[2], ps[1], 1e-6, 1e-6, g["n"], g["C"])
        assert_close(k + ".out", g["out"], y, tol, tol)
        gr = torch.autograd.grad(y, [x] + ps, g["g_out"], allow_unused=True)
        for i, (a, b) in enumerate(zip(g["grads"], gr)):
            if a is None:
                assert b is None or b.abs().max() == 0
                continue
            assert_close(f"{k}.grad{i}", a, b, tol, tol)
    g = golden["expand_n4"]
    assert torch.equal(O.stream_expand(g["x"], g["n"]), g["out"])


def test_config1_summary_matches_reference(golden):
    g = golden["config1_summary"]
    torch.manual_seed(0)
    x = torch.randn(2, 512, 4 * 512)
    phi = torch.randn(4 * 512, 24) * 0.02
    assert abs(x.double().sum().item() - g["x_sum"].item()) < 1e-6
    assert abs(phi.double().sum().item() - g["phi_sum"].item()) < 1e-9
    p = O.make_full_params(4, 512)
    p.phi_weight = phi
    with torch.no_grad():
        y = O.full_forward(x, p, lambda z: z, 4, 512, 20)
    assert_close("config1.rows", g["out_rows"], y.view(1024, -1)[g["rows"]], 1e-6, 1e-6)
    assert abs(y.double().sum().item() - g["out_sum"].item()) <= 1e-6 * abs(g["out_sum"].item()) + 1e-3
