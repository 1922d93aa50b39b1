"""Host-side pieces of the block-level chain API that need no GPU: the
RMSNorm backward the chain uses for the fused input norm, against autograd
through ``nn.RMSNorm``, and the argument checks."""

import pytest
import torch
import torch.nn as nn


def test_norm_backward_matches_autograd():
    from model.mhc_block import _norm_bwd
    torch.manual_seed(0)
    t, c = 37, 96
    z = torch.randn(t, c, dtype=torch.float64)
    norm = nn.RMSNorm(c, eps=1e-6).double()
    with torch.no_grad():
        norm.weight.add_(0.1 * torch.randn(c, dtype=torch.float64))
    zz = z.clone().requires_grad_(True)
    y = norm(zz)
    g = torch.randn_like(y)
    y.backward(g)
    dz, dw = _norm_bwd(g, z, norm.weight.detach(), 1e-6)
    assert torch.allclose(dz.double(), zz.grad, rtol=1e-5, atol=1e-6)
    assert torch.allclose(dw.double(), norm.weight.grad, rtol=1e-5, atol=1e-6)


def test_norm_arguments_are_checked():
    from model.mhc_block import _norm_args
    assert _norm_args(None, 8, torch.bfloat16, "cpu") == (None, 0.0)
    w, eps = _norm_args(nn.RMSNorm(8, eps=1e-5), 8, torch.bfloat16, "cpu")
    assert w.shape == (8,) and eps == 1e-5
    _, eps = _norm_args(nn.RMSNorm(8), 8, torch.bfloat16, "cpu")
    assert eps == torch.finfo(torch.bfloat16).eps
    with pytest.raises(ValueError):
        _norm_args(nn.RMSNorm(16), 8, torch.bfloat16, "cpu")
    with pytest.raises(TypeError):
        _norm_args(nn.LayerNorm(8), 8, torch.bfloat16, "cpu")


def test_chain_rejects_mixed_connections():
    from model.mhc_block import mhc_chain
    from model.mhc_fused import MHCConnection_Fused
    from model.mhc_fused_no_hres import MHCConnection_FusedNoHres
    x = torch.zeros(1, 2, 4 * 8)
    steps = [(MHCConnection_Fused(4, 8), None, None), (MHCConnection_FusedNoHres(4, 8), None, None)]
    with pytest.raises(ValueError):
        mhc_chain(x, steps)
    with pytest.raises(TypeError):
        mhc_chain(x, [(nn.Linear(8, 8), None, None)])
