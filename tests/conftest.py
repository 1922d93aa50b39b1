import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "minimind-mhc_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_PATH = os.path.join(ROOT, "tests", "golden", "golden.pt")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN_PATH, weights_only=False)


def golden_sublayer(g, to=None):
    """The sublayer function a golden module case was generated with."""
    import torch.nn.functional as F
    if g["sub"] == "mlp":
        w1, w2 = (g["w1"], g["w2"]) if to is None else (g["w1"].to(to), g["w2"].to(to))
        return lambda z: F.silu(z @ w1.t()) @ w2.t()
    if g["sub"] == "silu_half":
        return lambda z: F.silu(z) * 0.5
    return lambda z: z


def max_rel(ref: torch.Tensor, got: torch.Tensor) -> float:
    """max|ref - got| / max|ref| (the reference's own `_check` relative measure,
    model/mhc_fused.py:871-876)."""
    ref = ref.detach().float().cpu()
    got = got.detach().float().cpu()
    diff = (ref - got).abs().max().item()
    return diff / max(ref.abs().max().item(), 1e-8)


def assert_close(name, ref, got, atol, rtol):
    """Pass when abs < atol OR rel < rtol, rel measured against max|ref| — the
    acceptance rule of the reference self-tests (model/mhc_fused.py:871-876)."""
    ref = ref.detach().float().cpu()
    got = got.detach().float().cpu()
    assert ref.shape == got.shape, f"{name}: shape {tuple(ref.shape)} vs {tuple(got.shape)}"
    assert torch.isfinite(got).all(), f"{name}: non-finite values"
    diff = (ref - got).abs().max().item() if ref.numel() else 0.0
    rel = diff / max(ref.abs().max().item(), 1e-8) if ref.numel() else 0.0
    assert diff < atol or rel < rtol, f"{name}: abs={diff:.3e} rel={rel:.3e} (atol={atol}, rtol={rtol})"
