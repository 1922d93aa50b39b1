"""The model-level benchmark workloads (bench.py --workload c4 / c5) on a
small decoder: forward and one training step run through this build's mHC
modules, the loss is finite and every mHC parameter receives a finite,
non-zero gradient."""

import os
import sys

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


@pytest.mark.parametrize("moe", [False, True], ids=["dense", "moe"])
def test_small_decoder_trains_through_mhc_kernels(moe):
    import bench
    from model import _native as nat
    dev = torch.device("cuda")
    torch.manual_seed(0)
    m = bench._build_decoder(moe=moe, dev=dev, hidden=256, layers=2, heads=4, kv_heads=2, inter=512, vocab=512)
    ids = torch.randint(0, 512, (2, 256), device=dev)
    logits = m(ids)
    assert logits.shape == (2, 256, 512)
    loss = F.cross_entropy(logits.view(-1, 512).float(), ids.view(-1))
    assert torch.isfinite(loss)
    loss.backward()
    assert nat.lib().mhc_device_error(1) == 0
    mhc = [(n, p) for n, p in m.named_parameters() if "mhc" in n or n.startswith("exit.0")]
    assert mhc
    for n, p in mhc:
        assert p.dtype == torch.float32, n
        assert p.grad is not None and torch.isfinite(p.grad).all(), n
    assert sum(float(p.grad.abs().sum()) for _, p in mhc) > 0
