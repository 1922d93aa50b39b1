"""Checkpoint compatibility with the reference (trainer checkpoint format).

The reference trainer saves plain state_dicts, in fp16
(trainer/train_pretrain.py:63-71) and reloads them with load_state_dict
(trainer/trainer_utils.py:63-116).  This build's modules must therefore expose
the same state_dict keys, shapes and dtypes and the same deterministic
initial values; tests/golden/state_layout.json records the reference's
(tests/golden/make_state_layout.py).  CPU only: module construction needs no
GPU.
"""

import io
import json
import os

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _layout():
    with open(os.path.join(HERE, "golden", "state_layout.json")) as f:
        return json.load(f)


def _cls(name):
    from model.mhc_common import MHCHead, StreamExpand
    from model.mhc_fused import MHCConnection_Fused
    from model.mhc_fused_no_hres import MHCConnection_FusedNoHres
    return {"MHCConnection_Fused": MHCConnection_Fused, "MHCConnection_FusedNoHres": MHCConnection_FusedNoHres,
            "MHCHead": MHCHead, "StreamExpand": StreamExpand}[name]


CASES = sorted(_layout())


@pytest.mark.parametrize("key", CASES)
def test_state_dict_layout_matches_reference(key):
    name, n, c = key.split("/")
    ref = _layout()[key]
    m = _cls(name)(int(n), int(c))
    sd = m.state_dict()
    assert sorted(sd) == sorted(ref), (sorted(sd), sorted(ref))
    for k, e in ref.items():
        assert list(sd[k].shape) == e["shape"], k
        assert str(sd[k].dtype).replace("torch.", "") == e["dtype"], k
        if "value" in e:
            assert sd[k].reshape(-1).tolist() == pytest.approx(e["value"], rel=0, abs=0), k


@pytest.mark.parametrize("key", [k for k in CASES if not k.startswith("StreamExpand")])
def test_fp16_checkpoint_round_trip(key):
    """A reference-style fp16 checkpoint (random values in the reference's
    layout) loads into this build's module, and this module's own checkpoint
    reloads bit for bit."""
    name, n, c = key.split("/")
    ref = _layout()[key]
    gen = torch.Generator().manual_seed(3)
    ckpt = {k: torch.randn(e["shape"], generator=gen).half() for k, e in ref.items()}
    m = _cls(name)(int(n), int(c))
    m.load_state_dict(ckpt, strict=True)
    for k, v in m.state_dict().items():
        assert v.dtype == torch.float32
        assert torch.equal(v, ckpt[k].float()), k
    buf = io.BytesIO()
    torch.save(m.state_dict(), buf)
    buf.seek(0)
    m2 = _cls(name)(int(n), int(c))
    m2.load_state_dict(torch.load(buf, weights_only=True), strict=True)
    for k, v in m2.state_dict().items():
        assert torch.equal(v, m.state_dict()[k]), k
