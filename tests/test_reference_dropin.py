"""The drop-in on the CPU: this build's modules inside the reference's model.

* Option B of the integration notes: the reference's own
  ``model/model_minimind.py`` is imported with this build's ``mhc_fused``,
  ``mhc_fused_no_hres`` and ``mhc_common`` standing in for its own (its
  relative imports, ``model/model_minimind.py:11-13``, resolve to them).  The
  resulting ``MiniMindForCausalLM`` (``use_mhc`` 1 and 2, dense and MoE) must
  be built from this build's classes and have exactly the state_dict keys,
  shapes, dtypes and deterministic initial values of the pure reference model.
  Needs a checkout of the reference (``MINIMIND_REFERENCE``, or a directory
  named ``reference`` beside this repository); skipped without one.
* The benchmark decoder has the state_dict layout of the reference model
  recorded in tests/golden/model_golden.pt (no reference checkout needed).
Construction only: no kernel runs on the CPU.
"""

import importlib
import os
import sys
import types

import pytest
import torch

from conftest import ROOT

TINY = dict(hidden_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
            intermediate_size=256, vocab_size=512, max_position_embeddings=256, mhc_residual_expansion=4)


def _reference_root():
    for cand in (os.environ.get("MINIMIND_REFERENCE"), os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.exists(os.path.join(cand, "model", "model_minimind.py")):
            return cand
    return None


_CACHE = {}


def _load_model_module(ref_root, ours):
    """The reference's model_minimind module.  With ``ours``, it is imported as
    ``mhcref_ours.model_minimind`` whose package's mHC submodules are this
    build's.  Without, it is the unmodified reference package, imported as
    ``model`` (its files import each other by that absolute name) and then moved
    out of the way of this build's own ``model`` package."""
    if ours in _CACHE:
        return _CACHE[ours]
    from model import mhc_common, mhc_fused, mhc_fused_no_hres
    if ours:
        alias = "mhcref_ours"
        pkg = types.ModuleType(alias)
        pkg.__path__ = [os.path.join(ref_root, "model")]
        sys.modules[alias] = pkg
        sys.modules[alias + ".mhc_fused"] = mhc_fused
        sys.modules[alias + ".mhc_fused_no_hres"] = mhc_fused_no_hres
        sys.modules[alias + ".mhc_common"] = mhc_common
        mod = importlib.import_module(alias + ".model_minimind")
    else:
        mine = {k: v for k, v in sys.modules.items() if k == "model" or k.startswith("model.")}
        for k in mine:
            del sys.modules[k]
        sys.path.insert(0, ref_root)
        try:
            mod = importlib.import_module("model.model_minimind")
        finally:
            sys.path.remove(ref_root)
            for k in [k for k in sys.modules if k == "model" or k.startswith("model.")]:
                del sys.modules[k]
            sys.modules.update(mine)
        # transformers looks the classes' module up by name at construction;
        # this build's package has no module of that name
        sys.modules["model.model_minimind"] = mod
    _CACHE[ours] = mod
    return mod


def _layout(model):
    return {k: (tuple(v.shape), v.dtype) for k, v in model.state_dict().items()}


@pytest.mark.parametrize("use_mhc,moe", [(1, False), (2, False), (1, True)])
def test_reference_model_builds_on_this_builds_modules(use_mhc, moe):
    ref_root = _reference_root()
    if ref_root is None:
        pytest.skip("no reference checkout (set MINIMIND_REFERENCE)")
    ours = _load_model_module(ref_root, True)
    pure = _load_model_module(ref_root, False)
    from model.mhc_common import MHCHead, StreamExpand
    from model.mhc_fused import MHCConnection_Fused
    from model.mhc_fused_no_hres import MHCConnection_FusedNoHres

    kw = dict(TINY, use_mhc=use_mhc)
    if moe:
        kw.update(use_moe=True, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=128)
    models = []
    for mod in (ours, pure):
        torch.manual_seed(0)
        models.append(mod.MiniMindForCausalLM(mod.MiniMindConfig(**kw)))
    m_ours, m_pure = models
    want = MHCConnection_Fused if use_mhc == 1 else MHCConnection_FusedNoHres
    blk = m_ours.model.layers[0]
    assert type(blk.attn_mhc) is want and type(blk.mlp_mhc) is want
    assert type(m_ours.model.norm[0]) is MHCHead and type(m_ours.model.embed_up_norm[1]) is StreamExpand
    assert _layout(m_ours) == _layout(m_pure)
    sd_o, sd_p = m_ours.state_dict(), m_pure.state_dict()
    for k in sd_p:
        if "mhc" in k and "phi" not in k:
            assert torch.equal(sd_o[k], sd_p[k]), k
    # a reference checkpoint loads into the model built on this build's modules
    m_ours.load_state_dict(sd_p, strict=True)


def test_benchmark_decoder_has_the_reference_layout():
    import bench
    golden = torch.load(os.path.join(ROOT, "tests", "golden", "model_golden.pt"), weights_only=False)
    for case, g in golden.items():
        kw = g["config"]
        m = bench._build_decoder(
            moe=bool(kw.get("use_moe", False)), dev=torch.device("cpu"), n=kw["mhc_residual_expansion"],
            hidden=kw["hidden_size"], layers=kw["num_hidden_layers"], heads=kw["num_attention_heads"],
            kv_heads=kw["num_key_value_heads"], inter=kw["intermediate_size"], vocab=kw["vocab_size"],
            experts=kw.get("num_experts", 4), topk=kw.get("num_experts_per_tok", 1),
            moe_inter=kw.get("moe_intermediate_size"), use_mhc=kw["use_mhc"], dtype=torch.float32)
        ours = {k: tuple(v.shape) for k, v in m.state_dict().items()}
        ref = {k: tuple(v.shape) for k, v in g["state_dict"].items()}
        assert ours == ref, case
        m.load_state_dict({k: v.float() for k, v in g["state_dict"].items()}, strict=True)
        assert m.lm_head.weight.data_ptr() == m.model.embed_tokens.weight.data_ptr()
