"""The model-level workloads (bench.py --workload c4 / c5) and the drop-in
inside the reference's block structure.

* The benchmark decoder has the reference ``MiniMindForCausalLM``'s state_dict
  layout, so the reference's own weights (tests/golden/model_golden.pt, made
  by tests/golden/make_model_golden.py from the reference run on the CPU in
  fp32) load with ``strict=True``; its logits, next-token loss (plus the MoE
  auxiliary loss) and mHC parameter gradients must match the reference's.
  fp32 runs take the generic kernels and must agree to 1e-4 relative.  The
  bf16 run (mHC parameters fp32, as in the benchmark) takes the sm_100a
  kernels (n*C = 512); it is checked against the same bf16 decoder on the
  generic kernels (fp32 arithmetic, no tensor cores), which it must match
  closely, and against the fp32 reference, which it may miss only by the bf16
  model's own rounding noise: no more than the generic run misses it by.
* A small bf16 decoder trains through the kernels with finite, non-zero mHC
  gradients.
"""

import os
import sys

import pytest
import torch
import torch.nn.functional as F

from conftest import ROOT, max_rel

pytestmark = pytest.mark.gpu
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "model_golden.pt")


def _golden():
    return torch.load(GOLDEN, weights_only=False)


def _decoder_for(kw, dtype):
    import bench
    return bench._build_decoder(
        moe=bool(kw.get("use_moe", False)), dev=torch.device("cuda"), n=kw["mhc_residual_expansion"],
        hidden=kw["hidden_size"], layers=kw["num_hidden_layers"], heads=kw["num_attention_heads"],
        kv_heads=kw["num_key_value_heads"], inter=kw["intermediate_size"], vocab=kw["vocab_size"],
        experts=kw.get("num_experts", 4), topk=kw.get("num_experts_per_tok", 1),
        moe_inter=kw.get("moe_intermediate_size"), theta=kw["rope_theta"], eps=kw["rms_norm_eps"],
        iters=10, use_mhc=kw["use_mhc"], dtype=dtype)


def _run(g, dtype, policy=None):
    from model import _native as nat
    prev = nat.lib().mhc_set_path_policy(policy) if policy is not None else None
    try:
        return _run_policy(g, dtype)
    finally:
        if prev is not None:
            nat.lib().mhc_set_path_policy(prev)


def _run_policy(g, dtype):
    from model import _native as nat
    m = _decoder_for(g["config"], dtype)
    sd = {k: v.float() for k, v in g["state_dict"].items()}
    m.load_state_dict(sd, strict=True)
    m.train()
    ids = g["ids"].cuda()
    logits = m(ids)
    fwd_path = nat.lib().mhc_last_path()
    loss = F.cross_entropy(logits[:, :-1].float().reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))
    aux = m.aux_loss()
    total = loss + aux if aux is not None else loss
    params = dict(m.named_parameters())
    grads = torch.autograd.grad(total, [params[n] for n in g["grad_names"]])
    bwd_path = nat.lib().mhc_last_path()
    assert nat.device_error_code() == 0
    return logits, loss, aux, grads, (fwd_path, bwd_path)


@pytest.mark.parametrize("case", ["dense_mhc1", "moe_mhc2"])
def test_decoder_loads_reference_weights_and_matches_fp32(case):
    g = _golden()[case]
    logits, loss, aux, grads, _ = _run(g, torch.float32)
    assert max_rel(g["logits"], logits) < 1e-4
    assert abs(float(loss) - float(g["loss"])) < 1e-4 * float(g["loss"])
    if aux is not None:
        assert abs(float(aux) - float(g["aux_loss"])) < 1e-4 * max(float(g["aux_loss"]), 1e-6)
    for name, a, b in zip(g["grad_names"], g["grads"], grads):
        err = (a.float() - b.float().cpu()).abs().max().item()
        assert err < 1e-5 + 2e-3 * a.abs().max().item(), (name, err)


@pytest.mark.parametrize("case", ["dense_mhc1", "moe_mhc2"])
def test_decoder_bf16_on_fused_kernels_matches_reference(case):
    g = _golden()[case]
    logits, loss, _, grads, paths = _run(g, torch.bfloat16)
    assert paths[0] >= 1 and paths[1] == 1, "the sm_100a forward / tensor-core backward did not run"
    _, loss_g, _, grads_g, paths_g = _run(g, torch.bfloat16, policy=1)
    assert paths_g == (0, 0)
    assert max_rel(g["logits"], logits) < 5e-2
    assert abs(float(loss) - float(g["loss"])) < 1e-2 * float(g["loss"])
    assert abs(float(loss) - float(loss_g)) < 1e-3 * float(loss_g)
    big = max(a.abs().max().item() for a in g["grads"])
    num = den = 0.0
    for name, a, b, c in zip(g["grad_names"], g["grads"], grads, grads_g):
        a, b, c = a.float(), b.float().cpu(), c.float().cpu()
        # fused vs generic in the same bf16 model: only the projection's hi/lo
        # split and the reduction order differ (measured <= 1e-3 * big)
        assert (b - c).abs().max().item() < 2e-3 * big, name
        # vs the fp32 reference: the bf16 model's own noise, which the
        # generic run shows (gradients that are ~0 in the reference, such as
        # the layer-0 H_pre gates that see n identical streams, are all noise)
        err, err_g = (a - b).abs().max().item(), (a - c).abs().max().item()
        assert err <= 1.5 * err_g + 1e-3 * big, (name, err, err_g)
        num += ((a - b) ** 2).sum().item()
        den += (a ** 2).sum().item()
    assert (num / den) ** 0.5 < 0.1  # measured 0.007 (dense), 0.034 (MoE)


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
    if moe:
        loss = loss + m.aux_loss()
    assert torch.isfinite(loss)
    loss.backward()
    assert nat.lib().mhc_device_error(1) == 0
    mhc = [(n, p) for n, p in m.named_parameters() if "mhc" in n or n.startswith("model.norm.0")]
    assert mhc
    for n, p in mhc:
        assert p.dtype == torch.float32, n
        assert p.grad is not None and torch.isfinite(p.grad).all(), n
    assert sum(float(p.grad.abs().sum()) for _, p in mhc) > 0


@pytest.mark.parametrize("moe", [False, True], ids=["dense", "moe"])
def test_decoder_on_the_chain_api_matches_the_modules(moe):
    """The benchmark decoder with its sublayers run through mhc_chain (each
    block's input norms handed to the chain) against the same decoder calling
    the drop-in modules with the norms in the closures: same logits and
    gradients up to bf16 rounding."""
    import bench
    torch.manual_seed(0)
    dev = torch.device("cuda")
    m = bench._build_decoder(moe=moe, dev=dev, hidden=256, layers=2, heads=4, kv_heads=2, inter=512, vocab=512)
    ids = torch.randint(0, 512, (2, 256), device=dev)
    outs = []
    for chain in (False, True):
        m.model.use_chain = chain
        m.zero_grad(set_to_none=True)
        logits = m(ids)
        loss = F.cross_entropy(logits.view(-1, 512).float(), ids.view(-1))
        loss.backward()
        outs.append((logits.detach().float(), {n: p.grad.detach().float().clone() for n, p in m.named_parameters()
                                               if p.grad is not None}))
    (l0, g0), (l1, g1) = outs
    assert (l0 - l1).abs().max().item() <= 2e-2 * l0.abs().max().item()
    assert set(g0) == set(g1)
    for n in g0:
        assert (g0[n] - g1[n]).abs().max().item() <= 5e-2 * g0[n].abs().max().item() + 1e-6, n
