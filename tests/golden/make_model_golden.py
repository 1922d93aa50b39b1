"""Golden fixture of the reference's whole model with mHC on every sublayer.

Runs the REFERENCE's ``MiniMindForCausalLM`` (``model/model_minimind.py``,
imported from a read-only checkout given by ``--reference``) on the CPU in
fp32, for a tiny dense config (``use_mhc=1``, full mHC) and a tiny MoE config
(``use_mhc=2``, no H_res), and stores: the model config, every weight (rounded
to fp16 before the run so the fixture can store them in fp16 exactly), the
token ids, the logits, the next-token cross-entropy loss (plus the MoE
auxiliary loss the trainers add, ``trainer/train_pretrain.py:37``) and the
gradients of every mHC parameter.  The GPU test loads the weights into the
benchmark decoder (same state_dict keys) and compares logits and gradients,
which shows that the benchmark's model is the reference model and that this
build's modules work inside the reference's block structure
(``model/model_minimind.py:300-403``).  ``MiniMindBlock`` does not pass
``sinkhorn_iters``, so the reference runs with the module default of 10.

    python tests/golden/make_model_golden.py --reference /path/to/minimind-mhc
"""

from __future__ import annotations

import argparse
import os
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))

CONFIGS = {
    "dense_mhc1": dict(hidden_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       intermediate_size=256, vocab_size=512, rope_theta=1e6, rms_norm_eps=1e-6,
                       use_mhc=1, mhc_residual_expansion=4, max_position_embeddings=256),
    "moe_mhc2": dict(hidden_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                     intermediate_size=256, vocab_size=512, rope_theta=1e6, rms_norm_eps=1e-6,
                     use_mhc=2, mhc_residual_expansion=4, max_position_embeddings=256, use_moe=True,
                     num_experts=4, num_experts_per_tok=2, moe_intermediate_size=128),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a read-only checkout of the reference")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from model.model_minimind import MiniMindConfig, MiniMindForCausalLM  # noqa: E402  (reference)

    out = {}
    for name, kw in CONFIGS.items():
        torch.manual_seed(7)
        cfg = MiniMindConfig(**kw)
        model = MiniMindForCausalLM(cfg).float()
        gen = torch.Generator().manual_seed(11)
        with torch.no_grad():
            for pn, p in model.named_parameters():
                if "mhc" in pn or pn.startswith("model.norm.0"):
                    # mHC parameters: the constructor's init plus a perturbation
                    p.add_(torch.randn(p.shape, generator=gen) * 0.05)
                elif p.dim() >= 2:
                    p.copy_(torch.randn(p.shape, generator=gen) * 0.05)
                else:
                    p.copy_(1.0 + torch.randn(p.shape, generator=gen) * 0.1)
                p.copy_(p.half().float())  # stored exactly in fp16
        model.train()
        ids = torch.randint(0, kw["vocab_size"], (2, 48), generator=gen)
        res = model(ids)
        logits = res.logits
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))
        aux = res.aux_loss if res.aux_loss is not None else torch.zeros(())
        total = loss + aux
        names = [pn for pn, _ in model.named_parameters() if "mhc" in pn or pn.startswith("model.norm.0")]
        params = dict(model.named_parameters())
        grads = torch.autograd.grad(total, [params[pn] for pn in names])
        sd = {k: v.detach().half() for k, v in model.state_dict().items()}
        out[name] = dict(config=kw, state_dict=sd, ids=ids, logits=logits.detach(), loss=loss.detach(),
                         aux_loss=aux.detach(), grad_names=names, grads=[g.detach() for g in grads])
        print(name, "loss", float(loss), "aux", float(aux), "params", sum(v.numel() for v in sd.values()))
    path = os.path.join(HERE, "model_golden.pt")
    torch.save(out, path)
    print(f"wrote {path}: {os.path.getsize(path) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
