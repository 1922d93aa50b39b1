"""Generate the golden vectors that pin the oracle and the CUDA path.

Runs the REFERENCE implementation itself (Tshirt-hfk/minimind-mhc, imported
from a read-only checkout given by ``--reference``)
on small seeded CPU inputs and stores inputs, outputs and autograd gradients
under ``tests/golden/*.pt``.  The reference has no golden vectors or
known-answer tests of its own; its self-tests compare its Triton kernels with
its pure-PyTorch path on seeded ``torch.randn`` draws
(``model/mhc_fused.py:879-1025``), so these fixtures are made the same way: by
running that pure-PyTorch path.

The reference cannot travel to the GPU box, so the fixtures are committed and
the tests only read them.  Re-run with::

    python tests/golden/make_golden.py --reference /path/to/minimind-mhc
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _mlp(w1, w2):
    def f(z):
        return F.silu(z @ w1.t()) @ w2.t()
    return f


def _rand_like_list(ts, gen):
    return [torch.randn(t.shape, generator=gen, dtype=torch.float32).to(t.dtype) for t in ts]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a read-only checkout of the reference")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from model import mhc_fused as R            # noqa: E402  (reference)
    from model import mhc_fused_no_hres as RN   # noqa: E402
    from model import mhc_common as RC          # noqa: E402

    torch.manual_seed(0)
    gen = torch.Generator().manual_seed(1234)
    out = {}

    # ---------------- Sinkhorn (reference _sinkhorn_ref + autograd) -------------
    for n, iters, scale in [(4, 20, 1.0), (4, 10, 1.0), (4, 20, 0.02), (2, 20, 1.0), (8, 20, 1.0),
                            (1, 20, 1.0), (4, 1, 1.0)]:
        m = torch.randn(96, n, n, generator=gen) * scale
        if scale != 1.0:
            m = m + torch.eye(n)
        m.requires_grad_(True)
        y = R._sinkhorn_ref(m, iters, 1e-6)
        dy = torch.randn(y.shape, generator=gen)
        (dm,) = torch.autograd.grad(y, m, dy)
        out[f"sinkhorn_n{n}_it{iters}_s{scale}"] = dict(
            M=m.detach(), iters=iters, eps=1e-6, Y=y.detach(), dY=dy, dM=dm)

    # ---------------- PRE phase full (reference _pre_phase_full_ref) -------------
    def pre_full_case(n, c, dtype, init, bl=(2, 16)):
        b, l = bl
        fd = 2 * n + n * n
        x = (torch.randn(b, l, n * c, generator=gen)).to(dtype)
        if init == "bench":
            phi = (torch.randn(n * c, fd, generator=gen) * 0.02)
            b_res = torch.zeros(n, n)
            b_pre = torch.zeros(n)
            b_post = torch.zeros(n)
        else:
            bound = 1.0 / math.sqrt(fd)
            phi = torch.empty(n * c, fd).uniform_(-bound, bound, generator=gen)
            b_res = torch.eye(n)
            b_pre = torch.randn(n, generator=gen) * 0.1
            b_post = torch.randn(n, generator=gen) * 0.1
        params = [phi.to(dtype), torch.tensor(0.01).to(dtype), b_pre.to(dtype),
                  torch.tensor(0.02).to(dtype), b_post.to(dtype),
                  torch.tensor(0.015).to(dtype), b_res.to(dtype)]
        leaves = [x.clone().requires_grad_(True)] + [p.clone().requires_grad_(True) for p in params]
        z, hp, ho, hr, inv, mixes = R._pre_phase_full_ref(
            leaves[0], leaves[1], leaves[2], leaves[3], leaves[4], leaves[5], leaves[6], leaves[7],
            2.0, 1e-6, 1e-6, n, c)
        gz, gho, ghr = _rand_like_list([z, ho, hr], gen)
        g = torch.autograd.grad([z, ho, hr], leaves, [gz, gho, ghr])
        return dict(n=n, C=c, x=x, params=params, z=z.detach(), h_pre=hp.detach(), h_post=ho.detach(),
                    h_res_raw=hr.detach(), inv_rms=inv.detach(), mixes=mixes.detach(),
                    g_z=gz, g_h_post=gho, g_h_res_raw=ghr, grads=[t.detach() for t in g])

    out["pre_full_f32_bench"] = pre_full_case(4, 64, torch.float32, "bench")
    out["pre_full_f32_module"] = pre_full_case(4, 64, torch.float32, "module")
    out["pre_full_f32_n2"] = pre_full_case(2, 96, torch.float32, "module")
    out["pre_full_bf16_bench"] = pre_full_case(4, 64, torch.bfloat16, "bench")

    # ---------------- POST phase full (reference _post_phase_full_ref) -----------
    def post_full_case(n, c, dtype, bl=(2, 16)):
        b, l = bl
        x = torch.randn(b, l, n * c, generator=gen).to(dtype)
        h_res = R._sinkhorn_ref(torch.randn(b, l, n, n, generator=gen), 10, 1e-6).to(dtype)
        h_post = (torch.rand(b, l, n, generator=gen) * 2.0).to(dtype)
        f = torch.randn(b, l, c, generator=gen).to(dtype)
        leaves = [t.clone().requires_grad_(True) for t in (x, h_res, h_post, f)]
        o = R._post_phase_full_ref(leaves[0], leaves[1], leaves[2], leaves[3], n, c)
        go = torch.randn(o.shape, generator=gen).to(dtype)
        g = torch.autograd.grad(o, leaves, go)
        return dict(n=n, C=c, x=x, h_res=h_res, h_post=h_post, f=f, out=o.detach(), g_out=go,
                    grads=[t.detach() for t in g])

    out["post_full_f32"] = post_full_case(4, 64, torch.float32)
    out["post_full_bf16"] = post_full_case(4, 64, torch.bfloat16)
    out["post_full_f32_n8"] = post_full_case(8, 32, torch.float32)

    # ---------------- whole module (reference MHCConnection_Fused._forward_ref) --
    def module_full_case(n, c, dtype, init, iters, sub, bl=(2, 16)):
        b, l = bl
        torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
        mod = R.MHCConnection_Fused(n, c, sinkhorn_iters=iters)
        if init == "bench":
            with torch.no_grad():
                mod.phi_weight.copy_(torch.randn(n * c, 2 * n + n * n, generator=gen) * 0.02)
                mod.bias_res.zero_()
        else:
            with torch.no_grad():
                mod.bias_pre.copy_(torch.randn(n, generator=gen) * 0.1)
                mod.bias_post.copy_(torch.randn(n, generator=gen) * 0.1)
                mod.bias_res.add_(torch.randn(n, n, generator=gen) * 0.1)
        mod = mod.to(dtype)
        x = torch.randn(b, l, n * c, generator=gen).to(dtype).requires_grad_(True)
        if sub == "mlp":
            w1 = (torch.randn(2 * c, c, generator=gen) * 0.05).to(dtype)
            w2 = (torch.randn(c, 2 * c, generator=gen) * 0.05).to(dtype)
            fn = _mlp(w1, w2)
        else:
            w1 = w2 = None
            fn = (lambda z: z)
        y = mod._forward_ref(x, fn)
        loss = y.float().pow(2).mean()
        names = [k for k, _ in mod.named_parameters()]
        leaves = [x] + [p for _, p in mod.named_parameters()]
        g = torch.autograd.grad(loss, leaves)
        return dict(n=n, C=c, iters=iters, sub=sub, x=x.detach(), w1=w1, w2=w2,
                    param_names=names, params=[p.detach().clone() for _, p in mod.named_parameters()],
                    out=y.detach(), loss=loss.detach(), grads=[t.detach() for t in g])

    out["module_full_f32_bench_id"] = module_full_case(4, 64, torch.float32, "bench", 20, "id")
    out["module_full_f32_module_mlp"] = module_full_case(4, 64, torch.float32, "module", 10, "mlp")
    out["module_full_bf16_bench_mlp"] = module_full_case(4, 64, torch.bfloat16, "bench", 20, "mlp")
    out["module_full_f32_n2_mlp"] = module_full_case(2, 128, torch.float32, "module", 20, "mlp")

    # ---------------- no-H_res variant --------------------------------------------
    def pre_nohres_case(n, c, dtype, bl=(2, 16)):
        b, l = bl
        x = torch.randn(b, l, n * c, generator=gen).to(dtype)
        phi = torch.randn(n * c, 2 * n, generator=gen) * 0.05
        params = [phi.to(dtype), torch.tensor(0.01).to(dtype), (torch.randn(n, generator=gen) * 0.1).to(dtype),
                  torch.tensor(0.02).to(dtype), (torch.randn(n, generator=gen) * 0.1).to(dtype)]
        leaves = [x.clone().requires_grad_(True)] + [p.clone().requires_grad_(True) for p in params]
        z, hp, ho, inv, mixes = RN._pre_phase_ref(leaves[0], *leaves[1:], 2.0, 1e-6, 1e-6, n, c)
        gz, gho = _rand_like_list([z, ho], gen)
        g = torch.autograd.grad([z, ho], leaves, [gz, gho])
        return dict(n=n, C=c, x=x, params=params, z=z.detach(), h_pre=hp.detach(), h_post=ho.detach(),
                    inv_rms=inv.detach(), mixes=mixes.detach(), g_z=gz, g_h_post=gho,
                    grads=[t.detach() for t in g])

    out["pre_nohres_f32"] = pre_nohres_case(4, 64, torch.float32)
    out["pre_nohres_f32_n2"] = pre_nohres_case(2, 128, torch.float32)
    out["pre_nohres_bf16"] = pre_nohres_case(4, 64, torch.bfloat16)

    def post_nohres_case(n, c, dtype, bl=(2, 16)):
        b, l = bl
        x = torch.randn(b, l, n * c, generator=gen).to(dtype)
        h_post = (torch.rand(b, l, n, generator=gen) * 2.0).to(dtype)
        f = torch.randn(b, l, c, generator=gen).to(dtype)
        leaves = [t.clone().requires_grad_(True) for t in (x, h_post, f)]
        o = RN._post_phase_ref(leaves[0], leaves[1], leaves[2], n, c)
        go = torch.randn(o.shape, generator=gen).to(dtype)
        g = torch.autograd.grad(o, leaves, go)
        return dict(n=n, C=c, x=x, h_post=h_post, f=f, out=o.detach(), g_out=go,
                    grads=[t.detach() for t in g])

    out["post_nohres_f32"] = post_nohres_case(4, 64, torch.float32)
    out["post_nohres_bf16_n8"] = post_nohres_case(8, 32, torch.bfloat16)

    def module_nohres_case(n, c, dtype, bl=(2, 16)):
        b, l = bl
        torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
        mod = RN.MHCConnection_FusedNoHres(n, c)
        with torch.no_grad():
            mod.bias_pre.copy_(torch.randn(n, generator=gen) * 0.1)
            mod.bias_post.copy_(torch.randn(n, generator=gen) * 0.1)
        mod = mod.to(dtype)
        x = torch.randn(b, l, n * c, generator=gen).to(dtype).requires_grad_(True)
        w1 = (torch.randn(2 * c, c, generator=gen) * 0.05).to(dtype)
        w2 = (torch.randn(c, 2 * c, generator=gen) * 0.05).to(dtype)
        y = mod._forward_ref(x, _mlp(w1, w2))
        loss = y.float().pow(2).mean()
        names = [k for k, _ in mod.named_parameters()]
        leaves = [x] + [p for _, p in mod.named_parameters()]
        g = torch.autograd.grad(loss, leaves)
        return dict(n=n, C=c, sub="mlp", x=x.detach(), w1=w1, w2=w2, param_names=names,
                    params=[p.detach().clone() for _, p in mod.named_parameters()],
                    out=y.detach(), loss=loss.detach(), grads=[t.detach() for t in g])

    out["module_nohres_f32"] = module_nohres_case(4, 64, torch.float32)
    out["module_nohres_bf16"] = module_nohres_case(4, 64, torch.bfloat16)

    # ---------------- MHCHead / StreamExpand ---------------------------------------
    def head_case(n, c, dtype, bl=(2, 16)):
        b, l = bl
        torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
        mod = RC.MHCHead(n, c)
        with torch.no_grad():
            mod.bias.copy_(torch.randn(n, generator=gen) * 0.1)
            mod.alpha.fill_(0.05)
        mod = mod.to(dtype)
        x = torch.randn(b, l, n * c, generator=gen).to(dtype).requires_grad_(True)
        y = mod(x)  # CPU tensor -> reference's pure-PyTorch path
        gy = torch.randn(y.shape, generator=gen).to(dtype)
        names = [k for k, _ in mod.named_parameters()]
        leaves = [x] + [p for _, p in mod.named_parameters()]
        g = torch.autograd.grad(y, leaves, gy, allow_unused=True)
        return dict(n=n, C=c, x=x.detach(), param_names=names,
                    params=[p.detach().clone() for _, p in mod.named_parameters()],
                    out=y.detach(), g_out=gy,
                    grads=[(t.detach() if t is not None else None) for t in g])

    out["head_n4_f32"] = head_case(4, 64, torch.float32)
    out["head_n4_bf16"] = head_case(4, 64, torch.bfloat16)
    out["head_n1_f32"] = head_case(1, 96, torch.float32)
    out["head_n8_f32"] = head_case(8, 32, torch.float32)

    xe = torch.randn(2, 8, 48, generator=gen)
    out["expand_n4"] = dict(n=4, C=48, x=xe, out=RC.StreamExpand(4, 48)(xe))

    # ---------------- Config 1 summary ------------------------
    # x ~ N(0,1) [2,512,4*512], phi ~ N(0,0.02) [2048,24], alpha=0.01, biases 0,
    # 20 Sinkhorn iterations, f = identity, all drawn from seed 0 (x first, then phi).
    torch.manual_seed(0)
    n, c = 4, 512
    x1 = torch.randn(2, 512, n * c)
    phi1 = torch.randn(n * c, 2 * n + n * n) * 0.02
    mod = R.MHCConnection_Fused(n, c, sinkhorn_iters=20)
    with torch.no_grad():
        mod.phi_weight.copy_(phi1)
        mod.bias_res.zero_()
    with torch.no_grad():
        y1 = mod._forward_ref(x1, lambda z: z)
    rows = torch.arange(0, 1024, 33)
    out["config1_summary"] = dict(
        n=n, C=c, iters=20, x_sum=x1.double().sum(), x_sq=x1.double().pow(2).sum(),
        phi_sum=phi1.double().sum(), rows=rows, out_rows=y1.view(1024, -1)[rows].clone(),
        out_sum=y1.double().sum(), out_sq=y1.double().pow(2).sum())

    # ---------------- widths that take the sm_100a kernels ------------------------
    # n*C a multiple of 512 and C a multiple of 128: the fused tcgen05 forward and
    # the tensor-core backward run on these (the small cases above take the
    # generic kernels).  bf16 throughout, as the reference runs only with matching
    # activation / parameter dtypes; 136 tokens = one full and one partial
    # 128-token tile; an elementwise sublayer keeps the fixture small.
    gw = torch.Generator().manual_seed(4321)

    def module_wide_case(kind, n, c, iters, t=136):
        torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gw)))
        if kind == "full":
            mod = R.MHCConnection_Fused(n, c, sinkhorn_iters=iters)
            with torch.no_grad():
                mod.phi_weight.copy_(torch.randn(n * c, 2 * n + n * n, generator=gw) * 0.02)
                mod.bias_res.add_(torch.randn(n, n, generator=gw) * 0.1)
        else:
            mod = RN.MHCConnection_FusedNoHres(n, c)
            with torch.no_grad():
                mod.phi_weight.copy_(torch.randn(n * c, 2 * n, generator=gw) * 0.02)
        with torch.no_grad():
            mod.bias_pre.copy_(torch.randn(n, generator=gw) * 0.1)
            mod.bias_post.copy_(torch.randn(n, generator=gw) * 0.1)
        mod = mod.to(torch.bfloat16)
        x = torch.randn(1, t, n * c, generator=gw).bfloat16().requires_grad_(True)
        y = mod._forward_ref(x, lambda z: F.silu(z) * 0.5)
        loss = y.float().pow(2).mean()
        names = [k for k, _ in mod.named_parameters()]
        leaves = [x] + [p for _, p in mod.named_parameters()]
        g = torch.autograd.grad(loss, leaves)
        return dict(n=n, C=c, iters=iters, sub="silu_half", x=x.detach(), w1=None, w2=None,
                    param_names=names, params=[p.detach().clone() for _, p in mod.named_parameters()],
                    out=y.detach(), loss=loss.detach(), grads=[t.detach() for t in g])

    out["module_full_bf16_c768_wide"] = module_wide_case("full", 4, 768, 20)
    out["module_nohres_bf16_c1024_wide"] = module_wide_case("nohres", 4, 1024, 0)

    path = os.path.join(HERE, "golden.pt")
    torch.save(out, path)
    print(f"wrote {path}: {os.path.getsize(path) / 1e6:.2f} MB, {len(out)} cases")


if __name__ == "__main__":
    main()
