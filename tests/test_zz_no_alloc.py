"""mhc_pre_fwd_noalloc: the workspace-free variant of mhc_pre_fwd.

It must give bit-identical results to mhc_pre_fwd with a caller workspace
(same kernels, same inputs), on two calls in a row that reuse its fixed
device scratch, on the generic path (which uses the scratch) and on the fused
path; and it must reject batches larger than its scratch before any CUDA call.
The file name sorts last so the GPU test also runs after every other test.
"""

import ctypes

import pytest
import torch

N, C, T = 4, 256, 3000
FD = 2 * N + N * N
ARGS = dict(with_res=1, apply_sinkhorn=1, iters=20, post_mult=2.0, pre_eps=1e-6, rms_eps=1e-6, sk_eps=1e-6)


def _lib():
    from model import _native as nat
    return nat, nat.load_library()


def test_noalloc_rejects_batches_beyond_its_scratch():
    nat, L = _lib()
    big_t = 2_000_000  # T*n*4 bytes = 32 MB > 16 MiB
    P = ctypes.c_void_p(16)  # never dereferenced: rejected first
    st = L.mhc_pre_fwd_noalloc(P, nat.BF16, big_t, N, C, P, P, P, P, P, P, P, nat.F32, 1, 1, 20,
                               2.0, 1e-6, 1e-6, 1e-6, P, None, P, P, nat.F32, P, P, None)
    assert st == -5
    msg = L.mhc_last_error().decode()
    assert "fixed device scratch" in msg and "4194304" in msg


def _outputs(dev):
    return dict(z=torch.empty(T, C, device=dev, dtype=torch.bfloat16),
                h_pre=torch.empty(T, N, device=dev), h_post=torch.empty(T, N, device=dev),
                h_res=torch.empty(T, N * N, device=dev), inv=torch.empty(T, device=dev),
                mix=torch.empty(T, FD, device=dev))


def _params(dev, gen):
    ps = [torch.randn(N * C, FD, generator=gen) * 0.02, torch.tensor(0.3), torch.randn(N, generator=gen) * 0.1,
          torch.tensor(0.2), torch.randn(N, generator=gen) * 0.1, torch.tensor(0.25),
          torch.eye(N) + torch.randn(N, N, generator=gen) * 0.1]
    return [p.to(dev) for p in ps]


def _call(nat, L, x, ps, o, workspace):
    common = [nat.ptr(x), nat.BF16, T, N, C] + [nat.ptr(p) for p in ps] + [
        nat.F32, ARGS["with_res"], ARGS["apply_sinkhorn"], ARGS["iters"], ARGS["post_mult"], ARGS["pre_eps"],
        ARGS["rms_eps"], ARGS["sk_eps"], nat.ptr(o["z"]), nat.ptr(o["h_pre"]), nat.ptr(o["h_post"]),
        nat.ptr(o["h_res"]), nat.F32, nat.ptr(o["inv"]), nat.ptr(o["mix"])]
    s = torch.cuda.current_stream().cuda_stream
    if workspace is None:
        st = L.mhc_pre_fwd_noalloc(*common, s)
        name = "mhc_pre_fwd_noalloc"
    else:
        st = L.mhc_pre_fwd(*common, nat.ptr(workspace), workspace.numel(), s)
        name = "mhc_pre_fwd"
    nat.check(st, name)


@pytest.mark.gpu
@pytest.mark.parametrize("policy", [1, 0], ids=["generic", "auto"])
def test_noalloc_matches_workspace_entry_point_twice_in_a_row(policy):
    nat, L = _lib()
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(21)
    ps = _params(dev, gen)
    xs = [torch.randn(T, N * C, generator=gen).bfloat16().to(dev) for _ in range(2)]
    prev = L.mhc_set_path_policy(policy)
    try:
        # two calls in a row through the shared fixed scratch, no sync between
        got = [_outputs(dev) for _ in xs]
        for x, o in zip(xs, got):
            _call(nat, L, x, ps, o, None)
        ws = nat.workspace(L.mhc_pre_fwd_workspace(T, N, C, 1), dev)
        want = [_outputs(dev) for _ in xs]
        for x, o in zip(xs, want):
            _call(nat, L, x, ps, o, ws)
        torch.cuda.synchronize()
    finally:
        L.mhc_set_path_policy(prev)
    assert L.mhc_device_error(1) == 0
    for g, w in zip(got, want):
        for k in g:
            assert torch.equal(g[k], w[k]), k
    # the two inputs differ, so the second call did not reuse stale scratch
    assert not torch.equal(got[0]["z"], got[1]["z"])
