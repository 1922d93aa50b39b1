"""Failure detection without a GPU fault: the bounded wait that every fused
kernel uses gives up after its cycle limit (or as soon as the kernel's abort
flag is raised), the kernel records that and exits normally, and the CUDA
context stays usable for the next call.  Argument checks run on the CPU."""

import ctypes

import pytest
import torch


def _lib():
    from model import _native as nat
    return nat, nat.lib()


def _run(L, limit, use_abort):
    res = (ctypes.c_longlong * 2)()
    st = L.mhc_selftest_bounded_wait(limit, use_abort, ctypes.cast(res, ctypes.c_void_p))
    return st, res[0], res[1]


def test_selftest_rejects_bad_limits():
    nat, L = _lib()
    res = (ctypes.c_longlong * 2)()
    assert L.mhc_selftest_bounded_wait(0, 0, ctypes.cast(res, ctypes.c_void_p)) == -3
    assert L.mhc_selftest_bounded_wait(5_000_000_000, 0, ctypes.cast(res, ctypes.c_void_p)) == -3
    assert L.mhc_selftest_bounded_wait(1000, 0, None) == -3


@pytest.mark.gpu
def test_wait_runs_out_and_context_survives():
    nat, L = _lib()
    limit = 20_000_000  # ~10 ms at the B200's clock
    st, gave_up, cycles = _run(L, limit, 0)
    assert st == 0
    assert gave_up == 1
    assert limit <= cycles < 20 * limit
    # the abort flag ends the wait long before the limit
    st, gave_up, cycles = _run(L, 2_000_000_000, 1)
    assert st == 0
    assert gave_up == 1
    assert cycles < 50_000_000
    # the context is still usable: a fused-kernel call runs and agrees with the generic path
    from model.mhc_fused import MHCConnection_Fused
    torch.manual_seed(0)
    mod = MHCConnection_Fused(4, 256, sinkhorn_iters=20).cuda()
    x = torch.randn(1, 512, 4 * 256, device="cuda").bfloat16()
    y = mod(x, lambda z: z)
    prev = L.mhc_set_path_policy(1)
    y_gen = mod(x, lambda z: z)
    L.mhc_set_path_policy(prev)
    torch.cuda.synchronize()
    assert L.mhc_device_error(1) == 0
    assert (y.float() - y_gen.float()).abs().max().item() <= 2 ** -7 * y_gen.float().abs().max().item()
