"""Failure detection without a GPU fault: the bounded wait that every fused
kernel uses gives up after its cycle limit (or as soon as the kernel's abort
flag is raised), the kernel takes the fused kernels' give-up path (error code
in the device word and in the registered pinned host flag, NaN over the output
it owns) and exits normally, the Python layer raises on its next call, and the
CUDA context stays usable.  Argument checks and the Python-side check run on
the CPU."""

import ctypes

import pytest
import torch


def _lib():
    from model import _native as nat
    return nat, nat.lib()


def _run(L, limit, use_abort, poison=None):
    res = (ctypes.c_longlong * 2)()
    st = L.mhc_selftest_bounded_wait(limit, use_abort, ctypes.cast(res, ctypes.c_void_p),
                                     None if poison is None else poison.data_ptr(),
                                     0 if poison is None else poison.numel())
    return st, res[0], res[1]


def test_selftest_rejects_bad_limits():
    nat, L = _lib()
    res = (ctypes.c_longlong * 2)()
    r = ctypes.cast(res, ctypes.c_void_p)
    assert L.mhc_selftest_bounded_wait(0, 0, r, None, 0) == -3
    assert L.mhc_selftest_bounded_wait(5_000_000_000, 0, r, None, 0) == -3
    assert L.mhc_selftest_bounded_wait(1000, 0, None, None, 0) == -3
    assert L.mhc_selftest_bounded_wait(1000, 0, r, None, 8) == -3  # poison length without a buffer


def test_python_layer_raises_on_a_reported_give_up(monkeypatch):
    """The check every native call makes: a non-zero host error word raises
    before anything is launched; zero lets the call through."""
    nat, _ = _lib()
    word = ctypes.c_int(0)
    calls = []

    class FakeLib:
        def mhc_fake(self, *a):
            calls.append(a)
            return 0

    monkeypatch.setattr(nat, "_flag_word", word)
    monkeypatch.setattr(nat, "_lib", FakeLib())
    nat.call("mhc_fake", 1, 2)
    assert calls == [(1, 2)]
    word.value = 5
    with pytest.raises(RuntimeError, match="code 5: forward pre-aggregate"):
        nat.call("mhc_fake", 3)
    assert calls == [(1, 2)]
    word.value = 0
    nat.call("mhc_fake", 4)
    assert len(calls) == 2


def test_error_flag_must_be_pinned_host_memory():
    nat, L = _lib()
    pageable = (ctypes.c_int * 1)()
    st = L.mhc_set_error_flag(ctypes.cast(pageable, ctypes.c_void_p))
    assert st != 0


@pytest.mark.gpu
def test_wait_runs_out_and_context_survives():
    nat, L = _lib()
    nat.clear_device_error()
    nat._register_error_flag()
    limit = 20_000_000  # ~10 ms at the B200's clock
    poison = torch.zeros(1000, device="cuda")
    st, gave_up, cycles = _run(L, limit, 0, poison)
    assert st == 0
    assert gave_up == 1
    assert limit <= cycles < 20 * limit
    # the give-up path: NaN over the owned output, code 99 in both error words,
    # and the Python layer refuses the next call until the error is cleared
    assert torch.isnan(poison).all()
    assert nat.device_error_code() == 99
    with pytest.raises(RuntimeError, match="code 99"):
        nat.call("mhc_abi_version")
    assert L.mhc_device_error(0) == 99
    nat.clear_device_error()
    assert nat.device_error_code() == 0 and L.mhc_device_error(0) == 0
    # the abort flag ends the wait long before the limit
    st, gave_up, cycles = _run(L, 2_000_000_000, 1)
    assert st == 0
    assert gave_up == 1
    assert cycles < 50_000_000
    nat.clear_device_error()
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
