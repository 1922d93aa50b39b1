"""C-ABI library checks that need no GPU.

The shared library must load, export every entry point declared in
include/mhc_b200.h (and the Python binding must declare the same set), and
reject bad arguments on the host — before any CUDA call — with the documented
status codes.  No kernel is launched here.
"""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mhc_b200.h")


def _header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mhc_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from model import _native
    if not os.path.exists(_native.LIB_PATH):
        import __graft_entry__
        __graft_entry__.build()
    return _native.load_library()


def test_header_declares_entry_points():
    names = _header_functions()
    for must in ("mhc_pre_fwd", "mhc_post_fwd", "mhc_pre_bwd", "mhc_post_bwd", "mhc_sinkhorn_fwd",
                 "mhc_sinkhorn_bwd", "mhc_head_fwd", "mhc_head_bwd", "mhc_stream_expand_fwd",
                 "mhc_stream_expand_bwd"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    from model import _native
    names = _header_functions()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in mhc_b200.h but not exported"
    assert set(names) == set(_native.EXPORTED), "ctypes prototypes and header disagree"
    assert lib.mhc_abi_version() == 1


def test_host_validation_rejects_bad_arguments(lib):
    P = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # bad n
    st = lib.mhc_post_fwd(P, 1, P, 0, P, 0, P, 1, P, 8, 3, 64, 0, 0, 0.0, None, None)
    assert st == -3 and b"n must be" in lib.mhc_last_error()
    # bad dtype
    st = lib.mhc_post_fwd(P, 7, P, 0, P, 0, P, 1, P, 8, 4, 64, 0, 0, 0.0, None, None)
    assert st == -2
    # NULL input
    st = lib.mhc_post_fwd(None, 1, None, 0, P, 0, P, 1, P, 8, 4, 64, 0, 0, 0.0, None, None)
    assert st == -1
    # misaligned bf16 pointer
    st = lib.mhc_post_fwd(ctypes.c_void_p(17), 1, None, 0, P, 0, P, 1, P, 8, 4, 64, 0, 0, 0.0, None, None)
    assert st == -4
    # h_res_out without logits
    st = lib.mhc_post_fwd(P, 1, None, 0, P, 0, P, 1, P, 8, 4, 64, 0, 0, 0.0, P, None)
    assert st == -1
    # pre_fwd: workspace too small
    st = lib.mhc_pre_fwd(P, 1, 8, 4, 64, P, P, P, P, P, P, P, 0, 1, 1, 20, 2.0, 1e-6, 1e-6, 1e-6,
                         P, None, P, P, 0, P, P, P, 0, None)
    assert st == -5
    # sinkhorn bwd with a trajectory that cannot fit
    st = lib.mhc_sinkhorn_bwd(P, 0, P, 0, P, 0, 4, 16, 1000, 1e-6, None)
    assert st == -7
    # res gradients requested without the H_res segment
    st = lib.mhc_pre_bwd(P, 1, 8, 4, 64, P, P, P, P, P, None, None, 0, 0, 0, 0, 2.0, 1e-6, 1e-6, 0.0,
                         P, P, P, None, None, P, 0, None, P, P, P, P, P, P, None, None, P, 1 << 20, None)
    assert st == -1


def test_empty_batch_is_a_no_op(lib):
    # T == 0 returns OK without touching any pointer or the device
    assert lib.mhc_post_fwd(None, 1, None, 0, None, 0, None, 1, None, 0, 4, 64, 0, 0, 0.0, None, None) == 0
    assert lib.mhc_sinkhorn_fwd(None, 0, None, 0, 0, 4, 20, 1e-6, None) == 0
    assert lib.mhc_stream_expand_fwd(None, None, 1, 0, 4, 64, None) == 0


def test_path_policy_switch(lib):
    prev = lib.mhc_set_path_policy(1)
    assert lib.mhc_set_path_policy(0) == 1
    lib.mhc_set_path_policy(prev)
    assert lib.mhc_set_path_policy(prev) == prev


def test_workspace_queries(lib):
    a = lib.mhc_pre_fwd_workspace(32768, 4, 768, 1)
    assert a >= 32768 * 4 * 4
    b = lib.mhc_pre_bwd_workspace(32768, 4, 768, 1, 1, 20)
    assert b >= 32768 * 24 * 4
    assert lib.mhc_pre_bwd_workspace(1, 3, 768, 1, 1, 20) == 0  # invalid n


def test_first_native_call_loads_the_library_without_deadlock():
    """A process whose first native call is model._native.call() (the library
    not loaded yet) registers the error flag under the module lock, which loads
    the library under the same lock: the lock must be re-entrant.  Run in a
    fresh interpreter with pinning stubbed out (no GPU here); the flag
    registration then fails with a RuntimeError instead of hanging."""
    import subprocess
    import sys as _sys
    pkg = os.path.join(ROOT, "minimind-mhc_b200")
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import torch\n"
        "torch.Tensor.pin_memory = lambda self: self\n"
        "from model import _native as nat\n"
        "try:\n"
        "    nat.call('mhc_abi_version')\n"
        "except RuntimeError:\n"
        "    pass\n"
        "print('returned')\n" % pkg)
    r = subprocess.run([_sys.executable, "-c", code], capture_output=True, timeout=60)
    assert b"returned" in r.stdout, r.stderr.decode(errors="replace")[-2000:]
