"""ctypes binding of ``libmhc_b200.so`` (the C ABI in ``include/mhc_b200.h``).

This is the only place Python touches the native library.  Every call passes
raw device pointers, sizes, dtype codes and the current CUDA stream; a
non-zero status raises ``RuntimeError`` with the library's message.  There is
no CPU path: a CPU tensor, a missing library or a CUDA-less process is an
error, raised before anything is launched.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MHC_B200_LIB") or os.path.join(_HERE, "libmhc_b200.so")

F32, BF16, F16 = 0, 1, 2
_DTYPE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes)
_PROTOS = {
    "mhc_abi_version": (_I, []),
    "mhc_last_error": (ctypes.c_char_p, []),
    "mhc_device_sm_count": (_I, []),
    "mhc_pre_fwd_workspace": (_SZ, [_I64, _I, _I, _I]),
    "mhc_pre_fwd": (_I, [_P, _I, _I64, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I,
                         _F, _F, _F, _F, _P, _P, _P, _P, _I, _P, _P, _P, _SZ, _P]),
    "mhc_post_pre_fwd_workspace": (_SZ, [_I64, _I, _I, _I]),
    "mhc_post_pre_fwd": (_I, [_P, _I, _P, _P, _I, _P, _I, _P, _I64, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I,
                              _I, _I, _I, _F, _F, _F, _F, _P, _P, _P, _P, _I, _P, _P, _P, _I, _F, _P, _P,
                              _SZ, _P]),
    "mhc_post_fwd": (_I, [_P, _I, _P, _I, _P, _I, _P, _I, _P, _I64, _I, _I, _I, _I, _F, _P, _P]),
    "mhc_post_bwd": (_I, [_P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _P, _P, _P, _I64, _I, _I, _P]),
    "mhc_pre_bwd_workspace": (_SZ, [_I64, _I, _I, _I, _I, _I]),
    "mhc_pre_bwd": (_I, [_P, _I, _I64, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I,
                         _F, _F, _F, _F, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                         _P, _P, _P, _P, _SZ, _P]),
    "mhc_sinkhorn_fwd": (_I, [_P, _I, _P, _I, _I64, _I, _I, _F, _P]),
    "mhc_sinkhorn_bwd": (_I, [_P, _I, _P, _I, _P, _I, _I64, _I, _I, _F, _P]),
    "mhc_head_fwd_workspace": (_SZ, [_I64, _I, _I]),
    "mhc_head_fwd": (_I, [_P, _I, _I64, _I, _I, _P, _P, _P, _I, _F, _F, _P, _P, _P, _P, _SZ, _P]),
    "mhc_head_bwd_workspace": (_SZ, [_I64, _I, _I]),
    "mhc_head_bwd": (_I, [_P, _I, _I64, _I, _I, _P, _P, _P, _I, _F, _F, _P, _P, _P, _P, _P, _P,
                          _P, _P, _SZ, _P]),
    "mhc_stream_expand_fwd": (_I, [_P, _P, _I, _I64, _I, _I, _P]),
    "mhc_stream_expand_bwd": (_I, [_P, _P, _I, _I64, _I, _I, _P]),
    "mhc_set_path_policy": (_I, [_I]),
    "mhc_last_path": (_I, []),
    "mhc_device_error": (_I, [_I]),
    "mhc_set_error_flag": (_I, [_P]),
    "mhc_selftest_bounded_wait": (_I, [ctypes.c_longlong, _I, _P, _P, ctypes.c_longlong]),
    "mhc_pre_fwd_noalloc": (_I, [_P, _I, _I64, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I,
                                 _F, _F, _F, _F, _P, _P, _P, _P, _I, _P, _P, _P]),
}

PATH_AUTO, PATH_GENERIC, PATH_TWO_READ, PATH_SINGLE_READ, PATH_FUSED_POST_PRE = 0, 1, 2, 3, 4
# mhc_last_path() after a forward call: the kernel family that ran
RAN_GENERIC, RAN_TWO_READ, RAN_SINGLE_READ, RAN_POST_PRE, RAN_FP32_STREAM = 0, 1, 2, 3, 4

EXPORTED = tuple(_PROTOS)

_lib = None
# re-entrant: registering the error flag (under the lock) loads the library
# (which takes the lock again) when the first native call is a call()
_lock = threading.RLock()


def load_library(path: str | None = None):
    """Load (once) and return the ctypes handle; raises if the file is missing."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"mHC native library not found at {p}; build it with "
                f"`python minimind-mhc_b200/build.py` (there is no CPU fallback)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in _PROTOS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def lib():
    return _lib if _lib is not None else load_library()


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPE[t]
    except KeyError:
        raise TypeError(f"mHC kernels support float32/bfloat16/float16, got {t}") from None


def ptr(t):
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "mHC B200 kernels run on CUDA tensors only (this build has no CPU path); "
                f"got a tensor on {t.device}")


def check(status: int, what: str):
    if status != 0:
        msg = lib().mhc_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed with status {status}: {msg}")


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------------------
# Device-side give-ups reach the caller
#
# Every wait inside the fused kernels is bounded.  A kernel whose wait runs out
# writes its error code into a pinned host word registered here
# (mhc_set_error_flag), overwrites the outputs it owns with NaN and exits.
# Reading the word costs no synchronisation, so every call below checks it and
# raises once a kernel has given up (the give-up of one call is seen by a later
# one, as with CUDA's asynchronous errors).  The error stays raised until
# clear_device_error().
# ---------------------------------------------------------------------------

ERROR_ROLES = {1: "forward TMA producer", 2: "forward MMA issuer", 3: "forward row warps",
               4: "forward coefficient warp", 5: "forward pre-aggregate warps", 6: "forward Sinkhorn warp",
               11: "backward TMA producer", 12: "backward MMA issuer", 13: "backward epilogue",
               14: "backward prep warps", 21: "single-read forward TMA producer",
               22: "single-read forward MMA issuer", 23: "single-read forward ingest warps",
               24: "single-read forward coefficient warp", 25: "single-read forward Sinkhorn warps",
               26: "single-read forward z warps", 31: "merge + coefficient TMA producer",
               32: "merge + coefficient MMA issuer", 33: "merge + coefficient row warps",
               34: "merge + coefficient coefficient warp", 35: "merge + coefficient pre-aggregate warps",
               36: "merge + coefficient Sinkhorn warp", 37: "merge + coefficient merge warps",
               99: "bounded-wait self-test"}

_flag_tensor = None   # pinned int32 host tensor registered with the library
_flag_word = None     # ctypes view of its first element


def _register_error_flag():
    global _flag_tensor, _flag_word
    with _lock:
        if _flag_word is not None:
            return
        t = torch.zeros(4, dtype=torch.int32).pin_memory()
        check(lib().mhc_set_error_flag(t.data_ptr()), "mhc_set_error_flag")
        _flag_tensor = t
        _flag_word = ctypes.c_int.from_address(t.data_ptr())


def device_error_code() -> int:
    """The first give-up code a fused kernel wrote since the last clear (0 = none)."""
    return 0 if _flag_word is None else int(_flag_word.value)


def raise_if_device_error():
    code = device_error_code()
    if code:
        role = ERROR_ROLES.get(code, "unknown role")
        raise RuntimeError(
            f"an mHC kernel gave up on a bounded device wait (code {code}: {role}); the outputs it owned "
            f"were overwritten with NaN.  Call model._native.clear_device_error() to continue.")


def clear_device_error():
    """Resets the host word and the device error words (synchronises the device)."""
    if torch.cuda.is_available():
        lib().mhc_device_error(1)
    if _flag_word is not None:
        _flag_word.value = 0


def call(name: str, *args):
    if _flag_word is None:
        _register_error_flag()
    raise_if_device_error()
    check(getattr(lib(), name)(*args), name)
