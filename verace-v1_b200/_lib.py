"""ctypes binding of ``libverace_b200.so`` (the C ABI declared in include/verace_b200.h).

The library is built in-tree by ``build.py``.  There is no fallback: if the library
is missing, or a CUDA call fails, the caller gets a RuntimeError.
"""
import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libverace_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "verace_b200.h")

VERACE_OK = 0
F32, BF16, F16 = 0, 1, 2

_c_size = ctypes.c_size_t
_p = ctypes.c_void_p
_i = ctypes.c_int

# name -> (restype, argtypes)
_SIGNATURES = {
    "verace_version": (_i, []),
    "verace_last_error": (ctypes.c_char_p, []),
    "verace_kernel_launches": (ctypes.c_ulonglong, []),
    "verace_device_status": (_i, [_p]),
    "verace_sssd_scan_workspace": (_c_size, [_i, _i, _i, _i]),
    "verace_sssd_scan": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _c_size, _p]),
    "verace_sssd_scan_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p]),
    "verace_cham_scan_workspace": (_c_size, [_i, _i, _i, _i]),
    "verace_cham_scan": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p, _c_size, _p]),
    "verace_cham_unitarity_workspace": (_c_size, [_i, _i]),
    "verace_cham_unitarity": (_i, [_p, _p, _i, _i, _p, _p, _c_size, _p]),
    "verace_cham_scan_unitary": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p, _c_size, _p]),
    "verace_cham_retract_workspace": (_c_size, [_i, _i]),
    "verace_cham_retract": (_i, [_p, _p, _p, _p, _i, _i, _i, _p, _c_size, _p]),
    "verace_decode_workspace": (_c_size, [_i, _i]),
    "verace_decode_step": (_i, [_p] * 13 + [_i] * 6 + [_p, _c_size, _p]),
    "verace_mixer_prologue": (_i, [_p, ctypes.c_longlong] + [_p] * 5 + [ctypes.c_longlong] + [_i] * 5 + [_p]),
    "verace_decode_lazy_workspace": (_c_size, [_i, _i]),
    "verace_decode_pending_bytes": (_c_size, [_i, _i, _i]),
    "verace_decode_cham_lazy": (_i, [_p] * 7 + [_i, _p, _i, _i, _i, _p, _c_size, _p]),
    "verace_decode_cham_flush": (_i, [_p, _p, _p, _i, _i, _i, _p]),
    "verace_decode_cham_lazy_projected": (_i, [_p, ctypes.c_longlong, _p, _p, _p, _i, _p, _i, _i, _i, _p, _c_size,
                                               _p]),
    "verace_rmsnorm": (_i, [_p, _p, _p, ctypes.c_longlong, _i, ctypes.c_float, _i, _p]),
    "verace_add_rmsnorm": (_i, [_p, _p, _i, _p, ctypes.c_float, _p, ctypes.c_float, _p, ctypes.c_longlong, _i, _i,
                                _p]),
    "verace_mcmoe_workspace": (_c_size, [ctypes.c_longlong, _i, _i, _i, _i]),
    "verace_mcmoe_route": (_i, [_p, ctypes.c_longlong, _i, _i, _p, _p, _i, _p]),
    "verace_mcmoe_projection": (_i, [_p] * 6 + [_i, _p, ctypes.c_longlong, _i, _i, _i, _i, _i, _p, _c_size, _p]),
    "verace_situ_glu": (_i, [_p, _p, ctypes.c_longlong, _p, ctypes.c_longlong, _i, ctypes.c_float, ctypes.c_float,
                             _i, _p]),
}

_lib = None


def header_symbols(path=HEADER_PATH):
    """Names of every function declared in include/verace_b200.h."""
    text = open(path).read()
    return sorted(set(re.findall(r"VERACE_API\s+[\w\s\*]+?\b(verace_\w+)\s*\(", text)))


def lib():
    """Load (once) and return the ctypes library handle."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python verace-v1_b200/build.py` "
                "(there is no CPU or Python fallback for this path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc, what):
    if rc != VERACE_OK:
        msg = lib().verace_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")
