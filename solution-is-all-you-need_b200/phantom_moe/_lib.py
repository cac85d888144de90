"""ctypes binding of ``libphmoe.so`` (the C ABI declared in ``include/phmoe.h``).

The library is built in-tree (``phantom_moe/lib/libphmoe.so``) by
``phantom_moe._build``. There is no fallback: if the library is missing or
fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libphmoe.so"

PHMOE_OK = 0
PHMOE_ERR_INVALID_ARG = -1
PHMOE_ERR_UNSUPPORTED = -2
PHMOE_ERR_WORKSPACE = -3
PHMOE_ERR_CUDA = -4
PHMOE_ERR_ALIGNMENT = -5

DTYPE_F32 = 0
DTYPE_BF16 = 1

SCORING_SOFTMAX = 0
SCORING_SIGMOID = 1

PATH_AUTO = 0
PATH_DECODE = 1
PATH_PREFILL = 2
EP_HANDLE_BYTES = 64  # PHMOE_EP_HANDLE_BYTES

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/phmoe.h
SIGNATURES = {
    "phmoe_version": (_I, []),
    "phmoe_status_string": (ctypes.c_char_p, [_I]),
    "phmoe_last_error": (ctypes.c_char_p, []),
    "phmoe_workspace_size": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "phmoe_select_path": (_I, [_I, _I, _I, _I, _I, _I, _I, _I]),
    "phmoe_router": (_I, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "phmoe_dispatch_scratch_size": (_SZ, [_I, _I, _I]),
    "phmoe_dispatch": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _SZ, _P]),
    "phmoe_expert_ffn_decode": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _P,
                                     _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "phmoe_expert_ffn_prefill": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _P,
                                      _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "phmoe_combine": (_I, [_P, _P, _P, _I, _I, _I, _P, _I, _P]),
    "phmoe_fx_rows_size": (_SZ, [_LL, _I, _I]),
    "phmoe_fx_rows": (_I, [_P, _I, _LL, _I, _I, _P, _P]),
    "phmoe_gather_rows": (_I, [_P, _LL, _P, _I, _LL, _P, _P]),
    "phmoe_ep_create": (_I, [_I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "phmoe_ep_create_ex": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "phmoe_ep_connect": (_I, [_P, _P]),
    "phmoe_ep_destroy": (_I, [_P]),
    "phmoe_ep_workspace_size": (_SZ, [_P, _I]),
    "phmoe_ep_layer": (_I, [_P, _P, _I, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "phmoe_ep_layer_ex": (_I, [_P, _P, _I, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _SZ,
                               _P]),
    "phmoe_moe_layer": (_I, [_P, _I, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                             _P, _P, _P, _P, _SZ, _P]),
    "phmoe_moe_layer_noalloc": (_I, [_P, _I, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                     _P, _P, _P, _P]),
    "phmoe_router_ex": (_I, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _I, ctypes.c_float, _P, _P, _P, _P]),
    "phmoe_workspace_size_ex": (_SZ, [_I, _I, _I, _I, _I, _I, _I]),
    "phmoe_moe_layer_ex": (_I, [_P, _I, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _I, _I,
                                _I, _P, ctypes.c_float, _I, _P, _P, _P, _P, _SZ, _P]),
    "phmoe_gguf_q4_0_to_packed": (_I, [_P, _LL, _I, _P, _P, _P]),
    "phmoe_gguf_q4_k_to_packed": (_I, [_P, _LL, _I, _I, _P, _P, _P]),
    "phmoe_gguf_q4_k_dequantize": (_I, [_P, _LL, _P, _P]),
    "phmoe_quantize_int4": (_I, [_P, _I, _LL, _I, _I, _P, _P, _P]),
    "phmoe_kernel_launch_count": (ctypes.c_ulonglong, []),
    "phmoe_profile_begin": (_I, [_I]),
    "phmoe_profile_end": (_I, [_P, _I, _P]),
    "phmoe_device_error": (_I, [_I]),
}

NUM_STAGES = 5
STAGE_NAMES = ("router", "dispatch", "ffn_gateup", "ffn_down", "combine")


class PhmoeError(RuntimeError):
    """A libphmoe entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str):
        self.status = status
        super().__init__(f"{fn} failed with status {status}: {detail}")


_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"libphmoe.so not found at {p}; build it with `python -m phantom_moe._build` "
            "(or __graft_entry__.build()). There is no CPU fallback.")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(fn_name: str, status: int) -> None:
    if status != PHMOE_OK:
        lib = load()
        detail = (lib.phmoe_last_error() or b"").decode() or lib.phmoe_status_string(status).decode()
        raise PhmoeError(fn_name, status, detail)


def call(fn_name: str, *args) -> None:
    """Call an int-returning entry point and raise on a non-zero status."""
    lib = load()
    check(fn_name, getattr(lib, fn_name)(*args))
