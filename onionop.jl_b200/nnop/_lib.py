"""ctypes binding of ``libnnop_b200.so``.

This module is the Python counterpart of the Julia ``ccall`` shim: it declares
every entry point of ``include/nnop_b200.h`` with its C signature.  It has no
fallback: if the library is missing the import of :mod:`nnop` fails.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

from . import _build

LIB_PATH = pathlib.Path(os.environ.get("NNOP_B200_LIB", str(_build.LIB_PATH)))

F32, F16, BF16 = 0, 1, 2
OK, ERR_SHAPE, ERR_DTYPE, ERR_ARG, ERR_WORKSPACE, ERR_CUDA, ERR_ALIGN = 0, -1, -2, -3, -4, -5, -6

_vp = C.c_void_p
_i64 = C.c_int64
_int = C.c_int
_f = C.c_float
_sz = C.c_size_t

# name -> (restype, argtypes); mirrors include/nnop_b200.h
SIGNATURES = {
    "nnop_abi_version": (_int, []),
    "nnop_last_error": (C.c_char_p, []),
    "nnop_status_string": (C.c_char_p, [_int]),
    "nnop_device_wait_timeouts": (_int, []),
    "nnop_kernel_timing": (None, [_int]),
    "nnop_kernel_timing_read": (_int, [_int, C.POINTER(C.c_double), C.POINTER(_int)]),
    "nnop_flash_attention_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                        _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "nnop_flash_attention_fwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _int, _int]),
    "nnop_flash_attention_bwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _int, _int]),
    "nnop_flash_attention_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                        _vp, _sz, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "nnop_flash_attention_bwd_reuse": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                              _vp, _sz, _vp, _sz, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int,
                                              _vp]),
    "nnop_flash_attention_bwd_workspace_size_reuse": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _int, _sz, _int]),
    "nnop_flash_attention_fwd_pair_per_head": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                                      _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "nnop_flash_attention_bwd_pair_per_head_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _int]),
    "nnop_flash_attention_bwd_pair_per_head": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                                      _vp, _sz, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int,
                                                      _vp]),
    "nnop_flash_attention_rope_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                             _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "nnop_flash_attention_rope_bwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _int]),
    "nnop_flash_attention_rope_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                             _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "nnop_online_softmax_fwd": (_int, [_vp, _vp, _i64, _i64, _int, _vp]),
    "nnop_online_softmax_bwd": (_int, [_vp, _vp, _vp, _i64, _i64, _int, _vp]),
    "nnop_rms_norm_fwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _f, _f, _int, _vp]),
    "nnop_rms_norm_bwd_workspace_size": (_sz, [_i64, _i64]),
    "nnop_rms_norm_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _f, _int, _vp]),
    "nnop_rms_norm_bwd_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _int, _vp]),
    "nnop_add_rms_norm_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _f, _int, _vp]),
    "nnop_add_rms_norm_bwd_workspace_size": (_sz, [_i64, _i64]),
    "nnop_add_rms_norm_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _f, _int, _vp]),
    "nnop_layer_norm_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _int, _vp]),
    "nnop_layer_norm_bwd_workspace_size": (_sz, [_i64, _i64]),
    "nnop_layer_norm_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _int, _vp]),
    "nnop_llama_rope": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f, _int, _vp]),
    "nnop_llama_rope_cos_sin": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
}


class NNopError(RuntimeError):
    """A non-OK status from the library (the reference raises ``error(...)``)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class NNopShapeError(NNopError, ValueError):
    pass


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"libnnop_b200.so not found at {LIB_PATH}; build it with "
            "`python onionop.jl_b200/nnop/_build.py` (there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status: int) -> None:
    if status != OK:
        msg = lib.nnop_last_error().decode(errors="replace")
        if status == ERR_SHAPE:
            raise NNopShapeError(status, msg)
        raise NNopError(status, msg)
