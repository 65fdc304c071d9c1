"""Loader for libress_sm100.so, the C ABI declared in include/ress_sm100.h.

The library is the only compute path of this package.  There is no CPU or
PyTorch fallback: if the library or a CUDA device is missing, every kernel
wrapper raises.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libress_sm100.so")

RESS_OK = 0
RESS_E_ARG = -1
RESS_E_DTYPE = -2
RESS_E_SHAPE = -3
RESS_E_LAUNCH = -4
RESS_E_NO_DEVICE = -5
RESS_E_SCRATCH = -6
NOALLOC_SCRATCH_BYTES = 4 << 20
RESS_F32, RESS_BF16 = 0, 1
STATUS_HESS_NO_CONVERGENCE = 1
STATUS_ATTN_WAIT_TIMEOUT = 2
STATUS_LIST_OVERFLOW = 4

# every symbol include/ress_sm100.h declares, with its ctypes signature
_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_longlong
_F = ctypes.c_float
SIGNATURES = {
    "ress_version": (_I, []),
    "ress_check_scale_division": (_I, [_P, _P]),
    "ress_qkv_prologue": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _F, _P, _P, _P, _I, _P, _P, _P, _P]),
    "ress_qkv_prologue_scored": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _F, _P, _P, _P, _I, _P, _P, _P, _P, _P,
                                      _P, _P]),
    "ress_error_string": (ctypes.c_char_p, [_I]),
    "ress_workspace_size": (ctypes.c_size_t, [_I, _I, _I, _I]),
    "ress_score_quant": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _L, _L, _L,
                              _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "ress_pool_quant_q": (_I, [_P, _I, _I, _I, _I, _I, _I, _L, _L, _L, _P, _P, _P, _P]),
    "ress_pool_quant_kv": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _L, _L, _L, _P, _P, _P, _P, _P,
                                _P, _P, _P]),
    "ress_predict": (_I, [_I, _P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "ress_baseline": (_I, [_I, _P, _I, _I, _I, _F, _I, _P, _P]),
    "ress_hess_adjust": (_I, [_P, _P, _I, _I, _I, _I, _F, _F, _I, _I, _P, _P, _P]),
    "ress_restore_swap": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P,
                               _P, _P, _I, _I, _I, _P, _P, _P]),
    "ress_restore_swap_noalloc": (_I, [_I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P,
                                       _P, _P, _I, _I, _I, _P, _P]),
    "ress_select_prob": (_I, [_I, _P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _P, _P]),
    "ress_top_m_mask": (_I, [_I, _P, _P, _I, _I, _I, _P, _P]),
    "ress_round_step": (_I, [_P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F,
                             _P, _P, _P]),
    "ress_map_to_lists": (_I, [_P, _I, _I, _P, _P, _I, _P, _P]),
    "ress_sparse_attn": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _I, _F, _P, _L, _L, _I,
                              _I, _P, _P]),
    "ress_sparse_attn_sched": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _I, _F, _P, _L, _L, _I,
                                    _I, _P, _P, _P]),
    "ress_sparse_attn_split": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _I, _F, _P, _L, _L, _I,
                                    _I, _P, _P, _I, _P, _P, _P]),
    "ress_dense_attn": (_I, [_P, _P, _P, _I, _I, _I, _L, _L, _L, _L, _F, _P, _I, _I, _L, _L, _L, _I, _L, _I,
                             _P, _P]),
}

_lib = None


class RessError(RuntimeError):
    pass


def load(path: str = LIB_PATH):
    """Load the library (once) and bind every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RessError(f"{path} is missing: build it with `python -m ress_b200.build` "
                        "(this package has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(code: int, what: str):
    if code != RESS_OK:
        msg = load().ress_error_string(code).decode()
        raise RessError(f"{what} failed: {msg} (code {code})")
