"""The C-ABI library on the host: it loads without a GPU, exports every
symbol include/ress_sm100.h declares, and rejects bad arguments with an
error code before touching the device (no compute call is made here)."""

import ctypes
import os
import re

import pytest

from ress_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ress_sm100.h")


def _declared():
    src = open(HEADER).read()
    return set(re.findall(r"^\w[\w\s\*]*?\b(ress_\w+)\(", src, re.M))


def test_header_and_bindings_agree():
    assert _declared() == set(_lib.SIGNATURES)


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load()
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for name in _declared():
        assert hasattr(raw, name), name
    assert lib.ress_version() >= 1
    assert b"invalid argument" in lib.ress_error_string(_lib.RESS_OK - 1)


def test_workspace_size():
    lib = _lib.load()
    assert lib.ress_workspace_size(0, 1, 1, 1) == 0
    small = lib.ress_workspace_size(16, 5476, 5496, 85)
    big = lib.ress_workspace_size(16, 43808, 43968, 684)
    assert 0 < small < big


@pytest.mark.parametrize("call", [
    lambda L: L.ress_score_quant(None, None, None, 0, 1, 1, 1, 0, 64, 0, 0, 0, *([None] * 10), None),
    lambda L: L.ress_pool_quant_q(None, 0, 1, 1, 1, 0, 64, 0, 0, 0, None, None, None, None),
    lambda L: L.ress_predict(0, None, None, 1, 1, 1, 1, None, None, None),
    lambda L: L.ress_baseline(0, None, 1, 10, 0, 0.0, 3, None, None),
    lambda L: L.ress_hess_adjust(None, None, 1, 16, 4, 10, 0.0, 1.0, 1000, 2, None, None, None),
    lambda L: L.ress_restore_swap(1, None, None, None, None, 1, 16, 4, 10, 9, 5, None, 1, None, None, None,
                                  None, 10, 1, 0, None, None, None),
    lambda L: L.ress_select_prob(0, None, None, 4, 10, None, None, None, 10, 0, 0, None, None),
    lambda L: L.ress_top_m_mask(0, None, None, 4, 10, 1, None, None),
    lambda L: L.ress_round_step(None, None, None, 1, 0, None, None, None, None, None, 4, 10, 1, 0, 1, 1e-6,
                                None, None, None),
    lambda L: L.ress_map_to_lists(None, 4, 10, None, None, 10, None, None),
    lambda L: L.ress_sparse_attn(None, None, None, None, None, 1, 128, 64, None, None, 1, 0.125, None, 0, 0,
                                 128, 0, None, None),
    lambda L: L.ress_sparse_attn_sched(None, None, None, None, None, 1, 128, 64, None, None, 1, 0.125, None, 0, 0,
                                       128, 0, None, None, None),
    lambda L: L.ress_sparse_attn_split(None, None, None, None, None, 1, 128, 64, None, None, 1, 0.125, None, 0, 0,
                                       128, 0, None, None, 0, None, None, None),
    lambda L: L.ress_qkv_prologue(None, 1, 1, 16, 4, None, None, None, None, 1e-5, None, None, None, 0, None, None,
                                  None, None),
])
def test_bad_arguments_are_rejected_on_the_host(call):
    assert call(_lib.load()) == -1  # RESS_E_ARG


def test_dtype_and_shape_codes():
    lib = _lib.load()
    fake = ctypes.c_void_p(16)  # never dereferenced: rejected before any launch
    assert lib.ress_baseline(7, fake, 1, 10, 0, 0.0, 3, fake, None) == -2  # RESS_E_DTYPE
    assert lib.ress_baseline(0, fake, 1, 20000, 1, 0.97, 3, fake, None) == -3  # RESS_E_SHAPE
