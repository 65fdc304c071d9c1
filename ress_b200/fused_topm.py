"""Exact per-row top-m mask, ties to the lowest index.

Same contract as the reference's Triton ``scoring/fused_topm.py``
(``top_m_mask`` :109-136, ``can_use`` :97-100), served by the sm_100a kernel
``ress_top_m_mask``.  There is no 4096-column limit: rows up to 32 K
columns fit in shared memory.
"""

from __future__ import annotations

import torch

from . import kernels as K

MAX_K = 32768
_SUPPORTED_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def can_use(quality):
    return quality.is_cuda and quality.dtype in _SUPPORTED_DTYPES and 0 < quality.shape[-1] <= MAX_K


def top_m_mask(quality, counts, largest=True):
    """(..., k_blk) quality, (...) counts -> (..., k_blk) bool."""
    q = quality if quality.dtype != torch.float16 else quality.float()
    c = counts.clamp(min=0, max=quality.shape[-1])
    return K.top_m_mask(q, c, largest=largest)
