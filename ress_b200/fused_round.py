"""One restore-swap round over precomputed big tensors.

Same contract as the reference's Triton ``scoring/fused_round.py``
(``fused_round_step`` :234-277, ``can_use`` :219-231, ``_step_dtypes``
:202-216), served by the sm_100a kernel ``ress_round_step`` without the
4096-column limit.
"""

from __future__ import annotations

import torch

from . import kernels as K

MAX_K = 25600
_SUPPORTED = (torch.float32, torch.bfloat16)


def _step_dtypes(P, term_k, s_sq, big_dtype, knorm_dtype=None):
    raw_dtype = torch.promote_types(torch.promote_types(P.dtype, term_k.dtype), big_dtype)
    q_dtype = knorm_dtype if knorm_dtype is not None else torch.promote_types(raw_dtype, s_sq.dtype)
    return raw_dtype, q_dtype


def can_use(P, s_sq, term_k, drop_mask, big_dtype, knorm_dtype=None):
    if not P.is_cuda or big_dtype not in _SUPPORTED:
        return False
    if not (0 < P.shape[-1] <= MAX_K):
        return False
    if not (s_sq.shape == P.shape and term_k.shape == P.shape and drop_mask.shape == P.shape):
        return False
    return all(dt in _SUPPORTED for dt in _step_dtypes(P, term_k, s_sq, big_dtype, knorm_dtype))


def fused_round_step(P, term_k, s_sq, term_q, drop_mask, per_iter_count, big_dtype, g_norm_sq=None,
                     kept_mass=None, knorm_dtype=None, k_eps=1e-6):
    """Returns (new_drop_mask bool, restore_count int64) like the reference."""
    knorm = knorm_dtype is not None
    if not knorm == (g_norm_sq is not None) == (kept_mass is not None):
        raise AssertionError("the kept-mass objective uses g_norm_sq, kept_mass and knorm_dtype together: "
                             "pass all three or none")
    raw_dtype, q_dtype = _step_dtypes(P, term_k, s_sq, big_dtype, knorm_dtype)
    if P.dtype not in _SUPPORTED or s_sq.dtype not in _SUPPORTED:
        raise TypeError("the round step takes float32 or bfloat16 P, term_k and s_sq only")
    new_drop, cnt = K.round_step(P, term_k.to(P.dtype), s_sq, term_q, drop_mask, per_iter_count,
                                 raw_bf16=raw_dtype is torch.bfloat16, q_bf16=q_dtype is torch.bfloat16,
                                 g_norm_sq=g_norm_sq, kept_mass=kept_mass, k_eps=k_eps)
    return new_drop, cnt.to(torch.int64)
