"""The residual-drift criterion: W_O metric baking and restore-swap ordering.

Mirror of the reference's ``scoring/projected.py``: ``bake_M`` :214-232 and
``bake_and_attach_M`` :235-244 (torch, once per model load),
``kept_mass_norm_quality`` :191-211 (the closed-form single-move objective
change, kept for analysis), and ``restore_swap_rank_by`` :395-1058, which
runs here as one sm_100a kernel (``ress_restore_swap``) with the shipped
recipe: big tensors in bf16, kept-mass normalisation, track-best, lowest-
index ties.  It returns the same ``rank_by`` tensor the reference returns;
the fused forward never builds it and consumes the kernel's keep lists
directly.
"""

from __future__ import annotations

import torch

from . import kernels as K
from .wiring import global_blocks

KEPT_MASS_EPS = 1e-6


def kept_mass_norm_quality(G, K_, delta_G, u, eps=KEPT_MASS_EPS):
    """J - J_new = [G u (2K + u) / K^2 - delta_G] / (K + u)^2 (projected.py:191-211)."""
    Kc = K_.unsqueeze(-1)
    K_new = (Kc + u).clamp(min=eps)
    return (G.unsqueeze(-1) * u * (2.0 * Kc + u) / Kc.pow(2) - delta_G) / K_new.pow(2)


def bake_M(model):
    """(n_blocks, nh, hd, hd): M_h = (W_O^h)^T W_O^h per global block and head."""
    Ms = []
    with torch.no_grad():
        for block in global_blocks(model):
            W = block.attn.proj.weight
            nh = block.attn.num_heads
            hd = W.shape[1] // nh
            Ms.append(torch.stack([W[:, h * hd:(h + 1) * hd].T @ W[:, h * hd:(h + 1) * hd] for h in range(nh)]))
    return torch.stack(Ms)


def bake_and_attach_M(model):
    M = bake_M(model)
    for i, block in enumerate(global_blocks(model)):
        block.attn.M = M[i].to(next(block.attn.parameters()).device)
    return M


def restore_swap_rank_by(attn_pooled, v_bar, M, num_to_select, restore_frac=0.5, n_iters=1,
                         dtype=torch.float32, track_best=False, big_dtype=None, decay=0.5, renormalize=None,
                         n_cand=None, maximize=False, invert_cut=False):
    """Restore-swap ordering (projected.py:395-1058) on the GPU.

    attn_pooled (..., nh, q_blk, k_blk) over all pooled blocks, v_bar
    (..., nh, k_blk, hd), M (nh, hd, hd), num_to_select (..., nh, q_blk).
    Returns rank_by (..., nh, q_blk, n_cand) in bf16: s for dropped blocks,
    s + (max|s| + 1) for kept ones, as the reference does."""
    if big_dtype != torch.bfloat16 or dtype != torch.float32:
        raise NotImplementedError("the sm_100a path implements the shipped recipe: big_dtype=bf16, dtype=fp32")
    if maximize or invert_cut:
        raise NotImplementedError("the drift-maximisation controls are analysis-only and not ported")
    if renormalize is False:
        raise NotImplementedError("RESS_RENORM=0 (the unrenormalised cut) is not supported")
    k_blk = attn_pooled.shape[-1]
    n_cand = k_blk if n_cand is None else n_cand
    nq = attn_pooled.shape[-2]
    r = K.restore_swap(attn_pooled.reshape(-1, nq, k_blk), v_bar.reshape(-1, k_blk, v_bar.shape[-1]), M.float(),
                       num_to_select.reshape(-1), n_cand, n_iters=n_iters, track_best=track_best,
                       restore_frac=restore_frac, decay=decay, want_drop=True, want_s=True, want_lists=False)
    drop = r["drop"].bool()
    s = r["s"]
    keep_offset = s.abs().amax() + 1.0
    rank_by = torch.where(drop, s, s + keep_offset)
    return rank_by.view(*attn_pooled.shape[:-1], n_cand)
