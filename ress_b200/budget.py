"""Per-head block budgets: HeSS and the uniform baseline.

Mirror of the reference's ``budget/hess.py`` (``sum_normalize`` :46-48,
``combine_lambda`` :51-56, ``HessBudget`` :59-100), ``budget/uniform.py``
(``UniformBudget`` :23-37) and ``budget/_proportional.py``
(``adjust_attention_selection`` :149-215).  The table preparation is the same
torch arithmetic on the host; the per-input work (baseline count and the
cap-and-redistribute loop) runs in the sm_100a kernels ``ress_baseline`` and
``ress_hess_adjust``.  The objects keep the reference's plugin interface,
``num_to_select(layer_idx, attn_pooled, sparse_ratio, cdf_threshold, beta)``,
and additionally describe themselves (``spec``) so the fused layer can run
the budget without materialising ``attn_cond`` for a Python callback.
"""

from __future__ import annotations

import torch

from . import kernels as K
from .layer import BudgetSpec


def sum_normalize(scores: torch.Tensor) -> torch.Tensor:
    return scores / scores.sum(dim=-1, keepdim=True)


def combine_lambda(score_cam, score_pc, lam):
    return sum_normalize(lam * score_cam + (1 - lam) * score_pc)


def compute_baseline_num_to_select(pooled_score, sparse_ratio=None, cdf_threshold=None, eps=1e-5):
    """(B, nh, q_blk, k_blk) pooled map -> (B, nh, q_blk) long (attention.py:268-293)."""
    if eps != 1e-5:
        raise NotImplementedError("only the reference default eps=1e-5 is supported")
    return K.baseline(pooled_score, sparse_ratio, cdf_threshold).long()


def adjust_attention_selection(num_to_select, head_scores, beta, max_val, max_iters=1000, floor_frac=None):
    """HeSS re-allocation of (..., nh, q_blk) budgets (_proportional.py:149-215).
    Raises RuntimeError like the reference when a column does not converge
    (this check synchronises, as the reference's loop does)."""
    if floor_frac is not None:
        raise NotImplementedError("floor_frac is not used by any of the four modes")
    x = num_to_select
    lead = x.shape[:-2]
    nh, nq = x.shape[-2:]
    base = x.reshape(-1, nh, nq).to(torch.int32)
    out = K.hess_adjust(base, K.scores_norm(head_scores), max_val, beta=beta, max_iters=max_iters, min_clamp=0)
    K.check_status(base.device)
    return out.view(*lead, nh, nq).long()


class UniformBudget:
    """One budget for every head: the baseline count alone (uniform.py:23-37)."""

    def __init__(self, n_blocks=24, n_heads=16):
        self.head_scores = torch.ones(n_blocks, n_heads)

    @property
    def needs_v_bar(self):
        return False

    def num_to_select(self, layer_idx, attn_pooled, sparse_ratio=None, cdf_threshold=None, beta=1.0):
        return compute_baseline_num_to_select(attn_pooled, sparse_ratio, cdf_threshold)

    def spec(self, layer_idx, sparse_ratio, cdf_threshold, beta, device=None) -> BudgetSpec:
        return BudgetSpec("uniform", sparse_ratio=sparse_ratio, cdf_threshold=cdf_threshold, beta=beta)


class HessBudget:
    """Calibrated per-head importance -> per-(head, q-block) budget
    (hess.py:59-100): baseline count from this input's pooled map, then the
    proportional re-allocation by head score."""

    def __init__(self, score_cam_path, score_pc_path, lam=0.5, qkv_idx=0, floor_frac=None, layer_slice=None):
        raw_cam = torch.load(score_cam_path, weights_only=False)[qkv_idx]
        raw_pc = torch.load(score_pc_path, weights_only=False)[qkv_idx]
        if layer_slice is not None:
            raw_cam, raw_pc = raw_cam[layer_slice], raw_pc[layer_slice]
        self.score_cam = sum_normalize(raw_cam)
        self.score_pc = sum_normalize(raw_pc)
        self.lam = lam
        self.head_scores = combine_lambda(self.score_cam, self.score_pc, self.lam)
        if floor_frac is not None:
            raise NotImplementedError("floor_frac is not used by any of the four modes")
        self.floor_frac = floor_frac
        self._snorm = {}

    def num_to_select(self, layer_idx, attn_pooled, sparse_ratio=None, cdf_threshold=None, beta=1.0):
        baseline = compute_baseline_num_to_select(attn_pooled, sparse_ratio, cdf_threshold)
        return adjust_attention_selection(baseline, self.head_scores[layer_idx], beta, attn_pooled.shape[-1])

    def scores_norm(self, layer_idx, device):
        key = (layer_idx, str(device))
        if key not in self._snorm:
            self._snorm[key] = K.scores_norm(self.head_scores[layer_idx]).to(device)
        return self._snorm[key]

    def spec(self, layer_idx, sparse_ratio, cdf_threshold, beta, device=None) -> BudgetSpec:
        return BudgetSpec("hess", sparse_ratio=sparse_ratio, cdf_threshold=cdf_threshold, beta=beta,
                          scores_norm=self.scores_norm(layer_idx, device or "cuda"))
