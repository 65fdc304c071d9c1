"""Installing one attention mode on every global block.

Same contract as the reference's ``runtime/static.py`` (``set_static_budget``
:20-77): every call resets all per-call knobs of every global attention
module and installs a ``budget_fn(attn_pooled)`` closure (or
``perhead_budget_fn(attn_pooled, v_bar)`` for budgets that ask for V-bar), so
switching modes between forward passes leaves nothing stale behind.

The closures also carry ``ress_budget = (budget, layer, sparse_ratio,
cdf_threshold, beta)``: the fused forward recognises budgets of this package
by it and runs them on the device without a Python callback; any other
callable is simply called, exactly as the reference would.
"""

from __future__ import annotations

from .wiring import global_blocks


def set_static_budget(model, budget, sparse_ratio=None, cdf_threshold=None, beta=1.0,
                      block_criterion="probability", pooled_fallback=False, protect_own_frame=False):
    needs_v_bar = getattr(budget, "needs_v_bar", False)
    for i, block in enumerate(global_blocks(model)):
        attn = block.attn
        attn.dense = False
        attn.num_to_select = None
        attn.retain_output_grad = False
        attn.block_criterion = block_criterion
        attn.pooled_fallback = pooled_fallback
        attn.protect_own_frame = protect_own_frame
        attn.joint_select_fn = None
        attn.perhead_budget_fn = None
        attn.budget_fn = None
        if needs_v_bar:
            def _perhead_budget_fn(attn_pooled, v_bar, _layer=i):
                return budget.num_to_select(_layer, attn_pooled, sparse_ratio, cdf_threshold, beta, v_bar=v_bar)

            attn.perhead_budget_fn = _perhead_budget_fn
        else:
            def _budget_fn(attn_pooled, _layer=i):
                return budget.num_to_select(_layer, attn_pooled, sparse_ratio, cdf_threshold, beta)

            _budget_fn.ress_budget = (budget, i, sparse_ratio, cdf_threshold, beta)
            attn.budget_fn = _budget_fn
