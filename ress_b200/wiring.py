"""Wiring the sparse global attention into a backbone's blocks.

Same contract as the reference's ``models/wiring.py`` (``global_blocks`` :33,
``wire_ress_attention`` :49-109): each block's ``attn.forward`` is replaced
by a wrapper that reads the per-call configuration off the attention module
(``num_to_select``, ``budget_fn``, ``block_criterion``, ...) and calls
``ress_b200.attention.ress_attention_forward``; the block list is recorded
on the model for ``global_blocks``.
"""

from __future__ import annotations

from types import MethodType


def global_blocks(model):
    blocks = getattr(model, "ress_global_blocks", None)
    if blocks is not None:
        return blocks
    return model.aggregator.global_blocks


def global_attns(model):
    return [block.attn for block in global_blocks(model)]


def wire_ress_attention(model, blocks, aux_output_store=None, aux_full=True, num_special_tokens=5):
    from .attention import ress_attention_forward

    blocks = list(blocks)
    for i, block in enumerate(blocks):
        store = aux_output_store[i] if aux_output_store is not None else None

        def _fwd(self, x, pos=None, xpos=None, attn_bias=None, attn_mask=None, _store=store, _attn=block.attn):
            if attn_bias is not None or attn_mask is not None:
                raise AssertionError("the sparse global attention decides which key blocks each query block "
                                     "sees; a caller-side attn_bias or attn_mask has no place in it")
            return ress_attention_forward(
                _attn, x, pos if pos is not None else xpos,
                num_to_select=getattr(_attn, "num_to_select", None),
                budget_fn=getattr(_attn, "budget_fn", None),
                perhead_budget_fn=getattr(_attn, "perhead_budget_fn", None),
                joint_select_fn=getattr(_attn, "joint_select_fn", None),
                block_criterion=getattr(_attn, "block_criterion", "probability"),
                num_special_tokens=num_special_tokens,
                num_heads=_attn.num_heads,
                shape=getattr(_attn, "ress_shape", None),
                aux_store=_store,
                aux_full=aux_full,
                dense=getattr(_attn, "dense", False),
                retain_output_grad=getattr(_attn, "retain_output_grad", False),
                pooled_fallback=getattr(_attn, "pooled_fallback", False),
                protect_own_frame=getattr(_attn, "protect_own_frame", False),
            )

        block.attn.forward = MethodType(_fwd, block.attn)
    model.ress_global_blocks = blocks
    return blocks
