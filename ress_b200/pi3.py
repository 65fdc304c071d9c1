"""Pi3 backbone: which of its blocks take the sparse global attention.

Reference: ``src/ress/models/pi3.py:32-76``.  Pi3 runs frame and cross-frame
attention in one ``model.decoder`` list of 36 blocks that alternate: even
indices attend within one frame, odd indices over all frames jointly.  The
18 odd blocks are the global ones; their attention modules carry the same
``qkv`` / ``q_norm`` / ``k_norm`` / ``rope`` / ``num_heads`` / ``proj``
attributes as VGGT's, with ``model.patch_start_idx`` (5) special tokens per
frame, so ``wiring.wire_ress_attention`` patches them unchanged (the rotary
positions arrive as ``xpos=``, which the wrapper accepts).

Building the network needs Pi3's own source tree (``pi3`` package) and its
checkpoint; ``load_pi3`` raises with the reason when the package is absent.
``wire_pi3`` wires a Pi3 model the caller has built.
"""

from __future__ import annotations

from .wiring import wire_ress_attention

N_GLOBAL_BLOCKS = 18
PRETRAINED = "yyfz233/Pi3"


def global_block_indices(model) -> list:
    """Indices into ``model.decoder`` of the cross-frame blocks: the odd ones."""
    return [i for i in range(len(model.decoder)) if i % 2 == 1]


def checkpointable_blocks(model) -> list:
    """Every decoder block and every encoder block (for a backward pass through
    the whole network, e.g. calibration); inference does not use this."""
    return list(model.decoder) + list(model.encoder.blocks)


def wire_pi3(model, aux_output: bool = False, aux_full: bool = True, expect_blocks: int | None = N_GLOBAL_BLOCKS):
    """Route the global decoder blocks of a built Pi3 model through the sparse
    attention and tag the model for ``api.apply_*``.  ``expect_blocks``: the
    number of global blocks the checkpoint must have (None: any)."""
    blocks = [model.decoder[i] for i in global_block_indices(model)]
    if expect_blocks is not None and len(blocks) != expect_blocks:
        raise ValueError(f"a Pi3 decoder with {len(model.decoder)} blocks has {len(blocks)} cross-frame "
                         f"blocks; this backbone's tables are for {expect_blocks}")
    store = {i: {} for i in range(len(blocks))} if aux_output else None
    wire_ress_attention(model, blocks, aux_output_store=store, aux_full=aux_full,
                        num_special_tokens=model.patch_start_idx)
    model.aux_output_store = store
    model._ress_backbone = "pi3"
    return model


def load_pi3(pretrained: str = PRETRAINED, aux_output: bool = False, aux_full: bool = True, device: str = "cuda"):
    """A pretrained Pi3 with its global blocks wired (same contract as the
    reference's ``load_pi3``)."""
    try:
        from pi3.models.pi3 import Pi3
    except ImportError as e:
        raise RuntimeError("loading the pretrained pi3 backbone needs the `pi3` source tree (Pi3's repository "
                           "on the Python path) and its checkpoint; build the model yourself and call "
                           f"ress_b200.pi3.wire_pi3 on it ({e})") from None
    model = Pi3.from_pretrained(pretrained)
    wire_pi3(model, aux_output=aux_output, aux_full=aux_full)
    return model.to(device).eval()
