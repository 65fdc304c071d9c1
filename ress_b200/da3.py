"""Depth-Anything-3 backbone: which of its blocks take the sparse global
attention, and the per-view shape they cannot read from their positions.

Reference: ``src/ress/models/da3.py:56-151``.  DA3 is one DINOv2 tower
(``model.backbone.pretrained``); from ``alt_start`` on, its odd blocks attend
over all views jointly and the others within a view, so the global blocks are
the odd indices at or after ``alt_start`` (14 of the 40 blocks of the GIANT
preset).  Two things differ from VGGT and Pi3:

- one special (camera) token per view, not five;
- the cross-view blocks get all-ones positions for every patch token, so the
  patch grid cannot be recovered from ``pos``.  ``attach_shape_capture``
  wraps the tower's ``_get_intermediate_layers_not_chunked`` (which receives
  the (B, views, 3, H, W) images) to set ``ress_shape`` = {N, H, W} on every
  wired attention module before each forward; the layer reads it instead of
  ``pos``.

Building the network needs DA3's own source tree (``depth_anything_3``) and
its checkpoint; ``load_da3`` raises with the reason when they are absent.
``wire_da3`` wires a DA3 network the caller has built.
"""

from __future__ import annotations

from .wiring import wire_ress_attention

NUM_SPECIAL_TOKENS = 1
N_GLOBAL_BLOCKS = 14
PRETRAINED = "depth-anything/DA3-GIANT-1.1"


def _tower(model):
    """The DINOv2 tower inside a DA3 network."""
    return model.backbone.pretrained


def global_block_indices(model) -> list:
    """Indices into the tower's ``blocks`` of the cross-view blocks: odd and at
    or after ``alt_start``."""
    vit = _tower(model)
    if vit.alt_start == -1:
        raise ValueError("this DA3 preset has no cross-view blocks (alt_start == -1)")
    return [i for i in range(len(vit.blocks)) if i >= vit.alt_start and i % 2 == 1]


def checkpointable_blocks(model) -> list:
    return list(_tower(model).blocks)


def attach_shape_capture(model, blocks) -> None:
    """Before every forward of the tower, record (views, patch rows, patch
    columns) of the input images on the wired attention modules."""
    vit = _tower(model)
    inner = vit._get_intermediate_layers_not_chunked
    attns = [b.attn for b in blocks]
    patch = vit.patch_size

    def capture(x, *args, **kwargs):
        views, rows, cols = x.shape[1], x.shape[3] // patch, x.shape[4] // patch
        for a in attns:
            a.ress_shape = {"N": views, "H": rows, "W": cols}
        return inner(x, *args, **kwargs)

    vit._get_intermediate_layers_not_chunked = capture


def wire_da3(model, aux_output: bool = False, aux_full: bool = True, expect_blocks: int | None = None):
    """Route the cross-view blocks of a built DA3 network through the sparse
    attention, attach the shape capture and tag the model for ``api.apply_*``.
    ``expect_blocks``: the number of cross-view blocks the checkpoint must have
    (None: any; 14 for the GIANT preset)."""
    vit = _tower(model)
    blocks = [vit.blocks[i] for i in global_block_indices(model)]
    if expect_blocks is not None and len(blocks) != expect_blocks:
        raise ValueError(f"this DA3 tower has {len(blocks)} cross-view blocks, expected {expect_blocks}")
    store = {i: {} for i in range(len(blocks))} if aux_output else None
    wire_ress_attention(model, blocks, aux_output_store=store, aux_full=aux_full,
                        num_special_tokens=NUM_SPECIAL_TOKENS)
    attach_shape_capture(model, blocks)
    model.aux_output_store = store
    model._ress_backbone = "da3"
    return model


def load_da3(pretrained: str = PRETRAINED, aux_output: bool = False, aux_full: bool = True, device: str = "cuda"):
    """A pretrained DA3 network with its cross-view blocks wired (same contract
    as the reference's ``load_da3``)."""
    try:
        from depth_anything_3.api import DepthAnything3
    except ImportError as e:
        raise RuntimeError("loading the pretrained da3 backbone needs the `depth_anything_3` source tree and "
                           "its checkpoint; build the network yourself and call ress_b200.da3.wire_da3 on it "
                           f"({e})") from None
    net = DepthAnything3.from_pretrained(pretrained).model
    wire_da3(net, aux_output=aux_output, aux_full=aux_full, expect_blocks=N_GLOBAL_BLOCKS)
    return net.to(device).eval()
