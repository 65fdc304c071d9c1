"""Pi3 and DA3 wiring (ress_b200.pi3 / ress_b200.da3) on stand-in modules with
those backbones' structure (the real networks need their source trees and
checkpoints): which blocks are wired, the tags, the per-view shape capture of
DA3, and the loaders' error when the backbone's package is absent.  The
forward through the wired blocks runs on the GPU (test_gpu_wiring.py)."""

import types

import pytest
import torch
from torch import nn

from ress_b200 import api, backbones, da3, pi3, wiring
from ress_b200.vggt import Block, RotaryPosition2D


class Pi3Like(nn.Module):
    """Pi3's layout: one decoder list alternating frame (even) and cross-frame
    (odd) blocks, five special tokens per frame, an encoder with blocks."""

    def __init__(self, n_decoder=6, dim=128, heads=2):
        super().__init__()
        self.decoder = nn.ModuleList(Block(dim, heads, True, RotaryPosition2D(), 1.0) for _ in range(n_decoder))
        self.encoder = types.SimpleNamespace(blocks=[nn.Identity(), nn.Identity()])
        self.patch_start_idx = 5


class DA3Tower(nn.Module):
    """DA3's DINOv2 tower: cross-view blocks are the odd ones from alt_start on;
    _get_intermediate_layers_not_chunked receives the (B, views, 3, H, W)
    images (here it runs the cross-view blocks on given tokens)."""

    def __init__(self, n_blocks=7, alt_start=2, dim=128, heads=2):
        super().__init__()
        self.blocks = nn.ModuleList(Block(dim, heads, True, RotaryPosition2D(), 1.0) for _ in range(n_blocks))
        self.alt_start = alt_start
        self.patch_size = 14

    def _get_intermediate_layers_not_chunked(self, x, tokens=None, pos=None):
        for i, blk in enumerate(self.blocks):
            if i >= self.alt_start and i % 2 == 1 and tokens is not None:
                tokens = blk(tokens, pos=pos)
        return tokens


def _da3_like(**kw):
    m = nn.Module()
    m.backbone = nn.Module()
    m.backbone.pretrained = DA3Tower(**kw)
    return m


def _is_wired(block):
    return getattr(block.attn.forward, "__func__", None) is not type(block.attn).forward


def test_pi3_odd_decoder_blocks_are_wired():
    m = Pi3Like()
    assert pi3.global_block_indices(m) == [1, 3, 5]
    pi3.wire_pi3(m, aux_output=True, expect_blocks=None)
    assert [_is_wired(b) for b in m.decoder] == [False, True, False, True, False, True]
    assert wiring.global_blocks(m) == [m.decoder[i] for i in (1, 3, 5)]
    assert m._ress_backbone == "pi3" and backbones.infer_backbone(m).n_heads == 16
    assert set(m.aux_output_store) == {0, 1, 2}
    assert len(pi3.checkpointable_blocks(m)) == 8


def test_pi3_block_count_is_checked():
    with pytest.raises(ValueError, match="cross-frame"):
        pi3.wire_pi3(Pi3Like(n_decoder=6))  # 3 global blocks, the tables are for 18


def test_da3_cross_view_blocks_and_shape_capture():
    m = _da3_like(n_blocks=7, alt_start=2)
    assert da3.global_block_indices(m) == [3, 5]
    da3.wire_da3(m)
    vit = m.backbone.pretrained
    assert [_is_wired(b) for b in vit.blocks] == [False, False, False, True, False, True, False]
    assert m._ress_backbone == "da3" and backbones.infer_backbone(m).n_heads == 24
    # the tower's entry records (views, patch rows, patch columns) on every wired module
    vit._get_intermediate_layers_not_chunked(torch.zeros(1, 3, 3, 28, 42))
    for i in (3, 5):
        assert vit.blocks[i].attn.ress_shape == {"N": 3, "H": 2, "W": 3}
    vit._get_intermediate_layers_not_chunked(torch.zeros(1, 5, 3, 14 * 4, 14 * 4))
    assert vit.blocks[3].attn.ress_shape == {"N": 5, "H": 4, "W": 4}
    assert not hasattr(vit.blocks[2].attn, "ress_shape")


def test_da3_without_cross_view_blocks_raises():
    with pytest.raises(ValueError, match="alt_start"):
        da3.global_block_indices(_da3_like(alt_start=-1))


@pytest.mark.parametrize("name", ["pi3", "da3"])
def test_loaders_name_the_missing_package(name):
    with pytest.raises(RuntimeError, match="source tree"):
        api.load_backbone(name, device="cpu")


def test_wired_block_rejects_a_mask():
    m = Pi3Like()
    pi3.wire_pi3(m, expect_blocks=None)
    with pytest.raises(AssertionError):
        m.decoder[1].attn(torch.zeros(1, 4, 128), attn_mask=torch.ones(4, 4, dtype=torch.bool))
