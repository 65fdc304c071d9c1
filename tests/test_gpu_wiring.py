"""Forward through Pi3- and DA3-wired blocks on the GPU (stand-in modules with
those backbones' structure and head counts, random weights, bf16): the wired
global attention with every candidate block kept agrees with the unwired
module's dense attention in fp32 (torch SDPA), and DA3's cross-view blocks,
whose positions carry no patch grid, get their per-view shape from the
tower's entry."""

import copy

import pytest
import torch

from ress_b200 import da3, kernels as K, pi3
from test_backbone_wiring import Pi3Like, _da3_like

pytestmark = pytest.mark.gpu


def _grid_pos(views, special, h, w, ones=False):
    """(1, views*(special+h*w), 2) positions: (row, col) + 1 of each patch (or
    all ones, DA3's cross-view positions), zeros for the special tokens."""
    ys, xs = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
    patch = torch.stack([ys.reshape(-1), xs.reshape(-1)], -1) + 1
    if ones:
        patch = torch.ones_like(patch)
    frame = torch.cat([torch.zeros(special, 2, dtype=patch.dtype), patch], 0)
    return frame.repeat(views, 1)[None].cuda()


def _all_kept(attn, heads, views, special, hw):
    L = K.Layout(1, heads, views, special, hw)
    attn.num_to_select = torch.full((1, heads, L.nq), L.n_cand, dtype=torch.int32, device="cuda")


def _close(a, b):
    a, b = a.float(), b.float()
    assert torch.isfinite(a).all()
    err = (a - b).abs()
    assert err.max().item() <= 0.08 * b.abs().max().item(), (err.max().item(), b.abs().max().item())
    assert err.mean().item() <= 0.03 * b.abs().mean().item(), (err.mean().item(), b.abs().mean().item())


def test_pi3_wired_block_matches_dense():
    torch.manual_seed(0)
    views, special, h, w, heads = 3, 5, 16, 16, 16
    m = Pi3Like(n_decoder=2, dim=heads * 64, heads=heads).cuda().to(torch.bfloat16)
    ref = copy.deepcopy(m.decoder[1].attn).float()  # fp32 torch attention (SDPA) as the reference
    pi3.wire_pi3(m, expect_blocks=None)
    attn = m.decoder[1].attn
    _all_kept(attn, heads, views, special, h * w)
    x = torch.randn(1, views * (special + h * w), heads * 64, device="cuda", dtype=torch.bfloat16)
    pos = _grid_pos(views, special, h, w)
    with torch.no_grad():
        out = attn(x, xpos=pos)  # Pi3 passes the positions as xpos=
        want = ref(x.float(), pos=pos)
    torch.cuda.synchronize()
    K.check_status()
    _close(out, want)


def test_da3_wired_block_uses_the_captured_shape():
    torch.manual_seed(1)
    views, h, w, heads = 3, 16, 16, 24  # 771 tokens: an odd count cannot split into 2-token "views"
    m = _da3_like(n_blocks=2, alt_start=1, dim=heads * 64, heads=heads)
    m = m.cuda().to(torch.bfloat16)
    vit = m.backbone.pretrained
    ref = copy.deepcopy(vit.blocks[1].attn).float()
    da3.wire_da3(m)
    attn = vit.blocks[1].attn
    _all_kept(attn, heads, views, 1, h * w)
    x = torch.randn(1, views * (1 + h * w), heads * 64, device="cuda", dtype=torch.bfloat16)
    pos = _grid_pos(views, 1, h, w, ones=True)
    with torch.no_grad():
        # all-ones positions say nothing about the grid: without the captured
        # shape the grid read from them is 1 x 1 (here the token count does not
        # split that way and the layer refuses; other counts would split wrongly)
        with pytest.raises(AssertionError, match="token split"):
            attn(x, pos=pos)
        vit._get_intermediate_layers_not_chunked(torch.zeros(1, views, 3, 14 * h, 14 * w, device="cuda"))
        out = attn(x, pos=pos)
        want = ref(x.float(), pos=pos)
    torch.cuda.synchronize()
    K.check_status()
    _close(out, want)
