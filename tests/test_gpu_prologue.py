"""The fused q/k/v prologue (ress_qkv_prologue) against the torch path of
compute_qkv (reference src/ress/models/qkv.py:25-68): q/k LayerNorm, 2-D
rotary embedding, heads moved in front of the tokens.

v is a pure layout move and must be bit-identical.  The rotary step follows
torch's rounding points, so with the normalised values equal the outputs are
equal; the LayerNorm reduction order differs from torch's kernel, which can
move a normalised value by one unit in the last place.  Hence: fp32 within
1e-5 absolute; bf16 at least 97 % of elements bit-identical and every element
within 2 bf16 ulps of its magnitude (one from LayerNorm, one more through the
rotary sum)."""

import pytest
import torch

from ress_b200 import qkv as Q
from ress_b200 import vggt

pytestmark = pytest.mark.gpu


def _attn(dtype, dim=256, heads=4):
    torch.manual_seed(0)
    a = vggt.Attention(dim, heads, True, vggt.RotaryPosition2D(100.0))
    with torch.no_grad():
        for n in (a.q_norm, a.k_norm):
            n.weight.copy_(1 + 0.3 * torch.randn_like(n.weight))
            n.bias.copy_(0.2 * torch.randn_like(n.bias))
    return a.cuda().to(dtype).eval()


def _torch_path(a, lin, pos, nh, hd):
    B, T, _ = lin.shape
    q, k, v = lin.view(B, T, 3, nh, hd).permute(2, 0, 3, 1, 4).unbind(0)
    q, k = a.q_norm(q), a.k_norm(k)
    return a.rope(q, pos), a.rope(k, pos), v


def _inputs(a, frames, h, w, dtype):
    g = torch.Generator(device="cuda").manual_seed(7)
    T = frames * (h * w + 5)
    x = torch.randn(1, T, a.qkv.in_features, device="cuda", generator=g).to(dtype)
    ys, xs = torch.meshgrid(torch.arange(h, device="cuda"), torch.arange(w, device="cuda"), indexing="ij")
    patch = torch.stack([ys.reshape(-1), xs.reshape(-1)], dim=-1) + 1
    frame = torch.cat([torch.zeros(5, 2, dtype=patch.dtype, device="cuda"), patch], dim=0)
    pos = frame.repeat(frames, 1).reshape(1, T, 2)
    return x, pos


def _ulp(x):
    # bf16 unit in the last place of |x| (8 significant bits)
    e = torch.floor(torch.log2(x.abs().float().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("frames,h,w", [(3, 8, 8), (2, 37, 37)])
def test_prologue_matches_torch(dtype, frames, h, w):
    a = _attn(dtype)
    x, pos = _inputs(a, frames, h, w, dtype)
    nh, hd = a.num_heads, 64
    with torch.inference_mode():
        lin = a.qkv(x)
        got = Q._fused_prologue(a, lin, pos, nh, hd)
        assert got is not None, "the fused path must engage for LayerNorm(64) + RotaryPosition2D on CUDA"
        ref = _torch_path(a, lin, pos, nh, hd)
    for name, g_, r in zip("qkv", got, ref):
        assert g_.shape == r.shape and g_.dtype == r.dtype and g_.is_contiguous()
        if name == "v":
            assert torch.equal(g_, r)
            continue
        if dtype == torch.float32:
            assert (g_ - r).abs().max().item() <= 1e-5, name
        else:
            same = (g_ == r).float().mean().item()
            assert same >= 0.97, (name, same)
            diff = (g_.float() - r.float()).abs()
            assert bool((diff <= 2 * _ulp(r) + 1e-30).all()), (name, diff.max().item())


def test_prologue_without_rope_and_compute_qkv_route():
    a = _attn(torch.bfloat16)
    x, pos = _inputs(a, 2, 8, 8, torch.bfloat16)
    with torch.inference_mode():
        q, k, v, shp = Q.compute_qkv(a, x, pos, num_special_tokens=5, num_heads=a.num_heads)
        lin = a.qkv(x)
        ref = _torch_path(a, lin, pos, a.num_heads, 64)
        assert torch.equal(v, ref[2])
        assert (q.float() - ref[0].float()).abs().max().item() <= 0.05
        assert shp["N"] == 2 and shp["P"] == 69
        a.rope = None
        q2, k2, _ = Q._fused_prologue(a, lin, None, a.num_heads, 64)
        B, T, _ = lin.shape
        qr, kr, _ = lin.view(B, T, 3, a.num_heads, 64).permute(2, 0, 3, 1, 4).unbind(0)
        qr = a.q_norm(qr)
        assert (q2 == qr).float().mean().item() >= 0.97
