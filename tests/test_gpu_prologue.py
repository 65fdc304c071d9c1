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


def _inputs_s(a, frames, h, w, S, dtype):
    g = torch.Generator(device="cuda").manual_seed(11)
    T = frames * (h * w + S)
    x = torch.randn(1, T, a.qkv.in_features, device="cuda", generator=g).to(dtype)
    ys, xs = torch.meshgrid(torch.arange(h, device="cuda"), torch.arange(w, device="cuda"), indexing="ij")
    patch = torch.stack([ys.reshape(-1), xs.reshape(-1)], dim=-1) + 1
    frame = torch.cat([torch.zeros(S, 2, dtype=patch.dtype, device="cuda"), patch], dim=0)
    return x, frame.repeat(frames, 1).reshape(1, T, 2)


@pytest.mark.parametrize("frames,h,w,S,heads,rope,affine", [
    (3, 8, 8, 5, 4, True, True),        # 192 patch tokens: a ragged second window
    (2, 37, 37, 5, 4, True, True),      # windows that straddle frames
    (4, 10, 13, 1, 24, True, True),     # DA3's one special token and 24 heads
    (2, 16, 16, 0, 4, False, True),     # no special tokens, no rotary embedding
    (3, 9, 9, 5, 4, True, False),       # LayerNorm without weight and bias
])
def test_prologue_scored_equals_prologue_then_q_pass(frames, h, w, S, heads, rope, affine):
    """ress_qkv_prologue_scored (the q prologue fused into the Q pass) gives
    the bits of ress_qkv_prologue followed by ress_pool_quant_q: k, v, the
    special queries, the pooled queries, int8 Q and its scales."""
    from ress_b200 import kernels as K

    a = _attn(torch.bfloat16, dim=heads * 64, heads=heads)
    if not rope:
        a.rope = None
    x, pos = _inputs_s(a, frames, h, w, S, torch.bfloat16)
    L = K.Layout(1, heads, frames, S, h * w)
    with torch.inference_mode():
        lin = a.qkv(x).contiguous()
        args = Q._prologue_args(a, lin, pos, 64)
        assert args is not None
        if not affine:
            args.update(qn_weight=None, qn_bias=None, kn_weight=None, kn_bias=None)
        q, k, v = K.qkv_prologue(lin, heads, **args)
        qbar, q8, qs = K.pool_quant_q(q, L)
        sc = K.qkv_prologue_scored(lin, L, **args)
    torch.cuda.synchronize()
    assert torch.equal(sc["k"], k) and torch.equal(sc["v"], v)
    assert torch.equal(sc["qbar"], qbar) and torch.equal(sc["q8"], q8) and torch.equal(sc["qs"], qs)
    if S:
        special = q.view(1, heads, frames, S + h * w, 64)[:, :, :, :S].reshape(heads, frames * S, 64)
        assert torch.equal(sc["q_special"], special)
    else:
        assert sc["q_special"] is None


def test_attention_forward_takes_the_fused_route_bit_identically(monkeypatch):
    """ress_attention_forward on a bf16 block with LayerNorm q/k norms and the
    2-D rotary embedding runs the fused prologue (q never formed) and returns
    exactly what the unfused route (prologue, then the layer's own Q pass)
    returns."""
    from ress_b200 import attention as A
    from ress_b200 import kernels as K

    a = _attn(torch.bfloat16, dim=1024, heads=16)
    frames, h, w = 4, 16, 16
    x, pos = _inputs_s(a, frames, h, w, 5, torch.bfloat16)
    L = K.Layout(1, 16, frames, 5, h * w)
    nts = torch.full((1, 16, L.nq), max(2, L.n_cand // 2), dtype=torch.int32, device="cuda")
    calls = []
    real = A.compute_qkv_scored

    def spy(*args, **kw):
        r = real(*args, **kw)
        calls.append(r is not None)
        return r

    kw = dict(num_to_select=nts, num_special_tokens=5, num_heads=16, block_criterion="probability")
    monkeypatch.setattr(A, "FUSED_PROLOGUE", True)
    with torch.inference_mode():
        monkeypatch.setattr(A, "compute_qkv_scored", spy)
        fused = A.ress_attention_forward(a, x, pos, **kw)
        monkeypatch.setattr(A, "FUSED_PROLOGUE", False)
        plain = A.ress_attention_forward(a, x, pos, **kw)
    torch.cuda.synchronize()
    K.check_status()
    assert calls == [True]
    assert torch.equal(fused, plain)
