"""The dense bf16 attention kernel (ress_dense_attn) against torch fp32
attention on the same bf16 inputs: the special-token queries of a global
layer (reference src/ress/models/attention.py:404-412) and the aggregator's
frame attention (src/ress/models/vggt.py:72-86) run on it.  Tolerance: 2e-2
max-abs, 1e-3 mean-abs (P and the P.V operands are bf16)."""

import math

import pytest
import torch
import torch.nn.functional as F

from ress_b200 import kernels as K

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def _ref(q, k, v):
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float())


def _qkv(S, Tq, Tk, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(S, Tq, 64, device="cuda", generator=g) * scale).bfloat16()
    k = (torch.randn(S, Tk, 64, device="cuda", generator=g) * scale).bfloat16()
    v = torch.randn(S, Tk, 64, device="cuda", generator=g).bfloat16()
    return q, k, v


@pytest.mark.parametrize("S,Tq,Tk,scale", [(16, 1374, 1374, 1.0), (4, 128, 64, 2.0), (3, 1, 1, 1.0),
                                           (2, 300, 4100, 1.5), (32, 160, 5496, 1.0), (1, 257, 8191, 3.0)])
def test_dense_matches_torch(S, Tq, Tk, scale):
    q, k, v = _qkv(S, Tq, Tk, seed=S + Tq + Tk, scale=scale)
    ref = _ref(q, k, v)
    out = K.dense_attn(q, k, v, out_bf16=False)
    torch.cuda.synchronize()
    K.check_status()
    e = (out - ref).abs()
    assert e.max().item() < MAX_ABS and e.mean().item() < MEAN_ABS, (e.max().item(), e.mean().item())
    # the bf16 output is the fp32 output rounded
    ob = K.dense_attn(q, k, v)
    torch.cuda.synchronize()
    assert ob.dtype == torch.bfloat16
    assert torch.equal(ob, out.bfloat16())


def test_dense_strided_inputs_and_scattered_rows():
    """Rows addressed by strides (heads of a (B, T, 3, H, 64) buffer) and
    outputs scattered into a full token layout (group / period / offset)."""
    B, H, F_, Sp, HW = 1, 4, 3, 5, 37
    T = F_ * (Sp + HW)
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn(B, T, 3, H, 64, device="cuda", generator=g).bfloat16()
    q = qkv[:, :, 0].permute(0, 2, 1, 3)  # (B, H, T, 64), row stride 3*H*64, head stride 64
    k = qkv[:, :, 1].permute(0, 2, 1, 3)
    v = qkv[:, :, 2].permute(0, 2, 1, 3)
    qs = q.reshape(B, H, F_, Sp + HW, 64)[:, :, :, :Sp].reshape(B * H, F_ * Sp, 64)
    out = torch.full((B, H, T, 64), 7.0, device="cuda")
    K.dense_attn(qs, k[0], v[0], out=out, out_rows=(H, out.stride(0), out.stride(1), out.stride(2), Sp, Sp + HW, 0))
    torch.cuda.synchronize()
    ref = _ref(qs.view(B, H, F_ * Sp, 64), k, v).view(B, H, F_, Sp, 64)
    got = out.view(B, H, F_, Sp + HW, 64)
    assert (got[:, :, :, :Sp] - ref).abs().max().item() < MAX_ABS
    assert torch.all(got[:, :, :, Sp:] == 7.0)  # patch rows untouched


def test_dense_scale_argument():
    q, k, v = _qkv(2, 200, 333, seed=9)
    out = K.dense_attn(q, k, v, out_bf16=False, sm_scale=0.3)
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=0.3)
    torch.cuda.synchronize()
    assert (out - ref).abs().max().item() < MAX_ABS


def test_frame_attention_module_uses_kernel_and_matches_torch():
    """vggt.Attention in bf16 (prologue + dense kernel) against the same
    module's torch path in fp32."""
    from ress_b200 import vggt

    torch.manual_seed(0)
    rope = vggt.RotaryPosition2D()
    att = vggt.Attention(1024, 16, qk_norm=True, rope=rope).cuda()
    B, h, w = 2, 7, 9
    x = torch.randn(B, h * w + 5, 1024, device="cuda")
    pos = torch.zeros(B, h * w + 5, 2, dtype=torch.long, device="cuda")
    yy, xx = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
    pos[:, 5:, 0] = yy.reshape(-1).cuda() + 1
    pos[:, 5:, 1] = xx.reshape(-1).cuda() + 1
    ref = att(x, pos)  # fp32: torch path
    y = att.bfloat16()(x.bfloat16(), pos)
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16
    rel = (y.float() - ref).abs().max().item() / ref.abs().max().item()
    assert rel < 3e-2, rel
