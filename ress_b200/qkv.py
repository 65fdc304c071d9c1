"""Q/K/V projection and the patch/special token split.

Same arithmetic as the reference's ``models/qkv.py`` (``compute_patch_qkv``
:25-68, ``combine_special_and_patch`` :71-81, ``project_out`` :84-87) and
``models/tokens.py`` (:8-52).  ``compute_qkv`` returns q, k, v in the full
token layout without splitting: the sm_100a kernels take the layout instead
of split copies.
"""

from __future__ import annotations

import torch


def layer_shape(x, pos, num_special_tokens=5, num_heads=16, shape=None):
    B, NP, C = x.shape
    S = num_special_tokens
    if shape is not None:
        H, W, N = shape["H"], shape["W"], shape["N"]
    else:
        H = int(pos[0].max(0).values[0])
        W = int(pos[0].max(0).values[1])
        N = NP // (H * W + S)
    P = H * W + S
    assert N * P == NP, f"token split mismatch: N={N} x P={P} (= H*W+S = {H}*{W}+{S}) != {NP} tokens"
    return {"B": B, "N": N, "P": P, "head_dim": C // num_heads, "num_heads": num_heads, "H": H, "W": W, "S": S}


def _fusable_norm(m, hd):
    return (isinstance(m, torch.nn.LayerNorm) and tuple(m.normalized_shape) == (hd,) and m.elementwise_affine
            and m.bias is not None)


def _prologue_args(self, qkv, pos, hd):
    """The prologue kernel's norm and rotary arguments when the block's norms
    and rotary embedding are ones it reproduces (64-dim affine LayerNorm;
    this package's 2-D table RoPE or none), else None (torch path)."""
    if not qkv.is_cuda or qkv.dtype not in (torch.float32, torch.bfloat16) or hd != 64:
        return None
    if torch.is_autocast_enabled() or not (_fusable_norm(self.q_norm, hd) and _fusable_norm(self.k_norm, hd)):
        return None
    rope = getattr(self, "rope", None)
    cos = sin = None
    if rope is not None:
        from .vggt import RotaryPosition2D

        if type(rope) is not RotaryPosition2D or pos is None:
            return None
        cos, sin = rope._cos_sin(hd // 2, rope.MAX_POS, qkv.device, qkv.dtype)
    if self.q_norm.eps != self.k_norm.eps:
        return None
    return dict(qn_weight=self.q_norm.weight, qn_bias=self.q_norm.bias, kn_weight=self.k_norm.weight,
                kn_bias=self.k_norm.bias, eps=self.q_norm.eps, pos=pos if cos is not None else None,
                rope_cos=cos, rope_sin=sin)


def _fused_prologue(self, qkv, pos, nh, hd):
    """q, k, v from the sm_100a prologue kernel (see _prologue_args), else None."""
    args = _prologue_args(self, qkv, pos, hd)
    if args is None:
        return None
    from . import kernels as K

    return K.qkv_prologue(qkv.contiguous(), nh, **args)


def compute_qkv_scored(self, x, pos, num_special_tokens=5, num_heads=16, shape=None):
    """For a bf16 layer whose prologue the kernels reproduce: (k, v, scored,
    shp) with the patch queries already pooled and quantised by the fused
    prologue (kernels.qkv_prologue_scored; q itself is never formed), else
    None."""
    shp = layer_shape(x, pos, num_special_tokens, num_heads, shape)
    nh, hd = num_heads, x.shape[-1] // num_heads
    if x.dtype != torch.bfloat16 or self.qkv.weight.dtype != torch.bfloat16:
        return None
    args = _prologue_args(self, x, pos, hd)  # x: the Linear's output has its device and dtype
    if args is None:
        return None
    lin = self.qkv(x)
    from . import kernels as K

    L = K.Layout(shp["B"], nh, shp["N"], shp["S"], shp["P"] - shp["S"])
    scored = K.qkv_prologue_scored(lin.contiguous(), L, **args)
    return scored["k"], scored["v"], scored, shp


def compute_qkv(self, x, pos, num_special_tokens=5, num_heads=16, shape=None):
    """q, k, v as (B, nh, N*P, hd) views/tensors plus the shape dict."""
    shp = layer_shape(x, pos, num_special_tokens, num_heads, shape)
    B, NP, C = x.shape
    nh, hd = num_heads, C // num_heads
    lin = self.qkv(x)
    fused = _fused_prologue(self, lin, pos, nh, hd)
    if fused is not None:
        q, k, v = fused
        return q, k, v, shp
    qkv = lin.view(B, NP, 3, nh, hd).permute(2, 0, 3, 1, 4)
    q, k, v = qkv.unbind(0)
    q, k = self.q_norm(q), self.k_norm(k)
    if getattr(self, "rope", None) is not None:
        q = self.rope(q, pos)
        k = self.rope(k, pos)
    return q, k, v, shp


def get_patch_tokens(x, N, P, S):
    assert x.shape[-2] == N * P
    v = x.view(x.shape[:-2] + (N, P, x.shape[-1]))
    return v[..., S:, :].reshape(x.shape[:-2] + (N * (P - S), x.shape[-1])).contiguous()


def get_special_tokens(x, N, P, S):
    assert x.shape[-2] == N * P
    v = x.view(x.shape[:-2] + (N, P, x.shape[-1]))
    sp = v[..., :S, :].reshape(x.shape[:-2] + (N * S, x.shape[-1]))
    return None if sp.numel() == 0 else sp


def combine_special_and_patch(x_special, x_patch, shape):
    B, N, P, hd, nh, S = shape["B"], shape["N"], shape["P"], shape["head_dim"], shape["num_heads"], shape["S"]
    xp = x_patch.reshape(B, nh, N, P - S, hd)
    x = torch.cat([x_special.view(B, nh, N, S, hd), xp], dim=-2) if x_special is not None else xp
    return x.view(B, nh, N * P, hd)


def project_out(self, x, B, N, P, nh, hd):
    x = x.transpose(1, 2).reshape(B, N * P, nh * hd)
    w = self.proj.weight
    if x.dtype != w.dtype and not torch.is_autocast_enabled():
        # the sparse kernel writes fp32 (attention.py:243); a model held in
        # bf16 without autocast projects in its own dtype
        x = x.to(w.dtype)
    return self.proj_drop(self.proj(x))
