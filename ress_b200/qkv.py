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


def compute_qkv(self, x, pos, num_special_tokens=5, num_heads=16, shape=None):
    """q, k, v as (B, nh, N*P, hd) views/tensors plus the shape dict."""
    shp = layer_shape(x, pos, num_special_tokens, num_heads, shape)
    B, NP, C = x.shape
    nh, hd = num_heads, C // num_heads
    qkv = self.qkv(x).view(B, NP, 3, nh, hd).permute(2, 0, 3, 1, 4)
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
