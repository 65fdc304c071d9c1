"""A VGGT-1B-shaped aggregator for whole-model runs (random init).

The VGGT source and checkpoints are not available here, so this module
builds a network of the same shape from the architecture's published
description: a DINOv2 ViT-L/14 patch encoder with four register tokens
(518 x 518 images -> 37 x 37 patch tokens of width 1024), one camera and
four register tokens prepended to every frame (the 5 special tokens), then
24 pairs of transformer blocks that alternate attention within each frame
and attention over all frames ("global" blocks).  Blocks are pre-norm with
LayerScale, qk LayerNorm, 2-D rotary position embedding (frequency 100)
over the (row, column) patch positions, and a GELU MLP of ratio 4.  The
aggregator returns the concatenated frame/global outputs of layers 4, 11,
17 and 23, as VGGT's heads consume them.

The global blocks' ``attn`` modules carry the attribute set that
``ress_b200.wiring`` patches (qkv, q_norm, k_norm, rope, proj, proj_drop,
num_heads), so ``apply_*`` install the sparse global attention exactly as
on the original model.  Frame attention and the MLPs stay torch (cuBLAS
GEMMs, SDPA).

For view-sharded runs every global ``attn`` may carry ``ress_view =
(ViewGeom, gather)``; the frames of ``images`` are then this rank's frames
and the sparse layer all-gathers K and V itself.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class RotaryPosition2D(nn.Module):
    """Rotary embedding over 2-D integer positions: the first half of the
    head dimension is rotated by the row, the second half by the column,
    with angle p / frequency^(2i/d) on feature pairs (i, i + d/2)."""

    MAX_POS = 4096  # positions are patch rows / columns (+1), far below this

    def __init__(self, frequency: float = 100.0):
        super().__init__()
        self.frequency = frequency
        self._tables = {}

    def _cos_sin(self, dim: int, n: int, device, dtype):
        key = (dim, n, device, dtype)
        t = self._tables.get(key)
        if t is None:
            inv = 1.0 / (self.frequency ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
            ang = torch.outer(torch.arange(n, device=device, dtype=torch.float32), inv)
            ang = torch.cat([ang, ang], dim=-1)
            t = (ang.cos().to(dtype), ang.sin().to(dtype))
            self._tables[key] = t
        return t

    def forward(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        # x (B, nh, T, hd), pos (B, T, 2) integer
        d = x.shape[-1] // 2
        cos, sin = self._cos_sin(d, self.MAX_POS, x.device, x.dtype)  # fixed size: no host sync
        parts = []
        for axis in range(2):
            xa = x[..., axis * d:(axis + 1) * d]
            c = F.embedding(pos[..., axis], cos)[:, None]
            s = F.embedding(pos[..., axis], sin)[:, None]
            x1, x2 = xa.chunk(2, dim=-1)
            parts.append(xa * c + torch.cat([-x2, x1], dim=-1) * s)
        return torch.cat(parts, dim=-1)


class Attention(nn.Module):
    def __init__(self, dim: int, num_heads: int, qk_norm: bool, rope: RotaryPosition2D | None):
        super().__init__()
        self.num_heads = num_heads
        hd = dim // num_heads
        self.qkv = nn.Linear(dim, 3 * dim, bias=True)
        self.q_norm = nn.LayerNorm(hd) if qk_norm else nn.Identity()
        self.k_norm = nn.LayerNorm(hd) if qk_norm else nn.Identity()
        self.rope = rope
        self.proj = nn.Linear(dim, dim)
        self.proj_drop = nn.Identity()

    def forward(self, x, pos=None):
        B, T, C = x.shape
        nh = self.num_heads
        hd = C // nh
        lin = self.qkv(x)
        if x.is_cuda and x.dtype == torch.bfloat16 and hd == 64 and not torch.is_autocast_enabled():
            # bf16 on the GPU: the library's q/k prologue (norms and rotary
            # embedding in one pass) where it applies, then its dense bf16
            # attention writing token-major rows straight into proj's input
            from . import kernels as K
            from .qkv import _fused_prologue

            fused = _fused_prologue(self, lin, pos, nh, hd)
            if fused is None:
                q, k, v = lin.view(B, T, 3, nh, hd).permute(2, 0, 3, 1, 4).unbind(0)
                q, k = self.q_norm(q), self.k_norm(k)
                if self.rope is not None and pos is not None:
                    q, k = self.rope(q, pos), self.rope(k, pos)
                fused = (q.contiguous(), k.contiguous(), v.contiguous())
            q, k, v = fused
            o = torch.empty(B, T, C, dtype=x.dtype, device=x.device)
            K.dense_attn(q.reshape(B * nh, T, hd), k.reshape(B * nh, T, hd), v.reshape(B * nh, T, hd), out=o,
                         out_rows=(nh, T * C, hd, C, T, 0, 0))
            return self.proj_drop(self.proj(o))
        q, k, v = lin.view(B, T, 3, nh, hd).permute(2, 0, 3, 1, 4).unbind(0)
        q, k = self.q_norm(q), self.k_norm(k)
        if self.rope is not None and pos is not None:
            q, k = self.rope(q, pos), self.rope(k, pos)
        o = F.scaled_dot_product_attention(q, k, v)
        return self.proj_drop(self.proj(o.transpose(1, 2).reshape(B, T, C)))


class Mlp(nn.Module):
    def __init__(self, dim: int, ratio: int = 4):
        super().__init__()
        self.fc1 = nn.Linear(dim, ratio * dim)
        self.fc2 = nn.Linear(ratio * dim, dim)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x)))


class LayerScale(nn.Module):
    def __init__(self, dim: int, init: float):
        super().__init__()
        self.gamma = nn.Parameter(torch.full((dim,), init))

    def forward(self, x):
        return x * self.gamma


class Block(nn.Module):
    def __init__(self, dim: int, num_heads: int, qk_norm: bool, rope, ls_init: float):
        super().__init__()
        self.norm1 = nn.LayerNorm(dim)
        self.attn = Attention(dim, num_heads, qk_norm, rope)
        self.ls1 = LayerScale(dim, ls_init)
        self.norm2 = nn.LayerNorm(dim)
        self.mlp = Mlp(dim)
        self.ls2 = LayerScale(dim, ls_init)

    def forward(self, x, pos=None):
        x = x + self.ls1(self.attn(self.norm1(x), pos=pos))
        return x + self.ls2(self.mlp(self.norm2(x)))


class PatchEncoder(nn.Module):
    """DINOv2 ViT-L/14-shaped encoder with register tokens; returns the
    normalised patch tokens (B, hw, dim)."""

    def __init__(self, dim: int = 1024, depth: int = 24, num_heads: int = 16, patch: int = 14, img: int = 518,
                 registers: int = 4):
        super().__init__()
        self.patch = patch
        self.proj = nn.Conv2d(3, dim, patch, stride=patch)
        n = (img // patch) ** 2
        self.cls_token = nn.Parameter(torch.randn(1, 1, dim) * 0.02)
        self.reg_tokens = nn.Parameter(torch.randn(1, registers, dim) * 0.02)
        self.pos_embed = nn.Parameter(torch.randn(1, 1 + n, dim) * 0.02)
        self.blocks = nn.ModuleList([Block(dim, num_heads, False, None, 1e-5) for _ in range(depth)])
        self.norm = nn.LayerNorm(dim)
        self.n_prefix = 1 + registers

    def forward(self, images):
        x = self.proj(images).flatten(2).transpose(1, 2)
        B = x.shape[0]
        x = torch.cat([self.cls_token.expand(B, -1, -1), x], dim=1) + self.pos_embed
        x = torch.cat([x[:, :1], self.reg_tokens.expand(B, -1, -1), x[:, 1:]], dim=1)
        for blk in self.blocks:
            x = blk(x)
        return self.norm(x)[:, self.n_prefix:]


class Aggregator(nn.Module):
    def __init__(self, dim: int = 1024, depth: int = 24, num_heads: int = 16, img: int = 518, patch: int = 14,
                 encoder_depth: int = 24, intermediate=(4, 11, 17, 23)):
        super().__init__()
        self.patch_size = patch
        self.patch_embed = PatchEncoder(dim, encoder_depth, num_heads, patch, img)
        self.rope = RotaryPosition2D(100.0)
        self.frame_blocks = nn.ModuleList([Block(dim, num_heads, True, self.rope, 0.01) for _ in range(depth)])
        self.global_blocks = nn.ModuleList([Block(dim, num_heads, True, self.rope, 0.01) for _ in range(depth)])
        self.camera_token = nn.Parameter(torch.randn(1, 2, 1, dim) * 0.02)
        self.register_token = nn.Parameter(torch.randn(1, 2, 4, dim) * 0.02)
        self.patch_start_idx = 5
        self.intermediate = tuple(intermediate)
        self.register_buffer("_mean", torch.tensor([0.485, 0.456, 0.406]).view(1, 1, 3, 1, 1), persistent=False)
        self.register_buffer("_std", torch.tensor([0.229, 0.224, 0.225]).view(1, 1, 3, 1, 1), persistent=False)

    @staticmethod
    def _special(tok, B, N, first_frame: bool):
        # token (1, 2, k, C): index 0 for the first frame of the whole sequence, 1 for the others
        C = tok.shape[-1]
        if first_frame:
            t = torch.cat([tok[:, :1].expand(B, 1, -1, -1), tok[:, 1:].expand(B, N - 1, -1, -1)], dim=1)
        else:
            t = tok[:, 1:].expand(B, N, -1, -1)
        return t.reshape(B * N, -1, C)

    def positions(self, BN: int, h: int, w: int, device):
        ys, xs = torch.meshgrid(torch.arange(h, device=device), torch.arange(w, device=device), indexing="ij")
        patch = torch.stack([ys.reshape(-1), xs.reshape(-1)], dim=-1) + 1
        pos = torch.cat([torch.zeros(self.patch_start_idx, 2, dtype=patch.dtype, device=device), patch], dim=0)
        return pos.unsqueeze(0).expand(BN, -1, -1)

    def forward(self, images, first_frame: bool = True):
        """images (B, N, 3, H, W) in [0, 1] -> list of (B, N, P, 2*dim) at the
        intermediate layers (None elsewhere), patch_start_idx.
        ``first_frame`` says whether frame 0 of ``images`` is frame 0 of the
        sequence (False on the other ranks of a view-sharded run)."""
        B, N, _, H, W = images.shape
        x = ((images - self._mean) / self._std).view(B * N, 3, H, W).to(self.camera_token.dtype)
        patches = self.patch_embed(x)
        C = patches.shape[-1]
        tokens = torch.cat([self._special(self.camera_token, B, N, first_frame),
                            self._special(self.register_token, B, N, first_frame), patches], dim=1)
        P = tokens.shape[1]
        h, w = H // self.patch_size, W // self.patch_size
        pos = self.positions(B * N, h, w, images.device)
        outputs = []
        for i in range(len(self.frame_blocks)):
            tokens = self.frame_blocks[i](tokens.view(B * N, P, C), pos=pos)
            frame_out = tokens.view(B, N, P, C)
            tokens = self.global_blocks[i](tokens.view(B, N * P, C), pos=pos.reshape(B, N * P, 2))
            global_out = tokens.view(B, N, P, C)
            outputs.append(torch.cat([frame_out, global_out], dim=-1) if i in self.intermediate else None)
        return outputs, self.patch_start_idx


class VGGTAggregatorModel(nn.Module):
    """Holds ``aggregator`` like VGGT does, so ``model.aggregator.global_blocks``
    is where the method's wiring looks."""

    def __init__(self, **kw):
        super().__init__()
        self.aggregator = Aggregator(**kw)

    def forward(self, images, first_frame: bool = True):
        return self.aggregator(images, first_frame=first_frame)
