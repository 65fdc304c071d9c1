"""A small VGGT-shaped stack of global-attention blocks for API tests (random
init; the real VGGT source is not available).  Each block's ``attn`` has the
attribute set the reference's wiring relies on: qkv, q_norm, k_norm, rope,
proj, proj_drop, num_heads."""

import os

import torch
import torch.nn as nn

from ress_b200 import synth


class ToyAttention(nn.Module):
    def __init__(self, dim=1024, num_heads=16):
        super().__init__()
        self.num_heads = num_heads
        self.qkv = nn.Linear(dim, 3 * dim, bias=True)
        self.q_norm = nn.LayerNorm(dim // num_heads)
        self.k_norm = nn.LayerNorm(dim // num_heads)
        self.rope = None
        self.proj = nn.Linear(dim, dim)
        self.proj_drop = nn.Identity()


class ToyBlock(nn.Module):
    def __init__(self, dim=1024, num_heads=16):
        super().__init__()
        self.attn = ToyAttention(dim, num_heads)


class ToyAggregator(nn.Module):
    def __init__(self, n_blocks, dim=1024, num_heads=16):
        super().__init__()
        self.global_blocks = nn.ModuleList([ToyBlock(dim, num_heads) for _ in range(n_blocks)])


class ToyModel(nn.Module):
    def __init__(self, n_blocks=2, dim=1024, num_heads=16, seed=0):
        super().__init__()
        torch.manual_seed(seed)
        self.aggregator = ToyAggregator(n_blocks, dim, num_heads)


def positions(shape: synth.LayerShape, batch=1):
    """(B, N*P, 2): patches at (y+1, x+1), specials at 0 (VGGT's convention)."""
    ys, xs = torch.meshgrid(torch.arange(shape.grid_h), torch.arange(shape.grid_w), indexing="ij")
    patch = torch.stack([ys.reshape(-1), xs.reshape(-1)], -1) + 1
    frame = torch.cat([torch.zeros(shape.n_special, 2, dtype=patch.dtype), patch], 0)
    return frame.repeat(shape.n_frames, 1).unsqueeze(0).expand(batch, -1, -1).contiguous()


def write_tables(directory, name="vggt", n_layers=24, n_heads=16):
    os.makedirs(directory, exist_ok=True)
    torch.save(synth.fisher_table(n_layers, n_heads, seed=1), os.path.join(directory, f"fisher_scores_{name}_cam_pos.pt"))
    torch.save(synth.fisher_table(n_layers, n_heads, seed=3), os.path.join(directory, f"fisher_scores_{name}_pcd.pt"))
