"""Seeded synthetic inputs for one VGGT global-attention layer.

The reference measures on real VGGT activations; no dataset or checkpoint is
available here, so the benchmarks and parity tests use this generator instead.
It follows the configuration text of the benchmark: per head, Q, K and V are
built per 64-token block as a shared cluster mean ~N(0, 1) plus per-token noise
N(0, 0.5^2), and each (tensor, head) pair is then passed through its own random
orthogonal projection.

Machine independence matters more than the exact distribution: fixtures are
generated in one container and checked on another machine, so the generator
uses only operations whose results do not depend on the host CPU's vector
width:

* normals come from numpy's PCG64 ziggurat sampler (scalar code);
* the orthogonal projection is a randomised Walsh-Hadamard transform
  (random sign flips, the normalised 64x64 Hadamard butterfly, a random
  permutation, more sign flips).  Every step is an element-wise IEEE add,
  subtract or multiply by a power of two, so no BLAS or SIMD reduction order
  enters;
* the Fisher table uses the scalar libm ``exp`` per element.

Token layout (``vggt.py:46-58`` of the reference): N frames, each holding
S special tokens first and then H*W patch tokens.  The clusters are laid over
the patch-token sequence in frame-major order, i.e. the sequence the pooled
block map is built on (``models/attention.py:451``); the 5 special tokens of a
frame share one cluster of their own.  The reference's Hilbert permutation
(``models/hilbert.py:128-162``) only reorders patches inside a frame before
this sequence is formed, and the generator produces clusters directly in the
final order, which is what a Hilbert-ordered input looks like to the layer.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

HD = 64
KS_Q = 128
KS_K = 64


@dataclass(frozen=True)
class LayerShape:
    """Token layout of one global layer."""

    n_frames: int
    n_heads: int = 16
    head_dim: int = HD
    n_special: int = 5
    grid_h: int = 37
    grid_w: int = 37

    @property
    def hw(self) -> int:
        return self.grid_h * self.grid_w

    @property
    def tokens_per_frame(self) -> int:
        return self.hw + self.n_special

    @property
    def t_total(self) -> int:  # N * P, also the kernel key length Tk
        return self.n_frames * self.tokens_per_frame

    @property
    def t_patch(self) -> int:
        return self.n_frames * self.hw

    @property
    def t_special(self) -> int:
        return self.n_frames * self.n_special

    @property
    def q_blk(self) -> int:
        return -(-self.t_patch // KS_Q)

    @property
    def k_blk_pooled(self) -> int:
        return -(-self.t_patch // KS_K)

    @property
    def n_cand(self) -> int:
        # attention.py:453-456 -- floor when special tokens exist (sink protection on)
        if self.n_special > 0:
            return self.t_patch // KS_K
        return self.k_blk_pooled

    @property
    def k_blk_kernel(self) -> int:
        return -(-self.t_total // KS_K)

    @property
    def sink_blocks(self) -> int:
        return self.k_blk_kernel - self.n_cand


CONFIG1 = LayerShape(n_frames=4)
CONFIG2 = LayerShape(n_frames=32)
CONFIG4 = LayerShape(n_frames=200)


def _fwht64(x: np.ndarray) -> np.ndarray:
    """Normalised Walsh-Hadamard transform over the last axis (size 64), float32.

    Fixed butterfly order: h = 1, 2, 4, ..., 32; the pair (i, i + h) inside each
    block of 2h becomes (a + b, a - b).  The final scaling by 1/8 is exact."""
    y = x.astype(np.float32, copy=True)
    n = y.shape[-1]
    h = 1
    while h < n:
        y = y.reshape(y.shape[:-1] + (n // (2 * h), 2, h))
        a = y[..., 0, :].copy()
        b = y[..., 1, :].copy()
        y[..., 0, :] = a + b
        y[..., 1, :] = a - b
        y = y.reshape(y.shape[:-3] + (n,))
        h *= 2
    return y * np.float32(0.125)


def _random_orthogonal_apply(x: np.ndarray, rng: np.random.Generator) -> np.ndarray:
    """x: (T, 64) float32 -> x @ O for a random orthogonal O = D1 H P D2."""
    d1 = np.where(rng.integers(0, 2, size=HD) == 1, 1.0, -1.0).astype(np.float32)
    d2 = np.where(rng.integers(0, 2, size=HD) == 1, 1.0, -1.0).astype(np.float32)
    perm = rng.permutation(HD)
    y = _fwht64(x * d1)
    return np.ascontiguousarray(y[:, perm] * d2)


def _clustered_head(shape: LayerShape, rng: np.random.Generator) -> np.ndarray:
    """One head of one tensor, full token layout (N*P, 64) float32."""
    tp = shape.t_patch
    n_blk = -(-tp // KS_K)
    means = rng.standard_normal((n_blk, HD))
    noise = rng.standard_normal((tp, HD)) * 0.5
    patch = (np.repeat(means, KS_K, axis=0)[:tp] + noise).astype(np.float32)
    s = shape.n_special
    out = np.empty((shape.n_frames, shape.tokens_per_frame, HD), np.float32)
    out[:, s:, :] = patch.reshape(shape.n_frames, shape.hw, HD)
    if s > 0:
        smeans = rng.standard_normal((shape.n_frames, 1, HD))
        snoise = rng.standard_normal((shape.n_frames, s, HD)) * 0.5
        out[:, :s, :] = (smeans + snoise).astype(np.float32)
    flat = out.reshape(shape.t_total, HD)
    return _random_orthogonal_apply(flat, rng)


def layer_qkv(shape: LayerShape, seed: int = 0, dtype=torch.float32, device="cpu"):
    """Q, K, V of one global layer in the full token layout (1, nh, N*P, 64).

    ``device`` other than CPU switches to an on-device torch generator: fast,
    but not reproducible across machines; the parity tests always use the CPU
    path."""
    if torch.device(device).type != "cpu":
        return _layer_qkv_device(shape, seed, dtype, device)
    rng = np.random.Generator(np.random.PCG64(seed))
    tensors = []
    for _ in range(3):
        heads = [_clustered_head(shape, rng) for _ in range(shape.n_heads)]
        t = torch.from_numpy(np.stack(heads)).unsqueeze(0)
        tensors.append(t.to(dtype))
    return tuple(tensors)


def _layer_qkv_device(shape: LayerShape, seed, dtype, device):
    g = torch.Generator(device=device).manual_seed(seed)
    tp, nh = shape.t_patch, shape.n_heads
    out = []
    for _ in range(3):
        n_blk = -(-tp // KS_K)
        means = torch.randn(nh, n_blk, HD, generator=g, device=device)
        patch = means.repeat_interleave(KS_K, dim=1)[:, :tp]
        patch = patch + 0.5 * torch.randn(nh, tp, HD, generator=g, device=device)
        full = torch.empty(nh, shape.n_frames, shape.tokens_per_frame, HD, device=device)
        full[:, :, shape.n_special:] = patch.view(nh, shape.n_frames, shape.hw, HD)
        if shape.n_special:
            sm = torch.randn(nh, shape.n_frames, 1, HD, generator=g, device=device)
            full[:, :, :shape.n_special] = sm + 0.5 * torch.randn(
                nh, shape.n_frames, shape.n_special, HD, generator=g, device=device)
        q, _ = torch.linalg.qr(torch.randn(nh, HD, HD, generator=g, device=device))
        full = full.view(nh, -1, HD) @ q
        out.append(full.unsqueeze(0).to(dtype).contiguous())
    return tuple(out)


def fisher_table(n_layers: int = 24, n_heads: int = 16, seed: int = 1) -> torch.Tensor:
    """(3, n_layers, n_heads) log-normal(0, 1) head-importance table (float32)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    z = rng.standard_normal((3, n_layers, n_heads))
    vals = [math.exp(float(v)) for v in z.reshape(-1)]
    return torch.tensor(vals, dtype=torch.float32).view(3, n_layers, n_heads)


def out_proj_weight(dim: int = 1024, seed: int = 2) -> torch.Tensor:
    """Random-init W_O (dim, dim), uniform(-1/sqrt(dim), 1/sqrt(dim)) like nn.Linear."""
    rng = np.random.Generator(np.random.PCG64(seed))
    bound = 1.0 / math.sqrt(dim)
    w = rng.uniform(-bound, bound, size=(dim, dim)).astype(np.float32)
    return torch.from_numpy(w)


def metric_from_weight(w_o: torch.Tensor, n_heads: int = 16) -> torch.Tensor:
    """M_h = (W_O^h)^T W_O^h, (n_heads, hd, hd) float32 (reference projected.py:214-232).

    Formed in float64 and rounded once, so the result does not depend on the
    BLAS blocking of the host."""
    hd = w_o.shape[1] // n_heads
    w = w_o.double()
    ms = []
    for h in range(n_heads):
        wh = w[:, h * hd:(h + 1) * hd]
        ms.append(wh.T @ wh)
    return torch.stack(ms).float()


def split_tokens(x: torch.Tensor, shape: LayerShape):
    """(B, nh, N*P, hd) -> patch (B, nh, N*HW, hd), special (B, nh, N*S, hd).

    Same split as the reference's ``get_patch_tokens``/``get_special_tokens``
    (``models/tokens.py:8-52``)."""
    b, nh, _, hd = x.shape
    v = x.view(b, nh, shape.n_frames, shape.tokens_per_frame, hd)
    patch = v[:, :, :, shape.n_special:, :].reshape(b, nh, shape.t_patch, hd).contiguous()
    special = v[:, :, :, :shape.n_special, :].reshape(b, nh, shape.t_special, hd).contiguous()
    return patch, special


def checksum(t: torch.Tensor) -> str:
    """Bit-level digest of a tensor (for fixture drift detection)."""
    import hashlib
    a = t.detach().cpu().contiguous()
    if a.dtype == torch.bfloat16:
        a = a.view(torch.int16)
    return hashlib.sha256(a.numpy().tobytes()).hexdigest()[:16]
