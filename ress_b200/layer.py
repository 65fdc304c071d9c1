"""One sparse global-attention layer on the GPU, end to end.

This is the body of the reference's ``ress_attention_forward`` after the
Q/K/V projection (src/ress/models/attention.py:404-659), chained from the
library's kernels with no host synchronisation:

  1. ress_pool_quant_q / _kv   pooled means (a.3, a.4) and int8 Q/K, fp16 V
                               (a.12) in one read of Q, K and V each
  2. ress_predict              pooled softmax + candidate renormalisation (a.3, a.5)
  3. ress_baseline             CDF / ratio budget (a.6)
  4. ress_hess_adjust          HeSS per-head re-allocation (a.7), when the
                               budget is HeSS
  5. ress_restore_swap         ReSS ordering -> keep lists (a.8-a.11), or
     ress_select_prob          probability ordering -> keep lists (a.11)
  6. ress_sparse_attn          tcgen05 block-sparse attention (a.12), written
                               straight into the full token layout
  7. torch SDPA                the special-token queries attend densely to all
                               keys (a.2), on a side stream

The input tensors are the layer's q, k, v in the full token layout
(B, H, frames * (special + hw), 64): the patch/special split of the reference
(models/tokens.py) is folded into the kernels' index arithmetic, and the
output lands in the same layout, which is what combine_special_and_patch
(models/qkv.py:71-81) would have produced.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import kernels as K

MIN_NUM_TO_SELECT = 2  # attention.py:40


@dataclass
class BudgetSpec:
    """How many blocks each (head, q-block) keeps (budget/hess.py,
    budget/uniform.py).  kind: "uniform" or "hess"."""

    kind: str
    sparse_ratio: float | None = None
    cdf_threshold: float | None = None
    beta: float = 1.0
    scores_norm: torch.Tensor | None = None  # (H,) fp32 for "hess"; on the layer's device for graph capture


@dataclass
class OrderSpec:
    """Which blocks fill the budget.  kind: "probability", "restore_swap" or
    "random"."""

    kind: str = "probability"
    M: torch.Tensor | None = None  # (H, 64, 64) fp32, restore_swap
    n_iters: int = 5
    track_best: bool = True
    restore_frac: float = 0.5
    decay: float = 0.5


@dataclass
class HeadShard:
    """This process owns heads [h0, h0 + H_local) of h_total (heads split
    across GPUs).  HeSS couples the heads of a q-block column, so the
    baseline counts of all heads are gathered (``gather``: (B, H_local, nq)
    int32 -> (B, h_total, nq) int32, an NCCL all-gather) and the small
    re-allocation is computed redundantly on every GPU."""

    h0: int
    h_total: int
    gather: object
    heads: tuple | None = None  # this rank's global head indices when not the contiguous [h0, h0 + H_local)

    def select(self, full: torch.Tensor, H: int) -> torch.Tensor:
        if self.heads is None:
            return full[:, self.h0: self.h0 + H].contiguous()
        # the index lives on the device from the first (eager) call on: no host copy during graph capture
        cache = self.__dict__.setdefault("_idx", {})
        idx = cache.get(full.device)
        if idx is None:
            idx = cache[full.device] = torch.as_tensor(self.heads, dtype=torch.long, device=full.device)
        return full.index_select(1, idx)


@dataclass
class LayerResult:
    out: torch.Tensor                  # (B, H, N*P, 64) fp32, full token layout
    layout: K.Layout
    lists: torch.Tensor                # (B*H*nq, width) int32 keep lists
    counts: torch.Tensor               # (B*H*nq,) int32
    nts: torch.Tensor                  # (B, H, nq) int32 budgets
    attn_full: torch.Tensor | None = None
    attn_cond: torch.Tensor | None = None
    vbar: torch.Tensor | None = None
    extra: dict = field(default_factory=dict)

    @property
    def width(self) -> int:
        return self.layout.n_cand + self.layout.sink_blocks

    def sparsity(self) -> float:
        """1 - mean(final_map), sinks counted (attention.py:242).  Synchronises."""
        rows = self.counts.numel()
        return 1.0 - float(self.counts.sum().item()) / float(rows * self.width)

    def final_map(self) -> torch.Tensor:
        """Dense (B, H, nq, width) bool block map (API compatibility only)."""
        L = self.layout
        m = K.lists_to_map(self.lists, self.counts, self.width)
        return m.view(L.B, L.H, L.nq, self.width)


_random_gens = {}
_side_streams = {}


def _side_stream(dev):
    st = _side_streams.get(dev)
    if st is None:
        st = torch.cuda.Stream(device=dev)
        _side_streams[dev] = st
    return st


def _random_gen(device):
    """One generator per device for block_criterion="random", seeded once
    (attention.py:177-196)."""
    g = _random_gens.get(device)
    if g is None:
        g = torch.Generator(device=device).manual_seed(20260826)
        _random_gens[device] = g
    return g


def special_attention(q, k, v, L: K.Layout, out=None, q_special=None):
    """Dense attention of the special-token queries over all keys
    (attention.py:404-409; the key order does not change a softmax).
    bf16 layers with an fp32 full-layout ``out``: the library's dense bf16
    kernel writes the rows straight into their places in ``out`` and None is
    returned.  Otherwise (fp32 layers) torch SDPA's result is returned for
    the caller to place.  q_special: the special queries alone, (B*H,
    frames*special, 64) bf16 (the fused prologue's output), instead of q."""
    if L.special == 0:
        return None
    B, H = L.B, L.H
    if q_special is not None:
        if k.dtype != torch.bfloat16 or out is None or out.dtype != torch.float32 or out.stride(-1) != 1:
            raise K.RessError("special queries from the fused prologue take a bf16 layer and an fp32 output")
        k2, v2 = k.flatten(0, 1), v.flatten(0, 1)
        if k2.stride() != v2.stride():
            k2, v2 = k2.contiguous(), v2.contiguous()
        rows = (H, out.stride(0), out.stride(1), out.stride(2), L.special, L.special + L.hw, 0)
        K.dense_attn(q_special, k2, v2, out=out, out_rows=rows)
        return None
    qs = q.view(B, H, L.frames, L.special + L.hw, 64)[:, :, :, : L.special]
    if q.dtype == torch.bfloat16 and out is not None and out.dtype == torch.float32 and out.stride(-1) == 1:
        q2 = qs.reshape(B * H, L.Ts, 64)  # gathers the special rows (small)
        k2, v2 = k.flatten(0, 1), v.flatten(0, 1)
        if k2.stride() != v2.stride():
            k2, v2 = k2.contiguous(), v2.contiguous()
        rows = (H, out.stride(0), out.stride(1), out.stride(2), L.special, L.special + L.hw, 0)
        K.dense_attn(q2, k2, v2, out=out, out_rows=rows)
        return None
    return F.scaled_dot_product_attention(qs.reshape(B, H, L.Ts, 64), k, v)


def select_blocks(attn_full, attn_cond, vbar, B: int, H: int, nq: int, n_cand: int, sink_blocks: int,
                  budget: BudgetSpec | None, order: OrderSpec, *, num_to_select=None, budget_fn=None,
                  lead_blocks: int = 0, shard: HeadShard | None = None, ws=None):
    """Budget (a.6, a.7) and block order (a.8-a.11) of one layer's (head,
    q-block) rows -> (nts (B, H, nq) int32, dict(lists, counts)).
    attn_full (B*H, nq, nkp), attn_cond (B*H, nq, n_cand), vbar (B*H, nkp, 64)."""
    dev = attn_cond.device
    min_sel = min(MIN_NUM_TO_SELECT, n_cand)
    if num_to_select is not None:
        nts = num_to_select.to(device=dev, dtype=torch.int32).reshape(B, H, nq).clamp(min=min_sel)
    elif budget is not None:
        base = K.baseline(attn_cond, budget.sparse_ratio, budget.cdf_threshold).view(B, H, nq)
        if budget.kind == "hess" and shard is not None:
            full = shard.gather(base)
            nts_full = K.hess_adjust(full, budget.scores_norm, n_cand, beta=budget.beta, min_clamp=min_sel)
            nts = shard.select(nts_full, H)
        elif budget.kind == "hess":
            nts = K.hess_adjust(base, budget.scores_norm, n_cand, beta=budget.beta, min_clamp=min_sel)
        else:
            nts = base.clamp(min=min_sel)
    elif budget_fn is not None:
        nts = budget_fn(attn_cond.view(B, H, nq, n_cand))
        nts = nts.to(device=dev, dtype=torch.int32).reshape(B, H, nq).clamp(min=min_sel)
    else:
        raise AssertionError("num_to_select (or budget_fn) required unless dense=True")

    if order.kind == "restore_swap":
        r = K.restore_swap(attn_full, vbar, order.M, nts.view(-1), n_cand, n_iters=order.n_iters,
                           track_best=order.track_best, restore_frac=order.restore_frac, decay=order.decay,
                           sink_blocks=sink_blocks, lead_blocks=lead_blocks, ws=ws)
    elif order.kind == "probability":
        r = K.select_prob(attn_cond, nts.view(-1), sink_blocks=sink_blocks, lead_blocks=lead_blocks)
    elif order.kind == "random":
        key = torch.rand(attn_cond.shape, device=dev, dtype=torch.float32, generator=_random_gen(dev))
        keep = K.top_m_mask(key, nts.view(-1)).view(-1, n_cand)
        full_map = torch.cat([keep, torch.ones(keep.shape[0], sink_blocks, dtype=torch.bool, device=dev)], -1)
        if lead_blocks:
            full_map[:, :lead_blocks] = True
        lists, counts = K.map_to_lists(full_map)
        r = dict(lists=lists, counts=counts)
    else:
        raise ValueError(order.kind)
    return nts, r


def global_layer(q, k, v, L: K.Layout, budget: BudgetSpec | None, order: OrderSpec, *,
                 num_to_select: torch.Tensor | None = None, budget_fn=None, keep_pooled: bool = False,
                 lead_blocks: int = 0, out: torch.Tensor | None = None,
                 shard: HeadShard | None = None, joint_select_fn=None, map_hook=None,
                 attn_split=False, q_scored: dict | None = None) -> LayerResult:
    """Run one sparse global-attention layer.  q, k, v: (B, H, N*P, 64) CUDA,
    float32 or bfloat16.  Exactly one of ``budget``, ``num_to_select`` (a
    (B, H, nq) tensor) or ``budget_fn`` (callable(attn_cond) -> (B, H, nq))
    decides the per-row block count.  ``attn_split`` is the attention's
    ``split`` option (kernels.sparse_attn): None lets a layer with few rows
    (a head split over many GPUs) spread its longest rows over two CTAs.
    ``q_scored``: the fused prologue's output (kernels.qkv_prologue_scored:
    the patch queries pooled and quantised, the special queries apart); q is
    then None and the layer's own Q pass is skipped."""
    dev = k.device
    if k.stride() != v.stride():
        v = v.contiguous()
        k = k.contiguous()
    B, H = L.B, L.H
    n_cand = L.n_cand
    ws = K.workspace(dev, B * H, L.Tp, L.Tk, n_cand)
    if out is None:
        out = torch.empty(B, H, L.frames * (L.special + L.hw), 64, dtype=torch.float32, device=dev)
    main = torch.cuda.current_stream(dev)
    capturing = torch.cuda.is_current_stream_capturing()
    side = _side_stream(dev)
    side.wait_stream(main)
    q_special = None if q_scored is None else q_scored["q_special"]
    with torch.cuda.stream(side):
        # special rows of `out` (disjoint from the patch rows the main stream writes)
        x_special = special_attention(q, k, v, L, out, q_special=q_special)
    if not capturing:
        for t in (q, k, v, out, q_special):
            if t is not None:
                t.record_stream(side)

    if q_scored is None:
        qbar, q8, qs = K.pool_quant_q(q, L)
    else:
        qbar, q8, qs = q_scored["qbar"], q_scored["q8"], q_scored["qs"]
    kbar, vbar, k8, ks, v16, km = K.pool_quant_kv(k, v, L, ws=ws)
    need_full = order.kind == "restore_swap" or keep_pooled
    attn_full, attn_cond = K.predict(qbar, kbar, n_cand, full=need_full, cond=True)
    width = n_cand + L.sink_blocks
    if joint_select_fn is not None:
        # one-shot joint selection (attention.py:501-508): the callable returns the final map
        fm = joint_select_fn(attn_cond.view(B, H, L.nq, n_cand), vbar.view(B, H, L.nkp, 64)[:, :, :n_cand],
                             L.sink_blocks)
        if map_hook is not None:
            fm = map_hook(fm.view(B, H, L.nq, width), attn_cond.view(B, H, L.nq, n_cand))
        lists, counts = K.map_to_lists(fm.reshape(-1, width))
        K.sparse_attn(q8, qs, k8, ks, v16, lists, counts, out=out, out_layout=L, split=attn_split)
        main.wait_stream(side)
        if x_special is not None:
            if not capturing:
                x_special.record_stream(main)
            view = out.view(B, H, L.frames, L.special + L.hw, 64)
            view[:, :, :, : L.special] = x_special.view(B, H, L.frames, L.special, 64).float()
        return LayerResult(out=out, layout=L, lists=lists, counts=counts, nts=None, attn_full=attn_full,
                           attn_cond=attn_cond, vbar=vbar)
    nts, r = select_blocks(attn_full, attn_cond, vbar, B, H, L.nq, n_cand, L.sink_blocks, budget, order,
                           num_to_select=num_to_select, budget_fn=budget_fn, lead_blocks=lead_blocks, shard=shard,
                           ws=ws)

    if map_hook is not None:
        fm = K.lists_to_map(r["lists"], r["counts"], width).view(B, H, L.nq, width)
        fm = map_hook(fm, attn_cond.view(B, H, L.nq, n_cand))
        lists, counts = K.map_to_lists(fm.reshape(-1, width))
        r = dict(lists=lists, counts=counts)
    K.sparse_attn(q8, qs, k8, ks, v16, r["lists"], r["counts"], out=out, out_layout=L, split=attn_split)
    main.wait_stream(side)
    if x_special is not None:
        if not capturing:
            x_special.record_stream(main)
        view = out.view(B, H, L.frames, L.special + L.hw, 64)
        view[:, :, :, : L.special] = x_special.view(B, H, L.frames, L.special, 64).float()
    return LayerResult(out=out, layout=L, lists=r["lists"], counts=r["counts"], nts=nts,
                       attn_full=attn_full, attn_cond=attn_cond, vbar=vbar)


class CapturedLayer:
    """A layer call captured once into a CUDA graph and replayed.

    ``fn`` must read its inputs from and write its output to tensors that stay
    alive (static buffers); every kernel of the layer is stream-ordered with
    no host synchronisation, so the whole step -- the library's kernels, the
    side-stream SDPA and, under a head split, the NCCL all-gather -- becomes
    one graph launch.  Replays give the same bits as eager calls."""

    def __init__(self, fn, warmup: int = 2):
        dev = torch.cuda.current_device()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.result = fn()

    def replay(self):
        self.graph.replay()
        return self.result


def dense_layer(q, k, v, L: K.Layout) -> torch.Tensor:
    """The dense=True branch (attention.py:484-486): exact SDPA, torch."""
    return F.scaled_dot_product_attention(q, k, v)
