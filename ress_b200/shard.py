"""Splitting one sparse global-attention layer across the GPUs of a node.

Every stage of the layer is independent per attention head except the HeSS
budget (budget/_proportional.py:149-215), which re-allocates the baseline
counts of all heads of a q-block column.  Heads are therefore split across
ranks (balanced by their expected work, ranks may hold different numbers of
heads), and the only exchange is an all-gather of the (B, H_local, nq)
int32 baselines before ``ress_hess_adjust``, which then runs redundantly on
every rank over all heads (it is tiny).  The gather uses the list form of
``all_gather`` so the same code runs on NCCL and on gloo (CPU tests).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .layer import HeadShard


def head_range(n_heads: int, world: int, rank: int):
    if n_heads % world:
        raise ValueError(f"{n_heads} heads do not split evenly over {world} ranks")
    hl = n_heads // world
    return rank * hl, hl


def budget_shares(scores, cap: float | None = None) -> list:
    """Each head's expected share of the layer's blocks under HeSS, in units
    of the mean head budget: proportional to its score, capped at `cap` (all
    candidate blocks, i.e. n_cand / baseline = 1 / (1 - sparse_ratio)) with
    the excess spread over the uncapped heads in proportion, the way
    ``adjust_attention_selection`` re-allocates (budget/_proportional.py)."""
    s = [max(float(x), 0.0) for x in scores]
    H = len(s)
    tot = sum(s) or 1.0
    w = [x / tot * H for x in s]
    if cap is None:
        return w
    capped = [False] * H
    for _ in range(H):
        over = [i for i in range(H) if not capped[i] and w[i] > cap]
        if not over:
            break
        for i in over:
            capped[i] = True
        excess = sum(w[i] - cap for i in over)
        for i in over:
            w[i] = cap
        free = sum(w[i] for i in range(H) if not capped[i])
        if free <= 0:
            break
        for i in range(H):
            if not capped[i]:
                w[i] += excess * w[i] / free
    return w


# Per-head fixed cost of a rank, in units of the attention time of a head with
# the mean budget: scoring, pooled map, budget and restore-swap cost the same
# for every head (they run over all its candidates), attention grows with the
# kept blocks.  With few heads per GPU the per-head stages no longer fill the
# SMs and cost more per head than in a full layer (restore-swap of one head of
# the cfg2 layer: 0.136 ms, of sixteen: 1.16 ms).  Fitted to whole-layer times
# of head groups of the cfg2 layer on one B200 (groups of 1-4 heads, time =
# 0.21 + 0.118 * heads + 0.318 * budget share ms): 0.118 / 0.318 = 0.37.
HEAD_COST = 0.37


def balanced_heads(scores, world: int, cap: float | None = None, equal_size: bool = True,
                   head_cost: float = HEAD_COST) -> list:
    """Partition the heads over `world` ranks so that the ranks' expected
    work is even.  equal_size: groups of H / world heads balanced by their
    summed expected budgets (``budget_shares``), greedily (heaviest head first,
    to the lightest group with room).  Otherwise groups of any size (at
    least one head each) balanced by head_cost + budget share per head:
    longest-processing-time-first, then moves and swaps out of the heaviest
    group while they lower its load.  The result depends only on the scores,
    so every rank computes the same one."""
    s = budget_shares(scores, cap)
    H = len(s)
    if equal_size:
        if H % world:
            raise ValueError(f"{H} heads do not split evenly over {world} ranks")
        per = H // world
        groups = [[] for _ in range(world)]
        sums = [0.0] * world
        for h in sorted(range(H), key=lambda i: (-s[i], i)):
            g = min((i for i in range(world) if len(groups[i]) < per), key=lambda i: (sums[i], i))
            groups[g].append(h)
            sums[g] += s[h]
        return [sorted(g) for g in groups]
    if world > H:
        raise ValueError(f"{H} heads cannot give each of {world} ranks one")
    c = [x + head_cost for x in s]
    groups = [[] for _ in range(world)]
    load = [0.0] * world
    for h in sorted(range(H), key=lambda i: (-c[i], i)):
        g = min(range(world), key=lambda i: (load[i], i))
        groups[g].append(h)
        load[g] += c[h]
    for _ in range(64 * H):  # each step lowers the maximum load, so this ends long before
        mx = max(range(world), key=lambda i: (load[i], -i))
        top = load[mx]
        best = None  # (new max of the pair, kind, head, other group, other head)
        for o in range(world):
            if o == mx:
                continue
            for h in groups[mx]:
                if len(groups[mx]) > 1:
                    new = max(top - c[h], load[o] + c[h])
                    if new < top - 1e-12 and (best is None or new < best[0]):
                        best = (new, h, o, None)
                for h2 in groups[o]:
                    d = c[h] - c[h2]
                    if d > 0:
                        new = max(top - d, load[o] + d)
                        if new < top - 1e-12 and (best is None or new < best[0]):
                            best = (new, h, o, h2)
        if best is None:
            break
        _, h, o, h2 = best
        groups[mx].remove(h)
        groups[o].append(h)
        load[mx] -= c[h]
        load[o] += c[h]
        if h2 is not None:
            groups[o].remove(h2)
            groups[mx].append(h2)
            load[o] -= c[h2]
            load[mx] += c[h2]
    return [sorted(g) for g in groups]


def make_gather(world: int, group=None, order=None, sizes=None):
    """base (B, H_local, nq) int32 -> (B, H, nq): rank order, or global head
    order when `order` (the heads of every rank, rank after rank) is given.
    sizes: heads per rank when they differ; each rank's part then travels
    padded to the largest size.  One all_gather_into_tensor into a
    (world * B, pad, nq) buffer and one index_select that picks every head's
    slot in global order: three kernels at most inside a captured step."""
    if sizes is None:
        sizes = None if order is None else [len(order) // world] * world
    on_device = {}  # device copies of the slot index, made on the first (eager) call

    def slot_index(pad: int, h_local: int) -> torch.Tensor:
        # (rank, slot) of every head in global order, flattened over (rank, slot)
        sz = sizes if sizes is not None else [h_local] * world
        flat = []
        for r, n in enumerate(sz):
            flat.extend(r * pad + i for i in range(n))
        idx = torch.as_tensor(flat, dtype=torch.long)
        if order is not None:
            inv = torch.empty(len(order), dtype=torch.long)
            inv[torch.as_tensor(order, dtype=torch.long)] = torch.arange(len(order))
            idx = idx[inv]
        return idx

    def gather(base: torch.Tensor) -> torch.Tensor:
        B, h_local = base.shape[0], base.shape[1]
        pad = max(sizes) if sizes is not None else h_local
        if h_local == pad:
            send = base.contiguous()
        else:
            send = base.new_zeros(B, pad, *base.shape[2:])
            send[:, :h_local] = base
        buf = send.new_empty(world * B, *send.shape[1:])  # rank r's part: rows [r*B, (r+1)*B)
        dist.all_gather_into_tensor(buf, send, group=group)
        flat = buf.view(world * pad, *base.shape[2:]) if B == 1 else \
            buf.view(world, B, pad, *base.shape[2:]).transpose(0, 1).reshape(B, world * pad, *base.shape[2:])
        key = (base.device, pad, h_local)
        idx = on_device.get(key)
        if idx is None:
            idx = on_device[key] = slot_index(pad, h_local).to(base.device)
        if B == 1:
            return flat.index_select(0, idx).unsqueeze(0)
        return flat.index_select(1, idx)
    return gather


def make_head_shard(n_heads: int, world: int, rank: int, group=None, scores=None, cap=None,
                    equal_size: bool = True, head_cost: float = HEAD_COST) -> HeadShard:
    """Contiguous head ranges, or with `scores` (the layer's HeSS head scores)
    the balanced partition of ``balanced_heads`` (equal_size=False: ranks
    may hold different numbers of heads)."""
    if scores is None:
        h0, _ = head_range(n_heads, world, rank)
        return HeadShard(h0=h0, h_total=n_heads, gather=make_gather(world, group))
    parts = balanced_heads(scores, world, cap, equal_size=equal_size, head_cost=head_cost)
    order = [h for p in parts for h in p]
    return HeadShard(h0=parts[rank][0], h_total=n_heads,
                     gather=make_gather(world, group, order, sizes=[len(p) for p in parts]),
                     heads=tuple(parts[rank]))


# ----------------------------------------------------------------- views
# Whole-model runs with many views shard the frames: rank r owns frames
# [r * F, (r + 1) * F) of every layer (F = frames / world).  A global layer
# then needs every key and value, so K and V are all-gathered (the only
# large exchange), while each rank keeps its own queries.  The pooled-map
# q-blocks are 128 patch tokens of the global patch order, so a rank's
# first and last q-block can straddle a shard boundary; the up-to-127 patch
# queries it lacks come from its neighbours (each rank contributes its first
# and last 128 patch queries to a small all-gather), and the straddling
# q-block is computed on both sides, each keeping the rows of its own tokens.
# Every (head, q-block) row then sees exactly the inputs of the unsharded
# layer, so its budget, keep list and output are the same bits.

KS_Q = 128


@dataclass
class ViewGeom:
    """Where rank ``rank`` of ``world`` sits in a layer of ``frames`` frames."""

    frames: int
    special: int
    hw: int
    world: int
    rank: int

    def __post_init__(self):
        if self.frames % self.world:
            raise ValueError(f"{self.frames} frames do not split evenly over {self.world} ranks")
        if self.frames_local * self.hw < KS_Q:
            raise ValueError("each rank needs at least one q-block of its own patch tokens")

    @property
    def frames_local(self) -> int:
        return self.frames // self.world

    @property
    def f0(self) -> int:
        return self.rank * self.frames_local

    @property
    def p0(self) -> int:
        """First global patch index of this rank."""
        return self.f0 * self.hw

    @property
    def p1(self) -> int:
        return self.p0 + self.frames_local * self.hw

    @property
    def Tp(self) -> int:
        return self.frames * self.hw

    @property
    def b0(self) -> int:
        """First global q-block that holds one of this rank's patch tokens."""
        return self.p0 // KS_Q

    @property
    def b1(self) -> int:
        return -(-self.p1 // KS_Q)

    @property
    def lo(self) -> int:
        """Patch queries of the previous rank that this rank's first q-block needs."""
        return self.p0 - self.b0 * KS_Q

    @property
    def hi(self) -> int:
        """Patch queries of the next rank that this rank's last q-block needs."""
        return min(self.b1 * KS_Q, self.Tp) - self.p1


def patch_tokens(x: torch.Tensor, special: int, hw: int) -> torch.Tensor:
    """(B, H, F*(special+hw), 64) full layout -> (B, H, F*hw, 64) patch tokens."""
    B, H, T, D = x.shape
    f = T // (special + hw)
    return x.view(B, H, f, special + hw, D)[:, :, :, special:].reshape(B, H, f * hw, D)


def view_exchange_parts(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, geom: ViewGeom) -> dict:
    """What this rank contributes to the view exchange: its K and V and the
    first / last 128 patch queries (the neighbours' halos)."""
    qp = patch_tokens(q, geom.special, geom.hw)
    return dict(k=k.contiguous(), v=v.contiguous(), qhead=qp[:, :, :KS_Q].contiguous(),
                qtail=qp[:, :, -KS_Q:].contiguous())


def make_view_gather(world: int, group=None):
    """all_gather over the process group: (name, tensor) -> list of world tensors."""
    def gather(name: str, t: torch.Tensor):
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t, group=group)
        return parts
    return gather


def view_assemble(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, geom: ViewGeom, gather) -> tuple:
    """-> (qp, k_full, v_full): this rank's q-block queries (patch tokens
    [b0*128, min(b1*128, Tp)) of the global patch order, (B, H, n, 64)) and
    every key and value in the full token layout.  ``gather(name, t)``
    returns the list of every rank's ``t`` in rank order (an all-gather)."""
    mine = view_exchange_parts(q, k, v, geom)
    k_full = torch.cat(gather("k", mine["k"]), dim=2)
    v_full = torch.cat(gather("v", mine["v"]), dim=2)
    heads = gather("qhead", mine["qhead"])
    tails = gather("qtail", mine["qtail"])
    pieces = []
    if geom.lo:
        pieces.append(tails[geom.rank - 1][:, :, KS_Q - geom.lo:])
    pieces.append(patch_tokens(q, geom.special, geom.hw))
    if geom.hi:
        pieces.append(heads[geom.rank + 1][:, :, : geom.hi])
    return torch.cat(pieces, dim=2), k_full, v_full


@dataclass
class ViewLayerResult:
    out: torch.Tensor      # (B, H, F_local*(special+hw), 64) fp32, this rank's tokens
    lists: torch.Tensor    # (B*H*(b1-b0), width) int32 keep lists of q-blocks b0..b1-1
    counts: torch.Tensor
    nts: torch.Tensor      # (B, H, b1-b0) int32 budgets
    geom: ViewGeom


def view_sharded_layer(q, k, v, geom: ViewGeom, budget, order, gather, *, lead_blocks: int = 0) -> ViewLayerResult:
    """One sparse global-attention layer on this rank's frames.  q, k, v:
    (B, H, F_local*(special+hw), 64) CUDA, this rank's tokens in the full
    layout.  Same stages as ``layer.global_layer``; the pooled keys, the
    int8 keys, their mean and the fp16 values are formed from the gathered
    full K and V (identically on every rank)."""
    from . import kernels as K
    from . import layer as LY

    B, H = q.shape[0], q.shape[1]
    dev = q.device
    qp, k_full, v_full = view_assemble(q, k, v, geom, gather)
    Lk = K.Layout(B, H, geom.frames, geom.special, geom.hw)
    Lq = K.Layout(B, H, 1, 0, qp.shape[2])
    Ll = K.Layout(B, H, geom.frames_local, geom.special, geom.hw)
    ws = K.workspace(dev, B * H, Lk.Tp, Lk.Tk, Lk.n_cand)
    F_, S_, HW = geom.frames_local, geom.special, geom.hw
    out = torch.empty(B, H, F_ * (S_ + HW), 64, dtype=torch.float32, device=dev)
    main = torch.cuda.current_stream(dev)
    side = LY._side_stream(dev)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        # this rank's special rows of `out` (bf16 layers: written in place)
        x_special = LY.special_attention(q, k_full, v_full, Ll, out)
    for t in (q, k_full, v_full, out):
        t.record_stream(side)
    qbar, q8, qs = K.pool_quant_q(qp, Lq)
    kbar, vbar, k8, ks, v16, _ = K.pool_quant_kv(k_full, v_full, Lk, ws=ws)
    attn_full, attn_cond = K.predict(qbar, kbar, Lk.n_cand, full=order.kind == "restore_swap", cond=True)
    nts, r = LY.select_blocks(attn_full, attn_cond, vbar, B, H, Lq.nq, Lk.n_cand, Lk.sink_blocks, budget, order,
                              lead_blocks=lead_blocks, ws=ws)
    o = K.sparse_attn(q8, qs, k8, ks, v16, r["lists"], r["counts"]).view(B, H, qp.shape[2], 64)
    view = out.view(B, H, F_, S_ + HW, 64)
    view[:, :, :, S_:] = o[:, :, geom.lo: geom.lo + F_ * HW].view(B, H, F_, HW, 64)
    main.wait_stream(side)
    if x_special is not None:
        x_special.record_stream(main)
        view[:, :, :, :S_] = x_special.view(B, H, F_, S_, 64).float()
    return ViewLayerResult(out=out, lists=r["lists"], counts=r["counts"], nts=nts, geom=geom)
