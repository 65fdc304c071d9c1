"""ReSS block-sparse global attention: the replacement attention forward.

Mirror of the reference's ``models/attention.py`` interface: the constants,
``predict_attention`` :82-100, ``block_mean_value`` :103-109,
``same_frame_block_mask`` :112-144, ``build_block_mask`` :147-174,
``run_block_sparse_kernel`` :217-243, ``AttentionAux`` :246-265,
``compute_baseline_num_to_select`` :268-293 and ``ress_attention_forward``
:296-659, with the same arguments and results.  Everything between the Q/K/V
projection and the output projection runs on the sm_100a library through
``ress_b200.layer.global_layer``; there is no CPU or Triton path.

Only the defaults of the reference's import-time switches are supported
(RESS_SINK_MASS=0, RESS_SINK_PROTECT=1); other values raise at import.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import criterion as _criterion
from . import kernels as K
from .budget import compute_baseline_num_to_select  # noqa: F401  (re-exported, reference location)
from .layer import OrderSpec, global_layer
from .qkv import compute_qkv, compute_qkv_scored, get_patch_tokens, project_out

KS_Q = 128
KS_K = 64
KBLK = 64
MIN_NUM_TO_SELECT = 2
# True: bf16 layers whose q/k norms and rotary embedding the kernels reproduce
# take the fused prologue (kernels.qkv_prologue_scored: the patch queries pooled
# and quantised straight from the qkv Linear's output, never written).  Off by
# default: both routes give the same bits, and on a B200 the prologue and the
# Q pass are bound by instruction issue, not HBM, so the fused route, which
# saves 90 MB of traffic at 32 views but issues more instructions, measured
# slower (0.222 against 0.192 ms per layer)
FUSED_PROLOGUE = False

if os.environ.get("RESS_SINK_MASS", "0") != "0" or os.environ.get("RESS_SINK_PROTECT", "1") == "0":
    raise RuntimeError("ress_b200 implements the reference defaults RESS_SINK_MASS=0, RESS_SINK_PROTECT=1 only")


def _pool(x, blk):
    L = K.Layout.plain(x)
    xc = x if x.stride(-1) == 1 else x.contiguous()
    if blk == KS_Q:
        bar, _, _ = K.pool_quant_q(xc, L, quant=False)
    else:
        bar, _, _, _, _, _ = K.pool_quant_kv(xc, xc, L, quant=False)
    return bar.view(x.shape[0], x.shape[1], -1, x.shape[-1])


def predict_attention(query, key, ks_q=KS_Q, ks_k=KS_K, pool_mode="avg"):
    """softmax(avgpool128(Q) avgpool64(K)^T / sqrt(64)): (B, nh, q_blk, k_blk)."""
    if pool_mode != "avg" or ks_q != KS_Q or ks_k != KS_K or query.shape[-1] != 64:
        raise NotImplementedError("avg pooling with 128/64 blocks and head_dim 64 only")
    qbar, kbar = _pool(query, KS_Q), _pool(key, KS_K)
    B, nh = query.shape[:2]
    af, _ = K.predict(qbar.reshape(B * nh, -1, 64), kbar.reshape(B * nh, -1, 64), kbar.shape[2], cond=False)
    return af.view(B, nh, qbar.shape[2], kbar.shape[2])


def block_mean_value(value, ks_k=KS_K):
    if ks_k != KS_K or value.shape[-1] != 64:
        raise NotImplementedError("64-key blocks and head_dim 64 only")
    return _pool(value, KS_K)


def same_frame_block_mask(q_blk, k_blk, N, H, W, device):
    """(q_blk, k_blk) bool: query block and key block touch a common frame."""
    HW, T = H * W, N * H * W
    qs = torch.arange(q_blk, device=device) * KS_Q
    qe = (qs + KS_Q - 1).clamp(max=T - 1)
    ks = torch.arange(k_blk, device=device) * KS_K
    ke = (ks + KS_K - 1).clamp(max=T - 1)
    q0, q1, k0, k1 = qs // HW, qe // HW, ks // HW, ke // HW
    return ~((q1.unsqueeze(1) < k0.unsqueeze(0)) | (k1.unsqueeze(0) < q0.unsqueeze(1)))


def build_block_mask(pooled_score, num_to_select, sink_blocks, rank_by=None):
    """Keep the top num_to_select of each row (ties to the lowest index), then
    append sink_blocks always-kept columns: (B, nh, q_blk, k_blk + sink) bool."""
    key = pooled_score if rank_by is None else rank_by
    keep = K.top_m_mask(key if key.dtype in (torch.float32, torch.bfloat16) else key.float(),
                        num_to_select.reshape(-1)).view(key.shape)
    if sink_blocks > 0:
        ones = torch.ones(*keep.shape[:-1], sink_blocks, dtype=torch.bool, device=keep.device)
        keep = torch.cat([keep, ones], dim=-1)
    return keep


def run_block_sparse_kernel(query, key, value, final_map, dtype=torch.float16, out_dtype=torch.float32):
    """int8 per-block quantisation (Q 128-token, K - mean(K) 64-token blocks),
    block-sparse attention over final_map, (o, sparsity)."""
    if dtype != torch.float16:
        raise NotImplementedError("the kernel computes P.V in fp16 like the reference's dtype default")
    q = query.contiguous()
    k = key.contiguous()
    v = value.contiguous()
    _, q8, qs = K.pool_quant_q(q, K.Layout.plain(q), pool=False)
    _, _, k8, ks, v16, _ = K.pool_quant_kv(k, v, K.Layout.plain(k), pool=False)
    lists, counts = K.map_to_lists(final_map.reshape(-1, final_map.shape[-1]))
    o = K.sparse_attn(q8, qs, k8, ks, v16, lists, counts).view(q.shape)
    sparsity = 1 - final_map.float().mean().item()
    return o.to(out_dtype), sparsity


@dataclass
class AttentionAux:
    attn_pooled: torch.Tensor = None
    v_bar: torch.Tensor = None
    attn_full: torch.Tensor = None
    v_bar_full: torch.Tensor = None
    n_cand: int = None
    q_patch: torch.Tensor = None
    shape: dict = None
    sparsity: float = None
    output: torch.Tensor = None


def _order_for(self, block_criterion, hd, nh, device):
    if block_criterion == "probability":
        return OrderSpec("probability")
    if block_criterion == "random":
        return OrderSpec("random")
    if _criterion.is_restore_swap(block_criterion):
        spec = _criterion.parse_restore_swap(block_criterion)
        if spec.big_dtype != torch.bfloat16:
            raise NotImplementedError(f"{block_criterion!r}: only the bf16 restore-swap recipe (_bf16) is implemented")
        if spec.maximize or spec.invert_cut:
            raise NotImplementedError(f"{block_criterion!r}: drift-maximisation controls are not ported")
        if spec.use_wo:
            if getattr(self, "M", None) is None:
                raise AssertionError(f"{block_criterion!r} weighs drift by the output projection: attach the "
                                     "per-head metrics with bake_and_attach_M(model) before the forward")
            M = self.M.float().to(device)
        else:
            M = torch.eye(hd, device=device, dtype=torch.float32).expand(nh, hd, hd).contiguous()
        return OrderSpec("restore_swap", M=M, n_iters=spec.n_iters, track_best=spec.track_best,
                         restore_frac=spec.restore_frac, decay=spec.decay)
    if block_criterion in ("projected", "damage", "norm"):
        raise NotImplementedError(f"block_criterion={block_criterion!r} is not one of the four modes' orders")
    raise ValueError(block_criterion)


def _protect_own_frame_hook(shp, n_cand):
    """Budget-neutral own-frame protection (attention.py:583-618), torch glue."""
    def hook(final_map, attn_pooled):
        q_blk = final_map.shape[-2]
        same = same_frame_block_mask(q_blk, n_cand, shp["N"], shp["H"], shp["W"], final_map.device)
        same = same.expand_as(final_map[..., :n_cand])
        kept = final_map[..., :n_cand]
        missing = same & ~kept
        swappable = kept & ~same
        n_swap = torch.minimum(missing.sum(-1), swappable.sum(-1))
        out_pri = attn_pooled.float().masked_fill(~swappable, float("inf"))
        rank_out = torch.argsort(torch.argsort(out_pri, dim=-1, stable=True), dim=-1)
        in_pri = attn_pooled.float().masked_fill(~missing, float("-inf"))
        rank_in = torch.argsort(torch.argsort(in_pri, dim=-1, descending=True, stable=True), dim=-1)
        new_kept = (kept & ~(rank_out < n_swap.unsqueeze(-1))) | (rank_in < n_swap.unsqueeze(-1))
        return torch.cat([new_kept, final_map[..., n_cand:]], dim=-1)
    return hook


def ress_attention_forward(self, x, pos, num_to_select=None, budget_fn=None, perhead_budget_fn=None,
                           joint_select_fn=None, block_criterion="probability", pool_mode="avg",
                           num_special_tokens=5, num_heads=16, shape=None, aux_store=None, aux_full=True,
                           dense=False, retain_output_grad=False, pooled_fallback=False, protect_own_frame=False):
    """Replacement forward for a VGGT-family global-attention block
    (attention.py:296-659).  Same arguments and return value."""
    if pool_mode != "avg":
        raise NotImplementedError("pool_mode='avg' only")
    scored = None
    if (FUSED_PROLOGUE and not dense and aux_store is None and not retain_output_grad
            and getattr(self, "ress_view", None) is None):
        # bf16 layers whose prologue the kernels reproduce: the patch queries are
        # pooled and quantised straight from the qkv Linear's output (q is never formed)
        r = compute_qkv_scored(self, x, pos, num_special_tokens=num_special_tokens, num_heads=num_heads,
                               shape=shape)
        if r is not None:
            k, v, scored, shp = r
            q = None
    if scored is None:
        q, k, v, shp = compute_qkv(self, x, pos, num_special_tokens=num_special_tokens, num_heads=num_heads,
                                   shape=shape)
    B, N, P, hd, nh, S = shp["B"], shp["N"], shp["P"], shp["head_dim"], shp["num_heads"], shp["S"]
    L = K.Layout(B, nh, N, S, P - S)
    res = None
    if dense:
        x_out = F.scaled_dot_product_attention(q, k, v)
        sparsity = 0.0
    else:
        if hd != 64:
            raise NotImplementedError("the sm_100a kernels take head_dim 64")
        if q is not None:
            if q.dtype not in (torch.float32, torch.bfloat16):
                q, k, v = q.float(), k.float(), v.float()
            k = k if k.dtype == q.dtype else k.to(q.dtype)
            v = v if v.dtype == q.dtype else v.to(q.dtype)
        budget = None
        if joint_select_fn is None and perhead_budget_fn is None and budget_fn is not None:
            tag = getattr(budget_fn, "ress_budget", None)
            if tag is not None and hasattr(tag[0], "spec"):
                b, layer, sr, cdf, beta = tag
                budget = b.spec(layer, sr, cdf, beta, device=k.device)
                budget_fn = None
        order = _order_for(self, block_criterion, hd, nh, k.device)
        hook = _protect_own_frame_hook(shp, L.n_cand) if protect_own_frame else None
        pbf = None
        if perhead_budget_fn is not None:
            def pbf(attn_cond, _f=perhead_budget_fn):
                vb = block_mean_value(get_patch_tokens(v, N, P, S))[..., : L.n_cand, :]
                return _f(attn_cond, vb)
        view = getattr(self, "ress_view", None)
        if view is not None:
            # frames of this rank only; K/V are all-gathered inside (whole-model view sharding)
            if budget is None or joint_select_fn is not None or hook is not None or pbf is not None:
                raise NotImplementedError("view sharding runs the package's own budgets and orders")
            from .shard import view_sharded_layer

            geom, gather = view
            res = view_sharded_layer(q, k, v, geom, budget, order, gather)
            x_out = res.out
            sparsity = 0.0 if aux_store is None else None
            if aux_store is not None:
                raise NotImplementedError("aux outputs are not collected under view sharding")
        else:
            res = global_layer(q, k, v, L, budget, order, num_to_select=num_to_select,
                               budget_fn=pbf or budget_fn, keep_pooled=aux_store is not None,
                               joint_select_fn=joint_select_fn, map_hook=hook, q_scored=scored)
            x_out = res.out
        sparsity = None
    if aux_store is not None:
        if sparsity is None:
            sparsity = res.sparsity()
        if aux_full and res is not None:
            n_cand = L.n_cand
            attn_full = res.attn_full.view(B, nh, L.nq, L.nkp)
            v_bar_full = res.vbar.view(B, nh, L.nkp, hd)
            aux_store["value"] = AttentionAux(attn_pooled=attn_full[..., :n_cand], v_bar=v_bar_full[..., :n_cand, :],
                                              attn_full=attn_full, v_bar_full=v_bar_full, n_cand=n_cand,
                                              q_patch=get_patch_tokens(q, N, P, S), shape=shp, sparsity=sparsity)
        else:
            aux_store["value"] = AttentionAux(shape=shp, sparsity=sparsity)
    if retain_output_grad:
        x_out.retain_grad()
    if aux_store is not None and aux_full:
        aux_store["value"].output = x_out
    return project_out(self, x_out, B, N, P, nh, hd)
