"""Generate the golden fixtures by running the REFERENCE's own torch code.

Run only where the reference tree is available (it is not on the GPU box):

    python tests/golden/make_golden.py /path/to/libary753-ReSS [case ...]

(naming cases regenerates only those).

The reference's GPU-only dependency SpargeAttn (``spas_sage_attn``) is absent,
so its four imported symbols are stubbed; none of them is on the part of the
path this script runs (``fill_block_map_triton`` is restated below as the
scatter it performs).  The CPU eager path of the reference breaks top-m ties
with ``torch.topk``'s unspecified order; the reference's CUDA path
(``scoring/fused_topm.py:15-16``, ``scoring/fused_round.py:100-112``) breaks
them to the lowest index, and that is the rule this build pins, so
``projected._top_m_mask`` and ``build_block_mask``'s sort are swapped for
stable lowest-index versions here.  Nothing else in the reference is touched.

Each fixture stores: the generator's input checksums (to detect drift of the
synthetic generator between machines), the reference's pooled means as
checksums, the reference's pooled softmax map (the input of the
selection-only checks), the budgets, and the final block maps.
"""

from __future__ import annotations

import math
import os
import sys
import tempfile
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from ress_b200 import synth  # noqa: E402


def _install_reference(ref_root: str):
    for name in ["spas_sage_attn", "spas_sage_attn._qattn", "spas_sage_attn.quant_per_block",
                 "spas_sage_attn.utils"]:
        sys.modules[name] = types.ModuleType(name)

    def _absent(*a, **k):
        raise RuntimeError("SpargeAttn is not available here")

    sys.modules["spas_sage_attn._qattn"].qk_int8_sv_f16_accum_f16_block_sparse_attn_inst_buf_with_pv_threshold = _absent
    sys.modules["spas_sage_attn.quant_per_block"].per_block_int8 = _absent

    def fill_block_map(final_map, num_to_select, sorted_idx):
        ar = torch.arange(final_map.shape[-1])
        return final_map.scatter(-1, sorted_idx, (ar < num_to_select.unsqueeze(-1)).expand_as(sorted_idx))

    u = sys.modules["spas_sage_attn.utils"]
    u.fill_block_map_triton = fill_block_map
    u.block_map_lut_triton = _absent
    u.hyperparameter_check = _absent
    sys.path.insert(0, os.path.join(ref_root, "src"))

    from ress.models import attention as A
    from ress.scoring import projected as PJ

    def order_key(x, largest=True):
        b = x.float().contiguous().view(torch.int32).long()
        key = torch.where(b >= 0, b + (1 << 31), -1 - b)
        return key if largest else (1 << 32) - 1 - key

    def top_m_lowest(quality, counts, largest=True, k_max=None):
        key = order_key(quality, largest)
        n = quality.shape[-1]
        counts = counts.clamp(min=0, max=n)
        idx = torch.sort(key, dim=-1, descending=True, stable=True).indices
        pos = torch.arange(n).expand(idx.shape)
        return torch.zeros_like(quality, dtype=torch.bool).scatter(-1, idx, pos < counts.unsqueeze(-1))

    PJ._top_m_mask = top_m_lowest
    return A, PJ, fill_block_map


def build_block_mask_stable(fill, pooled_score, num_to_select, sink_blocks, rank_by=None):
    """attention.py:147-174 with a stable sort (ties to the lowest index)."""
    key = pooled_score if rank_by is None else rank_by
    idx = torch.sort(key, dim=-1, descending=True, stable=True).indices
    fm = fill(torch.zeros_like(pooled_score, dtype=torch.bool), num_to_select, idx)
    if sink_blocks > 0:
        shape = list(fm.shape)
        shape[-1] = sink_blocks
        fm = torch.cat([fm, torch.ones(shape, dtype=torch.bool)], dim=-1)
    return fm


def _store_map(x, as_bits):
    """A pooled map for the fixture: fp32 values, or -- for the large layers --
    the raw 16-bit patterns of a bf16 map (half the bytes)."""
    if as_bits and x.dtype == torch.bfloat16:
        return x.contiguous().view(torch.int16).numpy().view(np.uint16)
    return x.float().numpy()


def reference_layer(A, PJ, fill, shape, dtype, mode, sparse_ratio, cdf, lam=0.5, layer=0,
                    n_iters=5, heads=None):
    """One layer through the reference.  heads: store the pooled maps of
    these heads only (large layers); budgets and block maps cover all heads."""
    from ress.budget.hess import HessBudget

    q, k, v = synth.layer_qkv(shape, seed=0, dtype=dtype)
    qp, _ = synth.split_tokens(q, shape)
    kp, ks = synth.split_tokens(k, shape)
    vp, _ = synth.split_tokens(v, shape)
    M = synth.metric_from_weight(synth.out_proj_weight(), shape.n_heads)
    tmp = tempfile.mkdtemp()
    torch.save(synth.fisher_table(seed=1), os.path.join(tmp, "cam.pt"))
    torch.save(synth.fisher_table(seed=3), os.path.join(tmp, "pcd.pt"))
    hess = HessBudget(os.path.join(tmp, "cam.pt"), os.path.join(tmp, "pcd.pt"), lam=lam)

    # attention.py:446-581, _SINK_MASS=0 / _SINK_PROTECT=1 defaults
    attn_full = A.predict_attention(query=qp, key=kp)
    n_cand = kp.shape[-2] // A.KS_K
    attn_pooled = attn_full[..., :n_cand]
    attn_cond = attn_pooled / attn_pooled.sum(dim=-1, keepdim=True).clamp(min=1e-6)
    vbar_full = A.block_mean_value(vp)
    Tk = kp.shape[-2] + ks.shape[-2]
    sink_blocks = math.ceil(Tk / A.KBLK) - n_cand
    base = A.compute_baseline_num_to_select(attn_cond, sparse_ratio, cdf)
    nts = hess.num_to_select(layer, attn_cond, sparse_ratio, cdf, 1.0)
    nts = nts.clamp(min=min(A.MIN_NUM_TO_SELECT, n_cand))
    rank_by = None
    if mode == "ress":
        rank_by = PJ.restore_swap_rank_by(attn_full, vbar_full, M, nts, n_cand=n_cand,
                                          n_iters=n_iters, track_best=True,
                                          big_dtype=torch.bfloat16)
    final_map = build_block_mask_stable(fill, attn_cond, nts, sink_blocks, rank_by=rank_by)

    pooled_q = torch.nn.functional.avg_pool1d(qp.reshape(-1, qp.shape[-2], 64).transpose(1, 2),
                                              128, ceil_mode=True).transpose(1, 2)
    pooled_k = torch.nn.functional.avg_pool1d(kp.reshape(-1, kp.shape[-2], 64).transpose(1, 2),
                                              64, ceil_mode=True).transpose(1, 2)
    return dict(
        n_frames=shape.n_frames, n_heads=shape.n_heads, dtype=str(dtype), mode=mode,
        sparse_ratio=sparse_ratio, cdf=-1.0 if cdf is None else cdf, n_iters=n_iters,
        cs_q=synth.checksum(q), cs_k=synth.checksum(k), cs_v=synth.checksum(v),
        cs_M=synth.checksum(M),
        cs_qbar=synth.checksum(pooled_q.to(dtype)), cs_kbar=synth.checksum(pooled_k.to(dtype)),
        cs_vbar=synth.checksum(vbar_full),
        attn_full=_store_map(attn_full if heads is None else attn_full[:, heads], heads is not None),
        attn_cond=_store_map(attn_cond if heads is None else attn_cond[:, heads], heads is not None),
        heads=np.arange(shape.n_heads) if heads is None else np.asarray(heads),
        cs_attn_full=synth.checksum(attn_full), cs_attn_cond=synth.checksum(attn_cond),
        head_scores=hess.head_scores[layer].numpy(),
        baseline=base.int().numpy(),
        nts=nts.int().numpy(),
        final_map=np.packbits(final_map.numpy(), axis=-1),
        final_map_width=final_map.shape[-1],
        n_cand=n_cand, sink_blocks=sink_blocks,
    )


def budget_kats(PJ):
    """Known answers for adjust_attention_selection / compute_baseline_num_to_select
    on small hand-made inputs, including the degenerate-score and beta < 1
    branches (_proportional.py:184-215, attention.py:268-293)."""
    from ress.budget._proportional import adjust_attention_selection
    from ress.models.attention import compute_baseline_num_to_select

    rng = np.random.Generator(np.random.PCG64(7))
    out = {}
    base = torch.from_numpy(rng.integers(2, 40, size=(1, 8, 12))).long()
    scores = torch.from_numpy(np.exp(rng.standard_normal(8)).astype(np.float32))
    for tag, sc, beta, mx in (("plain", scores, 1.0, 40), ("capped", scores * torch.arange(1, 9).float() ** 2, 1.0, 30),
                              ("beta", scores, 0.25, 40), ("zero", torch.zeros(8), 1.0, 40)):
        out[f"adj_{tag}_in"] = base.int().numpy()
        out[f"adj_{tag}_scores"] = sc.float().numpy()
        out[f"adj_{tag}_beta"] = np.float64(beta)
        out[f"adj_{tag}_max"] = np.int64(mx)
        out[f"adj_{tag}_out"] = adjust_attention_selection(base, sc, beta, mx).int().numpy()
    # CDF budgets over rows with exact ties and a row whose mass never reaches tau
    cond = torch.from_numpy(rng.random((3, 5, 40)).astype(np.float32))
    cond[0, 0, :] = 1.0 / 40
    cond[1, 1, :10] = 0.0
    cond = cond / cond.sum(-1, keepdim=True)
    cond[2, 2, :] = 0.0
    out["cdf_cond"] = cond.numpy()
    for tag, sr, cdf in (("cdf", None, 0.9), ("both", 0.5, 0.97), ("ratio", 0.3, None)):
        out[f"cdf_{tag}_out"] = compute_baseline_num_to_select(cond.unsqueeze(0), sr, cdf)[0].int().numpy()
    cb = cond.bfloat16()
    out["cdfb_cond"] = cb.float().numpy()
    out["cdfb_cdf_out"] = compute_baseline_num_to_select(cb.unsqueeze(0), None, 0.9)[0].int().numpy()
    # top-m with ties (lowest index) and -0/+0
    q = torch.tensor([[0.5, 1.0, 1.0, -0.0, 0.0, 1.0, 0.25, 1.0],
                      [3.0, 3.0, 3.0, 3.0, 2.0, 2.0, 1.0, 0.0]])
    out["topm_q"] = q.numpy()
    out["topm_counts"] = np.array([3, 5], np.int32)
    out["topm_out"] = PJ._top_m_mask(q, torch.tensor([3, 5])).numpy()
    out["topm_small_out"] = PJ._top_m_mask(q, torch.tensor([2, 6]), largest=False).numpy()
    return out


def main(ref_root: str):
    torch.set_num_threads(os.cpu_count() or 1)
    A, PJ, fill = _install_reference(ref_root)
    # The cfg2 layer (32 frames, bf16, apply_hess sr .5 /
    # cdf .97 and apply_ress sr .5, HeSS lambda .5) stores the pooled maps of
    # two heads only -- the one with the largest HeSS score (capped at every
    # candidate) and the one with the smallest -- to keep the fixture small;
    # its budgets and block maps cover all 16 heads.
    cfg2_heads = [9, 3]
    cases = {
        "cfg1_ress": (synth.CONFIG1, torch.float32, "ress", 0.1, None, None),
        "cfg1_ress_sr50": (synth.CONFIG1, torch.float32, "ress", 0.5, None, None),
        "cfg1_hess_cdf": (synth.CONFIG1, torch.float32, "prob", 0.5, 0.97, None),
        "bf16_6f_ress": (synth.LayerShape(n_frames=6), torch.bfloat16, "ress", 0.5, None, None),
        "bf16_6f_hess_cdf": (synth.LayerShape(n_frames=6), torch.bfloat16, "prob", 0.5, 0.97, None),
        "cfg2_ress": (synth.LayerShape(n_frames=32), torch.bfloat16, "ress", 0.5, None, cfg2_heads),
        "cfg2_hess_cdf": (synth.LayerShape(n_frames=32), torch.bfloat16, "prob", 0.5, 0.97, cfg2_heads),
    }
    only = set(sys.argv[2:])
    pooled_keys = ("attn_full", "attn_cond", "head_scores", "heads", "cs_attn_full", "cs_attn_cond", "cs_q",
                   "cs_k", "cs_v", "cs_M", "cs_qbar", "cs_kbar", "cs_vbar")
    written = set()
    for name, (shape, dtype, mode, sr, cdf, heads) in cases.items():
        if only and name not in only:
            continue
        d = reference_layer(A, PJ, fill, shape, dtype, mode, sr, cdf, heads=heads)
        stem = name.split("_")[0] + "_" + name.split("_")[1] if name.startswith("bf16") else name.split("_")[0]
        if stem not in written:
            np.savez_compressed(os.path.join(HERE, f"{stem}_pooled.npz"),
                                **{k: d[k] for k in pooled_keys})
            written.add(stem)
        case = {k: v for k, v in d.items() if k not in pooled_keys}
        case["pooled"] = stem
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **case)
        print("wrote", name, d["final_map"].shape)
    if not only or "budget_kats" in only:
        np.savez_compressed(os.path.join(HERE, "budget_kats.npz"), **budget_kats(PJ))
        print("wrote budget_kats")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference tree> [case ...]")
    main(sys.argv[1])
