"""The oracle (CPU restatement) against the reference's own outputs.

The fixtures under tests/golden were produced by running the reference's
torch code (tests/golden/make_golden.py).  What must match exactly:
pooled means, budgets, and every block map whenever the oracle is handed the
reference's own pooled softmax map.  End to end, the oracle computes that map
itself with its own exp, which differs from torch's in the last bits; the
agreement is then measured and bounded (it is exact on the fp32 config)."""

import os

import numpy as np
import pytest
import torch

import oracle
from ress_b200 import synth

GOLD = os.path.join(os.path.dirname(__file__), "golden")
CASES = ["cfg1_ress", "cfg1_ress_sr50", "cfg1_hess_cdf", "bf16_6f_ress", "bf16_6f_hess_cdf", "cfg2_ress",
         "cfg2_hess_cdf"]
# minimum fraction of (head, q-block) rows identical end to end
E2E_FLOOR = {"cfg1_ress": 1.0, "cfg1_ress_sr50": 1.0, "cfg1_hess_cdf": 0.995,
             "bf16_6f_ress": 0.995, "bf16_6f_hess_cdf": 0.995, "cfg2_ress": 0.99, "cfg2_hess_cdf": 0.99}

_inputs = {}


def _load(name):
    case = dict(np.load(os.path.join(GOLD, f"{name}.npz")))
    pooled = dict(np.load(os.path.join(GOLD, f"{case['pooled']}_pooled.npz")))
    return case, pooled


def _shape_dtype(case):
    shape = synth.LayerShape(n_frames=int(case["n_frames"]), n_heads=int(case["n_heads"]))
    dtype = torch.bfloat16 if "bfloat16" in str(case["dtype"]) else torch.float32
    return shape, dtype


def _layer(case):
    shape, dtype = _shape_dtype(case)
    key = (shape, dtype)
    if key not in _inputs:
        q, k, v = synth.layer_qkv(shape, seed=0, dtype=dtype)
        _inputs[key] = (q, k, v)
    return shape, dtype, _inputs[key]


def _pooled_map(pooled, key, dtype):
    """A stored pooled map: fp32 values, or raw bf16 bit patterns (large layers)."""
    a = pooled[key]
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(a).to(dtype)


def _final_map(case):
    bits = np.unpackbits(case["final_map"], axis=-1)[..., : int(case["final_map_width"])]
    return torch.from_numpy(bits.astype(bool))


@pytest.mark.parametrize("name", CASES)
def test_generator_is_reproducible(name):
    case, pooled = _load(name)
    shape, dtype, (q, k, v) = _layer(case)
    assert synth.checksum(q) == str(pooled["cs_q"]), "synthetic generator drifted on this host"
    assert synth.checksum(k) == str(pooled["cs_k"])
    assert synth.checksum(v) == str(pooled["cs_v"])
    M = synth.metric_from_weight(synth.out_proj_weight(), shape.n_heads)
    assert synth.checksum(M) == str(pooled["cs_M"])


@pytest.mark.parametrize("name", CASES)
def test_pooled_means_bit_exact(name):
    case, pooled = _load(name)
    shape, dtype, (q, k, v) = _layer(case)
    qp, _ = synth.split_tokens(q, shape)
    kp, _ = synth.split_tokens(k, shape)
    vp, _ = synth.split_tokens(v, shape)
    rows = shape.n_heads
    assert synth.checksum(oracle.pool_mean(qp.reshape(rows, -1, 64), 128).unsqueeze(0).reshape(rows, -1, 64)) == str(pooled["cs_qbar"])
    assert synth.checksum(oracle.pool_mean(kp.reshape(rows, -1, 64), 64)) == str(pooled["cs_kbar"])
    assert synth.checksum(oracle.pool_mean(vp.reshape(rows, -1, 64), 64).unsqueeze(0)) == str(pooled["cs_vbar"])


@pytest.mark.parametrize("name", CASES)
def test_selection_bit_exact_given_reference_map(name):
    """Budgets + ordering + lists from the reference's own pooled map."""
    case, pooled = _load(name)
    shape, dtype, (q, k, v) = _layer(case)
    n_cand = int(case["n_cand"])
    heads = torch.from_numpy(pooled["heads"]).long()  # heads whose pooled maps the fixture holds
    attn_full = _pooled_map(pooled, "attn_full", dtype)
    cond = _pooled_map(pooled, "attn_cond", dtype)
    fm_ref = _final_map(case)[0]
    nts_ref = torch.from_numpy(case["nts"])
    nh, nq = nts_ref.shape[1], nts_ref.shape[2]
    sub = len(heads)
    # the budget: the baseline from the reference's attn_cond, then HeSS on the
    # reference's baselines of every head (it couples the heads of a q-block)
    sr = float(case["sparse_ratio"])
    cdf = float(case["cdf"])
    base = oracle.baseline(cond, sr, None if cdf < 0 else cdf)
    base_ref = torch.from_numpy(case["baseline"])
    assert torch.equal(base.view(1, sub, nq), base_ref[:, heads])
    nts = oracle.hess_adjust(base_ref.view(1, nh, nq), oracle.scores_norm(torch.from_numpy(pooled["head_scores"])),
                             n_cand, min_clamp=min(2, n_cand))
    assert torch.equal(nts, nts_ref)
    nts_sub = nts_ref[:, heads].reshape(-1)
    if str(case["mode"]) == "ress":
        vp = synth.split_tokens(v, shape)[0][:, heads]
        vbar = oracle.pool_mean(vp.reshape(sub, -1, 64), 64).to(torch.bfloat16)
        M = synth.metric_from_weight(synth.out_proj_weight(), nh)[heads]
        drop, _ = oracle.restore_swap(attn_full, vbar, M, nts_sub, n_cand)
        keep = ~drop
    else:
        keep = oracle.top_m_mask(cond.reshape(-1, n_cand), nts_sub)
    lists, counts = oracle.keep_lists(keep, int(case["sink_blocks"]))
    got = torch.zeros(sub * nq, fm_ref.shape[-1], dtype=torch.bool)
    for r in range(sub * nq):
        got[r, lists[r, : counts[r]].long()] = True
    assert torch.equal(got.view(sub, nq, -1), fm_ref[heads])


@pytest.mark.parametrize("name", CASES)
def test_end_to_end_agreement(name):
    case, pooled = _load(name)
    shape, dtype, (q, k, v) = _layer(case)
    qp, _ = synth.split_tokens(q, shape)
    kp, ks = synth.split_tokens(k, shape)
    vp, _ = synth.split_tokens(v, shape)
    M = synth.metric_from_weight(synth.out_proj_weight(), shape.n_heads)
    cdf = float(case["cdf"])
    o = oracle.layer_select(qp, kp, vp, ks.shape[-2], M, head_scores=torch.from_numpy(pooled["head_scores"]),
                            mode="ress" if str(case["mode"]) == "ress" else "prob",
                            sparse_ratio=float(case["sparse_ratio"]), cdf_threshold=None if cdf < 0 else cdf)
    heads = torch.from_numpy(pooled["heads"]).long()
    af_ref = _pooled_map(pooled, "attn_full", dtype).float()
    af = o["attn_full"].float().view(1, shape.n_heads, *af_ref.shape[-2:])[:, heads]
    rel = ((af - af_ref).abs() / af_ref.abs().clamp(min=1e-30)).max().item()
    assert rel < (1e-5 if dtype == torch.float32 else 1e-2)
    fm_ref = _final_map(case)[0, :, :, : o["n_cand"]]
    same = (o["keep"][0] == fm_ref).all(-1).float().mean().item()
    print(f"{name}: {same:.5f} of (head, q-block) rows identical end to end")
    assert same >= E2E_FLOOR[name], f"{name}: {same:.4f} of rows identical"


def test_budget_kats():
    g = dict(np.load(os.path.join(GOLD, "budget_kats.npz")))
    for tag in ("plain", "capped", "beta", "zero"):
        base = torch.from_numpy(g[f"adj_{tag}_in"])
        snorm = oracle.scores_norm(torch.from_numpy(g[f"adj_{tag}_scores"]))
        out = oracle.hess_adjust(base, snorm, int(g[f"adj_{tag}_max"]), beta=float(g[f"adj_{tag}_beta"]))
        assert torch.equal(out, torch.from_numpy(g[f"adj_{tag}_out"])), tag
    cond = torch.from_numpy(g["cdf_cond"])
    for tag, sr, cdf in (("cdf", None, 0.9), ("both", 0.5, 0.97), ("ratio", 0.3, None)):
        got = oracle.baseline(cond, sr, cdf)
        assert torch.equal(got, torch.from_numpy(g[f"cdf_{tag}_out"])), tag
    got = oracle.baseline(torch.from_numpy(g["cdfb_cond"]).bfloat16(), None, 0.9)
    assert torch.equal(got, torch.from_numpy(g["cdfb_cdf_out"]))
    q = torch.from_numpy(g["topm_q"])
    assert torch.equal(oracle.top_m_mask(q, torch.tensor([3, 5])), torch.from_numpy(g["topm_out"]))
    assert torch.equal(oracle.top_m_mask(q, torch.tensor([2, 6]), largest=False),
                       torch.from_numpy(g["topm_small_out"]))
