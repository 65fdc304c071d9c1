"""Host-side behaviour of the drop-in API (no GPU): mode installation and
reset, the criterion grammar, the HeSS table preparation against the
reference's own numbers, and the identities the reference's docstrings
state for its objective."""

import os

import numpy as np
import pytest
import torch

import ress_b200 as ress
from ress_b200 import budget as B
from ress_b200 import criterion, projected, static, wiring
from ress_b200.kernels import Layout
from ress_b200 import synth

from toy_model import ToyModel, write_tables

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture()
def tables(tmp_path, monkeypatch):
    write_tables(str(tmp_path))
    monkeypatch.setenv("RESS_CALIBRATION_DIR", str(tmp_path))
    return tmp_path


def test_criterion_grammar():
    s = criterion.parse_restore_swap("restore_swap_iter5_bf16_trackbest")
    assert (s.n_iters, s.track_best, s.big_dtype, s.use_wo, s.restore_frac, s.decay) == (5, True, torch.bfloat16, True, 0.5, 0.5)
    s = criterion.parse_restore_swap("damage_restore_swap_iter3_rf40_dc25_trackbest")
    assert (s.n_iters, s.use_wo, s.restore_frac, s.decay, s.big_dtype) == (3, False, 0.4, 0.25, None)
    s = criterion.parse_restore_swap("restore_swap_nowo_anti")
    assert (s.n_iters, s.use_wo, s.maximize, s.invert_cut) == (1, False, True, True)
    assert criterion.is_restore_swap("restore_swap_iter2_wo_bf16")
    assert not criterion.is_restore_swap("probability")
    with pytest.raises(ValueError):
        criterion.parse_restore_swap("projected")


def test_mode_switching_resets_every_knob(tables):
    """The reference's tests/test_runtime_mode_isolation.py contract: each
    apply_* clears what the previous mode installed (runtime/static.py:48-66)."""
    model = ToyModel(n_blocks=3)
    model._ress_backbone = "vggt"
    for blk in wiring.global_blocks(model):
        blk.attn.joint_select_fn = lambda *a: None
        blk.attn.perhead_budget_fn = lambda *a: None
        blk.attn.num_to_select = torch.ones(1)
        blk.attn.dense = True
    ress.apply_ress(model, sparse_ratio=0.5)
    for blk in wiring.global_blocks(model):
        a = blk.attn
        assert a.joint_select_fn is None and a.perhead_budget_fn is None and a.num_to_select is None
        assert a.dense is False and a.block_criterion == "restore_swap_iter5_bf16_trackbest"
        assert a.budget_fn.ress_budget[0].__class__.__name__ == "HessBudget"
        assert getattr(a, "M", None) is not None and a.M.shape == (16, 64, 64)
    ress.apply_sparse_vggt(model, 0.3, cdf_threshold=0.9)
    for i, blk in enumerate(wiring.global_blocks(model)):
        a = blk.attn
        assert a.block_criterion == "probability"
        b, layer, sr, cdf, beta = a.budget_fn.ress_budget
        assert isinstance(b, B.UniformBudget) and (layer, sr, cdf, beta) == (i, 0.3, 0.9, 1.0)
    ress.apply_dense(model)
    assert wiring.global_blocks(model)[0].attn.budget_fn.ress_budget[2] == 0.0
    ress.apply_hess(model, 0.5, 0.97)
    assert isinstance(wiring.global_blocks(model)[1].attn.budget_fn.ress_budget[0], B.HessBudget)


def test_budget_cache_and_backbone_errors(tables):
    model = ToyModel(n_blocks=1)
    with pytest.raises(ValueError):
        ress.apply_ress(model, 0.5)
    ress.apply_ress(model, 0.5, backbone="vggt")
    c1 = model._ress_budget_cache
    ress.apply_hess(model, 0.5, backbone="vggt")
    assert model._ress_budget_cache is c1
    with pytest.raises(ValueError):
        ress.get_backbone("nope")
    with pytest.raises(RuntimeError):
        ress.load_backbone("vggt")


def test_hess_tables_match_reference(tables):
    """HessBudget's head scores equal the reference's (fixture written by
    running the reference's HessBudget on the same synthetic tables)."""
    pooled = dict(np.load(os.path.join(GOLD, "cfg1_pooled.npz")))
    pcd, cam = ress.get_backbone("vggt").calibration_paths()
    hess = B.HessBudget(cam, pcd, lam=0.5)
    assert torch.equal(hess.head_scores[0], torch.from_numpy(pooled["head_scores"]))


def test_bake_M_matches_definition():
    model = ToyModel(n_blocks=2)
    M = projected.bake_M(model)
    W = model.aggregator.global_blocks[1].attn.proj.weight.detach()
    assert M.shape == (2, 16, 64, 64)
    assert torch.allclose(M[1, 5], W[:, 320:384].T @ W[:, 320:384])


def test_kept_mass_quality_matches_bruteforce():
    """The closed form equals J - J_new computed directly (the reference's
    tests/test_kept_mass_norm.py::test_quality_matches_bruteforce)."""
    g = torch.Generator().manual_seed(0)
    G = torch.rand(5, generator=g, dtype=torch.float64) + 0.1
    Kk = torch.rand(5, generator=g, dtype=torch.float64) * 0.5 + 0.4
    dG = torch.randn(5, 7, generator=g, dtype=torch.float64) * 0.01
    u = (torch.rand(5, 7, generator=g, dtype=torch.float64) - 0.5) * 0.2
    closed = projected.kept_mass_norm_quality(G, Kk, dG, u)
    brute = G.unsqueeze(-1) / Kk.unsqueeze(-1) ** 2 - (G.unsqueeze(-1) + dG) / (Kk.unsqueeze(-1) + u) ** 2
    assert torch.allclose(closed, brute, rtol=1e-10, atol=1e-12)


def test_single_drop_objective_is_renormalised_cut():
    """J({j}) = ||p_j (v_q - v_j)||_M^2 / (1 - p_j)^2 = (s_j / (1 - p_j))^2
    (criterion.py:31-34): the cut's key and the rounds' objective agree."""
    g = torch.Generator().manual_seed(1)
    nk, hd = 9, 4
    p = torch.softmax(torch.randn(nk, generator=g, dtype=torch.float64), 0)
    V = torch.randn(nk, hd, generator=g, dtype=torch.float64)
    A = torch.randn(hd, hd, generator=g, dtype=torch.float64)
    M = A.T @ A
    vq = p @ V
    for j in range(nk):
        gvec = p[j] * vq - p[j] * V[j]
        J = gvec @ M @ gvec / (1 - p[j]) ** 2
        s = p[j] * torch.sqrt((vq - V[j]) @ M @ (vq - V[j]))
        assert torch.allclose(J, (s / (1 - p[j])) ** 2)


def test_projected_score_with_identity_metric_is_the_damage_score():
    """With M = I the projected score p_j * sqrt(q.Mq - 2 q.Mk + k.Mk)
    (projected.py:259-288, 359-388) is the head-space damage score
    p_j * ||v_q - V_j|| -- the reduction the reference relies on for its
    "damage_restore_swap*" criteria (attention.py:562-568).  Checked on the
    oracle's per-candidate score s, which follows the reference's bf16
    expanded form; the bounds allow for that form's bf16 roundings."""
    import oracle

    g = torch.Generator().manual_seed(3)
    nq, nkp, n_cand = 6, 40, 39
    P = torch.softmax(torch.randn(nq, nkp, generator=g, dtype=torch.float64) * 2, -1).to(torch.bfloat16)
    vb = (torch.randn(1, nkp, 64, generator=g) * 0.5).to(torch.bfloat16)
    nts = torch.full((nq,), 10, dtype=torch.int32)
    _, s = oracle.restore_swap(P, vb, torch.eye(64).unsqueeze(0), nts, n_cand, n_iters=0, track_best=False)
    Pd, V = P.double(), vb[0].double()
    vq = Pd @ V
    dmg = Pd[:, :n_cand] * (vq.unsqueeze(1) - V[:n_cand].unsqueeze(0)).norm(dim=-1)
    scale = Pd[:, :n_cand] * (vq.norm(dim=-1, keepdim=True) + V[:n_cand].norm(dim=-1).unsqueeze(0))
    err = (s.double() - dmg).abs()
    assert float((err / scale).max()) < 0.02
    assert float((err / dmg).median()) < 0.01


@pytest.mark.parametrize("frames,special", [(4, 5), (32, 5), (12, 5), (6, 1)])
def test_no_special_key_is_a_candidate(frames, special):
    """Candidate blocks hold patch keys only; every special key lies in a sink
    block (attention.py:428-456, the reference's tests/test_special_key_protection.py)."""
    L = Layout(1, 16, frames, special, 37 * 37)
    assert L.n_cand * 64 <= L.Tp
    assert L.n_cand + L.sink_blocks == -(-L.Tk // 64)
    assert L.sink_blocks * 64 >= L.Ts
