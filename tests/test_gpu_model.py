"""The VGGT-shaped aggregator (ress_b200.vggt) wired through the public API:
apply_dense keeps every candidate block, so its global layers must match the
same model run with dense torch attention within the attention tolerance
(int8 Q/K and fp16 P in the sparse kernel); apply_ress runs and stays finite."""

import pytest
import torch

from ress_b200 import api, synth, vggt, wiring

pytestmark = pytest.mark.gpu


def _model():
    torch.manual_seed(0)
    m = vggt.VGGTAggregatorModel(dim=256, depth=2, num_heads=4, img=112, encoder_depth=1, intermediate=(0, 1))
    m = m.cuda().float().eval()
    return m


def _wire(m, tmp_path, monkeypatch):
    for name, seed in (("cam_pos", 1), ("pcd", 3)):
        torch.save(synth.fisher_table(24, 4, seed=seed), tmp_path / f"fisher_scores_vggt_{name}.pt")
    monkeypatch.setenv("RESS_CALIBRATION_DIR", str(tmp_path))
    wiring.wire_ress_attention(m, m.aggregator.global_blocks, num_special_tokens=5)
    m._ress_backbone = "vggt"


def test_dense_mode_matches_torch_attention(tmp_path, monkeypatch):
    m = _model()
    g = torch.Generator(device="cuda").manual_seed(1)
    images = torch.rand(1, 6, 3, 112, 112, device="cuda", generator=g)
    with torch.inference_mode():
        ref, _ = m(images)
    _wire(m, tmp_path, monkeypatch)
    api.apply_dense(m)
    with torch.inference_mode():
        got, _ = m(images)
    for a, b in zip(got, ref):
        rel = (a - b).abs().max() / b.abs().max()
        assert rel < 2e-2, float(rel)
    api.apply_ress(m, sparse_ratio=0.5, n_iters=5)
    with torch.inference_mode():
        out, _ = m(images)
    assert all(torch.isfinite(o).all() for o in out)
