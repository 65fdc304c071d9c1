"""The drop-in API on the GPU: apply_* on a wired VGGT-shaped model, then the
wired attention forward.  The forward must equal the fused layer run with the
budget and order the mode implies (bit for bit), and its keep lists must
equal the oracle's on the same Q/K/V."""

import pytest
import torch

import oracle
import ress_b200 as ress
from ress_b200 import attention as A
from ress_b200 import kernels as K
from ress_b200 import layer as LY
from ress_b200 import qkv as QKV
from ress_b200 import synth, wiring

from toy_model import ToyModel, positions, write_tables

pytestmark = pytest.mark.gpu
SHAPE = synth.CONFIG1


@pytest.fixture(scope="module")
def setup(tmp_path_factory):
    d = tmp_path_factory.mktemp("cal")
    write_tables(str(d))
    import os
    os.environ["RESS_CALIBRATION_DIR"] = str(d)
    dev = torch.device("cuda", 0)
    model = ToyModel(n_blocks=2).to(dev)
    store = {0: {}, 1: {}}
    wiring.wire_ress_attention(model, model.aggregator.global_blocks, aux_output_store=store)
    model._ress_backbone = "vggt"
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, SHAPE.t_total, 1024, generator=g).to(dev)
    pos = positions(SHAPE).to(dev)
    return model, store, x, pos, dev


def _manual(attn, x, pos, budget, order):
    q, k, v, shp = QKV.compute_qkv(attn, x, pos)
    L = K.Layout(1, 16, shp["N"], shp["S"], shp["P"] - shp["S"])
    res = LY.global_layer(q, k.contiguous(), v.contiguous(), L, budget, order)
    out = QKV.project_out(attn, res.out, 1, shp["N"], shp["P"], 16, 64)
    return out, res, (q, k, v), L


@pytest.mark.parametrize("mode", ["ress", "hess_cdf", "sparse_vggt", "dense"])
def test_apply_then_forward(setup, mode):
    model, store, x, pos, dev = setup
    if mode == "ress":
        ress.apply_ress(model, sparse_ratio=0.5)
    elif mode == "hess_cdf":
        ress.apply_hess(model, sparse_ratio=0.5, cdf_threshold=0.97)
    elif mode == "sparse_vggt":
        ress.apply_sparse_vggt(model, sparse_ratio=0.3)
    else:
        ress.apply_dense(model)
    uniform, hess = model._ress_budget_cache[1]
    for i, blk in enumerate(model.aggregator.global_blocks):
        attn = blk.attn
        with torch.no_grad():
            out_api = attn(x, pos=pos)
            if mode == "ress":
                budget = hess.spec(i, 0.5, None, 1.0, device=dev)
                order = LY.OrderSpec("restore_swap", M=attn.M.float())
            elif mode == "hess_cdf":
                budget, order = hess.spec(i, 0.5, 0.97, 1.0, device=dev), LY.OrderSpec("probability")
            elif mode == "sparse_vggt":
                budget, order = uniform.spec(i, 0.3, None, 1.0), LY.OrderSpec("probability")
            else:
                budget, order = uniform.spec(i, 0.0, None, 1.0), LY.OrderSpec("probability")
            out_man, res, (q, k, v), L = _manual(attn, x, pos, budget, order)
        torch.cuda.synchronize()
        K.check_status(dev)
        assert torch.equal(out_api, out_man)
        # keep lists against the oracle on the same Q/K/V
        qp = QKV.get_patch_tokens(q.cpu(), L.frames, L.special + L.hw, L.special)
        kp = QKV.get_patch_tokens(k.cpu(), L.frames, L.special + L.hw, L.special)
        vp = QKV.get_patch_tokens(v.cpu().contiguous(), L.frames, L.special + L.hw, L.special)
        hs = hess.head_scores[i] if mode in ("ress", "hess_cdf") else None
        sr = {"ress": 0.5, "hess_cdf": 0.5, "sparse_vggt": 0.3, "dense": 0.0}[mode]
        cdf = 0.97 if mode == "hess_cdf" else None
        o = oracle.layer_select(qp, kp, vp, L.Ts, attn.M.float().cpu(), head_scores=hs,
                                mode="ress" if mode == "ress" else "prob", sparse_ratio=sr, cdf_threshold=cdf)
        assert torch.equal(res.counts.cpu(), o["counts"])
        width = L.n_cand + L.sink_blocks
        assert torch.equal(K.lists_to_map(res.lists, res.counts, width).cpu(),
                           K.lists_to_map(o["lists"], o["counts"], width))
        aux = store[i]["value"]
        assert aux.n_cand == L.n_cand and aux.attn_pooled.shape[-1] == L.n_cand
        assert abs(aux.sparsity - res.sparsity()) < 1e-12
        if mode == "dense":
            assert aux.sparsity == pytest.approx(1 - width / width if L.sink_blocks == 0 else aux.sparsity)


def test_custom_budget_fn_goes_through_the_python_hook(setup):
    """A budget object this package does not know is called with attn_cond,
    as in the reference (runtime/static.py:74-77)."""
    model, store, x, pos, dev = setup
    calls = []

    class Fixed:
        def num_to_select(self, layer_idx, attn_pooled, sparse_ratio=None, cdf_threshold=None, beta=1.0):
            calls.append(tuple(attn_pooled.shape))
            return torch.full(attn_pooled.shape[:-1], 30, dtype=torch.long, device=attn_pooled.device)

    from ress_b200 import static
    static.set_static_budget(model, Fixed(), 0.5)
    attn = model.aggregator.global_blocks[0].attn
    with torch.no_grad():
        attn(x, pos=pos)
    torch.cuda.synchronize()
    assert calls and calls[0][-1] == SHAPE.n_cand
    assert store[0]["value"].sparsity > 0


def test_run_block_sparse_kernel_and_build_block_mask(setup):
    """The standalone reference functions on plain (B, H, T, 64) tensors."""
    model, store, x, pos, dev = setup
    g = torch.Generator().manual_seed(9)
    q = torch.randn(1, 4, 700, 64, generator=g).to(dev)
    k = torch.randn(1, 4, 900, 64, generator=g).to(dev)
    v = torch.randn(1, 4, 900, 64, generator=g).to(dev)
    af = A.predict_attention(q, k)
    assert af.shape == (1, 4, 6, 15)
    nts = A.compute_baseline_num_to_select(af, 0.5, 0.9)
    fm = A.build_block_mask(af, nts, sink_blocks=0)
    o, sparsity = A.run_block_sparse_kernel(q, k, v, fm)
    torch.cuda.synchronize()
    assert o.shape == q.shape and o.dtype == torch.float32
    assert abs(sparsity - (1 - fm.float().mean().item())) < 1e-12
    # against fp32 masked attention on the same map (int8 quantisation error only)
    mask = fm.repeat_interleave(128, dim=-2)[..., :700, :].repeat_interleave(64, dim=-1)[..., :900]
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    assert (o - ref).abs().max().item() < 0.1
