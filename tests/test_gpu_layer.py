"""The fused layer (ress_b200.layer.global_layer) against the oracle chained
the way ress_attention_forward chains the reference (attention.py:446-659):
keep lists bit-identical, patch outputs within 2e-2 max / 1e-3 mean abs of
the fp64 oracle attention, special-token outputs equal to dense attention."""

import pytest
import torch
import torch.nn.functional as F

import oracle
from ress_b200 import kernels as K
from ress_b200 import layer as LY
from ress_b200 import synth

pytestmark = pytest.mark.gpu

CASES = [
    ("1f-bf16-ress", synth.LayerShape(n_frames=1), torch.bfloat16, "ress", 0.5, None),
    ("cfg1", synth.CONFIG1, torch.float32, "ress", 0.1, None),
    ("cfg1-hess-cdf", synth.CONFIG1, torch.float32, "prob", 0.5, 0.97),
    ("6f-bf16-ress", synth.LayerShape(n_frames=6), torch.bfloat16, "ress", 0.5, None),
    ("cfg2", synth.CONFIG2, torch.bfloat16, "ress", 0.5, None),
    ("cfg2-hess-cdf", synth.CONFIG2, torch.bfloat16, "prob", 0.5, 0.97),
]
_inp = {}


def _data(shape, dtype):
    if (shape, dtype) not in _inp:
        _inp[(shape, dtype)] = synth.layer_qkv(shape, seed=0, dtype=dtype)
    return _inp[(shape, dtype)]


@pytest.mark.parametrize("name,shape,dtype,mode,sr,cdf", CASES, ids=[c[0] for c in CASES])
def test_layer_matches_oracle(name, shape, dtype, mode, sr, cdf):
    q, k, v = _data(shape, dtype)
    M = synth.metric_from_weight(synth.out_proj_weight())
    hs = synth.fisher_table(seed=1)[0, 3]
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    dev = torch.device("cuda", 0)
    budget = LY.BudgetSpec("hess", sparse_ratio=sr, cdf_threshold=cdf, scores_norm=K.scores_norm(hs))
    order = LY.OrderSpec("restore_swap", M=M.to(dev)) if mode == "ress" else LY.OrderSpec("probability")
    res = LY.global_layer(q.to(dev), k.to(dev), v.to(dev), L, budget, order)
    torch.cuda.synchronize()
    K.check_status(dev)
    qp, qsp = synth.split_tokens(q, shape)
    kp, ks = synth.split_tokens(k, shape)
    vp, vs = synth.split_tokens(v, shape)
    o = oracle.layer_select(qp, kp, vp, ks.shape[-2], M, head_scores=hs, mode=mode, sparse_ratio=sr,
                            cdf_threshold=cdf)
    assert torch.equal(res.nts.cpu(), o["nts"])
    assert torch.equal(res.counts.cpu(), o["counts"])
    lists = res.lists.cpu()
    for i in range(o["counts"].numel()):
        c = int(o["counts"][i])
        assert torch.equal(lists[i, :c], o["lists"][i, :c]), i
    # attention on sampled rows
    q8, qs, k8, ksc, _ = oracle.quantize_qk(qp, torch.cat([kp, ks], -2))
    g = torch.Generator().manual_seed(1)
    samples = [(int(torch.randint(0, 16, (1,), generator=g)), int(torch.randint(0, L.nq, (1,), generator=g)))
               for _ in range(12)] + [(15, L.nq - 1)]
    ref = oracle.sparse_attn_rows(q8, qs, k8, ksc, torch.cat([vp, vs], -2).reshape(16, -1, 64).to(torch.float16),
                                  o["lists"].view(16, L.nq, -1), o["counts"].view(16, L.nq), samples)
    out = res.out.cpu()
    patch, special = synth.split_tokens(out, shape)
    errs = []
    for i, (h, qb) in enumerate(samples):
        n = min(128, L.Tp - qb * 128)
        errs.append((patch[0, h, qb * 128: qb * 128 + n] - ref[i, :n]).abs().reshape(-1))
    e = torch.cat(errs)
    assert e.max().item() < 2e-2, e.max().item()
    assert e.mean().item() < 1e-3, e.mean().item()
    # special-token queries: dense attention over all keys (attention.py:404-409)
    exp = F.scaled_dot_product_attention(qsp.float(), torch.cat([kp, ks], -2).float(),
                                         torch.cat([vp, vs], -2).float())
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert (special - exp).abs().max().item() < tol
    # sparsity as the reference reports it (sinks counted)
    width = o["n_cand"] + o["sink_blocks"]
    assert abs(res.sparsity() - (1 - o["counts"].sum().item() / (o["counts"].numel() * width))) < 1e-12


def test_head_split_equals_full():
    """Heads split into 4 groups with the HeSS baseline exchange emulated on
    one GPU gives the same lists as the unsplit layer."""
    shape, dtype = synth.LayerShape(n_frames=6), torch.bfloat16
    q, k, v = _data(shape, dtype)
    dev = torch.device("cuda", 0)
    M = synth.metric_from_weight(synth.out_proj_weight()).to(dev)
    sn = K.scores_norm(synth.fisher_table(seed=1)[0, 5])
    budget = LY.BudgetSpec("hess", sparse_ratio=0.5, scores_norm=sn)
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    full = LY.global_layer(qd, kd, vd, L, budget, LY.OrderSpec("restore_swap", M=M))
    # baselines of every group first (what the all-gather delivers)
    Lg = K.Layout(1, 4, shape.n_frames, shape.n_special, shape.hw)
    bases = []
    for g in range(4):
        sl = slice(4 * g, 4 * g + 4)
        qbar, _, _ = K.pool_quant_q(qd[:, sl].contiguous(), Lg, quant=False)
        kbar, _, _, _, _, _ = K.pool_quant_kv(kd[:, sl].contiguous(), vd[:, sl].contiguous(), Lg, quant=False)
        _, ac = K.predict(qbar, kbar, Lg.n_cand, full=False)
        bases.append(K.baseline(ac, 0.5).view(1, 4, -1))
    gathered = torch.cat(bases, dim=1)
    for g in range(4):
        sl = slice(4 * g, 4 * g + 4)
        shard = LY.HeadShard(h0=4 * g, h_total=16, gather=lambda base, _g=gathered: _g)
        part = LY.global_layer(qd[:, sl].contiguous(), kd[:, sl].contiguous(), vd[:, sl].contiguous(), Lg, budget,
                               LY.OrderSpec("restore_swap", M=M[sl]), shard=shard)
        rows = slice(4 * g * L.nq, (4 * g + 4) * L.nq)
        assert torch.equal(part.counts, full.counts[rows])
        w = L.n_cand + L.sink_blocks
        assert torch.equal(K.lists_to_map(part.lists, part.counts, w), K.lists_to_map(full.lists[rows], full.counts[rows], w))
        pp, ps = synth.split_tokens(part.out.cpu(), shape)
        fp, fs = synth.split_tokens(full.out[:, sl].cpu(), shape)
        assert torch.equal(pp, fp)
        assert (ps - fs).abs().max().item() < 1e-2


@pytest.mark.parametrize("equal_size,world", [(True, 4), (False, 5)])
def test_balanced_head_split_equals_full(equal_size, world):
    """Heads split by the balanced partition (non-contiguous head sets per
    rank, equal or unequal numbers of heads), baselines gathered back into
    global head order: each rank's lists and patch outputs are the unsplit
    layer's."""
    from ress_b200 import shard as SH

    shape, dtype = synth.LayerShape(n_frames=6), torch.bfloat16
    q, k, v = _data(shape, dtype)
    dev = torch.device("cuda", 0)
    M = synth.metric_from_weight(synth.out_proj_weight()).to(dev)
    hs = synth.fisher_table(seed=1)[0, 5]
    sn = K.scores_norm(hs)
    budget = LY.BudgetSpec("hess", sparse_ratio=0.5, scores_norm=sn)
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    full = LY.global_layer(qd, kd, vd, L, budget, LY.OrderSpec("restore_swap", M=M))
    parts = SH.balanced_heads(hs, world, cap=2.0, equal_size=equal_size)
    assert sorted(h for p in parts for h in p) == list(range(16))
    assert any(p != list(range(p[0], p[0] + len(p))) for p in parts)  # not all contiguous
    if not equal_size:
        assert len({len(p) for p in parts}) > 1
    base_all = torch.empty(1, 16, L.nq, dtype=torch.int32, device=dev)
    for p in parts:
        hidx = torch.as_tensor(p, device=dev)
        Lg = K.Layout(1, len(p), shape.n_frames, shape.n_special, shape.hw)
        qbar, _, _ = K.pool_quant_q(qd.index_select(1, hidx).contiguous(), Lg, quant=False)
        kbar, _, _, _, _, _ = K.pool_quant_kv(kd.index_select(1, hidx).contiguous(),
                                              vd.index_select(1, hidx).contiguous(), Lg, quant=False)
        _, ac = K.predict(qbar, kbar, Lg.n_cand, full=False)
        base_all[:, hidx] = K.baseline(ac, 0.5).view(1, len(p), -1)
    w = L.n_cand + L.sink_blocks
    for p in parts:
        hidx = torch.as_tensor(p, device=dev)
        Lg = K.Layout(1, len(p), shape.n_frames, shape.n_special, shape.hw)
        sh = LY.HeadShard(h0=p[0], h_total=16, gather=lambda base, _g=base_all: _g, heads=tuple(p))
        part = LY.global_layer(qd.index_select(1, hidx).contiguous(), kd.index_select(1, hidx).contiguous(),
                               vd.index_select(1, hidx).contiguous(), Lg, budget,
                               LY.OrderSpec("restore_swap", M=M[hidx]), shard=sh)
        rows = (hidx[:, None] * L.nq + torch.arange(L.nq, device=dev)[None, :]).reshape(-1)
        assert torch.equal(part.counts, full.counts[rows])
        assert torch.equal(K.lists_to_map(part.lists, part.counts, w),
                           K.lists_to_map(full.lists[rows], full.counts[rows], w))
        pp, _ = synth.split_tokens(part.out.cpu(), shape)
        fp, _ = synth.split_tokens(full.out[:, hidx].cpu(), shape)
        assert torch.equal(pp, fp)


def test_cuda_graph_replay_equals_eager():
    """The layer captured in a CUDA graph (library kernels, side-stream SDPA)
    replays to the same bits as the eager call."""
    shape, dtype = synth.LayerShape(n_frames=6), torch.bfloat16
    q, k, v = (t.cuda() for t in _data(shape, dtype))
    dev = q.device
    M = synth.metric_from_weight(synth.out_proj_weight()).to(dev)
    sn = K.scores_norm(synth.fisher_table(seed=1)[0, 1]).to(dev)
    budget = LY.BudgetSpec("hess", sparse_ratio=0.5, scores_norm=sn)
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    order = LY.OrderSpec("restore_swap", M=M)
    eager = LY.global_layer(q, k, v, L, budget, order)
    out = torch.empty_like(eager.out)
    cap = LY.CapturedLayer(lambda: LY.global_layer(q, k, v, L, budget, order, out=out))
    for _ in range(2):
        r = cap.replay()
        torch.cuda.synchronize()
        assert torch.equal(r.out, eager.out)
        assert torch.equal(r.counts, eager.counts)


def test_cuda_graph_replay_with_split_attention():
    """The same with the split attention launch (attn_split=16: scratch
    allocated and the per-row counters zeroed inside the capture): replays
    give the eager call's bits, twice in a row."""
    shape, dtype = synth.LayerShape(n_frames=6), torch.bfloat16
    q, k, v = (t.cuda() for t in _data(shape, dtype))
    dev = q.device
    M = synth.metric_from_weight(synth.out_proj_weight()).to(dev)
    sn = K.scores_norm(synth.fisher_table(seed=1)[0, 1]).to(dev)
    budget = LY.BudgetSpec("hess", sparse_ratio=0.5, scores_norm=sn)
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    order = LY.OrderSpec("restore_swap", M=M)
    eager = LY.global_layer(q, k, v, L, budget, order, attn_split=16)
    out = torch.empty_like(eager.out)
    cap = LY.CapturedLayer(lambda: LY.global_layer(q, k, v, L, budget, order, out=out, attn_split=16))
    for _ in range(2):
        r = cap.replay()
        torch.cuda.synchronize()
        K.check_status(dev)
        assert torch.equal(r.out, eager.out)
        assert torch.equal(r.counts, eager.counts)


@pytest.mark.parametrize("world", [2, 4])
def test_view_sharded_layer_equals_full(world):
    """Frames sharded over `world` ranks, emulated in one process (the
    all-gather hands every rank the other ranks' contributions): each rank's
    budgets, keep lists and output rows are the unsharded layer's bits."""
    from ress_b200 import shard

    shape = synth.LayerShape(n_frames=8)
    dev = torch.device("cuda", 0)
    q, k, v = (t.to(dev) for t in synth.layer_qkv(shape, seed=2, dtype=torch.bfloat16, device=dev))
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    M = synth.metric_from_weight(synth.out_proj_weight()).to(dev)
    hs = synth.fisher_table(seed=1)[0, 4]
    budget = LY.BudgetSpec("hess", sparse_ratio=0.5, scores_norm=K.scores_norm(hs).to(dev))
    order = LY.OrderSpec("restore_swap", M=M)
    ref = LY.global_layer(q, k, v, L, budget, order)
    per = shape.n_frames // world * (shape.n_special + shape.hw)
    geoms = [shard.ViewGeom(shape.n_frames, shape.n_special, shape.hw, world, r) for r in range(world)]
    local = [tuple(t[:, :, r * per:(r + 1) * per].contiguous() for t in (q, k, v)) for r in range(world)]
    parts = [shard.view_exchange_parts(*local[r], geoms[r]) for r in range(world)]

    def gather(name, t):
        return [p[name] for p in parts]

    nq = L.nq
    for r in range(world):
        g = geoms[r]
        res = shard.view_sharded_layer(*local[r], g, budget, order, gather)
        torch.cuda.synchronize()
        K.check_status(dev)
        assert torch.equal(res.out, ref.out[:, :, r * per:(r + 1) * per])
        ref_rows = torch.arange(16, device=dev)[:, None] * nq + torch.arange(g.b0, g.b1, device=dev)[None, :]
        ref_rows = ref_rows.reshape(-1)
        assert torch.equal(res.nts.view(16, -1), ref.nts.view(16, nq)[:, g.b0:g.b1])
        assert torch.equal(res.counts, ref.counts[ref_rows])
        valid = torch.arange(res.lists.shape[1], device=dev)[None, :] < res.counts[:, None]
        assert torch.equal(torch.where(valid, res.lists, -1), torch.where(valid, ref.lists[ref_rows], -1))


def test_da3_shape_layer_matches_oracle():
    """The DA3 backbone's metadata (backbones.py: 24 heads, one special token)
    through the same kernels: budgets and keep lists bit-identical to the
    oracle chained like ress_attention_forward."""
    shape = synth.LayerShape(n_frames=4, n_heads=24, n_special=1, grid_h=28, grid_w=28)
    q, k, v = synth.layer_qkv(shape, seed=5, dtype=torch.bfloat16)
    H = 24
    M = synth.metric_from_weight(synth.out_proj_weight(dim=H * 64), H)
    hs = synth.fisher_table(n_heads=H, seed=7)[0, 2]
    L = K.Layout(1, H, shape.n_frames, shape.n_special, shape.hw)
    dev = torch.device("cuda", 0)
    budget = LY.BudgetSpec("hess", sparse_ratio=0.5, scores_norm=K.scores_norm(hs))
    res = LY.global_layer(q.to(dev), k.to(dev), v.to(dev), L, budget, LY.OrderSpec("restore_swap", M=M.to(dev)))
    torch.cuda.synchronize()
    K.check_status(dev)
    qp, _ = synth.split_tokens(q, shape)
    kp, ks = synth.split_tokens(k, shape)
    vp, _ = synth.split_tokens(v, shape)
    o = oracle.layer_select(qp, kp, vp, ks.shape[-2], M, head_scores=hs, mode="ress", sparse_ratio=0.5,
                            cdf_threshold=None)
    assert torch.equal(res.nts.cpu(), o["nts"])
    assert torch.equal(res.counts.cpu(), o["counts"])
    lists = res.lists.cpu()
    for i in range(o["counts"].numel()):
        c = int(o["counts"][i])
        assert torch.equal(lists[i, :c], o["lists"][i, :c]), i


@pytest.mark.parametrize("attn_split", [None, 16])
def test_layer_attn_split_option(attn_split):
    """global_layer's attn_split option (the split attention launch for layers
    with few rows: None lets the launch decide, and a 4-frame layer's 16 x 43
    rows are few enough on a B200 to split its long rows; 16 forces 16-block
    pieces): the keep lists are those of the default launch, and the outputs
    agree with it within 2e-3 max abs."""
    shape = synth.LayerShape(n_frames=4)
    q, k, v = (t.cuda() for t in _data(shape, torch.bfloat16))
    M = synth.metric_from_weight(synth.out_proj_weight()).cuda()
    hs = synth.fisher_table(seed=1)[0, 3]
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    budget = LY.BudgetSpec("hess", sparse_ratio=0.5, scores_norm=K.scores_norm(hs).cuda())
    order = LY.OrderSpec("restore_swap", M=M)
    ref = LY.global_layer(q, k, v, L, budget, order)
    res = LY.global_layer(q, k, v, L, budget, order, attn_split=attn_split)
    torch.cuda.synchronize()
    K.check_status()
    assert torch.equal(res.counts, ref.counts)
    assert (res.out - ref.out).abs().max().item() < 2e-3
