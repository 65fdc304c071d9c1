"""Config 4 at its full size: one global layer of 200 views (274,800 tokens
per head, 16 heads, 2,140 q-blocks, n_cand = 4,278 candidate blocks, 16 sink
blocks), apply_ress at sparse_ratio 0.75 with the HeSS budget — the layer
that runs the streamed large-layer restore-swap kernel and the longest
attention rows.  The oracle cannot run this layer end to end in seconds, so
the whole layer is held to size-independent properties and two heads to the
oracle stage by stage, each stage fed the GPU's own inputs of that stage:

* two runs give the same bits (lists, counts, outputs);
* every keep list is strictly ascending, ends with the 16 sink blocks and
  holds the row's budget plus the sinks (attention.py:147-174, 446-491);
* the budgets equal the oracle's HeSS re-allocation of the ratio baseline
  (attention.py:268-293, budget/_proportional.py:149-215), all rows;
* pooled means, the pooled softmax map, the key mean and the int8/fp16
  operands of two heads are bit-identical to the oracle's;
* restore-swap keep lists of sampled rows of those heads are bit-identical
  to the oracle's (projected.py:395-1058);
* sampled rows of the attention output, the longest and the ragged last
  q-block among them, are within 2e-2 max / 1e-3 mean abs of the oracle's
  fp64 attention on the same operands and lists."""

import pytest
import torch

import oracle
from ress_b200 import kernels as K
from ress_b200 import layer as LY
from ress_b200 import synth

pytestmark = pytest.mark.gpu

SPARSE_RATIO = 0.75
HEADS = (0, 15)


@pytest.fixture(scope="module")
def cfg4():
    dev = torch.device("cuda", 0)
    shape = synth.CONFIG4
    q, k, v = synth.layer_qkv(shape, seed=0, dtype=torch.bfloat16, device=dev)
    M = synth.metric_from_weight(synth.out_proj_weight()).to(dev)
    hs = synth.fisher_table(seed=1)[0, 3]
    L = K.Layout(1, 16, shape.n_frames, shape.n_special, shape.hw)
    budget = LY.BudgetSpec("hess", sparse_ratio=SPARSE_RATIO, scores_norm=K.scores_norm(hs).to(dev))
    order = LY.OrderSpec("restore_swap", M=M)
    res = LY.global_layer(q, k, v, L, budget, order)
    torch.cuda.synchronize()
    K.check_status(dev)
    return dict(shape=shape, q=q, k=k, v=v, M=M, hs=hs, L=L, budget=budget, order=order, res=res)


def test_config4_sizes(cfg4):
    L = cfg4["L"]
    assert (L.Tp, L.Tk, L.nq, L.n_cand, L.sink_blocks) == (273800, 274800, 2140, 4278, 16)


def test_config4_deterministic(cfg4):
    res = cfg4["res"]
    again = LY.global_layer(cfg4["q"], cfg4["k"], cfg4["v"], cfg4["L"], cfg4["budget"], cfg4["order"])
    torch.cuda.synchronize()
    assert torch.equal(again.counts, res.counts)
    # entries past a row's count are unspecified (the buffer is not cleared)
    valid = torch.arange(res.lists.shape[1], device=res.lists.device).unsqueeze(0) < res.counts.unsqueeze(1)
    assert torch.equal(torch.where(valid, again.lists, 0), torch.where(valid, res.lists, 0))
    assert torch.equal(again.out, res.out)


def test_config4_lists_and_budgets(cfg4):
    res, L = cfg4["res"], cfg4["L"]
    n_cand, sinks = L.n_cand, L.sink_blocks
    nts = res.nts.reshape(-1)
    counts = res.counts
    assert torch.equal(counts, nts + sinks)
    # budgets: the oracle's HeSS re-allocation of the ratio baseline (every
    # row's baseline is int(n_cand * (1 - r)) without a CDF threshold)
    base = torch.full((1, L.H, L.nq), int(n_cand * (1 - SPARSE_RATIO)), dtype=torch.int32)
    exp = oracle.hess_adjust(base, oracle.scores_norm(cfg4["hs"]), n_cand, min_clamp=2)
    assert torch.equal(res.nts.cpu().view(1, L.H, L.nq), exp)
    # lists: strictly ascending over the valid prefix, the sinks last
    lists = res.lists
    width = lists.shape[1]
    assert width == n_cand + sinks
    valid = torch.arange(1, width, device=lists.device).unsqueeze(0) < counts.unsqueeze(1)
    assert bool(((lists[:, 1:] > lists[:, :-1]) | ~valid).all())
    idx = (counts.long().unsqueeze(1) - sinks) + torch.arange(sinks, device=lists.device)
    tail = lists.gather(1, idx)
    assert bool((tail == n_cand + torch.arange(sinks, device=lists.device, dtype=lists.dtype)).all())
    assert int(lists[:, 0].min()) >= 0


def _head_inputs(cfg4, h):
    shape = cfg4["shape"]
    qp, _ = synth.split_tokens(cfg4["q"][:, h:h + 1], shape)
    kp, ks = synth.split_tokens(cfg4["k"][:, h:h + 1], shape)
    vp, vs = synth.split_tokens(cfg4["v"][:, h:h + 1], shape)
    return (qp[0].cpu(), kp[0].cpu(), vp[0].cpu(), torch.cat([kp, ks], -2)[0].cpu(),
            torch.cat([vp, vs], -2)[0].cpu())


@pytest.mark.parametrize("h", HEADS)
def test_config4_head_stages_match_oracle(cfg4, h):
    res, L, M = cfg4["res"], cfg4["L"], cfg4["M"]
    q, k, v = cfg4["q"], cfg4["k"], cfg4["v"]
    qp, kp, vp, key, value = _head_inputs(cfg4, h)
    qbar, q8, qs = K.pool_quant_q(q, L)
    kbar, vbar, k8, ks, v16, km = K.pool_quant_kv(k, v, L)
    torch.cuda.synchronize()
    # pooled means and the pooled softmax map
    assert torch.equal(qbar[h:h + 1].cpu(), oracle.pool_mean(qp, 128))
    assert torch.equal(kbar[h:h + 1].cpu(), oracle.pool_mean(kp, 64))
    assert torch.equal(vbar[h:h + 1].cpu(), oracle.pool_mean(vp, 64))
    af = oracle.predict(qbar[h:h + 1].cpu(), kbar[h:h + 1].cpu())
    assert torch.equal(res.attn_full[h:h + 1].cpu(), af)
    # quantised operands: the key mean over all 274,800 keys, then sampled blocks
    k16 = key.to(torch.float16).float()
    kmo = oracle.key_mean(k16)
    assert torch.equal(km[h:h + 1].cpu(), kmo)
    kc = (k16 - kmo.unsqueeze(1)).to(torch.float16).float()
    q16 = qp.to(torch.float16).float()
    for qb in (0, 1069, L.nq - 1):
        lo, hi = qb * 128, min(L.Tp, qb * 128 + 128)
        q8o, qso = oracle.quant_blocks(q16[:, lo:hi], 128)
        assert torch.equal(q8[h, lo:hi].cpu(), q8o[0]) and float(qs[h, qb]) == float(qso[0, 0])
    for kb in (0, 2000, L.n_cand - 1, L.nkb - 1):
        lo, hi = kb * 64, min(L.Tk, kb * 64 + 64)
        k8o, kso = oracle.quant_blocks(kc[:, lo:hi], 64)
        assert torch.equal(k8[h, lo:hi].cpu(), k8o[0]) and float(ks[h, kb]) == float(kso[0, 0])
    assert torch.equal(v16[h].cpu(), value[0].to(torch.float16))
    # restore-swap keep lists of sampled rows, fed the GPU's pooled map and values
    nts = res.nts.view(L.H, L.nq)[h]
    counts = res.counts.view(L.H, L.nq)[h]
    g = torch.Generator().manual_seed(h)
    longest = int(torch.argmax(counts))
    qsel = sorted({0, longest, L.nq - 1, *torch.randint(0, L.nq, (3,), generator=g).tolist()})
    drop, _ = oracle.restore_swap(res.attn_full[h, qsel].cpu(), res.vbar[h:h + 1].cpu(), M[h:h + 1].cpu(),
                                  nts[qsel].cpu(), L.n_cand)
    lo_lists, lo_counts = oracle.keep_lists(~drop, L.sink_blocks)
    lists = res.lists.view(L.H, L.nq, -1)[h]
    for i, qb in enumerate(qsel):
        c = int(lo_counts[i])
        assert c == int(counts[qb]), qb
        assert torch.equal(lists[qb, :c].cpu(), lo_lists[i, :c]), qb
    # attention of sampled rows (the longest and the ragged last q-block among them)
    samples = [(0, qb) for qb in (longest, L.nq - 1, qsel[1])]
    ref = oracle.sparse_attn_rows(q8[h:h + 1].cpu(), qs[h:h + 1].cpu(), k8[h:h + 1].cpu(), ks[h:h + 1].cpu(),
                                  v16[h:h + 1].cpu(), lists.cpu().unsqueeze(0), counts.cpu().unsqueeze(0), samples)
    patch, _ = synth.split_tokens(res.out[:, h:h + 1], cfg4["shape"])
    patch = patch[0, 0]
    errs = []
    for i, (_, qb) in enumerate(samples):
        n = min(128, L.Tp - qb * 128)
        errs.append((patch[qb * 128: qb * 128 + n].cpu() - ref[i, :n]).abs().reshape(-1))
    e = torch.cat(errs)
    assert e.max().item() < 2e-2, e.max().item()
    assert e.mean().item() < 1e-3, e.mean().item()
