"""Kernel-level parity on the GPU: every kernel against the CPU oracle on the
same seeded inputs.  Index/integer outputs must be bit-identical; the
attention output is held to the north-star tolerance (2e-2 max-abs,
1e-3 mean-abs) against the oracle's fp64 attention on the same int8 inputs."""

import pytest
import torch

import oracle
from ress_b200 import kernels as K
from ress_b200 import synth

pytestmark = pytest.mark.gpu

SMALL = synth.LayerShape(n_frames=6)
CASES = [(synth.CONFIG1, torch.float32), (SMALL, torch.bfloat16)]
_cache = {}


def _inputs(shape, dtype):
    key = (shape, dtype)
    if key not in _cache:
        q, k, v = synth.layer_qkv(shape, seed=0, dtype=dtype)
        _cache[key] = (q, k, v)
    return _cache[key]


def _layout(shape):
    return K.Layout(1, shape.n_heads, shape.n_frames, shape.n_special, shape.hw)


def _bits(t):
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16)
    if t.dtype == torch.float32:
        return t.view(torch.int32)
    return t


def _eq(a, b):
    return torch.equal(_bits(a), _bits(b))


@pytest.mark.parametrize("shape,dtype", CASES)
def test_pooling_and_quant_bit_exact(shape, dtype):
    q, k, v = _inputs(shape, dtype)
    L = _layout(shape)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    qbar, q8, qs = K.pool_quant_q(qd, L)
    kbar, vbar, k8, ks, v16, km = K.pool_quant_kv(kd, vd, L)
    torch.cuda.synchronize()
    qp, _ = synth.split_tokens(q, shape)
    kp, ksp = synth.split_tokens(k, shape)
    vp, vsp = synth.split_tokens(v, shape)
    H = shape.n_heads
    assert _eq(qbar, oracle.pool_mean(qp.reshape(H, -1, 64), 128))
    assert _eq(kbar, oracle.pool_mean(kp.reshape(H, -1, 64), 64))
    assert _eq(vbar, oracle.pool_mean(vp.reshape(H, -1, 64), 64))
    key = torch.cat([kp, ksp], dim=-2)
    val = torch.cat([vp, vsp], dim=-2)
    q8o, qso, k8o, kso, kmo = oracle.quantize_qk(qp, key)
    assert _eq(km, kmo)
    assert torch.equal(q8.cpu(), q8o) and _eq(qs, qso)
    assert torch.equal(k8.cpu(), k8o) and _eq(ks, kso)
    assert torch.equal(v16.cpu(), val.reshape(H, -1, 64).to(torch.float16))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pooling_and_quant_extreme_tiles(dtype):
    """Tiles whose values are all tiny (|x| maximum below 0.0157: the fp16
    rounding path), all zero, large (~1e4) or in fp16's subnormal range, in
    runs of 300 tokens so that whole 128-query and 64-key tiles fall inside
    one regime: the pooled means, int8 codes, scales and key mean stay
    bit-identical to the oracle."""
    shape = SMALL
    q, k, v = synth.layer_qkv(shape, seed=3, dtype=torch.float32)
    T = q.shape[-2]
    runs = torch.tensor([1.0, 1e-3, 0.0, 3e3, 1e-6, 1.0, 2e-4])
    f = runs[(torch.arange(T) // 300) % len(runs)].view(1, 1, T, 1)
    q, k, v = ((x * f * g).to(dtype) for x, g in ((q, 1.0), (k, 0.7), (v, 1.3)))
    L = _layout(shape)
    qbar, q8, qs = K.pool_quant_q(q.cuda(), L)
    kbar, vbar, k8, ks, v16, km = K.pool_quant_kv(k.cuda(), v.cuda(), L)
    torch.cuda.synchronize()
    qp, _ = synth.split_tokens(q, shape)
    kp, ksp = synth.split_tokens(k, shape)
    vp, vsp = synth.split_tokens(v, shape)
    H = shape.n_heads
    assert _eq(qbar, oracle.pool_mean(qp.reshape(H, -1, 64), 128))
    assert _eq(kbar, oracle.pool_mean(kp.reshape(H, -1, 64), 64))
    assert _eq(vbar, oracle.pool_mean(vp.reshape(H, -1, 64), 64))
    key = torch.cat([kp, ksp], dim=-2)
    val = torch.cat([vp, vsp], dim=-2)
    q8o, qso, k8o, kso, kmo = oracle.quantize_qk(qp, key)
    assert _eq(km, kmo)
    assert torch.equal(q8.cpu(), q8o) and _eq(qs, qso)
    assert torch.equal(k8.cpu(), k8o) and _eq(ks, kso)
    assert torch.equal(v16.cpu(), val.reshape(H, -1, 64).to(torch.float16))
    # the regimes were reached: zero, sub-window and large tiles among the Q scales
    qsc = qs.cpu().flatten()
    assert (qsc == 0).any() and ((qsc > 0) & (qsc < 0.0157 / 127)).any() and (qsc > 10).any()


@pytest.mark.parametrize("shape,dtype", CASES)
def test_predict_cond_baseline_bit_exact(shape, dtype):
    q, k, v = _inputs(shape, dtype)
    L = _layout(shape)
    qbar, _, _ = K.pool_quant_q(q.cuda(), L, quant=False)
    kbar, _, _, _, _, _ = K.pool_quant_kv(k.cuda(), v.cuda(), L, quant=False)
    af, ac = K.predict(qbar, kbar, L.n_cand)
    torch.cuda.synchronize()
    afo = oracle.predict(qbar.cpu(), kbar.cpu())
    assert _eq(af, afo)
    aco = oracle.attn_cond(afo, L.n_cand)
    assert _eq(ac, aco)
    for sr, cdf in ((0.5, 0.97), (None, 0.9), (0.1, None)):
        b = K.baseline(ac, sr, cdf)
        assert torch.equal(b.cpu(), oracle.baseline(aco, sr, cdf)), (sr, cdf)


def test_hess_adjust_bit_exact():
    g = torch.Generator().manual_seed(3)
    base = torch.randint(2, 60, (2, 16, 37), generator=g, dtype=torch.int32)
    for scale in (1.0, 30.0):
        hs = torch.exp(torch.randn(16, generator=g)) * torch.linspace(1, scale, 16)
        sn = K.scores_norm(hs)
        for beta in (1.0, 0.25):
            got = K.hess_adjust(base.cuda(), sn, 60, beta=beta, min_clamp=2)
            exp = oracle.hess_adjust(base, oracle.scores_norm(hs), 60, beta=beta, min_clamp=2)
            assert torch.equal(got.cpu(), exp), (scale, beta)
    K.check_status()


@pytest.mark.parametrize("shape,dtype", CASES)
@pytest.mark.parametrize("sr", [0.1, 0.5, 0.9])
def test_restore_swap_bit_exact(shape, dtype, sr):
    q, k, v = _inputs(shape, dtype)
    L = _layout(shape)
    qbar, _, _ = K.pool_quant_q(q.cuda(), L, quant=False)
    kbar, vbar, _, _, _, _ = K.pool_quant_kv(k.cuda(), v.cuda(), L, quant=False)
    af, ac = K.predict(qbar, kbar, L.n_cand)
    hs = synth.fisher_table(seed=1)[0, 0]
    nts = K.hess_adjust(K.baseline(ac, sr).view(1, 16, -1), K.scores_norm(hs), L.n_cand, min_clamp=2)
    M = synth.metric_from_weight(synth.out_proj_weight())
    r = K.restore_swap(af, vbar, M.cuda(), nts.view(-1), L.n_cand, sink_blocks=L.sink_blocks, want_drop=True,
                       want_s=True)
    torch.cuda.synchronize()
    drop_o, s_o = oracle.restore_swap(af.cpu(), vbar.cpu().to(torch.bfloat16), M, nts.cpu().view(-1), L.n_cand)
    assert _eq(r["s"], s_o)
    assert torch.equal(r["drop"].cpu().bool(), drop_o)
    lists_o, counts_o = oracle.keep_lists(~drop_o, L.sink_blocks)
    assert torch.equal(r["counts"].cpu(), counts_o)
    for i in range(counts_o.numel()):
        c = int(counts_o[i])
        assert torch.equal(r["lists"][i, :c].cpu(), lists_o[i, :c])
    K.check_status()


def test_restore_swap_large_layer_bit_exact():
    """60 frames: 1,283 candidate blocks, past the size at which a head's pooled
    V stays resident in shared memory, so the kernel that streams it through
    shared-memory stages runs.  Two heads keep the oracle quick."""
    shape = synth.LayerShape(n_frames=60)
    H = 2
    q, k, v = (t[:, :H].contiguous() for t in synth.layer_qkv(shape, seed=3, dtype=torch.bfloat16, device="cuda"))
    L = K.Layout(1, H, shape.n_frames, shape.n_special, shape.hw)
    assert L.n_cand > 1200
    qbar, _, _ = K.pool_quant_q(q, L, quant=False)
    kbar, vbar, _, _, _, _ = K.pool_quant_kv(k, v, L, quant=False)
    af, ac = K.predict(qbar, kbar, L.n_cand)
    hs = synth.fisher_table(seed=1)[0, 0, :H]
    nts = K.hess_adjust(K.baseline(ac, 0.6).view(1, H, -1), K.scores_norm(hs), L.n_cand, min_clamp=2)
    M = synth.metric_from_weight(synth.out_proj_weight())[:H].contiguous()
    r = K.restore_swap(af, vbar, M.cuda(), nts.view(-1), L.n_cand, sink_blocks=L.sink_blocks, want_drop=True,
                       want_s=True)
    torch.cuda.synchronize()
    drop_o, s_o = oracle.restore_swap(af.cpu(), vbar.cpu().to(torch.bfloat16), M, nts.cpu().view(-1), L.n_cand)
    assert _eq(r["s"], s_o)
    assert torch.equal(r["drop"].cpu().bool(), drop_o)
    lists_o, counts_o = oracle.keep_lists(~drop_o, L.sink_blocks)
    assert torch.equal(r["counts"].cpu(), counts_o)
    K.check_status()


@pytest.mark.parametrize("shape,dtype", CASES)
def test_select_prob_and_top_m(shape, dtype):
    q, k, v = _inputs(shape, dtype)
    L = _layout(shape)
    qbar, _, _ = K.pool_quant_q(q.cuda(), L, quant=False)
    kbar, _, _, _, _, _ = K.pool_quant_kv(k.cuda(), v.cuda(), L, quant=False)
    _, ac = K.predict(qbar, kbar, L.n_cand, full=False)
    nts = K.baseline(ac, 0.5, 0.97).view(-1)
    r = K.select_prob(ac, nts, sink_blocks=L.sink_blocks, lead_blocks=1, want_keep=True)
    keep_o = oracle.top_m_mask(ac.cpu().view(-1, L.n_cand), nts.cpu())
    assert torch.equal(r["keep"].cpu().bool(), keep_o)
    lists_o, counts_o = oracle.keep_lists(keep_o, L.sink_blocks, lead_blocks=1)
    assert torch.equal(r["counts"].cpu(), counts_o)
    # standalone top-m (fused_topm API), smallest-first too, with ties
    x = torch.randint(0, 7, (300, 777), dtype=torch.int32).float()
    c = torch.randint(0, 800, (300,), dtype=torch.int32)
    for largest in (True, False):
        got = K.top_m_mask(x.cuda(), c.cuda(), largest=largest)
        assert torch.equal(got.cpu(), oracle.top_m_mask(x, c, largest=largest))


def test_map_to_lists():
    g = torch.Generator().manual_seed(5)
    m = torch.rand(123, 700, generator=g) < 0.3
    lists, counts = K.map_to_lists(m.cuda())
    torch.cuda.synchronize()
    assert torch.equal(counts.cpu(), m.sum(-1).int())
    for i in range(0, 123, 17):
        assert torch.equal(lists[i, : counts[i]].cpu(), m[i].nonzero().view(-1).int())
    back = K.lists_to_map(lists, counts, 700)
    assert torch.equal(back.cpu(), m)


def _attn_case(shape, dtype, sr, lead=0):
    q, k, v = _inputs(shape, dtype)
    L = _layout(shape)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    qbar, q8, qs = K.pool_quant_q(qd, L)
    kbar, vbar, k8, ks, v16, km = K.pool_quant_kv(kd, vd, L)
    _, ac = K.predict(qbar, kbar, L.n_cand, full=False)
    nts = K.baseline(ac, sr).view(-1)
    sel = K.select_prob(ac, nts, sink_blocks=L.sink_blocks, lead_blocks=lead)
    return L, q8, qs, k8, ks, v16, sel


@pytest.mark.parametrize("shape,dtype", CASES)
@pytest.mark.parametrize("sr", [0.0, 0.5, 0.9])
def test_sparse_attention_tolerance(shape, dtype, sr):
    L, q8, qs, k8, ks, v16, sel = _attn_case(shape, dtype, sr)
    out = K.sparse_attn(q8, qs, k8, ks, v16, sel["lists"], sel["counts"])
    torch.cuda.synchronize()
    K.check_status()
    g = torch.Generator().manual_seed(11)
    rows = L.B * L.H
    samples = [(int(torch.randint(0, rows, (1,), generator=g)), int(torch.randint(0, L.nq, (1,), generator=g)))
               for _ in range(24)] + [(0, L.nq - 1), (rows - 1, 0)]
    ref = oracle.sparse_attn_rows(q8.cpu(), qs.cpu(), k8.cpu(), ks.cpu(), v16.cpu().float(),
                                  sel["lists"].view(rows, L.nq, -1).cpu(), sel["counts"].view(rows, L.nq).cpu(),
                                  samples)
    errs = []
    for i, (r, qb) in enumerate(samples):
        n = min(128, L.Tp - qb * 128)
        got = out[r, qb * 128: qb * 128 + n].cpu()
        errs.append((got - ref[i, :n]).abs())
    e = torch.cat([x.reshape(-1) for x in errs])
    assert e.max().item() < 2e-2, e.max().item()
    assert e.mean().item() < 1e-3, e.mean().item()


def test_sparse_attention_full_layout_and_leading_sink():
    shape, dtype = SMALL, torch.bfloat16
    L, q8, qs, k8, ks, v16, sel = _attn_case(shape, dtype, 0.7, lead=1)
    full = torch.full((1, L.H, shape.t_total, 64), float("nan"), device="cuda")
    K.sparse_attn(q8, qs, k8, ks, v16, sel["lists"], sel["counts"], out=full, out_layout=L)
    plain = K.sparse_attn(q8, qs, k8, ks, v16, sel["lists"], sel["counts"])
    torch.cuda.synchronize()
    patch, special = synth.split_tokens(full.cpu(), shape)
    assert torch.equal(patch[0], plain.cpu())
    assert torch.isnan(special).all()  # special rows are left for the dense branch
    lists = sel["lists"].cpu()
    assert (lists[:, 0] == 0).all()  # leading sink block forced in


@pytest.mark.parametrize("density", [0.1, 0.9])
def test_sparse_attention_random_maps(density):
    """Arbitrary keep lists (uniformly random per row, no structure) on a
    plain (patch-only) layout with a ragged key tail: sampled rows within
    2e-2 max / 1e-3 mean abs of the fp64 oracle."""
    g = torch.Generator().manual_seed(int(density * 10))
    T = 3000  # 24 q-blocks, 47 key blocks, last one ragged
    q, k, v = (torch.randn(1, 4, T, 64, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    L = K.Layout.plain(q)
    _, q8, qs = K.pool_quant_q(q, L, pool=False)
    _, _, k8, ks, v16, _ = K.pool_quant_kv(k, v, L, pool=False)
    m = torch.rand(4 * L.nq, L.nkb, generator=g) < density
    m[:, 0] = True  # every row keeps at least one block
    lists, counts = K.map_to_lists(m.cuda())
    out = K.sparse_attn(q8, qs, k8, ks, v16, lists, counts)
    torch.cuda.synchronize()
    K.check_status()
    samples = [(h, b) for h in range(4) for b in (0, 7, L.nq - 1)]
    ref = oracle.sparse_attn_rows(q8.cpu(), qs.cpu(), k8.cpu(), ks.cpu(), v16.cpu().float(),
                                  lists.view(4, L.nq, -1).cpu(), counts.view(4, L.nq).cpu(), samples)
    errs = []
    for i, (h, b) in enumerate(samples):
        n = min(128, T - b * 128)
        errs.append((out[h, b * 128: b * 128 + n].cpu() - ref[i, :n]).abs().reshape(-1))
    e = torch.cat(errs)
    assert e.max().item() < 2e-2, e.max().item()
    assert e.mean().item() < 1e-3, e.mean().item()


@pytest.mark.parametrize("chunk", [8, 30])
def test_split_rows_match_oracle_and_unsplit(chunk):
    """ress_sparse_attn_split: rows longer than `chunk` key blocks run as two
    pieces of their list (the kernel's limit) on separate CTAs, merged by the
    piece that finishes last.  Random keep lists with a ragged key tail (47
    key blocks, ~33 kept per row and one in five rows a single block: at
    chunk 8 every longer row splits, at chunk 30 about four in five):
    sampled rows within 2e-2 max / 1e-3 mean abs of the fp64 oracle, every
    row within 2e-3 of the one-CTA-per-row launch, and a second call on the
    same scratch (the per-row counters must be left at zero) gives the same
    bits as the first."""
    g = torch.Generator().manual_seed(chunk)
    T = 3000
    q, k, v = (torch.randn(1, 4, T, 64, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    L = K.Layout.plain(q)
    _, q8, qs = K.pool_quant_q(q, L, pool=False)
    _, _, k8, ks, v16, _ = K.pool_quant_kv(k, v, L, pool=False)
    m = torch.rand(4 * L.nq, L.nkb, generator=g) < 0.7
    m[:, 0] = True
    m[::5, 1:] = False  # some one-block rows, never split
    lists, counts = K.map_to_lists(m.cuda())
    plain = K.sparse_attn(q8, qs, k8, ks, v16, lists, counts, split=False)
    a = K.sparse_attn(q8, qs, k8, ks, v16, lists, counts, split=chunk)
    b = K.sparse_attn(q8, qs, k8, ks, v16, lists, counts, split=chunk)
    torch.cuda.synchronize()
    K.check_status()
    assert int((counts > chunk).sum()) > 10
    assert torch.equal(a, b)
    assert (a - plain).abs().max().item() < 2e-3
    samples = [(h, bq) for h in range(4) for bq in (0, 7, L.nq - 1)]
    ref = oracle.sparse_attn_rows(q8.cpu(), qs.cpu(), k8.cpu(), ks.cpu(), v16.cpu().float(),
                                  lists.view(4, L.nq, -1).cpu(), counts.view(4, L.nq).cpu(), samples)
    errs = []
    for i, (h, bq) in enumerate(samples):
        n = min(128, T - bq * 128)
        errs.append((a[h, bq * 128: bq * 128 + n].cpu() - ref[i, :n]).abs().reshape(-1))
    e = torch.cat(errs)
    assert e.max().item() < 2e-2, e.max().item()
    assert e.mean().item() < 1e-3, e.mean().item()


def test_scale_division_exhaustive():
    """The quantisers divide by RN(amax/127) with a reciprocal and one fma
    correction; over every fp16 amax and every fp16 |x| <= amax it must give
    the IEEE quotient."""
    import ctypes

    from ress_b200 import _lib

    n = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert _lib.load().ress_check_scale_division(ctypes.c_void_p(n.data_ptr()), stream) == 0
    torch.cuda.synchronize()
    assert int(n.item()) == 0


def test_scheduled_attention_equals_plain_order():
    """Rows launched in descending kept-block count give the same bits as the
    plain row order (each row's result does not depend on its CTA)."""
    L, q8, qs, k8, ks, v16, sel = _attn_case(SMALL, torch.bfloat16, 0.5)
    a = K.sparse_attn(q8, qs, k8, ks, v16, sel["lists"], sel["counts"], schedule=False)
    b = K.sparse_attn(q8, qs, k8, ks, v16, sel["lists"], sel["counts"], schedule=True)
    torch.cuda.synchronize()
    K.check_status()
    assert torch.equal(a, b)
