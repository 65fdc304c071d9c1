"""Head-split HeSS exchange on two gloo ranks (CPU): each rank gathers the
baselines of all heads, runs the re-allocation over all heads and keeps its
own slice; the slices must equal the single-process result."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from ress_b200 import shard


def _base():
    g = torch.Generator().manual_seed(4)
    return torch.randint(2, 60, (1, 16, 23), generator=g, dtype=torch.int32)


def _scores():
    g = torch.Generator().manual_seed(5)
    return torch.exp(torch.randn(16, generator=g)) * torch.linspace(1, 20, 16)


def _worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        h0, hl = shard.head_range(16, world, rank)
        local = _base()[:, h0:h0 + hl].contiguous()
        sh = shard.make_head_shard(16, world, rank)
        full = sh.gather(local)
        nts = oracle.hess_adjust(full, oracle.scores_norm(_scores()), 60, min_clamp=2)
        out_q.put((rank, full.clone(), nts[:, sh.h0:sh.h0 + hl].clone()))
    finally:
        dist.destroy_process_group()


def test_two_rank_hess_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (f, n)) for r, f, n in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = oracle.hess_adjust(_base(), oracle.scores_norm(_scores()), 60, min_clamp=2)
    for r in range(2):
        assert torch.equal(res[r][0], _base())
        assert torch.equal(res[r][1], ref[:, 8 * r:8 * r + 8])


# ----------------------------------------------------------------- views
_VIEW = dict(frames=6, special=5, hw=100)  # 600 patch tokens: q-blocks straddle every shard boundary


def _view_tensors():
    g = torch.Generator().manual_seed(9)
    T = _VIEW["frames"] * (_VIEW["special"] + _VIEW["hw"])
    return [torch.randn(1, 4, T, 64, generator=g) for _ in range(3)]


def _view_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        geom = shard.ViewGeom(world=world, rank=rank, **_VIEW)
        q, k, v = _view_tensors()
        per = geom.frames_local * (geom.special + geom.hw)
        sl = slice(rank * per, (rank + 1) * per)
        qp, kf, vf = shard.view_assemble(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(),
                                         v[:, :, sl].contiguous(), geom, shard.make_view_gather(world))
        out_q.put((rank, qp.numpy().copy(), kf.numpy().copy(), vf.numpy().copy()))  # by value
    finally:
        dist.destroy_process_group()


def test_view_exchange_two_and_three_ranks():
    """Each rank ends with every key and value, and with exactly the patch
    queries of the global q-blocks that hold its tokens (halo from the
    neighbours included)."""
    ctx = mp.get_context("spawn")
    q, k, v = _view_tensors()
    qpatch = shard.patch_tokens(q, _VIEW["special"], _VIEW["hw"])
    for world in (2, 3):
        oq = ctx.Queue()
        port = 30500 + os.getpid() % 1000 + world
        procs = [ctx.Process(target=_view_worker, args=(r, world, port, oq)) for r in range(world)]
        for p in procs:
            p.start()
        res = {r: tuple(torch.from_numpy(x) for x in (a, b, c)) for r, a, b, c in (oq.get(timeout=120) for _ in procs)}
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
        for r in range(world):
            geom = shard.ViewGeom(world=world, rank=r, **_VIEW)
            qp, kf, vf = res[r]
            assert torch.equal(kf, k) and torch.equal(vf, v)
            assert torch.equal(qp, qpatch[:, :, geom.b0 * 128: min(geom.b1 * 128, geom.Tp)])
            assert (geom.lo > 0) == (r > 0) or geom.p0 % 128 == 0


def test_view_geometry_config4():
    """200 views over 8 ranks: q-block ranges tile the global grid with one
    shared (straddling) block between neighbours."""
    gs = [shard.ViewGeom(frames=200, special=5, hw=1369, world=8, rank=r) for r in range(8)]
    assert gs[0].b0 == 0 and gs[-1].b1 == -(-200 * 1369 // 128)
    for a, b in zip(gs, gs[1:]):
        assert a.p1 == b.p0
        assert b.b0 == a.b1 - 1 if a.p1 % 128 else b.b0 == a.b1
        assert a.hi + b.lo == (128 if a.p1 % 128 else 0)


def _bal_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = shard.make_head_shard(16, world, rank, scores=_scores(), cap=2.0)
        local = _base().index_select(1, torch.as_tensor(sh.heads)).contiguous()
        full = sh.gather(local)
        nts = oracle.hess_adjust(full, oracle.scores_norm(_scores()), 60, min_clamp=2)
        out_q.put((rank, full.numpy().copy(), sh.select(nts, len(sh.heads)).numpy().copy(), list(sh.heads)))
    finally:
        dist.destroy_process_group()


def test_balanced_head_exchange_four_ranks():
    """Balanced (non-contiguous) head sets: the gathered baselines come back in
    global head order and each rank keeps its own heads' budgets."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 31500 + os.getpid() % 1000
    procs = [ctx.Process(target=_bal_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = {r: (f, n, h) for r, f, n, h in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = oracle.hess_adjust(_base(), oracle.scores_norm(_scores()), 60, min_clamp=2)
    seen = []
    for r in range(4):
        full, nts, heads = res[r]
        assert torch.equal(torch.from_numpy(full), _base())
        assert torch.equal(torch.from_numpy(nts), ref[:, heads])
        seen += heads
    assert sorted(seen) == list(range(16))


def _uneven_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = shard.make_head_shard(16, world, rank, scores=_scores(), cap=2.0, equal_size=False)
        local = _base().index_select(1, torch.as_tensor(sh.heads)).contiguous()
        full = sh.gather(local)
        nts = oracle.hess_adjust(full, oracle.scores_norm(_scores()), 60, min_clamp=2)
        # a batch of two layers: the gather keeps each batch entry's heads apart
        base2 = torch.cat([_base(), _base().flip(2) + 100], 0)
        full2 = sh.gather(base2.index_select(1, torch.as_tensor(sh.heads)).contiguous())
        assert torch.equal(full2, base2)
        out_q.put((rank, full.numpy().copy(), sh.select(nts, len(sh.heads)).numpy().copy(), list(sh.heads)))
    finally:
        dist.destroy_process_group()


def test_uneven_head_groups_three_ranks():
    """Ranks holding different numbers of heads: the padded all-gather returns
    every head's baselines in global order (also for a batch of two) and each
    rank keeps its own."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 32500 + os.getpid() % 1000
    procs = [ctx.Process(target=_uneven_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = {r: (f, n, h) for r, f, n, h in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = oracle.hess_adjust(_base(), oracle.scores_norm(_scores()), 60, min_clamp=2)
    seen, sizes = [], []
    for r in range(3):
        full, nts, heads = res[r]
        assert torch.equal(torch.from_numpy(full), _base())
        assert torch.equal(torch.from_numpy(nts), ref[:, heads])
        seen += heads
        sizes.append(len(heads))
    assert sorted(seen) == list(range(16))
    assert len(set(sizes)) > 1  # 16 heads over 3 ranks cannot be even


def test_budget_shares_cap():
    s = torch.tensor([10.0] + [1.0] * 7)
    w = shard.budget_shares(s, cap=2.0)
    assert abs(sum(w) - 8.0) < 1e-9 and abs(w[0] - 2.0) < 1e-9
    assert all(abs(x - 6.0 / 7.0) < 1e-9 for x in w[1:])
