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
