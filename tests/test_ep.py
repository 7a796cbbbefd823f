"""Expert parallelism, host side, on the CPU: the dispatch plan and the
exchange over torch.distributed with gloo ranks.

The three device steps are replaced by a fake with the same contract
(route -> top-k, weights, a quantized row; expert products of (row, expert)
pairs; combine in top-k order).  Sharding must leave the numbers untouched,
so the sharded result is compared with the fake run in one process, bit for
bit.  The real kernels are compared the same way in test_gpu_ep.py.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from motoria_b200.ep import ExpertParallelMoE, pack_records, peer_routes, plan_dispatch

D, E, K, XS = 16, 8, 3, 4


class FakeOps:
    """route: top-K of x @ R (distinct experts), softmax weights, an int8 row
    and per-row scales; experts: y = xq * (expert + 1) + dx[0]; combine:
    x += w_j y_j in j order.  Exact float arithmetic in a fixed order."""

    dim, K, E = D, K, E

    def __init__(self):
        g = torch.Generator().manual_seed(7)
        self.R = torch.randn((D, E), generator=g)

    def route(self, x):
        s = x @ self.R
        w, idx = torch.topk(s, K, dim=1)
        w = torch.softmax(w, dim=1)
        xq = torch.clamp(torch.round(x * 20), -127, 127).to(torch.int8)
        dx = torch.stack([x.abs().amax(1), x.sum(1), x[:, 0], x[:, 1]], 1)
        return idx.to(torch.int32), w, xq, dx

    plan = staticmethod(plan_dispatch)
    pack = staticmethod(pack_records)

    def experts(self, xq, dx, pair_row, pair_expert):
        r = pair_row.long()
        return xq[r].float() * (pair_expert.float() + 1)[:, None] + dx[r, :1]

    def combine(self, x, w, y, y_pos=None):
        T = x.shape[0]
        if y_pos is not None:
            y = y[y_pos.long()]
        yy = y.view(T, K, D)
        for j in range(K):
            x += w[:, j:j + 1] * yy[:, j]


def reference(ops, x):
    """The unsharded block with the same fake steps."""
    idx, w, xq, dx = ops.route(x)
    T = x.shape[0]
    rows = torch.arange(T * K, dtype=torch.int32) // K
    y = ops.experts(xq, dx, rows, idx.reshape(-1))
    ops.combine(x, w, y)
    return x


def tokens(rank, T):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn((T, D), generator=g)


def test_plan_sends_each_row_once_per_destination():
    ops = FakeOps()
    x = tokens(0, 50)
    idx = ops.route(x)[0]
    for world, placement in ((1, "contiguous"), (2, "contiguous"), (4, "contiguous"),
                             (8, "contiguous"), (4, "strided")):
        per = E // world
        plan = plan_dispatch(idx, per, world, placement)
        dest = idx.long() // per if placement == "contiguous" else idx.long() % world
        assert int(plan.pairs_per_dest.sum()) == idx.numel()
        pair_order = torch.argsort(plan.y_pos.long())
        assert torch.equal(torch.sort(plan.y_pos.long()).values, torch.arange(idx.numel()))
        r0 = p0 = 0
        for g in range(world):
            rows = plan.send_rows[r0:r0 + int(plan.rows_per_dest[g])].long()
            want = torch.nonzero((dest == g).any(1)).flatten()
            assert torch.equal(rows, want)              # each token once, ascending
            pairs = pair_order[p0:p0 + int(plan.pairs_per_dest[g])]
            assert torch.equal(pairs, torch.sort(pairs).values)
            meta = plan.pair_meta[p0:p0 + int(plan.pairs_per_dest[g])]
            assert torch.equal(rows[meta[:, 0].long()], pairs // K)   # record -> its row
            assert torch.equal(meta[:, 1], idx.reshape(-1)[pairs])
            assert bool((dest.reshape(-1)[pairs] == g).all())
            r0 += int(plan.rows_per_dest[g])
            p0 += int(plan.pairs_per_dest[g])


@pytest.mark.parametrize("world,placement", [(2, "contiguous"), (4, "strided"), (8, "contiguous")])
def test_peer_routes_land_where_the_origin_looks(world, placement):
    """The peer exchange: rank r stores the y row of each pair it received at
    an address from peer_routes; decoded, that must be the origin rank and
    the place its y_pos gives the pair (its send order)."""
    ops = FakeOps()
    T = (23, 0, 9, 31, 4, 17, 2, 11)[:world]
    plans = [plan_dispatch(ops.route(tokens(r, T[r]))[0], E // world, world, placement)
             for r in range(world)]
    counts = torch.stack([p.counts for p in plans])            # [src, dst, (rows, pairs)]
    BIG = 1 << 20                                              # rank s's rows at s * BIG
    for me in range(world):
        src_end, dst = peer_routes(counts, me, [s * BIG for s in range(world)], 1)
        start = 0
        for s in range(world):
            assert src_end[s] - start == int(counts[s, me, 1])
            order = torch.argsort(plans[s].y_pos.long())           # s's pairs in send order
            first = int(counts[s, :me, 1].sum())                   # s's pairs to lower ranks
            for i in range(src_end[s] - start):
                addr = dst[s] + i
                assert addr // BIG == s                            # stored at the origin
                pair = int(order[first + i])                       # the i-th pair s sent to me
                assert int(plans[s].y_pos[pair]) == addr % BIG     # where s's combine reads it
            start = src_end[s]


def test_peer_exchange_is_checked_at_construction():
    with pytest.raises(ValueError, match="exchange"):
        ExpertParallelMoE(FakeOps(), exchange="nvshmem")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, placement, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ops = FakeOps()
        ep = ExpertParallelMoE(ops, placement=placement)
        x = tokens(rank, T[rank])
        want = reference(ops, x.clone())
        got = ep.forward(x.clone())
        out[rank] = bool(torch.equal(got.view(torch.int32), want.view(torch.int32)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T,placement", [(2, (37, 21), "contiguous"),
                                               (4, (9, 0, 30, 5), "contiguous"),
                                               (4, (20, 11, 0, 7), "strided")])
def test_gloo_ranks_match_the_unsharded_block(world, T, placement):
    ctx = torch.multiprocessing.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, placement, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert all(out[r] for r in range(world)), dict(out)


def test_fake_reference_uses_every_expert():
    # sanity of the fixture: the routing spreads over all experts
    idx = FakeOps().route(tokens(0, 64))[0]
    assert len(np.unique(idx.numpy())) == E
