"""Expert parallelism for the MoE block: experts sharded over the GPUs of one
node, tokens exchanged with NCCL all-to-all.

The reference runs the block on one device (src/model/forward.c:167-197); the
sharded form here computes exactly the same numbers.  moe() is route ->
expert products -> combine, and only the middle step needs an expert's
weights, so:

1. every rank routes its own tokens (miag_route_async: top-k, weights, and
   the Q8_0 form of the normalised rows that the expert products read);
2. each token row goes once to every rank that holds one of its experts
   (contiguous placement: rank g holds experts [g*E/G, (g+1)*E/G)), with one
   (row, expert) record per pair, over all_to_all_single;
3. each rank runs the expert products of the pairs it received
   (miag_experts_async) -- the same kernels on the same bytes;
4. the results (one f32 row per pair) go back the reverse way, and
5. the origin combines them in top-k order (miag_combine_async).

Because the combine keeps the reference's order of adds (x + w_0 y_0 + w_1 y_1
+ ...), results come back per pair rather than as per-rank partial sums;
a partial sum would reassociate the adds.  The outputs therefore equal the
single-GPU block bit for bit.

The plan (who sends what where) and the send records are built by two
kernels of the library (miag_ep_plan_async, miag_ep_pack_async), so the
host reads only the per-rank counts that the collectives' split sizes need;
plan_dispatch and pack_records state the same in torch operations for the
CPU tests.  The collectives are torch.distributed's (NCCL on GPUs, gloo in
the CPU tests).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class DispatchPlan:
    """What one rank sends, for G ranks and its T tokens of K pairs each.
    Order, the same on every rank: rows grouped by destination, tokens
    ascending within a destination; pairs grouped by destination, pair id
    t*K + j ascending within a destination."""

    counts: torch.Tensor     # [G, 2] int64: rows and pairs to each destination
    send_rows: torch.Tensor  # [T*G] int32: the token of each row to send; the first
                             #   counts[:, 0].sum() are used
    pair_meta: torch.Tensor  # [T*K, 2] int32: (row within the destination's block from
                             #   this rank, expert), in pair order
    y_pos: torch.Tensor      # [T*K] int32: the place of pair t*K + j in pair order

    @property
    def rows_per_dest(self) -> torch.Tensor:
        return self.counts[:, 0]

    @property
    def pairs_per_dest(self) -> torch.Tensor:
        return self.counts[:, 1]


def owner(expert: torch.Tensor, experts_per_rank: int, world: int, placement: str) -> torch.Tensor:
    """Rank holding each expert: contiguous blocks of E/G experts (the
    specified placement), or strided, expert e on rank e mod G (spreads a
    skewed load such as config 3's Zipf bias over the ranks)."""
    if placement == "strided":
        return expert % world
    return expert // experts_per_rank


def plan_dispatch(idx: torch.Tensor, experts_per_rank: int, world: int,
                  placement: str = "contiguous") -> DispatchPlan:
    """idx [T][K] int32 top-k experts -> the rows and pair records to send,
    in torch operations: the statement of the plan that EngineOps.plan
    computes in one kernel (miag_ep_plan_async), used by the CPU tests.

    A row goes to a destination once however many of the token's experts
    live there."""
    T, K = idx.shape
    dev = idx.device
    dest = owner(idx.long(), experts_per_rank, world, placement)      # [T, K]
    hit = torch.zeros((T, world), dtype=torch.bool, device=dev)
    hit.scatter_(1, dest, True)
    # (g, t) keys of the hits first, ascending; misses after them
    key = torch.arange(world, device=dev)[:, None] * T + torch.arange(T, device=dev)[None, :]
    key = torch.where(hit.t(), key, torch.full_like(key, world * T))
    send_rows = (torch.sort(key.reshape(-1)).values % max(T, 1)).to(torch.int32)
    row_in_block = hit.long().cumsum(0) - 1                          # [T, G] index of t in g's block
    pair_ids = torch.arange(T * K, device=dev)
    pair_order = torch.argsort(dest.reshape(-1) * (T * K) + pair_ids)  # g-major, then pair order
    d_sorted = dest.reshape(-1)[pair_order]
    t_sorted = pair_order // K
    meta = torch.stack([row_in_block[t_sorted, d_sorted], idx.reshape(-1)[pair_order].long()], 1)
    y_pos = torch.empty(T * K, dtype=torch.int32, device=dev)
    y_pos[pair_order] = torch.arange(T * K, dtype=torch.int32, device=dev)
    counts = torch.stack([hit.sum(0), torch.bincount(d_sorted, minlength=world)], 1)
    return DispatchPlan(counts.to(torch.int64), send_rows, meta.to(torch.int32), y_pos)


def pack_records(xq: torch.Tensor, dx: torch.Tensor, plan: DispatchPlan,
                 all_counts: torch.Tensor, me: int, n_rows: int, n_pairs: int):
    """The send buffers of rank `me`, in torch operations (the statement of
    miag_ep_pack_async): one record per row to send (its int8 values, then
    its f32 scales as bytes), and the pair records with each row renumbered
    in the receiver's buffer, where the rows of lower ranks come first.
    all_counts [G][G][2]: every rank's plan.counts, in rank order."""
    rows = plan.send_rows[:n_rows].long()
    rec = torch.cat([xq[rows].view(torch.uint8), dx[rows].view(torch.uint8)], 1)
    G = all_counts.shape[0]
    dest = torch.repeat_interleave(torch.arange(G, device=xq.device), all_counts[me, :, 1])
    row_start = (all_counts[:, :, 0].cumsum(0) - all_counts[:, :, 0])[me]
    meta = plan.pair_meta[:n_pairs].clone()
    meta[:, 0] += row_start[dest].to(torch.int32)
    return rec, meta


def peer_routes(counts: torch.Tensor, me: int, peer_rows: list[int], row_bytes: int):
    """Where the y rows of the pairs rank `me` received go, for the peer
    exchange.  counts [G][G][2]: every rank's (rows, pairs) per destination,
    all-gathered.  The pairs arrive grouped by source rank; those from rank s
    go to s's exchange buffer (rows at address peer_rows[s]), after the pairs
    s sends to lower ranks: the place s's y_pos gives them.  Returns
    (src_end, dst): the end of each source's pairs in the received list, and
    the address of each source's first row."""
    G = counts.shape[0]
    src_end = [int(v) for v in counts[:, me, 1].cumsum(0)]
    dst = [peer_rows[s] + int(counts[s, :me, 1].sum()) * row_bytes for s in range(G)]
    return src_end, dst


class EngineOps:
    """The three device steps of a MoEEngine on torch tensors, enqueued on the
    tensors' device's current stream."""

    def __init__(self, engine, layer: int = 0):
        self.eng, self.layer = engine, layer
        sh = engine.shape
        self.dim, self.K, self.E = sh.dim, sh.n_active, sh.n_experts
        self.xs = engine.dx_stride()

    def _stream(self, t: torch.Tensor) -> int:
        # torch's default stream has handle 0, which the library reads as
        # "the context's own stream" (a non-blocking one, not ordered with
        # torch's work): name the legacy default stream explicitly instead
        # (cudaStreamLegacy == 1).
        return torch.cuda.current_stream(t.device).cuda_stream or 1

    def route(self, x: torch.Tensor):
        T, dev = x.shape[0], x.device
        idx = torch.empty((T, self.K), dtype=torch.int32, device=dev)
        w = torch.empty((T, self.K), dtype=torch.float32, device=dev)
        xq = torch.empty((T, self.dim), dtype=torch.int8, device=dev)
        dx = torch.empty((T, self.xs), dtype=torch.float32, device=dev)
        self.eng.route_device(x.data_ptr(), T, idx.data_ptr(), w.data_ptr(), xq.data_ptr(),
                              dx.data_ptr(), layer=self.layer, stream=self._stream(x))
        return idx, w, xq, dx

    def plan(self, idx: torch.Tensor, experts_per_rank: int, world: int,
             placement: str = "contiguous") -> DispatchPlan:
        """plan_dispatch in one kernel (miag_ep_plan_async)."""
        T, dev = idx.shape[0], idx.device
        plan = DispatchPlan(torch.empty((world, 2), dtype=torch.int64, device=dev),
                            torch.empty(T * world, dtype=torch.int32, device=dev),
                            torch.empty((T * self.K, 2), dtype=torch.int32, device=dev),
                            torch.empty(T * self.K, dtype=torch.int32, device=dev))
        self.eng.ep_plan_device(idx.data_ptr(), T, world, experts_per_rank,
                                placement == "strided", plan.counts.data_ptr(),
                                plan.send_rows.data_ptr(), plan.pair_meta.data_ptr(),
                                plan.y_pos.data_ptr(), stream=self._stream(idx))
        return plan

    def pack(self, xq: torch.Tensor, dx: torch.Tensor, plan: DispatchPlan,
             all_counts: torch.Tensor, me: int, n_rows: int, n_pairs: int):
        """pack_records in one kernel (miag_ep_pack_async)."""
        dev = xq.device
        rec = torch.empty((n_rows, xq.shape[1] + 4 * dx.shape[1]), dtype=torch.uint8, device=dev)
        meta = torch.empty((n_pairs, 2), dtype=torch.int32, device=dev)
        counts = all_counts.contiguous()
        self.eng.ep_pack_device(xq.data_ptr(), dx.data_ptr(), plan.send_rows.data_ptr(), n_rows,
                                plan.pair_meta.data_ptr(), n_pairs, counts.data_ptr(), me,
                                counts.shape[0], rec.data_ptr(), meta.data_ptr(),
                                stream=self._stream(xq))
        return rec, meta

    def experts(self, xq: torch.Tensor, dx: torch.Tensor, pair_row: torch.Tensor,
                pair_expert: torch.Tensor) -> torch.Tensor:
        P = pair_row.numel()
        y = torch.empty((P, self.dim), dtype=torch.float32, device=xq.device)
        self.eng.experts_device(xq.data_ptr(), dx.data_ptr(), xq.shape[0], pair_row.data_ptr(),
                                pair_expert.data_ptr(), P, y.data_ptr(), layer=self.layer,
                                stream=self._stream(xq))
        return y

    def experts_to_ranks(self, xq: torch.Tensor, dx: torch.Tensor, pair_row: torch.Tensor,
                         pair_expert: torch.Tensor, rank: int, src_end, dst, flags,
                         seq: int) -> None:
        """Expert products whose y rows are stored at the pairs' origin ranks
        (peer memory), then flagged there (miag_experts_to_ranks_async)."""
        P = pair_row.numel()
        self.eng.experts_to_ranks_device(xq.data_ptr() if P else 0, dx.data_ptr() if P else 0,
                                         xq.shape[0], pair_row.data_ptr() if P else 0,
                                         pair_expert.data_ptr() if P else 0, P, rank, src_end,
                                         dst, flags, seq, layer=self.layer,
                                         stream=self._stream(xq))

    def wait(self, flags: int, world: int, seq: int, like: torch.Tensor) -> None:
        """Enqueues the wait for every rank's y rows to have landed here."""
        self.eng.ep_wait_device(flags, world, seq, stream=self._stream(like))

    def combine_rows(self, x: torch.Tensor, w: torch.Tensor, y: int, y_pos: torch.Tensor) -> None:
        """combine() over y rows at a device address (the exchange buffer)."""
        self.eng.combine_device(x.data_ptr(), x.shape[0], w.data_ptr(), y, y_pos.data_ptr(),
                                stream=self._stream(x))

    def combine(self, x: torch.Tensor, w: torch.Tensor, y: torch.Tensor,
                y_pos: torch.Tensor | None = None) -> None:
        """x[t] += sum_j w[t][j] * y[row(t*K + j)]; row(p) = y_pos[p], or p."""
        self.eng.combine_device(x.data_ptr(), x.shape[0], w.data_ptr(), y.data_ptr(),
                                0 if y_pos is None else y_pos.data_ptr(), stream=self._stream(x))


def _a2a(dist, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group=None):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
    return out


class _PeerExchange:
    """The peer exchange of one engine: its buffer (y rows and one flag per
    rank, owned by the library context), the peers' buffers mapped here, and
    the step counter the flags are compared with.  All of it belongs to the
    context, so every ExpertParallelMoE over the same engine (one per layer,
    say) shares this one object: a second counter starting again at 1 would
    find the flags already at the first one's count and pass its wait before
    the rows land, and a second set of mappings would be freed under the
    first."""

    def __init__(self, eng, dist, group, world: int, rank: int):
        self.eng, self.dist, self.group, self.world, self.rank = eng, dist, group, world, rank
        self.cap, self.seq = 0, 0
        # every rank on a GPU of its own: the flag waits of two ranks must
        # never share one GPU
        dev = torch.cuda.current_device()
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        ids = [None] * world
        dist.all_gather_object(ids, uuid, group=group)
        if len(set(ids)) != world:
            raise ValueError("exchange='peer' needs one GPU per rank")

    @classmethod
    def of(cls, eng, dist, group, world: int, rank: int) -> "_PeerExchange":
        px = getattr(eng, "_peer_exchange", None)
        if px is None:
            px = cls(eng, dist, group, world, rank)
            eng._peer_exchange = px
        elif (px.world, px.rank) != (world, rank) or px.group is not group:
            raise ValueError("this engine's peer exchange belongs to another process group")
        return px

    def next_seq(self) -> int:
        self.seq += 1
        return self.seq

    def ensure(self, rows: int) -> None:
        """Buffers of at least `rows` y rows on every rank, mapped by every
        peer.  Every rank calls this with the same `rows` (derived from the
        all-gathered counts), so all grow together."""
        rows = max(rows, 1)  # buffers exist even when no rank has tokens yet
        if rows <= self.cap:
            return
        dist, eng, G, me = self.dist, self.eng, self.world, self.rank
        cap = max(rows, 2 * self.cap)
        torch.cuda.synchronize()
        if self.cap:
            eng.ep_close_peers()
        dist.barrier(group=self.group)  # nobody maps or writes the old buffers now
        y, flags, handle = eng.ep_buffer(cap)
        handles = [None] * G
        dist.all_gather_object(handles, handle, group=self.group)
        maps = [(y, flags) if r == me else eng.ep_open_peer(handles[r]) for r in range(G)]
        self.peer_y = [m[0] for m in maps]
        self.peer_flags = [m[1] for m in maps]
        self.own_y, self.own_flags = y, flags
        self.cap = cap
        dist.barrier(group=self.group)


class ExpertParallelMoE:
    """The MoE block over the ranks of a process group, one GPU each.

    `ops` runs the three device steps (EngineOps over this rank's MoEEngine,
    whose store must hold at least this rank's experts).  forward() updates
    the residual x [T][dim] (f32) in place, like miag_moe.

    exchange: how the y rows come back.  "collective": all_to_all_single.
    "peer": the down launch stores each row straight into the origin rank's
    exchange buffer over NVLink (CUDA IPC mappings), so the return overlaps
    the expert products, and a bounded device-side wait on per-rank flags
    orders the combine after it.  Peer needs one GPU per rank on one node.
    """

    def __init__(self, ops, group=None, placement: str = "contiguous",
                 exchange: str = "collective"):
        import torch.distributed as dist

        if placement not in ("contiguous", "strided"):
            raise ValueError(f"unknown placement {placement!r}")
        if exchange not in ("collective", "peer"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.dist = dist
        self.ops = ops
        self.group = group
        self.placement = placement
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if ops.E % self.world:
            raise ValueError(f"{ops.E} experts do not split evenly over {self.world} ranks")
        self.per_rank = ops.E // self.world
        self.exchange = exchange
        self._px = None
        if exchange == "peer":
            self._px = _PeerExchange.of(ops.eng, dist, group, self.world, self.rank)

    def experts_of(self, rank: int) -> list[int]:
        """The experts this placement puts on `rank` (its store must hold them)."""
        if self.placement == "strided":
            return list(range(rank, self.ops.E, self.world))
        return list(range(rank * self.per_rank, (rank + 1) * self.per_rank))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dist, ops, G, me = self.dist, self.ops, self.world, self.rank
        T, K, dev = x.shape[0], ops.K, x.device
        idx, w, xq, dx = ops.route(x)
        plan = ops.plan(idx, self.per_rank, G, self.placement)

        # Every rank's (rows, pairs) per destination: one all_gather, one
        # host synchronisation for the collectives' split sizes.
        M = torch.empty((G, G, 2), dtype=torch.int64, device=dev)      # [src, dst, (rows, pairs)]
        dist.all_gather_into_tensor(M.view(G * G, 2), plan.counts, group=self.group)
        Mh = M.cpu()
        rows_out, pairs_out = Mh[me, :, 0].tolist(), Mh[me, :, 1].tolist()
        rows_in, pairs_in = Mh[:, me, 0].tolist(), Mh[:, me, 1].tolist()
        R_out, R_in, P_in = sum(rows_out), sum(rows_in), sum(pairs_in)

        # dispatch: each row as one record (int8 values, then the f32 block
        # scales), and the pair records with rows numbered in the receiver
        rec, meta = ops.pack(xq, dx, plan, M, me, R_out, T * K)
        rec_w = rec.shape[1]
        rec_in = torch.empty((R_in, rec_w), dtype=torch.uint8, device=dev)
        meta_in = torch.empty((P_in, 2), dtype=torch.int32, device=dev)
        _a2a(dist, rec_in, rec, rows_in, rows_out, self.group)
        _a2a(dist, meta_in, meta, pairs_in, pairs_out, self.group)
        xq_in = rec_in[:, :xq.shape[1]].contiguous().view(torch.int8)
        dx_in = rec_in[:, xq.shape[1]:].contiguous().view(torch.float32)
        pair_row = meta_in[:, 0].contiguous()
        pair_expert = meta_in[:, 1].contiguous()
        self.last_received = (R_in, P_in, pair_expert)
        if self.exchange == "peer":
            # rows from source s go to rank s's buffer, after the rows that
            # s sends to lower ranks (its send order, the one y_pos indexes)
            px = self._px
            px.ensure(int(Mh[:, :, 1].sum(1).max()))
            src_end, dst = peer_routes(Mh, me, px.peer_y, ops.dim * 4)
            seq = px.next_seq()
            ops.experts_to_ranks(xq_in, dx_in, pair_row, pair_expert, me, src_end, dst,
                                 px.peer_flags, seq)
            ops.wait(px.own_flags, G, seq, x)
            ops.combine_rows(x, w, px.own_y, plan.y_pos)
            return x
        y_in = ops.experts(xq_in, dx_in, pair_row, pair_expert)

        # results back in this rank's send order; the combine finds pair p at
        # row y_pos[p] of it
        y_back = torch.empty((T * K, y_in.shape[1]), dtype=y_in.dtype, device=dev)
        _a2a(dist, y_back, y_in, pairs_out, pairs_in, self.group)
        ops.combine(x, w, y_back, plan.y_pos)
        return x


def simulate(ops, x: torch.Tensor, world: int, placement: str = "contiguous") -> torch.Tensor:
    """One process plays `world` ranks: the same plan, the exchange as local
    copies, each virtual rank's received pairs in an expert call of their
    own.  For tests without several GPUs.  x [G][T][dim]: each virtual
    rank's tokens; updated in place."""
    G, T, K = x.shape[0], x.shape[1], ops.K
    per = ops.E // world
    routed = []
    for r in range(G):
        idx, w, xq, dx = ops.route(x[r])
        routed.append((w, xq, dx, ops.plan(idx, per, G, placement)))
    y_back = [None] * G
    parts = [[] for _ in range(G)]
    for g in range(G):  # destination g receives from every source, in source order
        xq_in, dx_in, rows, exps, srcs, base = [], [], [], [], [], 0
        for s in range(G):
            w, xq, dx, plan = routed[s]
            r0 = int(plan.rows_per_dest[:g].sum()); r1 = r0 + int(plan.rows_per_dest[g])
            p0 = int(plan.pairs_per_dest[:g].sum()); p1 = p0 + int(plan.pairs_per_dest[g])
            sel = plan.send_rows[r0:r1].long()
            xq_in.append(xq[sel]); dx_in.append(dx[sel])
            rows.append(plan.pair_meta[p0:p1, 0].long() + base)
            exps.append(plan.pair_meta[p0:p1, 1])
            srcs.append((s, p1 - p0))
            base += r1 - r0
        y_g = ops.experts(torch.cat(xq_in).contiguous(), torch.cat(dx_in).contiguous(),
                          torch.cat(rows).to(torch.int32).contiguous(), torch.cat(exps).contiguous())
        off = 0
        for s, n in srcs:
            parts[s].append(y_g[off:off + n])
            off += n
    for r in range(G):
        w, xq, dx, plan = routed[r]
        y_back[r] = torch.cat(parts[r])  # destination-major: the plan's pair order
        ops.combine(x[r], w, y_back[r], plan.y_pos)
    return x
