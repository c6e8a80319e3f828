"""Row-sharded execution over one process per GPU (torch.distributed, NCCL over NVLink).

Low cardinality (dense keys): every shard reduces its rows to a mergeable per-group
state table (``Context.groupby_dense_state``), the tables are all-gathered and folded
in rank order (``Context.merge_states``) -- a few KB per GPU, latency-bound.

High cardinality (int64 keys): every shard routes its rows to the owner of their key,
one all-to-all moves each owner's rows to it, and the owner groups what it received.  The
result is sharded by owner.  Raw rows are shipped rather than per-shard partial tables:
with 2^28 distinct keys a shard's partial table is about as large as its rows.
  * count / sum / mean: the routing is the radix path's first pass (``Context.radix_route``:
    rows as (fmix64(key), value) ordered by the top 9 hash bits, rank r owning the digits
    [ceil(512 r / world), ceil(512 (r + 1) / world)); an f32 column travels as f32, 12 bytes a
    row), and the owner runs the remaining passes on its digits (``Context.radix_groupby_routed``),
    reading them in place from the senders' buffers over NVLink ("pull"), or after an NCCL
    all-to-all into its own buffer.
  * other outputs (extrema, variances): a stable owner partition (``Context.hash_partition``,
    senders concatenated in rank order, so every key's rows keep their global order and the
    +-0 tie rule of the extrema stays exact) and ``Context.groupby_hash`` on the owner.

The collective calls take any ``torch.distributed`` group, so the same code runs on
gloo with CPU tensors in the CPU test suite.
"""
from __future__ import annotations


def exchange_parts(dist, part_keys, part_vals, part_counts, recv_keys, recv_vals, group=None) -> int:
    """All-to-all of owner parts.  part_counts[p] rows of part p lie contiguously (in owner
    order) in part_keys / part_vals; rows received from rank r land after those of ranks < r.
    Returns the number of rows received; raises if they do not fit the receive buffers."""
    import torch

    send_counts = part_counts.to(torch.int64)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    s = [int(x) for x in send_counts.tolist()]
    r = [int(x) for x in recv_counts.tolist()]
    n_send, n_recv = sum(s), sum(r)
    # every rank takes the same collective steps, so a rank whose buffers are too small
    # still joins the exchange and raises afterwards
    fits = torch.tensor([1 if n_recv <= recv_keys.numel() and n_recv <= recv_vals.numel() else 0],
                        dtype=torch.int64, device=send_counts.device)
    dist.all_reduce(fits, op=dist.ReduceOp.MIN, group=group)
    if int(fits.item()) == 0:
        raise RuntimeError(f"receive buffers too small on some rank (this rank needs {n_recv} rows)")
    dist.all_to_all_single(recv_keys[:n_recv], part_keys[:n_send], r, s, group=group)
    dist.all_to_all_single(recv_vals[:n_recv], part_vals[:n_send], r, s, group=group)
    return n_recv


class ShardedDenseGroupby:
    """Row-sharded dense-key groupby: shard state -> all-gather -> fold in rank order.

    ``ctx`` is a ``winrapids_b200.Context`` (or an object with the same ``state_bytes`` /
    ``groupby_dense_state`` / ``merge_states`` methods); ``out`` holds the merged outputs
    on every rank."""

    def __init__(self, ctx, dist, world: int, n_groups: int, out: dict, device, group=None):
        import torch

        self.ctx, self.dist, self.world, self.G, self.group = ctx, dist, int(world), int(n_groups), group
        words = ctx.state_bytes(n_groups) // 8
        self.st_local = torch.empty(words, dtype=torch.float64, device=device)
        self.gathered = torch.empty(self.world * words, dtype=torch.float64, device=device)
        self.out = out

    def step(self, keys, vals, row_offset: int, mask=None):
        self.ctx.groupby_dense_state(keys, vals, self.G, row_offset=row_offset, mask=mask, state=self.st_local)
        self.dist.all_gather_into_tensor(self.gathered, self.st_local, group=self.group)
        self.ctx.merge_states(self.gathered, self.world, self.G, out=self.out)


class PeerMappingError(RuntimeError):
    """The exchange buffers could not be mapped across the ranks (raised on every rank)."""


def map_peers(ctx, dist, world: int, rank: int, own: int, device, group=None):
    """Every rank's buffer as mapped in this process, [own if q == rank else peer q's] for q in
    range(world), plus the list of the mappings made (to unmap).  The CUDA IPC handles travel
    once through ``dist.all_gather_object``; a failure on any rank raises PeerMappingError on
    every rank (each unmaps what it mapped), and a ``dist.barrier`` then makes sure every
    mapping exists before any rank stores into a peer's buffer."""
    import torch

    handles = [None] * world
    dist.all_gather_object(handles, ctx.peer_export(own), group=group)
    buffers, mapped, failure = [], [], None
    try:
        for q in range(world):
            if q == rank:
                buffers.append(own)
            else:
                p = ctx.peer_import(handles[q])
                mapped.append(p)
                buffers.append(p)
    except Exception as exc:  # every rank learns of it below, so none is left waiting
        failure = exc
    ok = torch.tensor([0 if failure else 1], dtype=torch.int32, device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    if int(ok.item()) == 0:
        for p in mapped:
            ctx.peer_close(p)
        raise PeerMappingError(f"peer memory mapping failed on rank {rank}: {failure}" if failure
                               else "peer memory mapping failed on another rank")
    dist.barrier(group=group)
    return buffers, mapped


class PeerShardedDenseGroupby:
    """Row-sharded dense-key groupby with the exchange over NVLink peer memory: each rank's
    state table is stored straight into every rank's exchange buffer and each rank folds the
    tables in rank order (tbgb_groupby_dense_sharded) -- no library collective in the step.
    Setup maps the buffers across the processes: the CUDA IPC handles travel once through
    ``dist.all_gather_object``; a ``dist.barrier`` then makes sure every mapping exists."""

    def __init__(self, ctx, dist, world: int, rank: int, n_groups: int, out: dict, device, group=None):
        self.ctx, self.dist, self.world, self.rank, self.G = ctx, dist, int(world), int(rank), int(n_groups)
        self.out, self.group = out, group
        self.own = ctx.exchange_alloc(self.world, self.G)
        self.mapped = []
        try:
            self.buffers, self.mapped = map_peers(ctx, dist, self.world, self.rank, self.own, device, group)
        except PeerMappingError:
            self.close()
            raise
        self.epoch = 0

    def step(self, keys, vals, row_offset: int, mask=None):
        self.epoch += 1
        self.ctx.groupby_dense_sharded(keys, vals, self.G, row_offset, self.rank, self.buffers, self.epoch,
                                       self.out, mask=mask)

    def close(self):
        """Unmap the peers' buffers and free the own one (finish() first when all ranks are alive)."""
        for p in self.mapped:
            self.ctx.peer_close(p)
        self.mapped = []
        if self.own:
            self.ctx.exchange_free(self.own)
            self.own = 0

    def finish(self):
        """Orderly teardown on every rank: unmap, wait until no rank maps this buffer, free it."""
        for p in self.mapped:
            self.ctx.peer_close(p)
        self.mapped = []
        self.dist.barrier(group=self.group)
        self.close()


RADIX_FIELDS = ("count", "sum", "mean")


RADIX_DIGITS = 512  # first-pass digits of the radix path (the top 9 bits of the key's hash)


def owned_digits(world: int):
    """First hash digit owned by each rank, world + 1 entries: rank r owns [lo[r], lo[r + 1])."""
    return [(RADIX_DIGITS * r + world - 1) // world for r in range(world + 1)]


class ShardedHashGroupby:
    """Owner-sharded int64-key groupby of one shard's rows (see the module docstring).

    ``ctx`` is a ``winrapids_b200.Context`` (or an object with the same methods).  Buffers
    are allocated once for shards of up to ``max_rows`` rows, receive buffers with
    ``recv_slack`` headroom over an even share.

    ``exchange`` says how routed rows (count / sum / mean) reach their owner:
      * "nccl": ``all_to_all_single`` into every owner's receive buffer;
      * "pull": no copy.  Every rank routes into a send buffer mapped into every process (CUDA
        IPC); after an all-gather of the 512 digit counts of every rank, each owner's second
        radix pass reads its digits straight from the senders' buffers (over NVLink for peers,
        the tiles of different senders interleaved), and a one-word all-reduce at the end of the
        step says that no owner reads a send buffer any more.  Raises PeerMappingError (on
        every rank) when the mapping fails.
    """

    def __init__(self, ctx, dist, world: int, max_rows: int, max_groups_per_owner: int, fields, device,
                 recv_slack: float = 1.25, group=None, exchange: str = "nccl"):
        import torch

        if exchange not in ("nccl", "pull"):
            raise ValueError(f"exchange must be 'nccl' or 'pull', not {exchange!r}")
        self.ctx, self.dist, self.world, self.group = ctx, dist, int(world), group
        self.rank = dist.get_rank(group) if group is not None else dist.get_rank()
        self.device = device
        self.max_rows = int(max_rows)
        self.max_groups = int(max_groups_per_owner)
        self.cap = int(max_rows * recv_slack) + 4096
        self.radix = set(fields) <= set(RADIX_FIELDS)
        self.mode = exchange if self.radix else "nccl"
        self.out_keys = torch.empty(self.max_groups, dtype=torch.int64, device=device)
        self.out = {f: torch.empty(self.max_groups, dtype=torch.float64, device=device) for f in fields}
        self.n_groups = torch.zeros(1, dtype=torch.int64, device=device)
        self.n_recv = 0
        self.value_bytes = 8
        self._vdtype = None
        self.own, self.mapped = 0, []
        if not self.radix:
            self.part_keys = torch.empty(max_rows, dtype=torch.int64, device=device)
            self.part_vals = torch.empty(max_rows, dtype=torch.float64, device=device)
            self.part_counts = torch.zeros(self.world, dtype=torch.int64, device=device)
            self.recv_keys = torch.empty(self.cap, dtype=torch.int64, device=device)
            self.recv_vals = torch.empty(self.cap, dtype=torch.float64, device=device)
            return
        self.lo = owned_digits(self.world)
        self.n_digits = self.lo[self.rank + 1] - self.lo[self.rank]
        self.digit_counts = torch.zeros(RADIX_DIGITS, dtype=torch.int64, device=device)
        self.seg_counts = torch.zeros(self.world * self.n_digits, dtype=torch.int64, device=device)
        if self.mode == "nccl":
            self.send_h = torch.empty(max_rows, dtype=torch.int64, device=device)
            self.recv_h = torch.empty(self.cap, dtype=torch.int64, device=device)
            return
        self.all_counts = torch.zeros(self.world * RADIX_DIGITS, dtype=torch.int64, device=device)
        self.one = torch.zeros(1, dtype=torch.int64, device=device)
        # the send buffer holds hashes, then values from `span` rows in (8 bytes a value at most):
        # one span on every rank, so any rank finds the values of any other
        span = torch.tensor([self.max_rows], dtype=torch.int64, device=device)
        dist.all_reduce(span, op=dist.ReduceOp.MAX, group=group)
        self.span = int(span.item())
        self.own = ctx.ipc_alloc(max(self.span, 1) * 16)
        try:
            self.bases, self.mapped = map_peers(ctx, dist, self.world, self.rank, self.own, device, group)
        except PeerMappingError:
            self.close()
            raise

    def _value_buffers(self, vb):
        import torch

        dt = torch.float32 if vb == 4 else torch.float64
        if self._vdtype != dt:
            if self.mode == "nccl":
                self.send_v = torch.empty(self.max_rows, dtype=dt, device=self.device)
                self.recv_v = torch.empty(self.cap, dtype=dt, device=self.device)
            self._vdtype = dt
            self.value_bytes = vb

    def step(self, keys, a, b=None, c=None, expr: str = "a", pred=None, threshold: float = 0.0, mask=None):
        """Route, exchange and group one shard; results stay in self.out_keys / self.out (the
        first self.n_groups entries)."""
        if keys.numel() > self.max_rows:
            raise ValueError("shard larger than the buffers")
        if not self.radix:
            self.ctx.hash_partition(keys, a, self.world, self.part_keys, self.part_vals, self.part_counts, b=b, c=c,
                                    expr=expr, pred=pred, threshold=threshold, mask=mask)
            self.n_recv = exchange_parts(self.dist, self.part_keys, self.part_vals, self.part_counts, self.recv_keys,
                                         self.recv_vals, group=self.group)
            self.ctx.groupby_hash_into(self.recv_keys[:self.n_recv], self.recv_vals[:self.n_recv], self.max_groups,
                                       self.out_keys, self.out, self.n_groups)
            return
        vb = self.ctx.radix_value_bytes(a, b, c, expr, pred, threshold)
        self._value_buffers(vb)
        if self.mode == "pull":
            send_h, send_v = self.own, self.own + self.span * 8
        else:
            send_h, send_v = self.send_h, self.send_v
        self.ctx.radix_route(keys, a, send_h, send_v, self.digit_counts, b=b, c=c, expr=expr, pred=pred,
                             threshold=threshold, mask=mask)
        if self.mode == "nccl":
            rows = self._exchange()
            hashes, vals = self.recv_h, self.recv_v
        else:
            rows, hashes, vals = self._senders_in_place(vb)
        self.n_recv = sum(rows)
        self.ctx.radix_groupby_routed(hashes, vals, rows, self.seg_counts, self.lo[self.rank], self.n_digits,
                                      self.max_groups, self.out_keys, self.out, self.n_groups, value_bytes=vb)
        if self.mode == "pull":  # every owner has read its rows: the send buffers may change again
            self.dist.all_reduce(self.one, group=self.group)

    def _exchange(self):
        """Digit counts to their owners, then the rows (senders concatenated in rank order, each
        sender's block in digit order).  Every rank takes the same collective steps; a rank whose
        receive buffers are too small makes every rank raise before the rows move.  Returns the
        rows received from each sender."""
        import torch

        dist, g, lo = self.dist, self.group, self.lo
        nd = [lo[r + 1] - lo[r] for r in range(self.world)]
        dist.all_to_all_single(self.seg_counts, self.digit_counts, [self.n_digits] * self.world, nd, group=g)
        dc = self.digit_counts.cpu().tolist()
        s = [int(sum(dc[lo[r]:lo[r + 1]])) for r in range(self.world)]
        rc = self.seg_counts.view(self.world, self.n_digits).sum(1).cpu().tolist()
        r = [int(x) for x in rc]
        n_send, n_recv = sum(s), sum(r)
        fits = torch.tensor([1 if n_recv <= self.cap else 0], dtype=torch.int64, device=self.digit_counts.device)
        dist.all_reduce(fits, op=dist.ReduceOp.MIN, group=g)
        if int(fits.item()) == 0:
            raise RuntimeError(f"receive buffers too small on some rank (this rank needs {n_recv} rows)")
        dist.all_to_all_single(self.recv_h[:n_recv], self.send_h[:n_send], r, s, group=g)
        dist.all_to_all_single(self.recv_v[:n_recv], self.send_v[:n_send], r, s, group=g)
        return r

    def _senders_in_place(self, vb):
        """Every rank's digit counts to every rank, then where this owner's rows start in each
        sender's buffer.  Returns (rows per sender, address of each sender's first row of this
        rank's digits, of its first value)."""
        dist, g, w = self.dist, self.group, self.world
        dist.all_gather_into_tensor(self.all_counts, self.digit_counts, group=g)
        table = self.all_counts.view(w, RADIX_DIGITS)
        lo, hi = self.lo[self.rank], self.lo[self.rank + 1]
        self.seg_counts.view(w, self.n_digits).copy_(table[:, lo:hi])
        counts = table.cpu().tolist()
        rows = [int(sum(counts[q][lo:hi])) for q in range(w)]
        before = [int(sum(counts[q][:lo])) for q in range(w)]  # sender q's rows of lower digits
        hashes = [self.bases[q] + 8 * before[q] for q in range(w)]
        vals = [self.bases[q] + self.span * 8 + vb * before[q] for q in range(w)]
        return rows, hashes, vals

    def close(self):
        """Unmap the peers' buffers and free the own one (finish() first when every rank is alive)."""
        for p in self.mapped:
            self.ctx.peer_close(p)
        self.mapped = []
        if self.own:
            self.ctx.ipc_free(self.own)
            self.own = 0

    def finish(self):
        """Orderly teardown on every rank: unmap, wait until no rank maps this rank's buffer, free it."""
        if self.mode == "nccl":
            return
        self.ctx.sync()
        for p in self.mapped:
            self.ctx.peer_close(p)
        self.mapped = []
        self.dist.barrier(group=self.group)
        self.close()

    @property
    def recv_bytes_per_row(self) -> int:
        return 8 + (self.value_bytes if self.radix else 8)

    def result(self):
        """(keys, {field: values}) of the groups this rank owns (host synchronisation)."""
        self.ctx.sync()
        g = int(self.n_groups.item())
        return self.out_keys[:g], {f: v[:g] for f, v in self.out.items()}
