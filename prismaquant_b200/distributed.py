"""Multi-GPU plumbing: one process per GPU, torch.distributed over NCCL.

The reference has no distributed code; it shards the cost pass by layer regex
into per-shard pickles merged on disk (incremental_measure_quant_cost.py:73-99,
179-221).  Here:
  * `partition_units` assigns whole units (Linears, expert tensors; fused
    siblings as one unit so their joint NVFP4 global needs no communication)
    to ranks, greedy by bytes (largest first onto the least-loaded rank);
  * `plan_pieces` does the same after cutting a 2-D unit larger than a rank's
    share (total / world) outside any sibling group (lm_head at large N) into
    row blocks; the blocks' NVFP4 maxima meet in ONE all_reduce(MAX)
    (`reduce_split_tmax`) before the scale pass;
  * `all_gather_costs` assembles the cost table with ONE all_gather of
    fixed-size float64 records (sse per format) per piece, summed by unit;
  * `all_reduce_traces` sums the per-Linear Fisher (raw trace, tokens) buffer
    across data-parallel ranks with ONE all_reduce.
Nothing else crosses GPUs: weights and packed outputs stay on their rank.
"""
from __future__ import annotations

import heapq
import math

import torch
import torch.distributed as dist


def partition_units(sizes: list[int], world: int, group_keys: list[str | None] | None = None) -> list[int]:
    """Rank of each unit.  Units sharing a non-None group key stay together."""
    n = len(sizes)
    keys = group_keys or [None] * n
    bundles: dict[object, list[int]] = {}
    for i, k in enumerate(keys):
        bundles.setdefault(("g", k) if k is not None else ("u", i), []).append(i)
    items = sorted(bundles.values(), key=lambda idx: (-sum(sizes[j] for j in idx), idx[0]))
    heap = [(0, r) for r in range(world)]
    rank = [0] * n
    for idx in items:
        load, r = heapq.heappop(heap)
        for j in idx:
            rank[j] = r
        heapq.heappush(heap, (load + sum(sizes[j] for j in idx), r))
    return rank


def plan_pieces(shapes, world: int, group_keys: list[str | None] | None = None):
    """Pieces of a model for `world` ranks and the rank of each: ([(unit, r0, r1)], [rank]).
    A unit is one piece, rows [0, rows), except a 2-D unit outside any sibling group whose size
    exceeds the per-rank share (total / world): it is cut into ceil(size / share) row blocks of
    near-equal height.  Pieces go to ranks as partition_units assigns units (siblings together,
    greedy by bytes).  shapes: [(name, shape)]."""
    keys = group_keys or [None] * len(shapes)
    sizes = [int(math.prod(sh)) for _, sh in shapes]
    share = sum(sizes) / max(world, 1)
    pieces, psizes, pkeys = [], [], []
    for u, ((_, sh), size, key) in enumerate(zip(shapes, sizes, keys)):
        rows = sh[0] if len(sh) == 2 else None
        k = math.ceil(size / share) if (world > 1 and key is None and rows and size > share) else 1
        k = min(k, rows or 1)
        for b in range(k):
            r0 = (rows or 0) * b // k if rows else 0
            r1 = (rows or 0) * (b + 1) // k if rows else (sh[0] if sh else 0)
            pieces.append((u, r0, r1))
            psizes.append(size * (r1 - r0) // max(sh[0], 1) if sh else size)
            pkeys.append(key)
    return pieces, partition_units(psizes, world, pkeys)


def reduce_split_tmax(tmax: torch.Tensor, slots: torch.Tensor, split_ids: torch.Tensor, n_split: int,
                      group=None) -> None:
    """The NVFP4 maxima of units cut into pieces, across ranks: `tmax` holds this rank's per-piece
    maxima (int32 bit patterns of non-negative floats, which order as the floats do), `slots` the
    positions of its pieces of split units and `split_ids` their split-unit numbers.  After ONE
    all_reduce(MAX) every piece of a split unit holds the unit's maximum (collective: every rank
    calls it, with empty slots if it holds no such piece)."""
    buf = torch.zeros(max(n_split, 1), dtype=torch.int32, device=tmax.device)
    if slots.numel():
        buf.scatter_reduce_(0, split_ids, tmax.index_select(0, slots), reduce="amax")
    dist.all_reduce(buf, op=dist.ReduceOp.MAX, group=group)
    if slots.numel():
        tmax.index_copy_(0, slots, buf.index_select(0, split_ids))


def max_units_per_rank(ranks: list[int], world: int) -> int:
    return max([ranks.count(r) for r in range(world)] + [0])


def all_gather_costs(local_ids: torch.Tensor, local_sse: torch.Tensor, n_units: int, cap: int,
                     group=None) -> torch.Tensor:
    """Gather [n_local, 4] sse records from every rank into a [n_units, 4] table.

    Every rank pads its records to `cap` (the largest per-rank record count,
    known to all ranks from the partition) and tags each with its unit id,
    so the table is assembled by index after ONE all_gather; records of the
    pieces of one unit add up."""
    world = dist.get_world_size(group)
    dev = local_sse.device
    rec = torch.full((cap, 5), -1.0, dtype=torch.float64, device=dev)
    rec[: local_sse.shape[0], 0] = local_ids.to(torch.float64)
    rec[: local_sse.shape[0], 1:] = local_sse
    out = torch.empty(world * cap, 5, dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(out, rec, group=group)
    # scatter by id without a device->host sync: padding rows (id -1) land in a spare last row
    ids = out[:, 0].long()
    ids = torch.where(ids >= 0, ids, torch.full_like(ids, n_units))
    table = torch.zeros(n_units + 1, 4, dtype=torch.float64, device=dev)
    table.index_add_(0, ids, out[:, 1:])
    return table[:n_units]


def all_reduce_traces(buf: torch.Tensor, group=None) -> torch.Tensor:
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    return buf


def all_reduce_fisher(acc, group=None):
    """Sum, in place over the ranks of a data-parallel probe, everything a FisherAccumulator holds
    before finalize: the (trace, tokens) buffer; with h_detail_dir also the exact (trace, w^2)
    sums and each per-weight diagonal; and the packed-expert accumulators.  Tensors are reduced in
    sorted name order, so every rank issues the same collectives.  Afterwards every rank's
    finalize gives the same stats; call it with file output on one rank only."""
    dist.all_reduce(acc._acc, op=dist.ReduceOp.SUM, group=group)
    if getattr(acc, "_detail", False):
        dist.all_reduce(acc._exact, op=dist.ReduceOp.SUM, group=group)
        for name in sorted(acc._h_full):
            dist.all_reduce(acc._h_full[name], op=dist.ReduceOp.SUM, group=group)
    for store in (acc._packed_grad_acc, acc._h_packed_channel, acc._packed_sample_count):
        for name in sorted(store):
            v = store[name]
            if isinstance(v, torch.Tensor):
                dist.all_reduce(v, op=dist.ReduceOp.SUM, group=group)
            else:   # a Python float (scalar grad-norm accumulator)
                t = torch.tensor([float(v)], dtype=torch.float64, device=acc._acc.device)
                dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
                store[name] = float(t.item())
    return acc


class RankLeft(RuntimeError):
    """A peer rank announced that it left the job."""


class RankTimeout(RuntimeError):
    """A peer rank did not reach a step within the monitor's timeout."""


class StepMonitor:
    """Host-side liveness between steps, over a key-value store (the process group's
    TCPStore, or any object with set / check).  A rank calls `arrive(step)` when it reaches a
    step, `check(step)` before that step's launches and collectives, and `leave()` when it stops
    taking part (only between steps: none of its kernels or collectives in flight).  `check`
    returns once every rank has reached `step`, raises RankLeft when a peer has left, and
    RankTimeout when a peer is still missing after `timeout` seconds, so the survivors find out
    on the host instead of blocking in their next collective."""

    def __init__(self, store, rank: int, world: int, timeout: float = 10.0, prefix: str = "pq_steps",
                 poll: float = 0.01):
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.prefix, self.poll = float(timeout), prefix, float(poll)

    def _key(self, kind: str, rank: int, step: int | None = None) -> str:
        return f"{self.prefix}/{kind}/{rank}" + ("" if step is None else f"/{step}")

    def arrive(self, step: int) -> None:
        self.store.set(self._key("step", self.rank, step), b"1")

    def leave(self) -> None:
        self.store.set(self._key("left", self.rank), b"1")

    def check(self, step: int) -> None:
        import time
        deadline = time.monotonic() + self.timeout
        pending = [r for r in range(self.world) if r != self.rank]
        while pending:
            still = []
            for r in pending:
                if self.store.check([self._key("step", r, step)]):
                    continue
                if self.store.check([self._key("left", r)]):
                    raise RankLeft(f"rank {r} left the job before step {step}")
                still.append(r)
            pending = still
            if pending:
                if time.monotonic() > deadline:
                    raise RankTimeout(f"rank(s) {pending} did not reach step {step} within {self.timeout:.1f} s")
                time.sleep(self.poll)
