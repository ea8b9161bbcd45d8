"""Direct agg pipeline: raw agg row groups -> request groups -> shuffle -> length buckets ->
packs -> ``PackedBatch``, without expanding every raw table into the flat candidate layout
first.

Counterpart of the reference's direct agg path (``RequestGroupBlock`` ``src/dataloader.py:11897``,
``iter_shuffled_request_groups`` ``:12645``, ``iter_packed_request_groups`` ``:12688``,
``iter_length_bucketed_packs`` ``:12741``, ``prepare_packed_axis_batch`` ``:13300``; routed by
``reader.agg_direct_mode``). Design here:

* one ``AggIndex`` per raw table (``data/agg.py``) holds the whole-array request /
  candidate / event structure; a *group* is one request position and its candidates
  (``RequestGroup``: source, position, a slice of its candidates, its sequence work);
* groups are shuffled through a bounded candidate-row buffer (seeded per rank; a group
  larger than the buffer passes straight through), routed to their length bucket
  (``reader.length_buckets``: bisect of the group's sequence work over the finite
  ``max_length`` bounds, the last bucket the catch-all), and packed per bucket: a group is
  split only when it alone exceeds the batch size, a pack is emitted when the next group
  would overflow it;
* a pack becomes two small Arrow tables per source -- the candidate-axis columns of its
  candidates and the event columns of its requests, gathered with ``take`` -- and one
  tensorizer call with the candidate -> request map, so each request's events are
  gathered and tensorized once (``reader.deduplicate_request_features``; without it the
  request rows are repeated per candidate);
* a source table is released when its last group has been packed.

``agg_direct_mode: compare`` trains on the legacy expansion and checks, for every raw
table, that the direct path tensorizes it to the same rows (candidates in request-group
order).
"""

from __future__ import annotations

import bisect
from dataclasses import dataclass
from typing import Iterable, Iterator, Sequence

import numpy as np
import torch

from .agg import AggIndex, AggPlan
from .batch import PackedBatch


@dataclass(frozen=True)
class RequestGroup:
    source: int          # id of the raw table (``AggIndex``) it lives in
    group: int           # index into the source's groups (one request position)
    lo: int              # first candidate of this slice, among the group's candidates
    count: int           # candidates in this slice
    work: int            # sequence work of the request (length-bucket key)
    last: bool = True    # the slice that ends the group (releases the source's reference)

    def split(self, n: int) -> tuple["RequestGroup", "RequestGroup"]:
        return (RequestGroup(self.source, self.group, self.lo, n, self.work, False),
                RequestGroup(self.source, self.group, self.lo + n, self.count - n, self.work, self.last))


class _Sources:
    """Raw tables by id, each released once all its groups have been packed."""

    def __init__(self) -> None:
        self.index: dict[int, AggIndex] = {}
        self.pending: dict[int, int] = {}
        self.next_id = 0

    def add(self, idx: AggIndex) -> int:
        sid = self.next_id
        self.next_id += 1
        self.index[sid] = idx
        self.pending[sid] = len(idx.group_gp)
        return sid

    def done(self, g: RequestGroup) -> None:
        if g.last:
            self.pending[g.source] -= 1
            if self.pending[g.source] == 0:
                del self.pending[g.source]
                del self.index[g.source]


def group_work(idx: AggIndex, tensorizer, metric: str = "max") -> np.ndarray:
    """Per group, the sequence work the tensorizer's ``sequence_lengths`` would report for
    its request row: over the model's sequences, the max (or sum) of the visible events,
    each capped at the sequence's ``max_length``."""

    p = idx.plan
    gps = idx.group_gp
    out = np.zeros(len(gps), dtype=np.int64)
    col_stream = {c: u for u in p.ups_types for c in p.sequence_columns.get(u, [])}
    col_stream.update({c: u for u, c in p.time_delta_outputs.items()})
    for q in tensorizer.sequences:
        if not q.fields:
            continue
        src = q.fields[0].source or q.fields[0].name
        u = col_stream.get(src)
        n = idx.ev_count[u][gps] if u is not None else np.zeros(len(gps), dtype=np.int64)
        if q.max_length:
            n = np.minimum(n, int(q.max_length))
        out = out + n if metric == "sum" else np.maximum(out, n)
    return out


def iter_groups(tables: Iterable, plan: AggPlan, tensorizer, sources: _Sources, metric: str = "max"):
    """Request groups of every raw table, in stored request order."""

    for table in tables:
        idx = AggIndex(table, plan)
        if not len(idx.group_gp):
            continue
        sid = sources.add(idx)
        work = group_work(idx, tensorizer, metric)
        for g in range(len(idx.group_gp)):
            yield RequestGroup(sid, g, 0, int(idx.group_count[g]), int(work[g]))


def shuffled(groups: Iterable[RequestGroup], buffer_rows: int, rng: np.random.Generator):
    """Bounded shuffle that keeps groups whole: groups wait in a buffer of at most
    ``buffer_rows`` candidates; making room emits uniformly chosen buffered groups.
    ``buffer_rows == 0`` keeps the stored order."""

    if buffer_rows <= 0:
        yield from groups
        return
    buf: list[RequestGroup] = []
    rows = 0

    def pop_random() -> RequestGroup:
        k = int(rng.integers(len(buf)))
        buf[k], buf[-1] = buf[-1], buf[k]
        return buf.pop()

    for g in groups:
        if g.count > buffer_rows:
            while buf:
                yield pop_random()
            rows = 0
            yield g
            continue
        while buf and rows + g.count > buffer_rows:
            out = pop_random()
            rows -= out.count
            yield out
        buf.append(g)
        rows += g.count
    while buf:
        yield pop_random()


class _Packer:
    """Groups into packs of at most ``size`` candidates; a group is split only when it
    alone exceeds ``size``."""

    def __init__(self, size: int) -> None:
        if size <= 0:
            raise ValueError("batch size must be positive")
        self.size = size
        self.buf: list[RequestGroup] = []
        self.rows = 0

    def add(self, g: RequestGroup) -> Iterator[list[RequestGroup]]:
        while g.count > self.size:
            if self.rows:
                yield self._flush()
            head, g = g.split(self.size)
            yield [head]
        if not g.count:
            return
        if self.rows and self.rows + g.count > self.size:
            yield self._flush()
        self.buf.append(g)
        self.rows += g.count
        if self.rows == self.size:
            yield self._flush()

    def _flush(self) -> list[RequestGroup]:
        out, self.buf, self.rows = self.buf, [], 0
        return out

    def rest(self) -> list[RequestGroup]:
        return self._flush() if self.rows else []


def packs(groups: Iterable[RequestGroup], batch_size: int, buckets: Sequence = ()):
    """``(bucket, pack)`` pairs; ``buckets``: ``(max_length or None, batch_size)`` in increasing
    length order, the last may be the catch-all ``None``."""

    if not buckets:
        packer = _Packer(batch_size)
        for g in groups:
            for p in packer.add(g):
                yield 0, p
        rest = packer.rest()
        if rest:
            yield 0, rest
        return
    bounds = [int(m) for m, _ in buckets if m is not None]
    catch_all = buckets[-1][0] is None
    packers = [_Packer(int(b)) for _, b in buckets]
    for g in groups:
        k = bisect.bisect_left(bounds, g.work)
        if k >= len(bounds) and not catch_all:
            raise ValueError("a request's sequence length exceeds every reader.length_buckets max_length "
                             "(add a catch-all bucket without max_length)")
        for p in packers[k].add(g):
            yield k, p
    for k, packer in enumerate(packers):
        rest = packer.rest()
        if rest:
            yield k, rest


def pack_tables(pack: Sequence[RequestGroup], sources: _Sources):
    """(candidate table, request table, candidate -> request row) of one pack."""

    import pyarrow as pa

    cand_parts, req_parts, ri = [], [], []
    by_source: dict[int, list[tuple[int, RequestGroup]]] = {}
    for r, g in enumerate(pack):
        by_source.setdefault(g.source, []).append((r, g))
    for sid, items in by_source.items():
        idx = sources.index[sid]
        gps = np.array([idx.group_gp[g.group] for _, g in items], dtype=np.int64)
        starts = np.array([idx.group_start[g.group] + g.lo for _, g in items], dtype=np.int64)
        counts = np.array([g.count for _, g in items], dtype=np.int64)
        from .parquet import _ragged

        cand = idx.cand_sorted[_ragged(starts, counts)]
        cand_parts.append(idx.candidate_table(cand))
        req_parts.append(idx.request_table(gps))
        ri.append(np.repeat(np.array([r for r, _ in items], dtype=np.int64), counts))
    # requests were numbered in pack order; candidates follow their source's order
    cand = pa.concat_tables(cand_parts, promote_options="default") if len(cand_parts) > 1 else cand_parts[0]
    req = pa.concat_tables(req_parts, promote_options="default") if len(req_parts) > 1 else req_parts[0]
    order = np.concatenate([[r for r, _ in items] for items in by_source.values()]).astype(np.int64)
    inverse = np.empty_like(order)
    inverse[order] = np.arange(len(order))
    req = req.take(pa.array(inverse))                          # request rows back in pack order
    for g in pack:
        sources.done(g)
    return cand, req, np.concatenate(ri)


class AggDirectBatches:
    """Iterable of ``PackedBatch`` from raw agg tables (the direct path)."""

    def __init__(self, tables: Iterable, plan: AggPlan, tensorizer, batch_size: int, *, shuffle_rows: int = 0,
                 seed: int = 0, rank: int = 0, length_buckets: Sequence = (), length_bucket_metric: str = "max",
                 drop_last: bool = True, pin: bool = False) -> None:
        self.tables, self.plan, self.tz = tables, plan, tensorizer
        self.batch_size = int(batch_size)
        self.shuffle_rows = int(shuffle_rows)
        self.rng = np.random.default_rng([int(seed), int(rank), 0xA66])
        self.buckets = [(None if m is None else int(m), int(b)) for m, b in length_buckets]
        self.metric = length_bucket_metric
        self.drop_last = drop_last
        self.pin = pin

    def __iter__(self) -> Iterator[PackedBatch]:
        sources = _Sources()
        groups = iter_groups(self.tables, self.plan, self.tz, sources, self.metric)
        sizes = [b for _, b in self.buckets] or [self.batch_size]
        for k, pack in packs(shuffled(groups, self.shuffle_rows, self.rng), self.batch_size, self.buckets):
            rows = sum(g.count for g in pack)
            if rows < sizes[k] and self.drop_last:
                for g in pack:
                    sources.done(g)
                continue
            cand, req, ri = pack_tables(pack, sources)
            yield self.tz(cand, pin=self.pin, requests=(req, ri))


def compare_direct_to_legacy(table, plan: AggPlan, tensorizer) -> None:
    """Raise unless the direct path tensorizes ``table`` to the legacy expansion's rows
    (candidates in request-group order; request rows deduplicated the same way)."""

    import pyarrow as pa

    idx = AggIndex(table, plan)
    flat = idx.flat_table().take(pa.array(idx.cand_sorted))
    legacy = tensorizer(flat)
    pack = [RequestGroup(0, g, 0, int(idx.group_count[g]), 0) for g in range(len(idx.group_gp))]
    sources = _Sources()
    sources.add(idx)
    cand, req, ri = pack_tables(pack, sources)
    direct = tensorizer(cand, requests=(req, ri))
    problems = []
    for name in ("ids", "offsets", "dense", "labels", "label_mask", "scenario_id"):
        a, b = getattr(legacy, name), getattr(direct, name)
        if (a is None) != (b is None) or (a is not None and not torch.equal(a, b)):
            problems.append(name)
    for name, seq in legacy.sequences.items():
        other = direct.sequences.get(name, {})
        for key, val in seq.items():
            if key not in other or not torch.equal(val, other[key]):
                problems.append(f"sequences.{name}.{key}")
    if problems:
        raise AssertionError(f"agg_direct_mode=compare: direct and legacy batches differ in {problems}")
