"""Aggregate ("agg") Parquet layout -> one row per candidate.

One physical row of the production layout holds several requests and their
candidates (reference ``DATA_FORMAT.md`` section 3.1, ``adapt_mdl_rankmixer_parquet``
``src/dataloader.py:6593-7425``):

* request-axis columns (``context_features``, ``request_columns``): one value per
  request position; ``context_indices`` names the request of every position;
* candidate-axis columns (``item_features``, labels): one value per candidate;
  ``target_indices`` names the request of every candidate;
* per user-behaviour stream ``<ups>``: event columns ``<ups>_x_<attr>`` (one value per
  event), event times ``<ups>_x_time`` and ``<ups>_x_indices`` (per event, the
  requests allowed to see it).

``AggAdapter`` expands a raw Arrow table into the flat layout the tensorizer reads:
per candidate its request's context values, its own item values and labels, the
request id, its position among its request's candidates, and per stream the events
visible to its request (stored order, the first ``sequence_max_lengths[ups]`` kept)
with their time delta to the request time (``<request_time> - <ups>_x_time``,
``log1p`` of the seconds under ``time_delta_transform: log1p_seconds``) in the
``time_delta_outputs`` column. Each request's events are gathered once and shared by
its candidates. With ``reader.deduplicate_request_features`` the tensorizer then keeps
one sequence row per request.

``write_mock_agg_parquet`` writes seeded files of this layout for a config (tests,
benchmarks of the data path).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

import numpy as np

AGG_ADAPTERS = ("src.dataloader:adapt_mdl_rankmixer_parquet", "mdl_b200.data.agg:AggAdapter")


@dataclass
class AggPlan:
    context_features: list[str]
    item_features: list[str]
    ups_types: list[str]
    request_columns: list[str] = field(default_factory=list)
    labels: dict[str, str] = field(default_factory=dict)
    sequence_max_lengths: dict[str, int] = field(default_factory=dict)
    request_time_column: str | None = None
    time_delta_outputs: dict[str, str] = field(default_factory=dict)
    time_delta_transform: str = "log1p_seconds"
    candidate_position_column: str | None = None
    request_id_column: str | None = None
    sequence_columns: dict[str, list[str]] = field(default_factory=dict)  # ups -> raw event columns

    @classmethod
    def from_config(cls, config, split: str = "train") -> "AggPlan":
        sp = getattr(config.data, split) or config.data.train
        if sp.adapter is None:
            raise ValueError(f"data.{split}: adapter_parquet needs an adapter section")
        if sp.adapter.callable not in AGG_ADAPTERS:
            raise ValueError(f"data.{split}.adapter.callable {sp.adapter.callable!r}: supported adapters are "
                             f"{AGG_ADAPTERS}")
        o = dict(sp.adapter.options or {})
        ups = list(o.get("ups_types") or [])
        tdo = dict(o.get("time_delta_outputs") or {})
        derived = set(tdo.values())
        seq_cols: dict[str, list[str]] = {u: [] for u in ups}
        for s in config.sequences:
            for fl in s.fields:
                src = fl.source or fl.name
                for u in ups:
                    if src.startswith(f"{u}_x_") and src not in derived and src not in seq_cols[u]:
                        seq_cols[u].append(src)
        labels = dict(o.get("labels") or sp.labels or {})
        return cls(context_features=list(o.get("context_features") or []),
                   item_features=list(o.get("item_features") or []), ups_types=ups,
                   request_columns=list(o.get("request_columns") or []), labels=labels,
                   sequence_max_lengths={k: int(v) for k, v in (o.get("sequence_max_lengths") or {}).items()},
                   request_time_column=o.get("request_time_column"), time_delta_outputs=tdo,
                   time_delta_transform=o.get("time_delta_transform", "log1p_seconds"),
                   candidate_position_column=o.get("candidate_position_column"),
                   request_id_column=sp.request_id, sequence_columns=seq_cols)

    def raw_columns(self) -> list[str]:
        cols = ["context_indices", "target_indices", *self.context_features, *self.item_features,
                *self.request_columns, *self.labels.values()]
        if self.request_time_column:
            cols.append(self.request_time_column)
        if self.request_id_column:
            cols.append(self.request_id_column)
        for u in self.ups_types:
            cols += [f"{u}_x_indices", f"{u}_x_time", *self.sequence_columns.get(u, [])]
        return list(dict.fromkeys(cols))


def _flat(arr):
    """Logical values of a list array (slices honoured, null lists empty) and per-row lengths."""

    import pyarrow.compute as pc

    lengths = np.asarray(pc.list_value_length(arr).fill_null(0).to_numpy(zero_copy_only=False), dtype=np.int64)
    return pc.list_flatten(arr), lengths


def _ints(arr) -> np.ndarray:
    return np.asarray(arr.fill_null(-1).to_numpy(zero_copy_only=False), dtype=np.int64)


class AggIndex:
    """Request / candidate / event structure of one raw agg table, built with whole-array
    operations (no per-row Python).

    * context position ``p`` (flattened ``context_indices``): one request of one raw row;
    * candidate ``c`` (flattened ``target_indices``) belongs to ``gp[c]``, the position of
      its request in its row (a ``(row, request)`` key looked up in the sorted context keys);
    * per stream ``u``: the events visible to each position, in stored order, the first
      ``sequence_max_lengths[u]`` kept (``ev_start[u][p]``, ``ev_count[u][p]`` into
      ``ev_event[u]``, the flattened event index).

    ``candidate_table`` / ``request_table`` gather the flat-layout columns of chosen
    candidates / request positions with Arrow ``take``; ``flat_table`` is the whole table in
    candidate order (the legacy adapter output)."""

    def __init__(self, table, plan: AggPlan) -> None:
        import pyarrow as pa

        from .parquet import _combined

        p = plan
        self.plan = p
        names = set(table.column_names)
        if "context_indices" not in names or "target_indices" not in names:
            raise ValueError("agg layout needs context_indices and target_indices columns")
        missing = [c for c in (*p.context_features, *p.item_features, *p.labels.values()) if c not in names]
        if missing:
            raise ValueError(f"agg table is missing columns {missing[:5]}")
        self.table = table
        self.rows = rows = table.num_rows
        self.col = {c: _combined(table.column(c)) for c in p.raw_columns() if c in names}
        ctx, self.ctx_len = _flat(self.col["context_indices"])
        tgt, self.tgt_len = _flat(self.col["target_indices"])
        ctx_req, tgt_req = _ints(ctx), _ints(tgt)
        self.ctx_row = np.repeat(np.arange(rows, dtype=np.int64), self.ctx_len)
        self.tgt_row = np.repeat(np.arange(rows, dtype=np.int64), self.tgt_len)
        self.ctx_req = ctx_req
        if (ctx_req < 0).any():
            raise ValueError("agg context_indices must be non-negative integers")
        self._M = int(max(ctx_req.max(initial=0), tgt_req.max(initial=0))) + 1
        keys = self.ctx_row * self._M + ctx_req
        self._order = np.argsort(keys, kind="stable")
        self._sorted = keys[self._order]
        dup = np.nonzero(self._sorted[1:] == self._sorted[:-1])[0]
        if len(dup):
            p0 = int(self._order[dup[0]])
            raise ValueError(f"agg row {int(self.ctx_row[p0])}: request {int(ctx_req[p0])} appears twice in "
                             "context_indices")
        gp = self._lookup(self.tgt_row, tgt_req)
        bad = np.nonzero(gp < 0)[0]
        if len(bad):
            c0 = int(bad[0])
            r0 = int(self.tgt_row[c0])
            local = c0 - int(np.cumsum(self.tgt_len)[r0] - self.tgt_len[r0])
            raise ValueError(f"agg row {r0}: candidate {local} targets request {int(tgt_req[c0])} without context")
        self.gp = gp
        # candidates grouped by request position (stable: stored order inside a request)
        self.cand_sorted = np.argsort(gp, kind="stable")
        gps, first, counts = np.unique(gp[self.cand_sorted], return_index=True, return_counts=True)
        self.group_gp, self.group_start, self.group_count = gps, first, counts
        # ordinal of every candidate among its request's candidates
        self.cand_rank = np.empty(len(gp), dtype=np.int64)
        self.cand_rank[self.cand_sorted] = np.arange(len(gp)) - np.repeat(first, counts)
        self.P = len(ctx_req)
        self._flats: dict[str, tuple] = {}
        self._events(pa)

    def flat(self, name: str):
        """``_flat`` of a raw list column, computed once per table."""

        got = self._flats.get(name)
        if got is None:
            got = self._flats[name] = _flat(self.col[name])
        return got

    def _lookup(self, row: np.ndarray, req: np.ndarray) -> np.ndarray:
        """Context position of each ``(row, request)`` pair, -1 where the row has no such request."""

        if not len(self._sorted):
            return np.full(len(row), -1, dtype=np.int64)
        key = row * self._M + np.clip(req, 0, self._M - 1)
        at = np.minimum(np.searchsorted(self._sorted, key), len(self._sorted) - 1)
        hit = (self._sorted[at] == key) & (req >= 0) & (req < self._M)
        return np.where(hit, self._order[at], -1)

    def _events(self, pa) -> None:
        p = self.plan
        self.ev_event: dict[str, np.ndarray] = {}
        self.ev_start: dict[str, np.ndarray] = {}
        self.ev_count: dict[str, np.ndarray] = {}
        self.ev_base: dict[str, np.ndarray] = {}     # first flattened event of every row
        for u in p.ups_types:
            if f"{u}_x_indices" in self.col:
                per_event, ev_len = self.flat(f"{u}_x_indices")    # one membership list per event
            else:
                per_event, ev_len = _flat(pa.nulls(self.rows, pa.list_(pa.list_(pa.int64()))))
            members, m_len = _flat(per_event)
            ev_row = np.repeat(np.arange(self.rows, dtype=np.int64), ev_len)
            m_event = np.repeat(np.arange(len(ev_row), dtype=np.int64), m_len)
            m_gp = self._lookup(ev_row[m_event], _ints(members)) if len(m_event) else np.zeros(0, np.int64)
            keep = m_gp >= 0
            m_gp, m_event = m_gp[keep], m_event[keep]
            order = np.argsort(m_gp, kind="stable")   # events of one position stay in stored order
            m_gp, m_event = m_gp[order], m_event[order]
            count = np.bincount(m_gp, minlength=self.P).astype(np.int64)
            start = np.cumsum(count) - count
            cap = p.sequence_max_lengths.get(u)
            self.ev_event[u] = m_event
            self.ev_start[u] = start
            self.ev_count[u] = count if cap is None else np.minimum(count, int(cap))
            self.ev_base[u] = np.cumsum(ev_len) - ev_len

    # ------------------------------------------------------------------ gathers
    def _per_position(self, name: str):
        """A request-axis column as one value per context position (``None``: not per position)."""

        arr = self.col.get(name)
        if arr is None:
            return None
        from .parquet import _is_list

        if _is_list(arr.type):
            vals, ln = self.flat(name)
            if np.array_equal(ln, self.ctx_len):
                return vals
        return None

    def _request_values(self, name: str, gps: np.ndarray):
        """Values of a request-axis column at context positions ``gps`` (a value per
        position, or the row's single value)."""

        import pyarrow as pa

        per = self._per_position(name)
        if per is not None:
            return per.take(pa.array(gps, type=pa.int64()))
        arr = self.col.get(name)
        if arr is None:
            return pa.nulls(len(gps))
        return arr.take(pa.array(self.ctx_row[gps], type=pa.int64()))

    def request_ids(self, gps: np.ndarray):
        import pyarrow as pa

        p = self.plan
        if p.request_id_column and p.request_id_column in self.col:
            return self._request_values(p.request_id_column, gps)
        return pa.array([f"{int(r)}:{int(q)}" for r, q in zip(self.ctx_row[gps], self.ctx_req[gps])])

    def candidate_table(self, cand: np.ndarray):
        """Candidate-axis columns (request context, items, labels, request id, candidate
        position) of candidates ``cand``, in that order."""

        import pyarrow as pa

        p = self.plan
        take = pa.array(cand, type=pa.int64())
        gps = self.gp[cand]
        out = {}
        for f in p.context_features:
            out[f] = self._request_values(f, gps)
        for f in p.request_columns:
            out[f] = self._request_values(f, gps)
        for f in p.item_features:
            out[f] = self.flat(f)[0].take(take)
        for lab in p.labels.values():
            arr = self.col[lab]
            from .parquet import _is_list

            out[lab] = self.flat(lab)[0].take(take) if _is_list(arr.type) else arr.take(
                pa.array(self.tgt_row[cand], type=pa.int64()))
        out[p.request_id_column or "__request_id"] = self.request_ids(gps)
        if p.candidate_position_column:
            out[p.candidate_position_column] = pa.array(self.cand_rank[cand], type=pa.int64())
        return pa.table(out)

    def request_table(self, gps: np.ndarray):
        """Per-request event columns (and time deltas) of context positions ``gps``."""

        import pyarrow as pa

        from .parquet import _ragged

        p = self.plan
        out = {}
        for u in p.ups_types:
            cnt = self.ev_count[u][gps]
            ev = self.ev_event[u][_ragged(self.ev_start[u][gps], cnt)]
            offsets = pa.array(np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32))
            take = pa.array(ev, type=pa.int64())
            for sc in p.sequence_columns.get(u, []):
                vals = self.flat(sc)[0] if sc in self.col else pa.nulls(0, pa.int64())
                out[sc] = pa.ListArray.from_arrays(offsets, vals.take(take) if len(vals) else pa.nulls(len(ev)))
            if u in p.time_delta_outputs:
                out[p.time_delta_outputs[u]] = pa.ListArray.from_arrays(
                    offsets, pa.array(self._deltas(u, gps, cnt, ev), type=pa.float32()))
        return pa.table(out) if out else pa.table({"__none": pa.nulls(len(gps))}).drop(["__none"])

    def _deltas(self, u: str, gps: np.ndarray, cnt: np.ndarray, ev: np.ndarray) -> np.ndarray:
        p = self.plan
        tcol = self.col.get(f"{u}_x_time")
        if tcol is None or not p.request_time_column or p.request_time_column not in self.col:
            return np.zeros(len(ev), dtype=np.float32)
        import pyarrow.compute as pc

        key = f"__times:{u}"
        if key not in self._flats:
            times, t_len = self.flat(f"{u}_x_time")
            self._flats[key] = (np.asarray(pc.cast(times, "float64").fill_null(np.nan).to_numpy(zero_copy_only=False)),
                                t_len, np.cumsum(t_len) - t_len)
        tv, t_len, t_base = self._flats[key]
        rt = self._request_values(p.request_time_column, gps)
        rtv = np.asarray(pc.cast(rt, "float64").fill_null(np.nan).to_numpy(zero_copy_only=False))
        row_of_req = self.ctx_row[gps]
        req_of_ev = np.repeat(np.arange(len(gps)), cnt)
        local = ev - self.ev_base[u][row_of_req[req_of_ev]]           # event index inside its row
        # an event beyond its row's time list has no time (delta 0)
        inside = local < t_len[row_of_req[req_of_ev]]
        et = np.full(len(ev), np.nan)
        et[inside] = tv[t_base[row_of_req[req_of_ev]][inside] + local[inside]]
        d = np.maximum(rtv[req_of_ev] - et, 0.0)
        if p.time_delta_transform == "log1p_seconds":
            d = np.log1p(d)
        return np.where(np.isnan(d), 0.0, d).astype(np.float32)

    def flat_table(self):
        """The legacy adapter output: every candidate in stored order, each with its
        request's context, items, labels, request id, position and visible events."""

        cand = np.arange(len(self.gp), dtype=np.int64)
        t = self.candidate_table(cand)
        req = self.request_table(self.gp)
        for name in req.column_names:
            t = t.append_column(name, req.column(name))
        return t


class AggAdapter:
    """Callable: raw agg Arrow table -> flat candidate-row Arrow table (``AggIndex.flat_table``)."""

    def __init__(self, plan: AggPlan) -> None:
        self.plan = plan

    def __call__(self, table):
        return AggIndex(table, self.plan).flat_table()


def write_mock_agg_parquet(config, path: str, rows: int, *, seed: int = 0, max_requests: int = 4,
                           max_candidates: int = 6, max_events: int = 40, row_group_size: int = 64,
                           split: str = "train") -> None:
    """Seeded agg-layout Parquet for ``config``'s adapter plan: ids drawn over each
    feature's table (``num_buckets`` / ``max_id``), bag features as short lists,
    labels Bernoulli(0.2), events shared by random subsets of a row's requests."""

    import pyarrow as pa
    import pyarrow.parquet as pq

    plan = AggPlan.from_config(config, split)
    rng = np.random.default_rng(seed)
    by_name = {f.name: f for f in config.features}
    by_source = {(f.source or f.name): f for f in config.features}
    seq_field = {(fl.source or fl.name): fl for s in config.sequences for fl in s.fields}

    def vocab(f) -> int:
        enc = getattr(f, "encoding", None)
        if enc is not None and enc.num_buckets:
            return int(enc.num_buckets)
        if enc is not None and enc.max_id:
            return int(enc.max_id)
        return 100

    def value(name: str):
        f = by_source.get(name) or by_name.get(name)
        if f is None:
            return int(rng.integers(1, 100))
        if f.kind == "dense":
            return [float(x) for x in rng.standard_normal(int(f.dimension))] if int(f.dimension) > 1 else \
                float(rng.standard_normal())
        v = int(rng.integers(1, vocab(f) + 1))
        if f.pooling != "none":
            return [int(x) for x in rng.integers(1, vocab(f) + 1, size=int(rng.integers(1, 5)))]
        return v

    data: dict[str, list] = {c: [] for c in plan.raw_columns()}
    next_request = 1
    for _ in range(rows):
        R = int(rng.integers(1, max_requests + 1))
        C = int(rng.integers(1, max_candidates + 1))
        ctx = list(range(next_request, next_request + R))
        next_request += R
        tgt = [ctx[int(rng.integers(0, R))] for _ in range(C)]
        data["context_indices"].append(ctx)
        data["target_indices"].append(tgt)
        for f in plan.context_features:
            data[f].append([value(f) for _ in range(R)])
        for f in plan.request_columns:
            data[f].append([int(rng.integers(1, 1000)) for _ in range(R)])
        for f in plan.item_features:
            data[f].append([value(f) for _ in range(C)])
        for lab in plan.labels.values():
            data[lab].append([float(rng.random() < 0.2) for _ in range(C)])
        req_time = [float(1.7e9 + rng.integers(0, 3600)) for _ in range(R)]
        if plan.request_time_column:
            data[plan.request_time_column].append(req_time)
        if plan.request_id_column and plan.request_id_column in data:
            data[plan.request_id_column].append([f"req{r}" for r in ctx])
        for u in plan.ups_types:
            E = int(rng.integers(0, max_events + 1))
            memb = []
            for _ in range(E):
                k = int(rng.integers(1, R + 1))
                memb.append(sorted(int(x) for x in rng.choice(ctx, size=k, replace=False)))
            data[f"{u}_x_indices"].append(memb)
            data[f"{u}_x_time"].append([float(min(req_time) - rng.integers(0, 86400 * 30)) for _ in range(E)])
            for sc in plan.sequence_columns.get(u, []):
                fl = seq_field.get(sc)
                vb = vocab(fl) if fl is not None and fl.kind == "categorical" else 100
                data[sc].append([int(x) for x in rng.integers(1, vb + 1, size=E)])
    pq.write_table(pa.table({k: pa.array(v) for k, v in data.items()}), path, row_group_size=row_group_size)
