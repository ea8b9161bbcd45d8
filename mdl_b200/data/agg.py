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


class AggAdapter:
    """Callable: raw agg Arrow table -> flat candidate-row Arrow table."""

    def __init__(self, plan: AggPlan) -> None:
        self.plan = plan

    def _delta(self, request_time, event_time) -> float:
        if request_time is None or event_time is None:
            return 0.0
        d = max(float(request_time) - float(event_time), 0.0)
        return math.log1p(d) if self.plan.time_delta_transform == "log1p_seconds" else d

    def __call__(self, table):
        import pyarrow as pa

        p = self.plan
        names = set(table.column_names)
        if "context_indices" not in names or "target_indices" not in names:
            raise ValueError("agg layout needs context_indices and target_indices columns")
        col = {c: table.column(c).to_pylist() for c in p.raw_columns() if c in names}
        missing = [c for c in (*p.context_features, *p.item_features, *p.labels.values()) if c not in col]
        if missing:
            raise ValueError(f"agg table is missing columns {missing[:5]}")
        out: dict[str, list[Any]] = {c: [] for c in (*p.context_features, *p.item_features, *p.request_columns,
                                                     *p.labels.values())}
        rid_col = p.request_id_column or "__request_id"
        out[rid_col] = []
        if p.candidate_position_column:
            out[p.candidate_position_column] = []
        for u in p.ups_types:
            for c in p.sequence_columns.get(u, []):
                out[c] = []
            if u in p.time_delta_outputs:
                out[p.time_delta_outputs[u]] = []
        for i in range(table.num_rows):
            ctx = list(col["context_indices"][i] or [])
            tgt = list(col["target_indices"][i] or [])
            pos = {}
            for k, r in enumerate(ctx):
                if r in pos:
                    raise ValueError(f"agg row {i}: request {r} appears twice in context_indices")
                pos[r] = k
            # events visible to each request, per stream (stored order)
            visible: dict[str, dict[Any, list[int]]] = {}
            for u in p.ups_types:
                memb = col.get(f"{u}_x_indices", [None] * table.num_rows)[i] or []
                by_req: dict[Any, list[int]] = {r: [] for r in ctx}
                for e, reqs in enumerate(memb):
                    for r in reqs or ():
                        if r in by_req:
                            by_req[r].append(e)
                visible[u] = by_req
            cache: dict[Any, dict[str, Any]] = {}
            ordinal: dict[Any, int] = {}
            for c, r in enumerate(tgt):
                if r not in pos:
                    raise ValueError(f"agg row {i}: candidate {c} targets request {r} without context")
                k = pos[r]
                if r not in cache:
                    req: dict[str, Any] = {}
                    for f in p.context_features:
                        req[f] = col[f][i][k]
                    for f in p.request_columns:
                        v = col.get(f, [None] * table.num_rows)[i]
                        req[f] = v[k] if isinstance(v, list) and len(v) == len(ctx) else v
                    rt = col.get(p.request_time_column, [None] * table.num_rows)[i] if p.request_time_column else None
                    rt = rt[k] if isinstance(rt, list) else rt
                    for u in p.ups_types:
                        keep = visible[u][r][:p.sequence_max_lengths.get(u, len(visible[u][r]))]
                        for sc in p.sequence_columns.get(u, []):
                            vals = col[sc][i] or []
                            req[sc] = [vals[e] for e in keep]
                        if u in p.time_delta_outputs:
                            times = col.get(f"{u}_x_time", [None] * table.num_rows)[i] or []
                            req[p.time_delta_outputs[u]] = [self._delta(rt, times[e] if e < len(times) else None)
                                                            for e in keep]
                    rid = col[p.request_id_column][i] if p.request_id_column in col else None
                    rid = rid[k] if isinstance(rid, list) else rid
                    req[rid_col] = rid if rid is not None else f"{i}:{r}"
                    cache[r] = req
                req = cache[r]
                for f, v in req.items():
                    out[f].append(v)
                for f in p.item_features:
                    out[f].append(col[f][i][c])
                for lab in p.labels.values():
                    v = col[lab][i]
                    out[lab].append(v[c] if isinstance(v, list) else v)
                if p.candidate_position_column:
                    out[p.candidate_position_column].append(ordinal.get(r, 0))
                ordinal[r] = ordinal.get(r, 0) + 1
        arrays = {}
        for name, values in out.items():
            if name in p.time_delta_outputs.values():
                arrays[name] = pa.array(values, type=pa.list_(pa.float32()))
            else:
                arrays[name] = pa.array(values)
        return pa.table(arrays)


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
