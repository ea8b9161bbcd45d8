"""The whole-array agg expansion and the direct agg pipeline (CPU).

* ``AggAdapter`` (``AggIndex.flat_table``) against a per-row statement of the expansion
  rules on seeded mock agg tables with edge cases (events shared by several requests,
  members that are not requests of the row, empty and null membership lists, rows without
  events);
* ``agg_direct_mode: compare``: the direct path tensorizes every raw table to the legacy
  expansion's rows, with and without request deduplication;
* the direct iterator: every candidate once, request groups whole unless larger than a
  batch, batch sizes, length buckets, a deterministic seeded shuffle, and training through
  the CLI with ``agg_direct_mode: direct``.
"""

import json
import math
import subprocess
import sys
from typing import Any

import numpy as np
import pyarrow as pa
import pyarrow.parquet as pq
import pytest
import yaml

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.agg import AggAdapter, AggIndex, AggPlan, write_mock_agg_parquet
from mdl_b200.data.agg_direct import (AggDirectBatches, RequestGroup, _Packer, compare_direct_to_legacy, packs,
                                      shuffled)
from mdl_b200.data.parquet import ParquetBatchIterator, Tensorizer

sys.path.insert(0, __file__.rsplit("/", 1)[0])
from test_agg_adapter import _mapping  # noqa: E402


def _delta(p, request_time, event_time) -> float:
    if request_time is None or event_time is None:
        return 0.0
    d = max(float(request_time) - float(event_time), 0.0)
    return math.log1p(d) if p.time_delta_transform == "log1p_seconds" else d


def _loop_flat_table(table, p):
    import pyarrow as pa

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
                        req[p.time_delta_outputs[u]] = [_delta(p, rt, times[e] if e < len(times) else None)
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



def _edge_table(cfg, seed):
    """A mock agg table plus rows that stress the membership rules."""

    import tempfile

    with tempfile.TemporaryDirectory() as d:
        write_mock_agg_parquet(cfg, f"{d}/a.parquet", rows=40, seed=seed, max_requests=5, max_candidates=9,
                               max_events=12)
        t = pq.read_table(f"{d}/a.parquet")
    rows = t.to_pylist()
    rng = np.random.default_rng(seed + 100)
    for r in rows[::3]:
        ctx = r["context_indices"]
        memb = r["impr_x_indices"]
        for e in range(len(memb)):
            x = rng.random()
            if x < 0.2:
                memb[e] = []
            elif x < 0.3:
                memb[e] = None
            elif x < 0.5:
                memb[e] = list(memb[e]) + [max(ctx) + 1000]        # not a request of this row
    rows[1]["impr_x_indices"], rows[1]["impr_x_time"], rows[1]["impr_x_cat_hn"] = [], [], []
    return pa.Table.from_pylist(rows, schema=t.schema)


def _sorted_rows(table):
    return sorted(json.dumps(r, sort_keys=True, default=str) for r in table.to_pylist())


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_vectorised_expansion_matches_row_rules(seed):
    cfg = app_config_from_mapping(_mapping())
    plan = AggPlan.from_config(cfg)
    table = _edge_table(cfg, seed)
    want = _loop_flat_table(table, plan)
    got = AggAdapter(plan)(table.slice(0))
    assert got.num_rows == want.num_rows
    for name in want.column_names:
        a, b = want.column(name).to_pylist(), got.column(name).to_pylist()
        if name.endswith("log1p_seconds"):
            for x, y in zip(a, b):
                np.testing.assert_allclose(np.array(y, np.float64), np.array(x, np.float64), rtol=1e-6, atol=1e-6)
        else:
            assert a == b, name
    # a sliced view of the raw table expands the same as the rows it shows
    part = table.slice(5, 20)
    assert _sorted_rows(AggAdapter(plan)(part)) == _sorted_rows(_loop_flat_table(part, plan))


def test_expansion_errors():
    cfg = app_config_from_mapping(_mapping())
    plan = AggPlan.from_config(cfg)
    t = _edge_table(cfg, 0)
    rows = t.to_pylist()
    rows[2]["target_indices"] = list(rows[2]["target_indices"]) + [10 ** 6]
    with pytest.raises(ValueError, match="without context"):
        AggIndex(pa.Table.from_pylist(rows, schema=t.schema), plan)
    rows = t.to_pylist()
    rows[0]["context_indices"] = [rows[0]["context_indices"][0]] * 2
    rows[0]["site_hn"] = [rows[0]["site_hn"][0]] * 2
    with pytest.raises(ValueError, match="appears twice"):
        AggIndex(pa.Table.from_pylist(rows, schema=t.schema), plan)


@pytest.mark.parametrize("dedup", [True, False])
def test_compare_mode_direct_equals_legacy(dedup):
    m = _mapping()
    m["data"]["train"]["reader"]["deduplicate_request_features"] = dedup
    cfg = app_config_from_mapping(m)
    plan = AggPlan.from_config(cfg)
    tz = Tensorizer(cfg, _plan(cfg), seq_names=["impr"])
    for seed in range(3):
        compare_direct_to_legacy(_edge_table(cfg, seed), plan, tz)


def _plan(cfg):
    from mdl_b200.models.factory import build_model

    return build_model(cfg, device="cpu", base_seed=0).encoder.batch_plan


def test_packer_and_shuffle_rules():
    g = [RequestGroup(0, i, 0, c, 0) for i, c in enumerate([3, 5, 9, 2, 4, 1])]
    out = []
    p = _Packer(6)
    for x in g:
        out += list(p.add(x))
    out.append(p.rest())
    sizes = [[y.count for y in pk] for pk in out]
    assert sizes == [[3], [5], [6], [3, 2], [4, 1]]            # the 9-row group split 6 + 3
    assert [y.last for y in out[2]] == [False] and out[3][0].last
    # bounded shuffle keeps every group once, is seeded, and differs from stored order
    groups = [RequestGroup(0, i, 0, 1 + i % 4, 0) for i in range(200)]
    a = [x.group for x in shuffled(groups, 32, np.random.default_rng(7))]
    b = [x.group for x in shuffled(groups, 32, np.random.default_rng(7))]
    assert a == b and sorted(a) == list(range(200)) and a != list(range(200))
    # buckets by sequence work
    gw = [RequestGroup(0, i, 0, 2, w) for i, w in enumerate([1, 7, 3, 12, 4, 9])]
    got = list(packs(gw, 4, [(4, 4), (8, 2), (None, 2)]))
    for k, pk in got:
        for x in pk:
            assert (k == 0 and x.work <= 4) or (k == 1 and 4 < x.work <= 8) or (k == 2 and x.work > 8)


@pytest.mark.parametrize("shuffle,buckets", [(0, ()), (64, ()), (0, [(3, 16), (None, 24)])])
def test_direct_iterator_covers_every_candidate_once(tmp_path, shuffle, buckets):
    cfg = app_config_from_mapping(_mapping())
    plan = AggPlan.from_config(cfg)
    tz = Tensorizer(cfg, _plan(cfg), seq_names=["impr"])
    paths = []
    for i in range(2):
        write_mock_agg_parquet(cfg, str(tmp_path / f"a{i}.parquet"), rows=60, seed=i, row_group_size=15,
                               max_candidates=12)
        paths.append(str(tmp_path / f"a{i}.parquet"))
    legacy = AggAdapter(plan)
    all_rows = pa.concat_tables([legacy(pq.read_table(p)) for p in paths])
    want = sorted(zip(all_rows.column("search_id").to_pylist(), all_rows.column("candidate_position").to_pylist()))
    it = ParquetBatchIterator(paths, tz, 16, adapter=legacy, agg_direct_mode="direct", shuffle_rows=shuffle,
                              seed=3, drop_last=False, prefetch=0, length_buckets=buckets)
    seen = []
    goods = []
    for b in it:
        sizes = [s for _, s in buckets] or [16]
        assert b.rows <= max(sizes)
        ri = b.sequences["impr"]["row_indices"].numpy()
        assert (np.diff(ri) >= 0).all() or shuffle  # requests numbered in pack order
        assert b.sequences["impr"]["lengths"].numel() == ri.max() + 1
        seen.append(b.rows)
        goods += b.ids.numpy()[:int(b.offsets[-1])].tolist()
    assert sum(seen) == len(want)
    # the same candidate feature ids as the legacy expansion, each candidate once
    assert sorted(goods) == sorted(tz(all_rows).ids.numpy().tolist())


def test_cli_trains_with_direct_agg_pipeline(tmp_path):
    for i in range(2):
        write_mock_agg_parquet(app_config_from_mapping(_mapping()), str(tmp_path / f"agg-{i}.parquet"), rows=120,
                               seed=i, row_group_size=20)
    m = _mapping(str(tmp_path))
    m["data"]["train"]["reader"].update({"agg_direct_mode": "direct", "shuffle_buffer_rows": 64})
    cfg_path = tmp_path / "agg.yaml"
    cfg_path.write_text(yaml.safe_dump(m))
    out = subprocess.run([sys.executable, "-m", "mdl_b200", "train", "--config", str(cfg_path), "--max-steps", "4"],
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    done = [l for l in lines if l.get("done")]
    assert done and done[-1]["steps"] == 4, out.stdout[-2000:]
    assert all(math.isfinite(l["loss"]) for l in lines if "loss" in l)


@pytest.mark.parametrize("mode", ["legacy", "direct"])
def test_data_stage_costs(tmp_path, mode):
    """data-stages: read / expand / tensorize seconds of the agg pipeline, every timed
    candidate row counted once, the slowest stage named."""

    m = _mapping(str(tmp_path))
    m["data"]["train"]["reader"]["agg_direct_mode"] = mode
    cfg = app_config_from_mapping(m)
    write_mock_agg_parquet(cfg, str(tmp_path / "a.parquet"), rows=60, seed=0, row_group_size=20)
    from mdl_b200.benchmark.data_stages import stage_costs

    res = stage_costs(cfg, [str(tmp_path / "a.parquet")], _plan(cfg), ["impr"], max_tables=2, warmup=1,
                      batch_size=16)
    flat = AggAdapter(AggPlan.from_config(cfg))(pq.ParquetFile(str(tmp_path / "a.parquet")).read_row_group(1))
    flat2 = AggAdapter(AggPlan.from_config(cfg))(pq.ParquetFile(str(tmp_path / "a.parquet")).read_row_group(2))
    assert res["mode"] == mode and res["rows"] == flat.num_rows + flat2.num_rows
    assert set(res["stages"]) >= {"read", "expand", "tensorize"} and res["bottleneck"] in res["stages"]
    assert abs(sum(s["share"] for s in res["stages"].values()) - 1.0) < 1e-3
    cfg_path = tmp_path / "agg.yaml"
    cfg_path.write_text(yaml.safe_dump(m))
    out = subprocess.run([sys.executable, "-m", "mdl_b200", "data-stages", "--config", str(cfg_path),
                          "--max-tables", "2"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    assert json.loads(out.stdout.strip().splitlines()[-1])["rows"] > 0
