"""Scenario discovery: distinct raw scene ids from Parquet, the JSON cache, and the MDL
template expansion of the scenario prior feature and scenario token."""

import json

import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import baseline_config, scaled_config
from mdl_b200.data.scenarios import discover_scenario_values, resolve_auto_scenarios


def _files(tmp_path):
    d = tmp_path / "data"
    d.mkdir()
    pq.write_table(pa.table({"scene_id": [3, 7, 3, -2], "x": [1, 2, 3, 4]}), d / "a.parquet", row_group_size=2)
    pq.write_table(pa.table({"scene_id": [7, 11], "x": [5, 6]}), d / "b.parquet")
    return str(d)


def test_discover_and_cache(tmp_path):
    m, _ = baseline_config(1)
    cache = tmp_path / "cache" / "scenes.json"
    m["data"] = {"train": {"inputs": [_files(tmp_path)]}}
    m["scenarios"] = {"source": "scene_id", "auto_discover": True, "discovery_cache_path": str(cache)}
    cfg = app_config_from_mapping(m)
    assert discover_scenario_values(cfg) == (-2, 3, 7, 11)
    assert json.loads(cache.read_text())["values"] == [-2, 3, 7, 11]
    res = resolve_auto_scenarios(cfg)
    assert res.scenarios.names == ("-2", "3", "7", "11") and not res.scenarios.auto_discover
    # the cache answers without reading Parquet once the signature matches
    cache.write_text(json.dumps({"signature": json.loads(cache.read_text())["signature"], "values": [1, 2]}))
    assert discover_scenario_values(cfg) == (1, 2)


def test_mdl_template_expansion(tmp_path):
    m, _ = scaled_config(3, 1e-4, num_fields=8, batch=32)
    m["features"].append({"name": "scenario_prior_scene_id_hn", "kind": "categorical", "source": "scene_prior",
                          "embedding_dim": 16, "embedding_scope": "scenario",
                          "encoding": {"type": "identity", "max_id": 100}})
    m["tokenization"]["scenario_tokens"] = [
        {"name": "__auto__", "important_inputs": ["scene_id"], "prior_inputs": ["scenario_prior_scene_id_hn"]},
        {"name": "global", "important_inputs": ["scene_id"]}]
    m["data"] = {"train": {"inputs": [_files(tmp_path)]}}
    m["scenarios"] = {"source": "scene_id", "auto_discover": True}
    cfg = app_config_from_mapping(m)
    res = resolve_auto_scenarios(cfg, [7, -2])
    names = [f.name for f in res.features]
    assert "scenario_neg_2_prior_scene_id_hn" in names and "scenario_7_prior_scene_id_hn" in names
    assert "scenario_prior_scene_id_hn" not in names
    toks = {t.name: t for t in res.tokenization.scenario_tokens}
    assert set(toks) == {"-2", "7", "global"}
    assert toks["7"].prior_inputs == ("scenario_7_prior_scene_id_hn",)
    with pytest.raises(ValueError):
        resolve_auto_scenarios(cfg, [1, 1])


def test_cardinality_audit_reports_scalar_multis(tmp_path):
    from mdl_b200.data.audit import audit_cardinality

    m, _ = baseline_config(1)
    cfg = app_config_from_mapping(m)
    cats = [f for f in cfg.features if f.kind == "categorical"]
    single, other = cats[0], cats[1]
    path = tmp_path / "x.parquet"
    pq.write_table(pa.table({single.source or single.name: pa.array([[1], [2, 3], None, [4, 5, 6]]),
                             other.source or other.name: pa.array([7, 8, 9, 10])}), path)
    out = audit_cardinality(cfg, [str(path)])
    st = out["scalar_stats"][single.name]
    assert out["raw_rows_seen"] == 4 and st["multi_rows"] == 2 and st["nulls"] == 1 and st["max_len"] == 3
    assert st["samples"] == [[2, 3], [4, 5, 6]]
    assert out["scalar_multis"] == [single.name] and not out["passed"]
    assert out["scalar_stats"][other.name]["multi_rows"] == 0
