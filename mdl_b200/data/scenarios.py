"""Scenario discovery (``scenarios.auto_discover``).

Reference: ``discover_scenario_values`` / ``resolve_auto_scenarios``
(``src/dataloader.py:9672-9830``) with the JSON discovery cache (``:9517-9583``).

* ``discover_scenario_values`` reads only the ``scenarios.source`` column of the
  split's Parquet files and returns the sorted distinct integer values (at most
  ``scenarios.max_discovered``). With ``scenarios.discovery_cache_path`` the
  result is cached as JSON under a signature of (source column, split inputs).
* ``resolve_auto_scenarios`` returns a new config whose scenario names are the
  discovered values (raw encoding). For the MDL models it also expands the
  templates: the feature ``scenario_prior_scene_id_hn`` becomes one feature
  ``scenario_<v>_prior_scene_id_hn`` per value and the scenario token
  ``__auto__`` one token per value whose prior inputs name that feature.
* ``resolve_auto_scenarios_distributed``: rank 0 discovers, the values are
  broadcast, every rank resolves the same config.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

AUTO_TOKEN = "__auto__"
AUTO_PRIOR = "scenario_prior_scene_id_hn"
MDL_MODELS = ("mdl_rankmixer", "mdl_onetrans", "mdl_mixformer")


def _signature(config, split: str) -> str:
    sp = getattr(config.data, split) or config.data.train
    payload = {"version": 1, "source": config.scenarios.source, "inputs": list(sp.inputs)}
    return hashlib.sha256(json.dumps(payload, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def _read_cache(config, split: str) -> tuple[int, ...] | None:
    path = config.scenarios.discovery_cache_path
    if not path or not Path(path).is_file():
        return None
    payload = json.loads(Path(path).read_text())
    if payload.get("signature") != _signature(config, split):
        return None
    values = payload.get("values")
    if not isinstance(values, list) or not values or not all(isinstance(v, int) for v in values):
        raise ValueError(f"scenario discovery cache {path}: values must be a non-empty list of integers")
    return tuple(sorted(set(values)))


def _write_cache(config, split: str, values: tuple[int, ...]) -> None:
    path = config.scenarios.discovery_cache_path
    if not path:
        return
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    tmp = p.with_name(f".{p.name}.{os.getpid()}.tmp")
    tmp.write_text(json.dumps({"signature": _signature(config, split), "values": list(values)}, indent=2) + "\n")
    os.replace(tmp, p)


def discover_scenario_values(config, split: str = "train") -> tuple[int, ...]:
    import pyarrow.compute as pc
    import pyarrow.parquet as pq

    from .parquet import discover_parquet_inputs

    sc = config.scenarios
    if not sc.source:
        raise ValueError("scenario discovery needs scenarios.source")
    cached = _read_cache(config, split)
    if cached is not None:
        return cached
    sp = getattr(config.data, split) or config.data.train
    values: set[int] = set()
    for path in discover_parquet_inputs(sp.inputs):
        f = pq.ParquetFile(path)
        if sc.source not in f.schema_arrow.names:
            raise ValueError(f"scenario discovery: {path} has no column {sc.source!r}")
        for g in range(f.metadata.num_row_groups):
            col = f.read_row_group(g, columns=[sc.source]).column(0)
            uniq = pc.unique(col.combine_chunks() if hasattr(col, "combine_chunks") else col)
            for v in uniq.to_pylist():
                if v is None:
                    continue
                if isinstance(v, bool) or not isinstance(v, int):
                    raise ValueError(f"scenario source {sc.source!r} must hold integers, found {v!r}")
                values.add(int(v))
            if len(values) > sc.max_discovered:
                raise ValueError(f"more than scenarios.max_discovered={sc.max_discovered} scenario values")
    if not values:
        raise ValueError(f"scenario discovery found no values in {sc.source!r}")
    out = tuple(sorted(values))
    _write_cache(config, split, out)
    return out


def _prior_name(v: int) -> str:
    return f"scenario_{'neg_' + str(-v) if v < 0 else v}_prior_scene_id_hn"


def resolve_auto_scenarios(config, values=None):
    """A config with the discovered scenarios filled in (unchanged without auto_discover)."""

    from ..config.loader import app_config_from_mapping
    from ..config.schema import thaw

    sc = config.scenarios
    if not sc.auto_discover:
        return config
    vals = discover_scenario_values(config) if values is None else tuple(values)
    ordered = tuple(sorted({int(v) for v in vals}))
    if not ordered or len(ordered) != len(vals):
        raise ValueError("auto scenario values must be a non-empty set of distinct integers")
    if len(ordered) > sc.max_discovered:
        raise ValueError(f"auto scenario values exceed scenarios.max_discovered={sc.max_discovered}")
    m = thaw(config)
    m.pop("extends", None)
    m["scenarios"].update({"names": [str(v) for v in ordered], "auto_discover": False, "source_encoding": "raw"})
    if config.model.name in MDL_MODELS:
        feats = m["features"]
        templ = [f for f in feats if f["name"] == AUTO_PRIOR]
        if len(templ) != 1:
            raise ValueError(f"auto scenarios on an MDL model need one template feature {AUTO_PRIOR!r}")
        tok = m["tokenization"]
        ttempl = [t for t in tok.get("scenario_tokens", []) if t["name"] == AUTO_TOKEN]
        if len(ttempl) != 1 or AUTO_PRIOR not in ttempl[0].get("prior_inputs", []):
            raise ValueError(f"auto scenarios need one scenario token {AUTO_TOKEN!r} whose prior_inputs name "
                             f"{AUTO_PRIOR!r}")
        expanded = []
        for f in feats:
            if f["name"] == AUTO_PRIOR:
                expanded.extend({**f, "name": _prior_name(v)} for v in ordered)
            else:
                expanded.append(f)
        m["features"] = expanded
        t0 = ttempl[0]
        tokens = [{**t0, "name": str(v),
                   "prior_inputs": [_prior_name(v) if n == AUTO_PRIOR else n for n in t0.get("prior_inputs", [])]}
                  for v in ordered]
        tokens += [t for t in tok.get("scenario_tokens", []) if t["name"] != AUTO_TOKEN]
        tok["scenario_tokens"] = tokens
    return app_config_from_mapping(m)


def resolve_auto_scenarios_distributed(config, rank: int = 0, world: int = 1, group=None):
    if not config.scenarios.auto_discover:
        return config
    payload = [discover_scenario_values(config) if rank == 0 else None]
    if world > 1:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.broadcast_object_list(payload, src=0, group=group)
    return resolve_auto_scenarios(config, payload[0])
