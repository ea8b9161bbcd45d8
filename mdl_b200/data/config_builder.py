"""Model configs from a field contract and a data profile (offline: reads YAML / JSON only).

Counterpart of the reference's production config builder
(``scripts/build_production_configs.py``: coarse ``rankmixer`` / ``mdl_rankmixer`` /
``onetrans`` / ``mdl_onetrans`` contracts, ``*_fine`` siblings, profile-driven table sizes,
``--estimate-from-names``, an embedding memory summary). The reference hard-codes its
production field list; here the fields come from a *contract* file:

.. code-block:: yaml

    request_id: search_id                 # agg layout request key (optional)
    request_time_column: impr_time        # for event time deltas (optional)
    context_features: [site_hn, ...]      # request axis
    item_features: [goods_id_hn, ...]     # candidate axis
    bag_features: [query_terms_hn]        # multi-valued (else read from the profile)
    dense_features: {price: 1}            # name -> dimension
    labels: {click: label_click}          # task -> column
    ups:                                  # user behaviour streams of the agg layout
      impr: {fields: [impr_x_goods_id_hn, impr_x_cat_hn], max_length: 200}
    scene_column: scene_id                # MDL scenes (coarse) ...
    scenes: [home, search]
    fine_scene_column: fine_scene_id      # ... and their fine siblings (optional)
    fine_scenes: [home_a, home_b, search_a]

Sizes come from, in order: ``recommend-shapes`` output (``num_embeddings``,
``embedding_dim`` per feature), a ``profile_columns`` report of the raw files (distinct
values scaled by ``growth`` and the load; bags and their lengths from the list nesting),
or name heuristics
(``estimate_from_names``, marked as such in the summary). Encodings come from
``recommend_encodings`` on the profile, else ``pre_hashed`` for ``*_hn`` columns and
``hash`` otherwise. The memory summary plans the tables with the framework's sharding
planner (``parallel/sharding.py``) for a world size and reports the largest rank's bytes
(fp32 weights plus row-wise Adagrad state) against a per-GPU budget.
"""

from __future__ import annotations

import copy
import math
import re
from dataclasses import dataclass, field
from typing import Any, Mapping

FAMILIES = ("rankmixer", "mdl_rankmixer", "onetrans", "mdl_onetrans")


@dataclass
class FieldContract:
    context_features: list[str]
    item_features: list[str]
    labels: dict[str, str]
    ups: dict[str, dict] = field(default_factory=dict)
    bag_features: list[str] = field(default_factory=list)
    dense_features: dict[str, int] = field(default_factory=dict)
    request_id: str | None = None
    request_time_column: str | None = None
    scene_column: str | None = None
    scenes: list[str] = field(default_factory=list)
    fine_scene_column: str | None = None
    fine_scenes: list[str] = field(default_factory=list)

    @classmethod
    def from_mapping(cls, m: Mapping[str, Any]) -> "FieldContract":
        known = set(cls.__dataclass_fields__)
        unknown = sorted(set(m) - known)
        if unknown:
            raise ValueError(f"field contract: unknown key(s) {unknown}")
        c = cls(context_features=list(m.get("context_features") or []),
                item_features=list(m.get("item_features") or []), labels=dict(m.get("labels") or {}),
                ups={k: dict(v or {}) for k, v in (m.get("ups") or {}).items()},
                bag_features=list(m.get("bag_features") or []),
                dense_features={k: int(v) for k, v in (m.get("dense_features") or {}).items()},
                request_id=m.get("request_id"), request_time_column=m.get("request_time_column"),
                scene_column=m.get("scene_column"), scenes=[str(s) for s in m.get("scenes") or []],
                fine_scene_column=m.get("fine_scene_column"),
                fine_scenes=[str(s) for s in m.get("fine_scenes") or []])
        if not c.labels:
            raise ValueError("field contract: labels must name at least one task")
        if not (c.context_features or c.item_features):
            raise ValueError("field contract: no context or item features")
        dup = sorted({f for f in c.context_features if f in set(c.item_features)})
        if dup:
            raise ValueError(f"field contract: features on both axes: {dup[:5]}")
        for u, spec in c.ups.items():
            if not spec.get("fields"):
                raise ValueError(f"field contract: ups {u!r} lists no fields")
        return c


# ------------------------------------------------------------------ sizing
_NAME_BUCKETS = (  # (pattern over the column name, log2 rows) -- first match wins
    (r"(goods|sku|item|product|user|uid|query_hash|query_arr|title|name_bigram|ner|tfidf)", 22),
    (r"(query|term|q2q|q2i|session|sess)", 20),
    (r"(mall|shop|brand|cluster|spec|prpty|cat4|cat3|leaf)", 18),
    (r"(cat|category|tag|page)", 14),
    (r"(cnt|count|num|dis|level|ratio|rate|price|sales|rank|score|bucket)", 10),
    (r"(site|lang|language|region|plat|currency|timezone|scene|method|country|device|os)", 8),
)


def estimated_bits(column: str) -> int:
    name = column.lower()
    for pattern, bits in _NAME_BUCKETS:
        if re.search(pattern, name):
            return bits
    return 18


def fourth_root_dim(rows: float, lo: int = 8, hi: int = 64) -> int:
    """``6 * rows^0.25`` rounded to a multiple of 8, clamped to [lo, hi]."""

    return int(min(hi, max(lo, round(6.0 * max(rows, 1.0) ** 0.25 / 8.0) * 8)))


@dataclass
class Sizing:
    rows: int
    dim: int
    encoding: str
    bag_length: int | None
    source: str          # "shapes", "profile" or "name estimate"


def size_features(contract: FieldContract, *, profile: Mapping | None = None, shapes: Mapping | None = None,
                  load: float = 0.5, growth: float = 4.0, max_dim: int = 64, max_bits: int = 28) -> dict[str, Sizing]:
    """Table rows, width, encoding and bag length of every categorical column (features
    and behaviour-stream fields), keyed by column name.

    ``profile``: a ``profile_columns`` report of the raw agg files (entries carry their
    ``column``); a feature column nested one list level deeper than its axis (a list per
    request or candidate) is a bag, ``4 x`` its mean length rounded up to a power of two
    (4 to 64) being its ``max_length``. ``shapes``: ``recommend_shapes`` output over two
    such profiles, keyed like the profile."""

    from .profile import recommend_encodings

    entries = dict((profile or {}).get("features") or {})
    col_of = {k: v.get("column", k) for k, v in entries.items()}
    prof = {col_of[k]: v for k, v in entries.items()}
    shp = {col_of.get(k, k): v for k, v in ((shapes or {}).get("features") or {}).items()}
    enc_rec = {col_of.get(k, k): v["encoding"] for k, v in recommend_encodings(profile).items()} if profile else {}
    cols = list(contract.context_features) + list(contract.item_features)
    stream_cols = list(dict.fromkeys(c for spec in contract.ups.values() for c in spec["fields"]))
    cols += [c for c in stream_cols if c not in cols]
    out: dict[str, Sizing] = {}
    for col in cols:
        if col in contract.dense_features:
            continue
        if col in shp:
            rows, dim, how = int(shp[col]["num_embeddings"]), int(shp[col]["embedding_dim"]), "shapes"
        elif col in prof:
            distinct = max(1, int(prof[col]["distinct"]))
            bits = min(max_bits, max(4, math.ceil(math.log2(distinct * growth / load))))
            rows, dim, how = 1 << bits, fourth_root_dim(distinct * growth, hi=max_dim), "profile"
        else:
            bits = min(max_bits, estimated_bits(col))
            rows, dim, how = 1 << bits, fourth_root_dim(float(1 << bits) * load, hi=max_dim), "name estimate"
        bag = None
        if col not in stream_cols:
            entry = prof.get(col)
            if entry is not None and entry.get("depth", 1) >= 2:
                mean = float(entry.get("inner_mean_length") or 1.0)
                bag = int(min(64, max(4, 1 << math.ceil(math.log2(max(1.0, 4.0 * mean))))))
            elif col in contract.bag_features:
                bag = 16
        rec = enc_rec.get(col)
        if rec in ("pre_hashed", "identity"):
            encoding = rec
        elif rec == "remixed_pre_hashed":
            encoding = "hash"        # a salted hash of the text remixes clustered low bits
        else:                        # vocab needs a fitted vocabulary: hash into the planned table offline
            encoding = "pre_hashed" if col.endswith("_hn") and rec is None else "hash"
        if encoding == "identity" and col in prof:
            rows = max(rows, int(prof[col]["max_id"]) + 1)
        out[col] = Sizing(rows, dim, encoding, bag, how)
    return out


def _encoding(s: Sizing) -> dict:
    if s.encoding == "identity":
        return {"type": "identity", "max_id": s.rows - 1, "out_of_range": "zero"}
    return {"type": s.encoding, "num_buckets": s.rows}


def _feature_name(col: str) -> str:
    return re.sub(r"_hn$", "", col)


# ------------------------------------------------------------------ builder
def build_config(contract: FieldContract, family: str, *, sizes: Mapping[str, Sizing], fine: bool = False,
                 batch_size: int = 2048, token_dim: int | None = None, layers: int | None = None,
                 inputs: list[str] | None = None) -> dict:
    """A complete config mapping (same schema as the YAML files) for ``family``."""

    if family not in FAMILIES:
        raise ValueError(f"family must be one of {FAMILIES}")
    mdl = family.startswith("mdl_")
    onetrans = family.endswith("onetrans")
    feats: list[dict] = []
    for col in contract.context_features + contract.item_features:
        if col in contract.dense_features:
            feats.append({"name": _feature_name(col), "kind": "dense", "source": col,
                          "dimension": contract.dense_features[col]})
            continue
        s = sizes[col]
        f = {"name": _feature_name(col), "kind": "categorical", "source": col, "embedding_dim": s.dim,
             "encoding": _encoding(s)}
        if s.bag_length:
            f.update({"pooling": "mean", "max_length": s.bag_length, "truncation": "tail"})
        feats.append(f)
    names = [f["name"] for f in feats]
    if len(set(names)) != len(names):
        raise ValueError("two columns map to the same feature name")
    seqs = []
    time_outputs = {}
    for u, spec in contract.ups.items():
        fields = []
        for col in spec["fields"]:
            s = sizes[col]
            fields.append({"name": re.sub(rf"^{re.escape(u)}_x_", "", _feature_name(col)), "kind": "categorical",
                           "source": col, "embedding_dim": s.dim, "encoding": _encoding(s)})
        if contract.request_time_column:
            time_outputs[u] = f"{u}_x_time_delta_log1p_seconds"
            fields.append({"name": "age", "kind": "dense", "source": time_outputs[u], "dimension": 1})
        seq = {"name": u, "fields": fields, "max_length": int(spec.get("max_length", 100)),
               "sequence_order": "newest_to_oldest", "truncation": "head"}
        if onetrans:
            seq["encoder"] = "raw"
        else:
            seq.update({"encoder": "mean_pool", "pool_dim": 64})
        if contract.request_time_column:
            seq["time_delta_field"] = "age"
        seqs.append(seq)
    adapter = {"callable": "mdl_b200.data.agg:AggAdapter",
               "options": {"context_features": [c for c in contract.context_features],
                           "item_features": [c for c in contract.item_features],
                           "ups_types": list(contract.ups), "labels": dict(contract.labels),
                           "sequence_max_lengths": {u: int(s.get("max_length", 100)) for u, s in contract.ups.items()},
                           "candidate_position_column": "candidate_position"}}
    if contract.request_time_column:
        adapter["options"].update({"request_time_column": contract.request_time_column,
                                   "time_delta_outputs": time_outputs, "time_delta_transform": "log1p_seconds"})
    reader = {"shuffle_buffer_rows": 8 * batch_size, "agg_direct_mode": "direct", "pin_memory": True,
              "prefetch_batches": 4, "deduplicate_request_features": bool(contract.request_id)}
    m: dict[str, Any] = {
        "runtime": {"device": "cuda", "precision": "bf16", "distributed": "none"},
        "data": {"train": {"format": "adapter_parquet", "inputs": list(inputs or []), "labels": dict(contract.labels),
                           "adapter": adapter, "reader": reader,
                           **({"request_id": contract.request_id} if contract.request_id else {})}},
        "features": feats,
        "sequences": seqs,
        "model": {"name": family},
        "training": {"batch_size": batch_size, "embedding_distribution": "sharded",
                     "embedding_sharding": {"strategy": "auto", "table_wise_max_rows": 65536},
                     "sparse_optimizer": "rowwise_adagrad", "dense_optimizer": "rmsprop", "lr_dense": 1e-4,
                     "lr_sparse": 0.05, "lr_warmup_steps": 5000, "rmsprop_alpha": 0.99999,
                     "loss_reduction": "mean_per_task"},
    }
    token_inputs = names + [q["name"] for q in seqs if not onetrans]
    if onetrans:
        d = token_dim or 256
        m["tokenization"] = {"feature_tokenizer": "auto_split", "num_feature_tokens": 32,
                             "sequence_tokens": [{"name": q["name"], "inputs": [q["name"]]} for q in seqs]}
        m["model"].update({"embedding_dim": 64, "token_dim": d, "num_layers": layers or 6, "num_heads": max(1, d // 32),
                           "hidden_dim": 4 * d, "task_head_hidden_dim": 4 * d, "ffn_activation": "gelu",
                           "ns_tokenizer": "auto_split", "num_ns_tokens": 32, "use_pyramid": True,
                           "pyramid_schedule": "linear", "use_sep_tokens": len(seqs) > 1,
                           "max_position_embeddings": sum(q["max_length"] for q in seqs) + len(seqs) + 32})
    else:
        d = token_dim or 768
        T = int(min(32, max(8, 1 << math.ceil(math.log2(max(1, len(token_inputs) / 8))))))
        m["tokenization"] = {"feature_tokenizer": "rankmixer", "num_feature_tokens": T,
                             "feature_token_inputs": token_inputs}
        m["model"].update({"embedding_dim": 64, "token_dim": d, "num_layers": layers or 2, "num_heads": T,
                           "hidden_dim": 2 * d, "task_head_hidden_dim": 2 * d, "ffn_activation": "gelu"})
    if mdl:
        col = contract.fine_scene_column if fine else contract.scene_column
        scenes = contract.fine_scenes if fine else contract.scenes
        if not col or not scenes:
            raise ValueError(f"{family}: the contract needs {'fine_' if fine else ''}scene_column and "
                             f"{'fine_' if fine else ''}scenes")
        _add_scenarios(m, col, scenes, list(contract.labels), onetrans)
        if col not in contract.context_features and col not in contract.item_features:
            adapter["options"].setdefault("request_columns", []).append(col)   # expanded per candidate
    elif fine:
        raise ValueError("fine siblings exist for the MDL families only")
    return m


def _add_scenarios(m: dict, column: str, scenes: list[str], tasks: list[str], onetrans: bool) -> None:
    """Scene id (scope ``scenario``) feeding one token per scene plus the global token;
    one scene-scoped prior table per scene and one task-scoped prior per task (the
    token-unique prior inputs), all read from the scene column."""

    feats = m["features"]
    n = len(scenes)
    feats.append({"name": "scene_id", "kind": "categorical", "source": column, "embedding_dim": 64,
                  "embedding_scope": "scenario", "encoding": {"type": "hash", "num_buckets": max(8, 2 * n)}})
    for s in scenes:
        feats.append({"name": f"prior_{s}", "kind": "categorical", "source": column, "embedding_dim": 64,
                      "embedding_scope": "scenario", "encoding": {"type": "hash", "num_buckets": max(8, 2 * n)}})
    for t in tasks:
        feats.append({"name": f"prior_{t}", "kind": "categorical", "source": column, "embedding_dim": 64,
                      "embedding_scope": "task", "encoding": {"type": "hash", "num_buckets": max(8, 2 * n)}})
    m["scenarios"] = {"names": list(scenes), "source": column}
    m["tokenization"]["scenario_tokens"] = (
        [{"name": s, "important_inputs": ["scene_id"], "prior_inputs": [f"prior_{s}"]} for s in scenes]
        + [{"name": "global", "important_inputs": ["scene_id"]}])
    m["tokenization"]["task_tokens"] = [{"name": t, "important_inputs": [f"prior_{t}"],
                                         "prior_inputs": [f"prior_{t}"]} for t in tasks]
    m["model"].update({"use_task_tokens": True, "use_scenario_tokens": True, "use_global_scenario_token": True,
                       "use_task_feature_interaction": True, "use_scenario_feature_interaction": True,
                       "tokens_per_scenario": 1})
    if onetrans:
        m["model"]["experimental_model_acknowledged"] = True


# ------------------------------------------------------------------ memory
def memory_summary(mapping: Mapping, *, world_size: int, budget_gb: float | None = None) -> dict:
    """Embedding rows and bytes, and the largest rank's share under the sharding plan."""

    from ..parallel.sharding import EmbeddingTableSpec, embedding_local_bytes, plan_embedding_shards

    tables = []
    for f in mapping.get("features", []):
        if f.get("kind") == "categorical":
            enc = f.get("encoding") or {}
            rows = int(enc.get("num_buckets") or (enc.get("max_id", 0) + 1))
            tables.append(EmbeddingTableSpec(f["name"], rows, int(f["embedding_dim"])))
    for q in mapping.get("sequences", []):
        for fl in q.get("fields", []):
            if fl.get("kind") == "categorical":
                enc = fl.get("encoding") or {}
                rows = int(enc.get("num_buckets") or (enc.get("max_id", 0) + 1))
                tables.append(EmbeddingTableSpec(f"{q['name']}.{fl['name']}", rows, int(fl["embedding_dim"])))
    shard = (mapping.get("training") or {}).get("embedding_sharding") or {}
    plan = plan_embedding_shards(tables, world_size=world_size, strategy=shard.get("strategy", "auto"),
                                 table_wise_max_rows=int(shard.get("table_wise_max_rows", 65536)),
                                 optimizer_state_layout="rowwise")
    per_rank = [0] * world_size
    for t in tables:
        s = plan.tables[t.name]
        for r in range(world_size):
            per_rank[r] += embedding_local_bytes(rows=s.local_rows(t.num_embeddings, r), embedding_dim=t.embedding_dim,
                                                 weight_element_size=4, optimizer_state_layout="rowwise")
    out = {"tables": len(tables), "rows": sum(t.num_embeddings for t in tables),
           "bytes": sum(embedding_local_bytes(rows=t.num_embeddings, embedding_dim=t.embedding_dim,
                                              weight_element_size=4, optimizer_state_layout="rowwise")
                        for t in tables),
           "world_size": world_size, "max_rank_bytes": max(per_rank), "min_rank_bytes": min(per_rank)}
    if budget_gb is not None:
        out["budget_bytes"] = int(budget_gb * 2 ** 30)
        out["fits"] = out["max_rank_bytes"] <= out["budget_bytes"]
    return out


def render(mapping: Mapping, summary: Mapping, sizes: Mapping[str, Sizing]) -> str:
    """YAML text with the sizing provenance and the memory summary as a header comment."""

    import yaml

    how: dict[str, int] = {}
    for s in sizes.values():
        how[s.source] = how.get(s.source, 0) + 1
    lines = ["# generated by `python -m mdl_b200 build-config`",
             "# table sizes from: " + ", ".join(f"{k} ({v})" for k, v in sorted(how.items()))]
    if how.get("name estimate"):
        lines.append("# ESTIMATED: some tables were sized from column names; profile the data "
                     "(profile-data, recommend-shapes) before production training")
    lines.append("# embeddings: {tables} tables, {rows:,} rows, {gb:.2f} GiB with row-wise Adagrad state; "
                 "largest rank at world size {world_size}: {rgb:.2f} GiB".format(
                     gb=summary["bytes"] / 2 ** 30, rgb=summary["max_rank_bytes"] / 2 ** 30, **summary))
    if "fits" in summary:
        lines.append(f"# per-GPU budget {summary['budget_bytes'] / 2 ** 30:.1f} GiB: "
                     + ("fits" if summary["fits"] else "DOES NOT FIT"))
    return "\n".join(lines) + "\n" + yaml.safe_dump(copy.deepcopy(dict(mapping)), sort_keys=False)
