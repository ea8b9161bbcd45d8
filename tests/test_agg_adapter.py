"""The aggregate ("agg") Parquet layout: expansion of multi-request rows into
candidate rows (request context, candidate items, labels, request ids, candidate
positions, the events each request may see with their time deltas), and training
from seeded mock agg files through the CLI on two gloo ranks."""

import json
import math
import subprocess
import sys

import pyarrow as pa
import pytest
import yaml

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.agg import AggAdapter, AggPlan, write_mock_agg_parquet


def _mapping(path="", batch=32):
    feats = [
        {"name": "site", "kind": "categorical", "source": "site_hn", "embedding_dim": 8,
         "encoding": {"type": "pre_hashed", "num_buckets": 64}},
        {"name": "query_terms", "kind": "categorical", "source": "query_terms_hn", "embedding_dim": 8,
         "pooling": "mean", "max_length": 4, "encoding": {"type": "pre_hashed", "num_buckets": 128}},
        {"name": "goods", "kind": "categorical", "source": "goods_id_hn", "embedding_dim": 8,
         "encoding": {"type": "pre_hashed", "num_buckets": 256}},
        {"name": "price", "kind": "categorical", "source": "price_hn", "embedding_dim": 8,
         "encoding": {"type": "pre_hashed", "num_buckets": 32}},
    ]
    seq = {"name": "impr", "max_length": 8, "encoder": "mean_pool", "pool_dim": 8, "sequence_order": "newest_to_oldest",
           "truncation": "head", "time_delta_field": "age",
           "fields": [{"name": "age", "kind": "dense", "source": "impr_x_time_delta_log1p_seconds", "dimension": 1},
                      {"name": "cat", "kind": "categorical", "source": "impr_x_cat_hn", "embedding_dim": 8,
                       "encoding": {"type": "pre_hashed", "num_buckets": 64}}]}
    adapter = {"callable": "src.dataloader:adapt_mdl_rankmixer_parquet",
               "options": {"context_features": ["site_hn", "query_terms_hn"],
                           "item_features": ["goods_id_hn", "price_hn"], "ups_types": ["impr"],
                           "labels": {"click": "label_click"}, "sequence_max_lengths": {"impr": 8},
                           "request_time_column": "impr_time",
                           "time_delta_outputs": {"impr": "impr_x_time_delta_log1p_seconds"},
                           "time_delta_transform": "log1p_seconds",
                           "candidate_position_column": "candidate_position"}}
    return {"data": {"train": {"format": "adapter_parquet", "inputs": [path] if path else [],
                               "request_id": "search_id", "labels": {"click": "label_click"},
                               "adapter": adapter,
                               "reader": {"deduplicate_request_features": True, "shuffle_buffer_rows": 0}}},
            "features": feats, "sequences": [seq],
            "tokenization": {"feature_tokenizer": "rankmixer", "num_feature_tokens": 4,
                             "feature_token_inputs": ["site", "query_terms", "goods", "price", "impr"]},
            "model": {"name": "rankmixer", "token_dim": 32, "num_layers": 1, "num_heads": 2, "hidden_dim": 64,
                      "task_head_hidden_dim": 16},
            "runtime": {"device": "cpu", "precision": "fp32"},
            "training": {"batch_size": batch, "lr_dense": 1e-3, "lr_warmup_steps": 0, "save_checkpoint": False,
                         "embedding_sharding": {"strategy": "row_wise"}}}


def test_agg_row_expands_to_candidate_rows():
    cfg = app_config_from_mapping(_mapping())
    plan = AggPlan.from_config(cfg)
    assert plan.sequence_columns == {"impr": ["impr_x_cat_hn"]}
    table = pa.table({
        "context_indices": [[10, 20]],
        "target_indices": [[10, 20, 10]],
        "site_hn": [[5, 6]],
        "query_terms_hn": [[[1, 2], [3]]],
        "goods_id_hn": [[100, 200, 300]],
        "price_hn": [[1, 2, 3]],
        "label_click": [[1.0, 0.0, 0.0]],
        "impr_time": [[1000.0, 2000.0]],
        "search_id": [["a", "b"]],
        "impr_x_indices": [[[10], [10, 20], [20]]],
        "impr_x_time": [[900.0, 1500.0, 1990.0]],
        "impr_x_cat_hn": [[7, 8, 9]],
    })
    flat = AggAdapter(plan)(table).to_pydict()
    assert flat["search_id"] == ["a", "b", "a"]
    assert flat["site_hn"] == [5, 6, 5]
    assert flat["query_terms_hn"] == [[1, 2], [3], [1, 2]]
    assert flat["goods_id_hn"] == [100, 200, 300]
    assert flat["label_click"] == [1.0, 0.0, 0.0]
    assert flat["candidate_position"] == [0, 0, 1]
    # request 10 sees events 0 and 1; request 20 sees events 1 and 2
    assert flat["impr_x_cat_hn"] == [[7, 8], [8, 9], [7, 8]]
    ages = flat["impr_x_time_delta_log1p_seconds"]
    assert ages[0] == pytest.approx([math.log1p(100.0), 0.0], abs=1e-5)  # event 1 is after request 10's time
    assert ages[1] == pytest.approx([math.log1p(500.0), math.log1p(10.0)], abs=1e-5)


def test_train_from_mock_agg_files_on_two_gloo_ranks(tmp_path):
    for i in range(2):
        cfg0 = app_config_from_mapping(_mapping())
        write_mock_agg_parquet(cfg0, str(tmp_path / f"agg-{i}.parquet"), rows=160, seed=i, row_group_size=20)
    m = _mapping(str(tmp_path))
    cfg_path = tmp_path / "agg.yaml"
    cfg_path.write_text(yaml.safe_dump(m))
    out = subprocess.run([sys.executable, "-m", "mdl_b200", "train", "--config", str(cfg_path), "--max-steps", "4",
                          "--nproc-per-node", "2", "--master-port", "29587"], capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    done = [l for l in lines if l.get("done")]
    assert done and done[-1]["steps"] == 4, out.stdout[-2000:]
    assert all(math.isfinite(l["loss"]) for l in lines if "loss" in l), out.stdout[-2000:]
