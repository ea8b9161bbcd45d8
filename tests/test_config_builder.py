"""build-config: model config YAMLs of the four families (and the MDL fine siblings) from a
field contract, sized by name estimates or by a profile of raw agg files; every written
config validates, plans its embedding memory, and trains on the agg files it describes."""

import json
import subprocess
import sys

import pytest
import yaml

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.agg import write_mock_agg_parquet
from mdl_b200.data.config_builder import FieldContract, build_config, estimated_bits, memory_summary, size_features

CONTRACT = {
    "request_id": "search_id",
    "request_time_column": "impr_time",
    "context_features": ["site_hn", "query_terms_hn"],
    "item_features": ["goods_id_hn", "price_hn", "cat1_id_hn"],
    "bag_features": ["query_terms_hn"],
    "labels": {"click": "label_click", "buy": "label_buy"},
    "ups": {"impr": {"fields": ["impr_x_goods_id_hn", "impr_x_cat_hn"], "max_length": 16}},
    "scene_column": "scene_hn",
    "scenes": ["home", "search"],
    "fine_scene_column": "fine_scene_hn",
    "fine_scenes": ["home_a", "home_b", "search_a"],
}


def _run(*args):
    return subprocess.run([sys.executable, "-m", "mdl_b200", *args], capture_output=True, text=True, timeout=900)


def test_name_estimates_and_memory_plan():
    c = FieldContract.from_mapping(CONTRACT)
    sizes = size_features(c)
    assert sizes["goods_id_hn"].rows > sizes["cat1_id_hn"].rows > sizes["site_hn"].rows
    assert estimated_bits("goods_id_hn") == 22 and sizes["site_hn"].source == "name estimate"
    assert sizes["query_terms_hn"].bag_length == 16 and sizes["goods_id_hn"].bag_length is None
    m = build_config(c, "mdl_rankmixer", sizes=sizes, token_dim=32, layers=1)
    app_config_from_mapping(m)
    s1 = memory_summary(m, world_size=1, budget_gb=1000.0)
    s8 = memory_summary(m, world_size=8, budget_gb=0.001)
    assert s1["max_rank_bytes"] == s1["bytes"] and s1["fits"]
    assert s8["bytes"] == s1["bytes"] and s8["max_rank_bytes"] < s1["bytes"] and not s8["fits"]
    with pytest.raises(ValueError, match="fine siblings"):
        build_config(c, "rankmixer", sizes=sizes, fine=True)
    with pytest.raises(ValueError, match="both axes"):
        FieldContract.from_mapping({**CONTRACT, "item_features": ["site_hn"]})


def test_cli_builds_every_family_and_trains_from_profile(tmp_path):
    contract = tmp_path / "contract.yaml"
    contract.write_text(yaml.safe_dump(CONTRACT))
    out = _run("build-config", "--contract", str(contract), "--out-dir", str(tmp_path / "est"),
               "--family", "rankmixer")
    assert out.returncode == 2 and "no sizing source" in out.stderr
    out = _run("build-config", "--contract", str(contract), "--out-dir", str(tmp_path / "est"), "--fine",
               "--estimate-from-names", "--token-dim", "32", "--layers", "1", "--batch-size", "32")
    assert out.returncode == 0, out.stderr[-3000:]
    written = json.loads(out.stdout.strip().splitlines()[-1])["configs"]
    names = sorted(p["path"].rsplit("/", 1)[1] for p in written)
    assert names == ["mdl_onetrans.yaml", "mdl_onetrans_fine.yaml", "mdl_rankmixer.yaml", "mdl_rankmixer_fine.yaml",
                     "onetrans.yaml", "rankmixer.yaml"]
    text = (tmp_path / "est" / "rankmixer.yaml").read_text()
    assert text.startswith("# generated") and "ESTIMATED" in text
    fine = yaml.safe_load((tmp_path / "est" / "mdl_rankmixer_fine.yaml").read_text())
    assert fine["scenarios"] == {"names": ["home_a", "home_b", "search_a"], "source": "fine_scene_hn"}
    # mock raw agg files laid out as the contract says, then configs sized from their profile
    est = app_config_from_mapping(yaml.safe_load((tmp_path / "est" / "mdl_rankmixer.yaml").read_text()))
    data = tmp_path / "data"
    data.mkdir()
    for i in range(2):
        write_mock_agg_parquet(est, str(data / f"agg-{i}.parquet"), rows=80, seed=i, row_group_size=20)
    out = _run("build-config", "--contract", str(contract), "--out-dir", str(tmp_path / "prof"), "--family",
               "mdl_rankmixer", "--profile-inputs", str(data), "--token-dim", "32", "--layers", "1",
               "--batch-size", "32", "--inputs", str(data), "--world-size", "2", "--budget-gb", "1")
    assert out.returncode == 0, out.stderr[-3000:]
    text = (tmp_path / "prof" / "mdl_rankmixer.yaml").read_text()
    assert "profile (" in text and "ESTIMATED" not in text and "fits" in text
    m = yaml.safe_load(text)
    by_name = {f["name"]: f for f in m["features"]}
    assert by_name["query_terms"]["pooling"] == "mean"          # nested one level below the request axis
    assert by_name["goods_id"]["encoding"]["num_buckets"] <= 1 << 14   # sized from what the files hold
    m["runtime"].update({"device": "cpu", "precision": "fp32"})
    m["training"].update({"save_checkpoint": False, "lr_warmup_steps": 0})
    cfg_path = tmp_path / "train.yaml"
    cfg_path.write_text(yaml.safe_dump(m))
    out = _run("train", "--config", str(cfg_path), "--max-steps", "2")
    assert out.returncode == 0, out.stderr[-3000:]
    done = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{") and '"done"' in l]
    assert done and done[-1]["steps"] == 2
