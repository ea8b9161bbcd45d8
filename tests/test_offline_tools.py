"""Offline tools: data profiles, embedding-shape and encoding recommendations, batch-size
tuning and benchmark summaries (CPU)."""

import json
import math

import numpy as np
import pytest

from mdl_b200.benchmark.tools import load_reports, markdown, summarize_benchmarks
from mdl_b200.data.profile import (collision_fraction, heaps_exponent, recommend_encodings, recommend_shapes,
                                   splitmix64)


def test_splitmix64_reference_value_and_collisions():
    # first output of SplitMix64 from state 0 (the generator's published test value)
    assert int(splitmix64(np.array([0], dtype=np.uint64))[0]) == 0xE220A8397B1DCDAF
    v = np.arange(0, 1 << 12, dtype=np.uint64) << np.uint64(8)   # low 8 bits all zero
    assert collision_fraction(v, 8) == 1.0                          # raw low bits: one slot
    assert collision_fraction(splitmix64(v), 16) < 0.2              # remixed: spread out


def test_heaps_and_shape_recommendation():
    assert heaps_exponent(100, 400, 1000, 16000) == pytest.approx(0.5)
    small = {"rows": 1000, "features": {"a": {"distinct": 100}, "b": {"distinct": 50}}}
    large = {"rows": 16000, "features": {"a": {"distinct": 400}, "b": {"distinct": 50}}}
    rec = recommend_shapes(small, large, horizon_rows=256000, load=0.5)
    a, b = rec["features"]["a"], rec["features"]["b"]
    assert a["growth_exponent"] == pytest.approx(0.5) and a["projected_distinct"] == 1600
    assert a["num_embeddings"] == 4096 and a["projected_load"] <= 0.5         # 2^ceil(log2(3200))
    assert b["growth_exponent"] == 0.0 and b["num_embeddings"] == 128         # saturated vocabulary
    assert a["embedding_dim"] % 8 == 0 and 8 <= a["embedding_dim"] <= 128
    assert a["embedding_dim"] == int(round(6 * 1600 ** 0.25 / 8)) * 8


def test_encoding_recommendation():
    prof = {"features": {
        "dense_ids": {"distinct": 900, "min_id": 0, "max_id": 999, "collisions_raw": {"20": 0.0},
                      "collisions_remixed": {"20": 0.0}},
        "words": {"distinct": 5000, "min_id": -9e18, "max_id": 9e18, "collisions_raw": {"20": 0.0},
                  "collisions_remixed": {"20": 0.0}},
        "good_hash": {"distinct": 10 ** 6, "min_id": -9e18, "max_id": 9e18, "collisions_raw": {"20": 0.6},
                      "collisions_remixed": {"20": 0.6}},
        "bad_hash": {"distinct": 10 ** 6, "min_id": 0, "max_id": 2 ** 40, "collisions_raw": {"20": 0.99},
                     "collisions_remixed": {"20": 0.6}}}}
    rec = recommend_encodings(prof)
    assert [rec[k]["encoding"] for k in ("dense_ids", "words", "good_hash", "bad_hash")] == [
        "identity", "vocab", "pre_hashed", "remixed_pre_hashed"]


def test_summarize_benchmarks(tmp_path):
    lines = [{"metric": "train samples/sec", "value": 100.0, "n_gpus": 1, "config": {"model": "m"}},
             {"metric": "train samples/sec", "value": 190.0, "n_gpus": 2, "config": {"model": "m"}},
             {"metric": "train samples/sec", "value": 360.0, "n_gpus": 4, "config": {"model": "m"}},
             {"impl": "reference", "metric": "train samples/sec", "value": 10.0, "n_gpus": 1,
              "config": {"model": "m"}}]
    p = tmp_path / "b.log"
    p.write_text("noise\n" + "\n".join(json.dumps(x) for x in lines) + "\n")
    s = summarize_benchmarks(load_reports([str(p)]))
    eff = {(r["impl"], r["n_gpus"]): r["weak_scaling_efficiency"] for r in s["rows"]}
    assert eff[("mdl_b200", 2)] == 0.95 and eff[("mdl_b200", 4)] == 0.9 and eff[("reference", 1)] == 1.0
    assert "| mdl_b200 | m |" in markdown(s)


def _run(*args):
    import subprocess
    import sys

    out = subprocess.run([sys.executable, "-m", "mdl_b200", *args], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]


def test_cli_profile_recommend_and_tune(tmp_path):
    data = tmp_path / "data"
    _run("make-synthetic-parquet", "--benchmark", "1", "--files", "1", "--rows", "512", "--out", str(data))
    over = ["--benchmark-config", "1", "--set", f"data.train.inputs=[{str(data)}]"]
    prof = tmp_path / "p.json"
    res = _run("profile-data", *over, "--max-rows", "400", "--out", str(prof))[-1]
    assert res["rows"] == 400 and res["features"] > 0
    report = json.loads(prof.read_text())
    f0 = next(iter(report["features"].values()))
    assert 0 < f0["distinct"] <= f0["values"] and set(f0["collisions_raw"]) == {"16", "18", "20", "22", "24"}
    enc = _run("recommend-encodings", "--profile", str(prof))
    assert enc and all(v["encoding"] in ("identity", "vocab", "pre_hashed", "remixed_pre_hashed")
                       for v in enc[-1].values())
    tuned = _run("tune-batch-size", "--benchmark-config", "1", "--batch-sizes", "32", "64", "--steps", "2",
                 "--warmup", "1")[-1]
    assert [r["batch_size"] for r in tuned["results"]] == [32, 64]
    assert tuned["recommended_batch_size"] in (32, 64)
    assert not math.isnan(tuned["results"][0]["samples_per_s"])
