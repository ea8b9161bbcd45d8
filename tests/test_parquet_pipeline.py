"""Flat Parquet pipeline on CPU: round trip of synthetic batches, encodings, rank
sharding covering every row group exactly once, vocab fitting, training from Parquet."""

import numpy as np
import pytest
import torch

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import baseline_config
from mdl_b200.data.parquet import (CategoricalEncoder, ParquetBatchIterator, Tensorizer, discover_parquet_inputs,
                                   fit_vocabs, load_vocab_map, plan_row_groups, stable_hash_bucket,
                                   validate_matching_schemas, write_synthetic_parquet)
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.train.trainer import Trainer


def _setup(tmp_path, n_files=3, rows=256):
    m, spec = baseline_config(1)
    cfg = app_config_from_mapping(m)
    model = build_model(cfg, device="cpu", base_seed=0)
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    batches = [gen.batch(rows) for _ in range(n_files)]
    for i, b in enumerate(batches):
        write_synthetic_parquet(str(tmp_path / f"part-{i}.parquet"), b, model.encoder.batch_plan, cfg, 64)
    return cfg, model, batches


def test_round_trip(tmp_path):
    cfg, model, batches = _setup(tmp_path)
    paths = discover_parquet_inputs([str(tmp_path)])
    assert len(paths) == 3
    tz = Tensorizer(cfg, model.encoder.batch_plan)
    validate_matching_schemas(paths, tz.columns())
    it = ParquetBatchIterator(paths, tz, 256, prefetch=2)
    got = list(it)
    assert len(got) == 3
    for a, b in zip(got, batches):
        assert torch.equal(a.ids, b.ids) and torch.equal(a.offsets, b.offsets)
        torch.testing.assert_close(a.dense, b.dense)
        torch.testing.assert_close(a.labels, b.labels)


def test_same_thread_overlapped_prepare(tmp_path):
    """prefetch 0: batches prepared on the consuming thread; ``schedule_next`` prepares the
    next one between steps (overlap), and the batches equal the threaded reader's."""

    from mdl_b200.data.parquet import OverlappedPrepareIterator

    cfg, model, batches = _setup(tmp_path)
    paths = discover_parquet_inputs([str(tmp_path)])
    tz = Tensorizer(cfg, model.encoder.batch_plan)
    threaded = list(ParquetBatchIterator(paths, tz, 256, prefetch=2))
    it = iter(ParquetBatchIterator(paths, tz, 256, prefetch=0))
    assert isinstance(it, OverlappedPrepareIterator)
    got = []
    for b in it:
        got.append(b)
        it.schedule_next()  # what the training loop does after launching a step
    assert it.prepared_ahead == 2 and len(got) == 3
    for a, b in zip(got, threaded):
        assert torch.equal(a.ids, b.ids) and torch.equal(a.offsets, b.offsets)
    plain = list(ParquetBatchIterator(paths, tz, 256, prefetch=0, overlap=False))
    assert len(plain) == 3 and torch.equal(plain[0].ids, threaded[0].ids)


def test_row_group_sharding_covers_everything_once(tmp_path):
    _setup(tmp_path, n_files=4)
    paths = discover_parquet_inputs([str(tmp_path / "*.parquet")])
    for world in (1, 2, 3, 8):
        seen = []
        for r in range(world):
            seen += [(x.path, x.index) for x in plan_row_groups(paths, r, world)]
        assert len(seen) == len(set(seen)) == 16


def test_encodings():
    from types import SimpleNamespace as NS

    enc = NS(type="pre_hashed", num_buckets=8, max_id=None, out_of_range="error", salt=None)
    e = CategoricalEncoder(NS(name="x", encoding=enc))
    out = e.encode(np.array([-1, 8, None, 17], dtype=object))
    assert out.tolist() == [8, 1, 0, 2]
    h = CategoricalEncoder(NS(name="h", encoding=NS(type="hash", num_buckets=100, salt="s", max_id=None,
                                                    out_of_range="error")))
    assert h.encode(np.array(["a", None, "a"], dtype=object)).tolist() == [stable_hash_bucket("a", 100, "s"), 0,
                                                                             stable_hash_bucket("a", 100, "s")]
    ident = CategoricalEncoder(NS(name="i", encoding=NS(type="identity", max_id=10, out_of_range="clip",
                                                        num_buckets=None, salt=None)))
    assert ident.encode(np.array([3, 12, None], dtype=object)).tolist() == [3, 10, 0]


def test_fit_vocab(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq

    pq.write_table(pa.table({"c": ["x", "y", "x", None, "z", "x", "y"]}), str(tmp_path / "d.parquet"))
    m, _ = baseline_config(1)
    m["features"] = [{"name": "c", "kind": "categorical", "source": "c",
                      "encoding": {"type": "vocab", "min_count": 2, "artifact": "c.parquet"}}]
    m["tokenization"] = {"feature_tokenizer": "rankmixer", "num_feature_tokens": 1}
    cfg = app_config_from_mapping(m)
    out = fit_vocabs(cfg, [str(tmp_path / "d.parquet")], str(tmp_path / "vocab"))
    assert load_vocab_map(out["c"]) == {"x": 1, "y": 2}


def test_train_from_parquet(tmp_path):
    cfg, model, _ = _setup(tmp_path, n_files=2)
    torch.manual_seed(0)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    it = ParquetBatchIterator(discover_parquet_inputs([str(tmp_path)]), Tensorizer(cfg, model.encoder.batch_plan),
                              128, shuffle_rows=256, seed=1)
    losses = [float(tr.train_step(b).loss) for b in it]
    assert len(losses) == 4 and all(np.isfinite(losses))
    assert it.position == len(it.refs)


def _failing_factory(n):
    yield from ()
    raise ValueError(f"broken reader {n}")


def test_host_prepare_process_matches_in_process(tmp_path):
    from mdl_b200.cli import main
    from mdl_b200.config.schema import thaw
    from mdl_b200.data.prepare_process import ProcessBatchIterator, parquet_batches

    data = tmp_path / "data"
    assert main(["make-synthetic-parquet", "--benchmark", "1", "--files", "2", "--rows", "256",
                 "--out", str(data)]) == 0
    m, _ = baseline_config(1)
    m["runtime"]["device"] = "cpu"
    cfg = app_config_from_mapping(m)
    model = build_model(cfg, device="cpu", base_seed=0)
    plan = model.encoder.batch_plan
    paths = discover_parquet_inputs([str(data)])
    ref = list(ParquetBatchIterator(paths, Tensorizer(cfg, plan), 128))
    it = ProcessBatchIterator(parquet_batches, (thaw(cfg), plan, paths, 128, 0, 1, "train", False, 0, 0))
    got = list(it)
    it.close()
    assert len(got) == len(ref) == 4
    for a, b in zip(got, ref):
        assert torch.equal(a.ids, b.ids) and torch.equal(a.offsets, b.offsets) and torch.equal(a.labels, b.labels)
    bad = ProcessBatchIterator(_failing_factory, (7,))
    with pytest.raises(RuntimeError, match="broken reader 7"):
        list(bad)
    bad.close()


def _stalling_factory(seconds):
    import time as _t

    _t.sleep(seconds)
    yield from ()


def test_host_prepare_startup_timeout():
    from mdl_b200.data.prepare_process import ProcessBatchIterator

    # heartbeats keep a slow start alive; a child silent past the limit is reported. The
    # limit leaves room for a spawned child to import its modules on a loaded host (over
    # 12 s with eight test workers on eight cores); the stall outlasts it.
    it = ProcessBatchIterator(_stalling_factory, (40.0,), startup_timeout_s=30.0, beat_s=0.5)
    assert list(it) == []
    it.close()
    it = ProcessBatchIterator(_stalling_factory, (30.0,), startup_timeout_s=1.0, beat_s=60.0)
    with pytest.raises(TimeoutError):
        list(it)
    it.close(join_timeout_s=1.0)


def test_length_buckets_group_rows_by_sequence_work(tmp_path):
    """reader.length_buckets: every batch holds rows of one length bucket, in that
    bucket's batch size; no row is lost or duplicated."""

    import pyarrow as pa
    import pyarrow.parquet as pq

    from mdl_b200.ops.embedding import LookupFeature, LookupPlan

    rng = np.random.default_rng(0)
    n = 200
    lengths = rng.integers(0, 12, size=n)
    hist = [list(range(1, int(k) + 1)) for k in lengths]
    table = pa.table({"f": pa.array(np.arange(1, n + 1) % 50, type=pa.int64()),
                      "hist_item": pa.array(hist, type=pa.list_(pa.int64())),
                      "click": pa.array(rng.integers(0, 2, size=n).astype(np.float32))})
    pq.write_table(table, str(tmp_path / "part.parquet"), row_group_size=50)
    m = {"data": {"train": {"format": "flat_parquet", "inputs": [str(tmp_path)], "labels": {"click": "click"},
                            "reader": {"length_buckets": [{"max_length": 4, "batch_size": 16},
                                                          {"batch_size": 8}]}}},
         "features": [{"name": "f", "kind": "categorical", "source": "f", "embedding_dim": 8,
                       "encoding": {"type": "identity", "max_id": 100}}],
         "sequences": [{"name": "hist", "max_length": 10, "encoder": "mean_pool", "pool_dim": 8,
                        "fields": [{"name": "item", "kind": "categorical", "source": "hist_item", "embedding_dim": 8,
                                    "encoding": {"type": "identity", "max_id": 100}}]}],
         "model": {"name": "rankmixer", "token_dim": 16, "num_layers": 1, "hidden_dim": 32},
         "tokenization": {"feature_tokenizer": "rankmixer", "num_feature_tokens": 2},
         "runtime": {"device": "cpu", "precision": "fp32"}, "training": {"batch_size": 16}}
    cfg = app_config_from_mapping(m)
    plan = LookupPlan([LookupFeature("f", "f", width=8)], out_width=8)
    tz = Tensorizer(cfg, plan, seq_names=["hist"])
    r = cfg.data.train.reader
    it = ParquetBatchIterator([str(tmp_path / "part.parquet")], tz, 16, drop_last=False, shuffle_rows=0,
                              length_buckets=[(b.max_length, b.batch_size) for b in r.length_buckets])
    seen = []
    for b in it:
        ln = b.sequences["hist"]["lengths"].numpy()
        short = ln <= 4
        assert short.all() or (~short).all(), ln
        full = 16 if short.all() else 8
        assert b.rows <= full
        seen += (b.ids[:b.rows].numpy() - 1).tolist()  # f = (row + 1) % 50 identifies rows up to 50
    assert len(seen) == n
