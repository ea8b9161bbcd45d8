"""The whole-array tensorizer against a per-row definition of the same rules (CPU):
scalar and list categoricals with nulls (a null is one padding id), ``head`` / ``tail``
truncation of bags, identity clipping, low-bit ``pre_hashed`` buckets, salted ``hash``
of the value's text, fitted vocabularies, dense scalars and lists with a presence column,
labels with nulls (mask 0), a label-mask column and named scenes."""

from hashlib import sha256

import numpy as np
import pyarrow as pa
import pytest

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.parquet import Tensorizer
from mdl_b200.ops.embedding import LookupFeature, LookupPlan


def _config():
    feats = [
        {"name": "uid", "kind": "categorical", "source": "uid", "embedding_dim": 4,
         "encoding": {"type": "identity", "max_id": 50, "out_of_range": "clip"}},
        {"name": "ph", "kind": "categorical", "source": "ph", "embedding_dim": 4,
         "encoding": {"type": "pre_hashed", "num_buckets": 64}},
        {"name": "hs", "kind": "categorical", "source": "hs", "embedding_dim": 4,
         "encoding": {"type": "hash", "num_buckets": 97, "salt": "s1"}},
        {"name": "voc", "kind": "categorical", "source": "voc", "embedding_dim": 4,
         "encoding": {"type": "vocab"}},
        {"name": "tags_t", "kind": "categorical", "source": "tags", "embedding_dim": 4, "pooling": "mean",
         "max_length": 3, "truncation": "tail", "encoding": {"type": "identity", "max_id": 200}},
        {"name": "tags_h", "kind": "categorical", "source": "tags", "embedding_dim": 4, "pooling": "mean",
         "max_length": 2, "truncation": "head", "encoding": {"type": "hash", "num_buckets": 31}},
        {"name": "age", "kind": "dense", "source": "age", "dimension": 1},
        {"name": "vec", "kind": "dense", "source": "vec", "dimension": 3, "presence": False},
    ]
    m = {"data": {"train": {"format": "flat_parquet", "inputs": [], "labels": {"click": "click", "buy": "buy"},
                            "label_masks": {"buy": "buy_mask"}}},
         "features": feats,
         "scenarios": {"source": "scene", "names": ["home", "search", "feed"]},
         "model": {"name": "rankmixer", "token_dim": 16, "num_layers": 1, "hidden_dim": 32},
         "tokenization": {"feature_tokenizer": "rankmixer", "num_feature_tokens": 2},
         "runtime": {"device": "cpu", "precision": "fp32"}, "training": {"batch_size": 16}}
    return app_config_from_mapping(m)


def _table(rows: int, seed: int):
    rng = np.random.default_rng(seed)

    def maybe(v, p=0.2):
        return None if rng.random() < p else v

    tags = []
    for _ in range(rows):
        r = rng.random()
        if r < 0.15:
            tags.append(None)
        elif r < 0.25:
            tags.append([])
        else:
            tags.append([maybe(int(x), 0.1) for x in rng.integers(1, 150, size=rng.integers(1, 6))])
    return pa.table({
        "uid": pa.array([maybe(int(x)) for x in rng.integers(-3, 80, size=rows)], type=pa.int64()),
        "ph": pa.array([maybe(int(x)) for x in rng.integers(0, 1 << 40, size=rows)], type=pa.int64()),
        "hs": pa.array([maybe(f"v{int(x)}") for x in rng.integers(0, 30, size=rows)], type=pa.string()),
        "voc": pa.array([maybe(f"w{int(x)}") for x in rng.integers(0, 8, size=rows)], type=pa.string()),
        "tags": pa.array(tags, type=pa.list_(pa.int64())),
        "age": pa.array([maybe(float(x)) for x in rng.normal(size=rows)], type=pa.float64()),
        "vec": pa.array([maybe([maybe(float(x), 0.1) for x in rng.normal(size=rng.integers(1, 5))])
                         for _ in range(rows)], type=pa.list_(pa.float32())),
        "click": pa.array([maybe(float(x)) for x in rng.integers(0, 2, size=rows)], type=pa.float32()),
        "buy": pa.array([bool(x) for x in rng.integers(0, 2, size=rows)], type=pa.bool_()),
        "buy_mask": pa.array([maybe(float(x)) for x in rng.integers(0, 2, size=rows)], type=pa.float32()),
        "scene": pa.array([maybe(["home", "search", "feed", "other"][int(x)]) for x in rng.integers(0, 4, rows)]),
    })


def _bucket(text: str, n: int, salt=None) -> int:
    prefix = "" if salt is None else f"{salt}:"
    return int.from_bytes(sha256((prefix + text).encode()).digest()[:8], "little") % n + 1


def _encode_one(f, v, vocab):
    if v is None:
        return 0
    e = f.encoding
    if e.type == "identity":
        v = int(v)
        if v > e.max_id:
            v = e.max_id if e.out_of_range == "clip" else 0
        return max(v, 0)
    if e.type == "pre_hashed":
        return (int(v) & (e.num_buckets - 1)) + 1
    if e.type == "hash":
        return _bucket(str(v), e.num_buckets, e.salt)
    return vocab.get(str(v), 0)


def _expected(cfg, table, vocab):
    rows = table.num_rows
    ids, lengths = [], []
    dense_cols = []
    for f in cfg.features:
        col = table.column(f.source).to_pylist()
        if f.kind == "dense":
            d = f.dimension
            out = np.zeros((rows, d + (1 if f.presence else 0)), np.float32)
            for i, v in enumerate(col):
                if v is None:
                    continue
                vals = v if isinstance(v, list) else [v]
                vals = [0.0 if x is None else float(x) for x in vals[:d]]
                out[i, :len(vals)] = vals
                if f.presence:
                    out[i, d] = 1.0
            dense_cols.append(out)
            lengths.append(np.zeros(rows, np.int64))
            continue
        ln = np.zeros(rows, np.int64)
        for i, v in enumerate(col):
            if isinstance(v, list):
                if f.max_length is not None and len(v) > f.max_length:
                    v = v[-f.max_length:] if f.truncation == "tail" else v[:f.max_length]
                ids += [_encode_one(f, x, vocab) for x in v]
                ln[i] = len(v)
            else:
                ids.append(_encode_one(f, v, vocab))
                ln[i] = 1
        lengths.append(ln)
    labels = np.zeros((rows, 2), np.float32)
    mask = np.ones((rows, 2), np.float32)
    for t, name in enumerate(["click", "buy"]):
        for i, v in enumerate(table.column(name).to_pylist()):
            if v is None:
                mask[i, t] = 0.0
            else:
                labels[i, t] = float(v)
    mask[:, 1] *= np.array([0.0 if v is None else v for v in table.column("buy_mask").to_pylist()], np.float32)
    names = {"home": 0, "search": 1, "feed": 2}
    scen = np.array([names.get(str(v), 0) for v in table.column("scene").to_pylist()], np.int64)
    return np.array(ids, np.int64), np.concatenate(lengths), np.concatenate(dense_cols, 1), labels, mask, scen


@pytest.mark.parametrize("seed,rows,chunks", [(0, 64, 1), (1, 200, 3), (2, 7, 1)])
def test_tensorizer_matches_row_definition(seed, rows, chunks):
    cfg = _config()
    dense_col = 0
    plan_feats = []
    for f in cfg.features:
        if f.kind == "dense":
            plan_feats.append(LookupFeature(f.name, None, width=f.dimension, dense_col=dense_col))
            dense_col += f.dimension + (1 if f.presence else 0)
        else:
            plan_feats.append(LookupFeature(f.name, f.name, width=4))
    plan = LookupPlan(plan_feats, out_width=0, dense_width=dense_col)
    vocab = {f"w{k}": k + 1 for k in range(5)}           # w5..w7 are unseen -> 0
    tz = Tensorizer(cfg, plan, vocab_maps={"voc": vocab})
    table = _table(rows, seed)
    if chunks > 1:  # several record batches and a sliced view, as the batch iterator hands them over
        parts = [table.slice(k * rows // chunks, rows // chunks) for k in range(chunks)]
        table = pa.concat_tables(parts + [table.slice(chunks * (rows // chunks))]).slice(3, rows - 5)
    b = tz(table)
    ids, lengths, dense, labels, mask, scen = _expected(cfg, table, vocab)
    n = table.num_rows
    np.testing.assert_array_equal(np.diff(b.offsets.numpy()), lengths)
    np.testing.assert_array_equal(b.ids.numpy()[:len(ids)], ids)
    np.testing.assert_allclose(b.dense.numpy(), dense, rtol=1e-6)
    np.testing.assert_array_equal(b.labels.numpy(), labels)
    np.testing.assert_array_equal(b.label_mask.numpy(), mask)
    np.testing.assert_array_equal(b.scenario_id.numpy(), scen)
    assert b.rows == n


@pytest.mark.parametrize("truncation,order,anchor", [("tail", "oldest_to_newest", True),
                                                     ("head", "newest_to_oldest", True),
                                                     ("tail", "oldest_to_newest", False)])
def test_sequences_null_anchor_and_request_rows(truncation, order, anchor):
    """Event sequences: steps whose anchor value is null leave every field (before the
    ``max_length`` window), other nulls are padding values; with request deduplication one
    sequence row per distinct request id, in order of first appearance, plus the
    candidate -> request map."""

    L = 4
    m = {"data": {"train": {"format": "flat_parquet", "inputs": [], "labels": {"click": "click"},
                            "request_id": "rid", "reader": {"deduplicate_request_features": True}}},
         "features": [{"name": "f", "kind": "categorical", "source": "f", "embedding_dim": 4,
                       "encoding": {"type": "identity", "max_id": 100}}],
         "sequences": [{"name": "h", "max_length": L, "truncation": truncation, "sequence_order": order,
                        "encoder": "mean_pool", "pool_dim": 8,
                        **({"null_anchor_field": "item"} if anchor else {}),
                        "fields": [{"name": "item", "kind": "categorical", "source": "h_item", "embedding_dim": 4,
                                    "encoding": {"type": "identity", "max_id": 1000}},
                                   {"name": "dt", "kind": "dense", "source": "h_dt", "dimension": 1}]}],
         "model": {"name": "rankmixer", "token_dim": 16, "num_layers": 1, "hidden_dim": 32},
         "tokenization": {"feature_tokenizer": "rankmixer", "num_feature_tokens": 2},
         "runtime": {"device": "cpu", "precision": "fp32"}, "training": {"batch_size": 16}}
    cfg = app_config_from_mapping(m)
    rng = np.random.default_rng(5)
    rows = 40
    rid = [f"r{int(x)}" for x in rng.integers(0, 12, size=rows)]
    items, dts = {}, {}
    for r in sorted(set(rid)):
        n = int(rng.integers(0, 9))
        items[r] = [None if rng.random() < 0.3 else int(x) for x in rng.integers(1, 999, size=n)]
        dts[r] = [None if rng.random() < 0.2 else float(x) for x in rng.normal(size=n)]
    table = pa.table({"f": pa.array(rng.integers(1, 50, size=rows), type=pa.int64()),
                      "rid": pa.array(rid),
                      "h_item": pa.array([items[r] for r in rid], type=pa.list_(pa.int64())),
                      "h_dt": pa.array([dts[r] for r in rid], type=pa.list_(pa.float64())),
                      "click": pa.array(rng.integers(0, 2, size=rows).astype(np.float32))})
    plan = LookupPlan([LookupFeature("f", "f", width=4)], out_width=4)
    b = Tensorizer(cfg, plan, seq_names=["h"])(table.slice(2))
    seq = b.sequences["h"]
    order_seen = list(dict.fromkeys(rid[2:]))
    np.testing.assert_array_equal(seq["row_indices"].numpy(), [order_seen.index(r) for r in rid[2:]])
    ids = seq["ids"].numpy().reshape(-1, L)
    dense = seq["dense"].numpy().reshape(-1, L)
    assert ids.shape[0] == len(order_seen)
    for k, r in enumerate(order_seen):
        steps = list(zip(items[r], dts[r]))
        if anchor:
            steps = [s for s in steps if s[0] is not None]
        steps = steps[-L:] if truncation == "tail" else steps[:L]
        if order == "newest_to_oldest":
            steps = steps[::-1]
        want_ids = [0] * (L - len(steps)) + [0 if i is None else i for i, _ in steps]
        want_dt = [0.0] * (L - len(steps)) + [0.0 if d is None else d for _, d in steps]
        assert seq["lengths"][k] == len(steps)
        np.testing.assert_array_equal(ids[k], want_ids)
        np.testing.assert_allclose(dense[k], want_dt, rtol=1e-6)
