"""Offline data tools: categorical profiles of Parquet inputs and the embedding-shape and
encoding recommendations built on them.

Counterparts of the reference's offline scripts ``scripts/profile_prehashed_parquet.py``,
``scripts/recommend_embedding_shapes.py`` and ``scripts/recommend_categorical_encodings.py``
(redesigned; the reports are this framework's own JSON):

* ``profile_parquet``: per categorical feature (and sequence field) of a config, over the
  first ``max_rows`` rows of the inputs -- values seen, distinct values, the largest id,
  null rows, and for candidate power-of-two table sizes the fraction of distinct values
  that collide when the id's low bits index the table, raw and after a SplitMix64 remix
  (Steele, Lea, Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014).
* ``recommend_shapes``: two profiles of nested prefixes of the same data give a Heaps'
  law growth exponent per feature (``V(n) = K n^beta``, Heaps 1978); the cardinality is
  projected to a horizon and the table gets the smallest power of two that keeps the
  projected load at ``load`` and an embedding width from the fourth-root rule
  ``~ 6 * V^(1/4)`` (Google's feature-column guideline), rounded to a multiple of 8 and
  clipped to ``[min_dim, max_dim]``.
* ``recommend_encodings``: ``identity`` for dense small id ranges, ``vocab`` for small
  vocabularies, ``pre_hashed`` (low bits) when raw low bits collide no more than a remix
  would, else ``remixed_pre_hashed``.
"""

from __future__ import annotations

import math

import numpy as np

MASK64 = (1 << 64) - 1


def splitmix64(x: np.ndarray) -> np.ndarray:
    """SplitMix64 finaliser of uint64 values (vectorised)."""

    z = (x.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15))
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def collision_fraction(values: np.ndarray, bits: int) -> float:
    """Fraction of distinct values sharing a table row with another value when the low
    ``bits`` bits index the table."""

    if values.size == 0:
        return 0.0
    slots = values & np.uint64((1 << bits) - 1)
    _, counts = np.unique(slots, return_counts=True)
    return float(counts[counts > 1].sum()) / float(values.size)


def _flat_values(col) -> tuple[np.ndarray, int, int, float]:
    """(distinct-able uint64 values, null rows, list depth, mean length of the innermost lists)."""

    import pyarrow as pa
    import pyarrow.compute as pc

    col = col.combine_chunks() if isinstance(col, pa.ChunkedArray) else col
    nulls = int(col.null_count)
    depth, inner = 0, 0.0
    while pa.types.is_list(col.type) or pa.types.is_large_list(col.type):
        depth += 1
        ln = pc.list_value_length(col).drop_null()
        inner = float(pc.mean(ln).as_py() or 0.0) if len(ln) else 0.0
        col = col.flatten()
    if pa.types.is_integer(col.type):
        vals = np.asarray(col.drop_null().to_numpy(zero_copy_only=False)).astype(np.int64).view(np.uint64)
    else:  # strings or other: a stable 64-bit hash of the text
        from pandas.util import hash_array

        vals = hash_array(np.asarray(col.drop_null().cast(pa.string()).to_numpy(zero_copy_only=False),
                                     dtype=object), categorize=False)
    return vals.astype(np.uint64), nulls, depth, inner


def profile_parquet(config, paths, *, max_rows: int = 1_000_000, bucket_bits=(16, 18, 20, 22, 24)) -> dict:
    """Categorical profile of the first ``max_rows`` rows of ``paths`` (see module doc)."""

    columns: dict[str, str] = {}
    for f in config.features:
        if f.kind == "categorical":
            columns[f.source or f.name] = f.name
    for q in config.sequences:
        for fl in q.fields:
            if fl.kind == "categorical":
                columns[fl.source or fl.name] = f"{q.name}.{fl.name}"
    return profile_columns(paths, columns, max_rows=max_rows, bucket_bits=bucket_bits)


def profile_columns(paths, columns: dict[str, str], *, max_rows: int = 1_000_000,
                    bucket_bits=(16, 18, 20, 22, 24)) -> dict:
    """The profile of named columns (``{column: report name}``); besides the counts, each
    entry has the column's list ``depth`` and the mean length of its innermost lists
    (``inner_mean_length``: bag length in a flat file, values per request / candidate /
    event position in an agg file)."""

    import pyarrow.parquet as pq

    seen: dict[str, list[np.ndarray]] = {c: [] for c in columns}
    nulls = {c: 0 for c in columns}
    shape = {c: [0, 0.0, 0] for c in columns}          # depth, sum of inner means, row groups
    rows = 0
    for path in paths:
        pf = pq.ParquetFile(path)
        present = [c for c in columns if c in pf.schema_arrow.names]
        for i in range(pf.num_row_groups):
            if rows >= max_rows:
                break
            t = pf.read_row_group(i, columns=present)
            take = min(t.num_rows, max_rows - rows)
            t = t.slice(0, take)
            rows += take
            for c in present:
                v, n, depth, inner = _flat_values(t.column(c))
                seen[c].append(v)
                nulls[c] += n
                shape[c][0] = max(shape[c][0], depth)
                shape[c][1] += inner
                shape[c][2] += 1
        if rows >= max_rows:
            break
    report = {"rows": rows, "features": {}}
    for c, name in columns.items():
        vals = np.concatenate(seen[c]) if seen[c] else np.zeros(0, np.uint64)
        distinct = np.unique(vals)
        raw = {str(b): round(collision_fraction(distinct, b), 6) for b in bucket_bits}
        mixed = {str(b): round(collision_fraction(splitmix64(distinct), b), 6) for b in bucket_bits}
        report["features"][name] = {
            "column": c, "values": int(vals.size), "distinct": int(distinct.size), "null_rows": nulls[c],
            "max_id": int(distinct.view(np.int64).max()) if distinct.size else 0,
            "min_id": int(distinct.view(np.int64).min()) if distinct.size else 0,
            "depth": shape[c][0], "inner_mean_length": round(shape[c][1] / max(1, shape[c][2]), 4),
            "collisions_raw": raw, "collisions_remixed": mixed,
        }
    return report


def heaps_exponent(v_small: int, v_large: int, n_small: int, n_large: int) -> float:
    """``beta`` of ``V(n) = K n^beta`` through two (rows, distinct) points, in [0, 1]."""

    if v_small <= 0 or v_large <= 0 or n_large <= n_small or n_small <= 0:
        return 1.0
    beta = math.log(v_large / v_small) / math.log(n_large / n_small)
    return float(min(1.0, max(0.0, beta)))


def recommend_shapes(small: dict, large: dict, *, horizon_rows: int, load: float = 0.5, min_dim: int = 8,
                     max_dim: int = 128, max_bits: int = 30) -> dict:
    """Per-feature table sizes and embedding widths from two nested-prefix profiles."""

    out = {"horizon_rows": int(horizon_rows), "load": load, "features": {}}
    for name, lg in large["features"].items():
        sm = small["features"].get(name)
        v2 = max(1, lg["distinct"])
        beta = heaps_exponent(sm["distinct"] if sm else v2, v2, small["rows"], large["rows"]) if sm else 1.0
        projected = v2 * (max(horizon_rows, large["rows"]) / max(1, large["rows"])) ** beta
        bits = max(1, math.ceil(math.log2(max(2.0, projected / load))))
        bits = min(bits, max_bits)
        dim = int(round(6.0 * projected ** 0.25 / 8.0)) * 8
        dim = int(min(max_dim, max(min_dim, dim)))
        out["features"][name] = {"distinct_seen": lg["distinct"], "growth_exponent": round(beta, 4),
                                 "projected_distinct": int(projected), "num_embeddings": 1 << bits,
                                 "embedding_dim": dim, "projected_load": round(projected / (1 << bits), 4)}
    return out


def recommend_encodings(profile: dict, *, identity_max_id: int = 1 << 20, identity_density: float = 0.25,
                        vocab_max: int = 200_000, bits: int = 20) -> dict:
    """One encoding per categorical feature with the evidence behind it."""

    out = {}
    for name, f in profile["features"].items():
        span = f["max_id"] - min(f["min_id"], 0) + 1
        density = f["distinct"] / span if span > 0 else 0.0
        raw = f["collisions_raw"].get(str(bits))
        mixed = f["collisions_remixed"].get(str(bits))
        if 0 <= f["min_id"] and f["max_id"] < identity_max_id and density >= identity_density:
            enc, why = "identity", f"ids within [0, {f['max_id']}] at density {density:.2f}"
        elif f["distinct"] <= vocab_max:
            enc, why = "vocab", f"{f['distinct']} distinct values"
        elif raw is not None and mixed is not None and raw <= 1.1 * mixed + 1e-6:
            enc, why = "pre_hashed", f"low-bit collisions {raw:.4f} vs remixed {mixed:.4f} at {bits} bits"
        else:
            enc, why = "remixed_pre_hashed", f"low-bit collisions {raw} vs remixed {mixed} at {bits} bits"
        out[name] = {"encoding": enc, "reason": why}
    return out
