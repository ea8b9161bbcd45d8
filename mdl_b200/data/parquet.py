"""Flat Parquet input pipeline: discovery, rank sharding, encodings, tensorization, prefetch.

Counterparts in the reference: input discovery and schema checks
(``src/dataloader.py:2326-2460``), the Parquet scanner with row-group LPT
sharding, column pruning and threaded prefetch (``:2809``, ``:3232-4045``),
tensorization into one batch per step (``:9200-9600``), categorical encodings
(``src/features.py:150-365``), the pinned host pool and coalesced H2D
(``src/train.py:2923-3108``, ``src/dataloader.py:11586-11790``) and the device
prefetch iterator on a side stream (``src/train.py:4547-4713``).

One sample per Parquet row (``data.train.format: flat_parquet``). A categorical
feature's column holds a scalar or a list (a bag); a dense feature's column a
scalar or a fixed-length list. Batches come out as ``PackedBatch`` in the CSR
order of a lookup plan's batch layout (``FeatureEncoder.batch_plan``), with all
int64 leaves in one pinned buffer and all fp32 leaves in another.
"""

from __future__ import annotations

import glob
import os
import queue
import threading
from dataclasses import dataclass
from hashlib import sha256
from typing import Any, Iterator, Sequence

import numpy as np
import torch

from .batch import PackedBatch


def _pa():
    import pyarrow as pa
    import pyarrow.parquet as pq

    return pa, pq


# ------------------------------------------------------------------ discovery
def discover_parquet_inputs(inputs: Sequence[str]) -> list[str]:
    """Expand globs and directories (recursively) into a sorted list of Parquet files."""

    out: list[str] = []
    for item in inputs:
        if any(ch in item for ch in "*?["):
            out.extend(p for p in glob.glob(item, recursive=True) if os.path.isfile(p))
        elif os.path.isdir(item):
            for root, _dirs, files in os.walk(item):
                out.extend(os.path.join(root, f) for f in files if f.endswith(".parquet"))
        elif os.path.isfile(item):
            out.append(item)
        else:
            raise FileNotFoundError(f"no Parquet input at {item!r}")
    return sorted(dict.fromkeys(out))


def validate_matching_schemas(paths: Sequence[str], required: Sequence[str]) -> None:
    """Every file has every required column, with one type per column across files."""

    _, pq = _pa()
    seen: dict[str, Any] = {}
    for p in paths:
        schema = pq.read_schema(p)
        names = set(schema.names)
        missing = [c for c in required if c not in names]
        if missing:
            raise ValueError(f"{p}: missing columns {missing}")
        for c in required:
            t = schema.field(c).type
            if c in seen and seen[c] != t:
                raise ValueError(f"column {c!r} has type {seen[c]} in one file and {t} in {p}")
            seen[c] = t


@dataclass(frozen=True)
class RowGroupRef:
    path: str
    index: int
    rows: int


def plan_row_groups(paths: Sequence[str], rank: int, world: int, unit: str = "row_group") -> list[RowGroupRef]:
    """Deterministic shard of the input across ranks: longest-processing-time over rows
    (largest units first, ties to the lowest rank), in file order within a rank."""

    _, pq = _pa()
    units: list[tuple[int, int, RowGroupRef]] = []
    order = 0
    for p in paths:
        meta = pq.ParquetFile(p).metadata
        if unit == "file":
            units.append((meta.num_rows, order, RowGroupRef(p, -1, meta.num_rows)))
            order += 1
            continue
        for g in range(meta.num_row_groups):
            units.append((meta.row_group(g).num_rows, order, RowGroupRef(p, g, meta.row_group(g).num_rows)))
            order += 1
    load = [0] * world
    mine: list[tuple[int, RowGroupRef]] = []
    for rows, o, ref in sorted(units, key=lambda u: (-u[0], u[1])):
        r = min(range(world), key=lambda i: (load[i], i))
        load[r] += rows
        if r == rank:
            mine.append((o, ref))
    return [ref for _, ref in sorted(mine, key=lambda x: x[0])]


# ------------------------------------------------------------------ encodings
def stable_hash_bucket(value: Any, num_buckets: int, salt: str | None = None) -> int:
    """``sha256("<salt>:<value>")`` low 8 bytes (little-endian) mod n, plus 1 (0 is padding)."""

    prefix = "" if salt is None else f"{salt}:"
    return int.from_bytes(sha256((prefix + str(value)).encode("utf-8")).digest()[:8], "little") % num_buckets + 1


class CategoricalEncoder:
    """Raw column values -> table ids (0 = padding / null / out of vocabulary)."""

    def __init__(self, feature, vocab: dict[str, int] | None = None) -> None:
        enc = feature.encoding
        self.name = feature.name
        self.type = enc.type if enc is not None else "identity"
        self.enc = enc
        self.vocab = vocab
        if self.type in ("vocab", "shared_vocab") and vocab is None:
            raise ValueError(f"feature {feature.name!r}: vocab encoding needs a fitted vocabulary")
        if self.type == "pre_hashed":
            n = int(enc.num_buckets or 0)
            if n <= 0 or n & (n - 1):
                raise ValueError(f"feature {feature.name!r}: pre_hashed needs a power-of-two num_buckets")

    def encode(self, values: np.ndarray) -> np.ndarray:
        """``values``: 1-D object/int array with None for nulls."""

        n = len(values)
        if n == 0:
            return np.zeros(0, dtype=np.int64)
        enc = self.enc
        if self.type == "identity":
            mask = np.array([v is not None for v in values]) if values.dtype == object else np.ones(n, bool)
            out = np.zeros(n, dtype=np.int64)
            out[mask] = values[mask].astype(np.int64)
            max_id = int(enc.max_id) if enc is not None and enc.max_id else None
            if max_id is not None:
                bad = out > max_id
                if bad.any():
                    policy = enc.out_of_range
                    if policy == "error":
                        raise ValueError(f"feature {self.name!r}: ids above max_id {max_id}")
                    out[bad] = max_id if policy == "clip" else 0
            out[out < 0] = 0
            return out
        if self.type == "pre_hashed":
            mask = np.array([v is not None for v in values]) if values.dtype == object else np.ones(n, bool)
            nb = np.uint64(int(enc.num_buckets))
            raw = np.zeros(n, dtype=np.int64)
            raw[mask] = values[mask].astype(np.int64)
            out = (raw.view(np.uint64) & (nb - np.uint64(1))).astype(np.int64) + 1
            out[~mask] = 0
            return out
        # hash / vocab: map each distinct value once
        keys = np.array(["" if v is None else str(v) for v in values], dtype=object)
        nulls = np.array([v is None for v in values])
        uniq, inv = np.unique(keys, return_inverse=True)
        if self.type == "hash":
            nbk, salt = int(enc.num_buckets), enc.salt
            mapped = np.array([stable_hash_bucket(u, nbk, salt) for u in uniq], dtype=np.int64)
        else:
            mapped = np.array([self.vocab.get(u, 0) for u in uniq], dtype=np.int64)
        out = mapped[inv]
        out[nulls] = 0
        return out

    def encode_arrow(self, values) -> np.ndarray:
        """``values``: a flat Arrow array (nulls allowed). Numeric encodings convert the
        buffer at once; ``hash`` / ``vocab`` encode each distinct value once (Arrow
        ``dictionary_encode``), so the Python work is per distinct value, not per row."""

        import pyarrow as pa
        import pyarrow.compute as pc

        n = len(values)
        if n == 0:
            return np.zeros(0, dtype=np.int64)
        nulls = values.is_null().to_numpy(zero_copy_only=False) if values.null_count else None
        if self.type in ("identity", "pre_hashed") and not (pa.types.is_integer(values.type)
                                                            or pa.types.is_floating(values.type)
                                                            or pa.types.is_boolean(values.type)):
            values = pc.cast(values, pa.int64())
        if self.type in ("identity", "pre_hashed"):
            raw = np.asarray(values.fill_null(0).to_numpy(zero_copy_only=False)).astype(np.int64, copy=False)
            enc = self.enc
            if self.type == "pre_hashed":
                nb = np.uint64(int(enc.num_buckets))
                out = (raw.view(np.uint64) & (nb - np.uint64(1))).astype(np.int64) + 1
            else:
                out = raw.copy()
                max_id = int(enc.max_id) if enc is not None and enc.max_id else None
                if max_id is not None:
                    bad = out > max_id
                    if bad.any():
                        if enc.out_of_range == "error":
                            raise ValueError(f"feature {self.name!r}: ids above max_id {max_id}")
                        out[bad] = max_id if enc.out_of_range == "clip" else 0
                out[out < 0] = 0
            if nulls is not None:
                out[nulls] = 0
            return out
        d = pc.dictionary_encode(values)
        uniq = d.dictionary.to_pylist()
        if self.type == "hash":
            nbk, salt = int(self.enc.num_buckets), self.enc.salt
            mapped = np.array([stable_hash_bucket(u, nbk, salt) for u in uniq], dtype=np.int64)
        else:
            mapped = np.array([self.vocab.get(str(u), 0) for u in uniq], dtype=np.int64)
        idx = np.asarray(d.indices.fill_null(0).to_numpy(zero_copy_only=False), dtype=np.int64)
        out = mapped[idx] if len(mapped) else np.zeros(n, dtype=np.int64)
        if nulls is not None:
            out[nulls] = 0
        return out


def fit_vocabs(config, paths: Sequence[str], out_dir: str) -> dict[str, str]:
    """Count values of every ``vocab``-encoded feature and write ``value, id, count`` Parquet
    artifacts (ids by descending count then value, from 1; ``min_count`` / ``max_size``)."""

    pa, pq = _pa()
    from collections import Counter

    feats = [f for f in config.features if f.kind == "categorical" and f.encoding is not None
             and f.encoding.type == "vocab"]
    counters = {f.name: Counter() for f in feats}
    for p in paths:
        cols = list(dict.fromkeys(f.source or f.name for f in feats))
        table = pq.read_table(p, columns=cols)
        for f in feats:
            col = table.column(f.source or f.name).to_pylist()
            for v in col:
                if isinstance(v, list):
                    counters[f.name].update(str(x) for x in v if x is not None)
                elif v is not None:
                    counters[f.name][str(v)] += 1
    os.makedirs(out_dir, exist_ok=True)
    written = {}
    for f in feats:
        min_count = f.encoding.min_count or 1
        cands = sorted(((v, c) for v, c in counters[f.name].items() if c >= min_count), key=lambda x: (-x[1], x[0]))
        if f.encoding.max_size is not None:
            cands = cands[:f.encoding.max_size]
        path = os.path.join(out_dir, f.encoding.artifact or f"{f.name}.vocab.parquet")
        pq.write_table(pa.table({"value": [v for v, _ in cands], "id": list(range(1, len(cands) + 1)),
                                 "count": [c for _, c in cands]}), path)
        written[f.name] = path
    return written


def load_vocab_map(path: str) -> dict[str, int]:
    _, pq = _pa()
    t = pq.read_table(path)
    return {str(v): int(i) for v, i in zip(t["value"].to_pylist(), t["id"].to_pylist())}


# ------------------------------------------------------------------ tensorization
def group_keys(column) -> np.ndarray:
    """int64 key per row of a group-id column (QAUC / UAUC groups): integer ids as they
    are, anything else by a deterministic 64-bit hash of its text (the same on every
    rank and process); missing values share key -1."""

    import pyarrow as pa

    col = column.combine_chunks() if hasattr(column, "combine_chunks") else column
    if pa.types.is_integer(col.type):
        return np.asarray(col.fill_null(-1).to_numpy(zero_copy_only=False), dtype=np.int64)
    from pandas.util import hash_array

    vals = col.cast(pa.string()).to_numpy(zero_copy_only=False)
    missing = np.array([v is None for v in vals])
    keys = hash_array(np.where(missing, "", vals).astype(object), categorize=False).view(np.int64)
    keys = keys & np.int64(0x7FFFFFFFFFFFFFFF)
    keys[missing] = -1
    return keys


def _combined(col):
    """One contiguous Arrow array for a (chunked) column."""

    import pyarrow as pa

    return col.combine_chunks() if isinstance(col, pa.ChunkedArray) else col


def _is_list(t) -> bool:
    import pyarrow as pa

    return pa.types.is_list(t) or pa.types.is_large_list(t) or pa.types.is_fixed_size_list(t)


def _list_layout(arr) -> tuple[np.ndarray, np.ndarray | None]:
    """``(offsets [n+1] into arr.values, null rows or None)`` of a list array; offsets
    honour a sliced array (they index the unsliced child ``arr.values``)."""

    import pyarrow as pa

    if pa.types.is_fixed_size_list(arr.type):
        size = arr.type.list_size
        offs = (arr.offset + np.arange(len(arr) + 1, dtype=np.int64)) * size
    else:
        offs = np.asarray(arr.offsets.to_numpy(), dtype=np.int64)
    nulls = arr.is_null().to_numpy(zero_copy_only=False) if arr.null_count else None
    return offs, nulls


def _ragged(starts: np.ndarray, counts: np.ndarray) -> np.ndarray:
    """Concatenation of ``arange(starts[i], starts[i] + counts[i])`` over i."""

    total = int(counts.sum())
    if total == 0:
        return np.zeros(0, dtype=np.int64)
    first = np.cumsum(counts) - counts
    return np.repeat(starts.astype(np.int64) - first, counts) + np.arange(total, dtype=np.int64)


def _float_values(arr) -> np.ndarray:
    """float32 numpy copy of a flat Arrow array, nulls as 0."""

    import pyarrow as pa
    import pyarrow.compute as pc

    if not pa.types.is_floating(arr.type):
        arr = pc.cast(arr, pa.float64())
    return np.asarray(arr.fill_null(0.0).to_numpy(zero_copy_only=False), dtype=np.float32)


class Tensorizer:
    """Arrow table (one sample per row) -> ``PackedBatch`` for a batch layout.

    Every column is converted with whole-array Arrow / NumPy operations (list offsets,
    ragged gathers, ``dictionary_encode`` for hashed and vocabulary features); Python
    runs per feature and per distinct hashed value, not per row."""

    def __init__(self, config, batch_plan, *, split: str = "train", vocab_maps: dict[str, dict] | None = None,
                 seq_names=None):
        self.config = config
        self.plan = batch_plan
        by_name = {f.name: f for f in config.features}
        self.features = [by_name[lf.name] for lf in batch_plan.features]
        vocab_maps = vocab_maps or {}
        self.encoders = {}
        for f in self.features:
            if f.kind != "categorical":
                continue
            enc = f.encoding
            share = enc.share_with if enc is not None and enc.type == "shared_vocab" else None
            self.encoders[f.name] = CategoricalEncoder(f, vocab_maps.get(share or f.name))
        sp = getattr(config.data, split) or config.data.train
        self.labels = dict(sp.labels)
        self.label_masks = dict(sp.label_masks)
        self.tasks = list(config.task_names)
        self.dense_width = batch_plan.dense_width
        sc = config.scenarios
        self.scene_source = sc.source
        self.scene_index = {str(n): i for i, n in enumerate(sc.names)}
        self.scene_encoding = sc.source_encoding
        # event sequences (one list column per field) and request-level deduplication
        by_seq = {q.name: q for q in config.sequences}
        self.sequences = [by_seq[n] for n in (seq_names or [])]
        self.seq_encoders = {}
        for q in self.sequences:
            for fl in q.fields:
                if fl.kind == "categorical":
                    self.seq_encoders[(q.name, fl.name)] = CategoricalEncoder(fl, vocab_maps.get(f"{q.name}.{fl.name}"))
        for q in self.sequences:
            if q.null_anchor_field is not None and q.null_anchor_field not in {fl.name for fl in q.fields}:
                raise ValueError(f"sequence {q.name!r} null_anchor_field {q.null_anchor_field!r} is not one of "
                                 "its fields")
        self.request_id = sp.request_id if sp.reader.deduplicate_request_features else None
        self.group_id = sp.group_id
        if sp.reader.deduplicate_request_features and not sp.request_id:
            raise ValueError("reader.deduplicate_request_features needs the split's request_id column")

    def columns(self) -> list[str]:
        cols = [f.source or f.name for f in self.features]
        cols += [self.labels.get(t, t) for t in self.tasks if self.labels.get(t, t)]
        cols += list(self.label_masks.values())
        if self.scene_source:
            cols.append(self.scene_source)
        if self.group_id:
            cols.append(self.group_id)
        for q in self.sequences:
            cols += [fl.source or fl.name for fl in q.fields]
        if self.request_id:
            cols.append(self.request_id)
        return list(dict.fromkeys(cols))

    def _event_matrix(self, q, col, rows: int, anchor=None) -> tuple[np.ndarray, np.ndarray]:
        """``[rows, L]`` positions into the column's flat values (-1 = padding) and lengths.

        With ``anchor`` (the ``null_anchor_field`` column, aligned with ``col``) the events
        whose anchor value is null are dropped from every field first (reference
        ``_compact_direct_sequence_by_anchor``, ``src/dataloader.py:9312``); other nulls stay
        as padding values. Truncation then keeps the first (``head``) or last (``tail``)
        ``max_length`` events of the stored order; the kept events are laid out oldest to
        newest and left-padded, the layout the sequence models read (valid events at the end)."""

        L = int(q.max_length)
        col = _combined(col)
        offs = col.offsets.to_numpy().astype(np.int64)
        starts, ends = offs[:-1], offs[1:]
        if col.null_count:
            nul = col.is_null().to_numpy(zero_copy_only=False)
            ends = np.where(nul, starts, ends)
        kept = None
        if anchor is not None:
            anchor = _combined(anchor)
            aoffs = anchor.offsets.to_numpy().astype(np.int64)
            if not np.array_equal(np.diff(aoffs), np.diff(offs)):
                raise ValueError(f"sequence {q.name!r}: null_anchor_field lists differ in length from the "
                                 "other fields")
            ok = np.ones(len(col.values), dtype=bool)
            if anchor.values.null_count:      # anchor validity moved to this column's flat positions
                aok = ~anchor.values.is_null().to_numpy(zero_copy_only=False)
                n_all = offs[1:] - offs[:-1]
                ok[_ragged(offs[:-1], n_all)] = aok[_ragged(aoffs[:-1], n_all)]
            kept = np.nonzero(ok)[0]
            before = np.concatenate([[0], np.cumsum(ok)])      # kept events before each flat position
            starts, ends = before[starts], before[ends]
        n = ends - starts
        keep = np.minimum(n, L)
        src0 = starts if q.truncation == "head" else ends - keep
        j = np.arange(L)[None, :] - (L - keep)[:, None]          # rank among the kept events
        valid = j >= 0
        if q.sequence_order == "newest_to_oldest":
            pos = src0[:, None] + (keep[:, None] - 1 - j)
        else:
            pos = src0[:, None] + j
        if kept is not None:
            pos = kept[np.where(valid, pos, 0)] if len(kept) else np.zeros_like(pos)
        return np.where(valid, pos, -1), keep

    def _sequence(self, q, table, rows: int) -> dict:
        import pyarrow as pa

        L = int(q.max_length)
        cats = [fl for fl in q.fields if fl.kind == "categorical"]
        dens = [fl for fl in q.fields if fl.kind == "dense"]
        first = table.column((cats or dens)[0].source or (cats or dens)[0].name)
        anchor = None
        if q.null_anchor_field is not None:
            fa = next(fl for fl in q.fields if fl.name == q.null_anchor_field)
            anchor = table.column(fa.source or fa.name)
        pos, lengths = self._event_matrix(q, first, rows, anchor)
        ids = np.zeros((len(cats), rows, L), dtype=np.int64)
        for k, fl in enumerate(cats):
            col = table.column(fl.source or fl.name)
            col = col.combine_chunks() if isinstance(col, pa.ChunkedArray) else col
            flat = self.seq_encoders[(q.name, fl.name)].encode_arrow(col.values)
            safe = np.clip(pos, 0, max(0, len(flat) - 1))
            ids[k] = np.where(pos >= 0, flat[safe] if len(flat) else 0, 0)
        out = {"ids": torch.from_numpy(ids.reshape(len(cats), rows * L)), "lengths": torch.from_numpy(lengths)}
        if dens:
            width = sum(int(fl.dimension) for fl in dens)
            dense = np.zeros((rows, L, width), dtype=np.float32)
            c = 0
            for fl in dens:
                col = table.column(fl.source or fl.name)
                col = col.combine_chunks() if isinstance(col, pa.ChunkedArray) else col
                d = int(fl.dimension)
                flat = _float_values(col.values).reshape(-1, d)
                safe = np.clip(pos, 0, max(0, len(flat) - 1))
                dense[:, :, c:c + d] = np.where((pos >= 0)[..., None], flat[safe] if len(flat) else 0.0, 0.0)
                c += d
            out["dense"] = torch.from_numpy(dense.reshape(rows * L, width))
        return out

    def sequence_lengths(self, table, metric: str = "max") -> np.ndarray:
        """Per-row sequence work (reference ``_table_effective_sequence_lengths``
        ``src/train.py:1936-1952``): over the model's sequences, the max (or sum) of each
        row's event count, capped at each sequence's ``max_length``."""

        import pyarrow as pa

        out = np.zeros(table.num_rows, dtype=np.int64)
        for q in self.sequences:
            if not q.fields:
                continue
            fl = q.fields[0]
            col = table.column(fl.source or fl.name)
            col = col.combine_chunks() if isinstance(col, pa.ChunkedArray) else col
            offs = col.offsets.to_numpy().astype(np.int64)
            n = offs[1:] - offs[:-1]
            if col.null_count:
                n = np.where(col.is_null().to_numpy(zero_copy_only=False), 0, n)
            if q.max_length:
                n = np.minimum(n, int(q.max_length))
            out = out + n if metric == "sum" else np.maximum(out, n)
        return out

    def _sequences(self, table, requests=None) -> dict:
        """Sequence payloads; with request deduplication one row per distinct ``request_id``
        (in order of first appearance) plus ``row_indices`` (candidate -> request row).

        ``requests``: ``(request table, candidate -> request row)`` built by the caller (the
        direct agg path); its rows are used as they are with deduplication, repeated per
        candidate without it."""

        if not self.sequences:
            return {}
        ri = None
        src = table
        if requests is not None:
            req, rows = requests
            rows = np.asarray(rows, dtype=np.int64)
            if self.request_id:
                ri = torch.from_numpy(rows)
                src = req
            else:
                import pyarrow as pa

                src = req.take(pa.array(rows))
        elif self.request_id:
            import pyarrow.compute as pc

            # dictionary indices number the requests in order of first appearance (nulls: one request)
            d = pc.dictionary_encode(_combined(table.column(self.request_id)), null_encoding="encode")
            inv = np.asarray(d.indices.to_numpy(zero_copy_only=False), dtype=np.int64)
            _, first = np.unique(inv, return_index=True)
            ri = torch.from_numpy(inv)
            src = table.take(first)
        out = {}
        for q in self.sequences:
            seq = self._sequence(q, src, src.num_rows)
            if ri is not None:
                seq["row_indices"] = ri
            out[q.name] = seq
        return out

    def _bag(self, f, col) -> tuple[np.ndarray, np.ndarray]:
        """(encoded ids, lengths) of one categorical column; scalars are bags of one, a
        null (scalar or list) is one padding id, lists keep the first (``head``) or last
        (``tail``) ``max_length`` values."""

        arr = _combined(col)
        rows = len(arr)
        enc = self.encoders[f.name]
        if not _is_list(arr.type):
            return enc.encode_arrow(arr), np.ones(rows, dtype=np.int64)
        offs, nulls = _list_layout(arr)
        starts, n = offs[:-1], offs[1:] - offs[:-1]
        if nulls is not None:
            n = np.where(nulls, 0, n)
        cap = f.max_length
        if cap is not None:
            keep = np.minimum(n, int(cap))
            if f.truncation == "tail":
                starts = starts + n - keep
            n = keep
        vals = enc.encode_arrow(arr.values.take(_ragged(starts, n)))
        if nulls is None:
            return vals, n
        lengths = np.where(nulls, 1, n)
        out = np.zeros(int(lengths.sum()), dtype=np.int64)
        out[_ragged(np.cumsum(lengths) - lengths, n)] = vals
        return out, lengths

    def _dense(self, f, col) -> np.ndarray:
        """``[rows, dimension (+1 presence)]``: a scalar fills the first column, a list its
        first ``dimension`` values; null values are 0, a null row has presence 0."""

        arr = _combined(col)
        rows = len(arr)
        dim = int(f.dimension)
        out = np.zeros((rows, dim + (1 if f.presence else 0)), dtype=np.float32)
        if _is_list(arr.type):
            offs, nulls = _list_layout(arr)
            n = offs[1:] - offs[:-1]
            if nulls is not None:
                n = np.where(nulls, 0, n)
            k = np.minimum(n, dim)
            vals = _float_values(arr.values.take(_ragged(offs[:-1], k)))
            row = np.repeat(np.arange(rows), k)
            out[row, _ragged(np.zeros(rows, dtype=np.int64), k)] = vals
        else:
            nulls = arr.is_null().to_numpy(zero_copy_only=False) if arr.null_count else None
            out[:, 0] = _float_values(arr)
        if f.presence:
            out[:, dim] = 1.0 if nulls is None else (~nulls).astype(np.float32)
        return out

    def __call__(self, table, pin: bool = False, requests=None) -> PackedBatch:
        rows = table.num_rows
        ids_parts, len_parts = [], []
        dense = np.zeros((rows, self.dense_width), dtype=np.float32)
        for lf, f in zip(self.plan.features, self.features):
            col = table.column(f.source or f.name)
            if f.kind == "dense":
                d = self._dense(f, col)
                dense[:, lf.dense_col:lf.dense_col + d.shape[1]] = d
                len_parts.append(np.zeros(rows, dtype=np.int64))
                continue
            ids, lengths = self._bag(f, col)
            ids_parts.append(ids)
            len_parts.append(lengths)
        offsets = np.zeros(len(self.plan.features) * rows + 1, dtype=np.int64)
        np.cumsum(np.concatenate(len_parts) if len_parts else np.zeros(0, np.int64), out=offsets[1:])
        ids = np.concatenate(ids_parts) if ids_parts else np.zeros(0, dtype=np.int64)
        labels = np.zeros((rows, len(self.tasks)), dtype=np.float32)
        mask = np.ones((rows, len(self.tasks)), dtype=np.float32)
        any_mask = False
        for t, task in enumerate(self.tasks):
            name = self.labels.get(task, task)
            if name not in table.column_names:
                mask[:, t] = 0.0
                any_mask = True
                continue
            arr = _combined(table.column(name))
            labels[:, t] = _float_values(arr)
            if arr.null_count:
                mask[:, t] = (~arr.is_null().to_numpy(zero_copy_only=False)).astype(np.float32)
                any_mask = True
            mname = self.label_masks.get(task)
            if mname and mname in table.column_names:
                mask[:, t] *= _float_values(_combined(table.column(mname)))
                any_mask = True
        scen = np.zeros(rows, dtype=np.int64)
        if self.scene_source and self.scene_source in table.column_names:
            arr = _combined(table.column(self.scene_source))
            if self.scene_encoding == "index":
                scen = np.asarray(arr.fill_null(0).to_numpy(zero_copy_only=False)).astype(np.int64)
            else:
                import pyarrow.compute as pc

                d = pc.dictionary_encode(arr, null_encoding="encode")
                names = np.array([self.scene_index.get(str(v), 0) for v in d.dictionary.to_pylist()], np.int64)
                scen = names[np.asarray(d.indices.to_numpy(zero_copy_only=False), dtype=np.int64)]
        group = None
        if self.group_id and self.group_id in table.column_names:
            group = torch.from_numpy(group_keys(table.column(self.group_id)))
        return PackedBatch.pack(torch.from_numpy(ids), torch.from_numpy(offsets),
                                torch.from_numpy(dense) if self.dense_width else None, torch.from_numpy(labels),
                                torch.from_numpy(mask) if any_mask else None, torch.from_numpy(scen), rows,
                                sequences=self._sequences(table, requests), pin=pin, group_key=group)


# ------------------------------------------------------------------ iteration
class ParquetBatchIterator:
    """This rank's batches: its row groups (``plan_row_groups``) read with column pruning,
    optionally shuffled through a row buffer, cut into ``batch_size`` rows and tensorized,
    ``prefetch`` batches ahead on a background thread. ``position`` counts the row groups
    consumed (the data cursor of a checkpoint)."""

    def __init__(self, paths: Sequence[str], tensorizer: Tensorizer, batch_size: int, *, rank: int = 0,
                 world: int = 1, shard_unit: str = "row_group", shuffle_rows: int = 0, seed: int = 0,
                 drop_last: bool = True, prefetch: int = 2, pin: bool = False, start_position: int = 0,
                 loop: bool = False, io_policy=None, length_buckets: Sequence = (),
                 length_bucket_metric: str = "max", adapter=None, overlap: bool = True,
                 agg_direct_mode: str = "legacy") -> None:
        """``length_buckets``: ``(max_length or None, batch_size)`` pairs in increasing
        length order (the last may be the catch-all ``None``): rows are grouped by their
        sequence work (``Tensorizer.sequence_lengths``) and each bucket yields batches of
        its own size, so short-history rows are not padded to the longest history
        (reference ``_iter_length_bucketed_tables`` ``src/train.py:1955-2077``).

        ``agg_direct_mode`` (with an agg ``adapter``): ``legacy`` expands every raw table into
        candidate rows first; ``direct`` / ``direct_arrow`` build batches from request groups
        of the raw tables (``data/agg_direct.py``: groups stay whole, each request's events
        are gathered once); ``compare`` trains on ``legacy`` and checks every raw table
        against ``direct``."""

        self.refs = plan_row_groups(paths, rank, world, shard_unit)
        # adapter: raw Arrow table -> flat rows (e.g. the agg layout, ``data/agg.py``);
        # the files are then read with the adapter's raw columns
        self.adapter = adapter
        if agg_direct_mode not in ("legacy", "direct", "direct_arrow", "compare"):
            raise ValueError("reader.agg_direct_mode must be legacy, direct, direct_arrow or compare")
        self.agg_mode = agg_direct_mode if adapter is not None else "legacy"
        self.seed = seed
        self.buckets = [(None if m is None else int(m), int(b)) for m, b in length_buckets]
        self.bucket_metric = length_bucket_metric
        self.io = io_policy  # RemoteIoPolicy: timeouts, retries and skips of remote reads
        self.rank = rank
        self.tz = tensorizer
        self.batch_size = batch_size
        self.shuffle_rows = shuffle_rows
        self.rng = np.random.default_rng([seed, rank])
        self.drop_last = drop_last
        # prefetch = 0: batches are prepared on the consuming thread (``overlap``: scheduled
        # by ``OverlappedPrepareIterator.schedule_next`` between steps)
        self.prefetch_thread = prefetch > 0
        self.overlap = overlap
        self.prefetch = max(1, prefetch)
        self.pin = pin
        self.position = start_position
        self.loop = loop
        self._q: queue.Queue = queue.Queue(maxsize=self.prefetch)
        self._thread: threading.Thread | None = None
        self._stop = threading.Event()

    def _tables(self, raw: bool = False):
        pa, pq = _pa()
        cols = self.adapter.plan.raw_columns() if self.adapter is not None else self.tz.columns()
        while not self._stop.is_set():
            if self.io is not None and self.position == 0:
                self.io.stagger(self.rank)
            while self.position < len(self.refs) and not self._stop.is_set():
                ref = self.refs[self.position]

                def read(ref=ref):
                    f = pq.ParquetFile(ref.path)
                    present = [c for c in cols if c in f.schema_arrow.names]
                    return f.read(columns=present) if ref.index < 0 else f.read_row_group(ref.index, columns=present)

                t = read() if self.io is None else self.io.run(read, f"read {ref.path}#{ref.index}", opening=True,
                                                                 path=ref.path)
                self.position += 1
                if t is None:
                    continue
                if raw or self.adapter is None:
                    yield t
                    continue
                if self.agg_mode == "compare":
                    from .agg_direct import compare_direct_to_legacy

                    compare_direct_to_legacy(t, self.adapter.plan, self.tz)
                yield self.adapter(t)
            if not self.loop or not self.refs:
                return
            self.position = 0

    def _bucketed(self):
        """Length-bucketed batches: shuffled rows routed to their bucket's buffer."""

        pa, _ = _pa()
        bounds = np.array([m for m, _ in self.buckets if m is not None], dtype=np.int64)
        bufs: list = [None] * len(self.buckets)
        for t in self._tables():
            if self.shuffle_rows:
                t = t.take(pa.array(self.rng.permutation(t.num_rows)))
            which = np.searchsorted(bounds, self.tz.sequence_lengths(t, self.bucket_metric), side="left")
            if self.buckets[-1][0] is not None and (which >= len(self.buckets)).any():
                raise ValueError("a row's sequence length exceeds every reader.length_buckets max_length "
                                 "(add a catch-all bucket without max_length)")
            for k, (_m, size) in enumerate(self.buckets):
                sel = np.nonzero(which == k)[0]
                if not len(sel):
                    continue
                part = t.take(pa.array(sel))
                bufs[k] = part if bufs[k] is None else pa.concat_tables([bufs[k], part])
                while bufs[k].num_rows >= size:
                    yield self.tz(bufs[k].slice(0, size), pin=self.pin)
                    bufs[k] = bufs[k].slice(size)
        for k, buf in enumerate(bufs):
            if buf is not None and buf.num_rows and not self.drop_last:
                yield self.tz(buf, pin=self.pin)

    def _batches(self):
        if self.agg_mode in ("direct", "direct_arrow"):
            from .agg_direct import AggDirectBatches

            yield from AggDirectBatches(self._tables(raw=True), self.adapter.plan, self.tz, self.batch_size,
                                        shuffle_rows=self.shuffle_rows, seed=self.seed, rank=self.rank,
                                        length_buckets=self.buckets if self.tz.sequences else (),
                                        length_bucket_metric=self.bucket_metric, drop_last=self.drop_last,
                                        pin=self.pin)
            return
        if self.buckets and self.tz.sequences:
            yield from self._bucketed()
            return
        pa, _ = _pa()
        buf = None
        for t in self._tables():
            buf = t if buf is None else pa.concat_tables([buf, t])
            need = max(self.batch_size, self.shuffle_rows)
            while buf.num_rows >= need:
                if self.shuffle_rows:
                    idx = self.rng.permutation(buf.num_rows)
                    buf = buf.take(pa.array(idx))
                yield self.tz(buf.slice(0, self.batch_size), pin=self.pin)
                buf = buf.slice(self.batch_size)
        while buf is not None and buf.num_rows >= self.batch_size:
            yield self.tz(buf.slice(0, self.batch_size), pin=self.pin)
            buf = buf.slice(self.batch_size)
        if buf is not None and buf.num_rows and not self.drop_last:
            yield self.tz(buf, pin=self.pin)

    def _worker(self):
        try:
            for b in self._batches():
                while not self._stop.is_set():
                    try:
                        self._q.put(b, timeout=0.1)
                        break
                    except queue.Full:
                        continue
                if self._stop.is_set():
                    return
            self._q.put(StopIteration())
        except BaseException as error:  # surfaced to the consumer
            self._q.put(error)

    def __iter__(self) -> Iterator[PackedBatch]:
        if self.prefetch_thread is False:
            # no background thread: the caller's thread prepares every batch, and with
            # ``overlap`` it does so when the training loop calls ``schedule_next`` right
            # after launching a step (the device drains the step meanwhile)
            it = OverlappedPrepareIterator(self._batches())
            if not self.overlap:
                return iter(it)
            return it
        self._stop.clear()
        self._thread = threading.Thread(target=self._worker, daemon=True)
        self._thread.start()
        return self._threaded()

    def _threaded(self) -> Iterator[PackedBatch]:
        while True:
            item = self._q.get()
            if isinstance(item, StopIteration):
                return
            if isinstance(item, BaseException):
                raise item
            yield item

    def close(self) -> None:
        self._stop.set()
        while self._thread is not None and self._thread.is_alive():
            try:  # unblock a producer waiting on a full queue
                self._q.get_nowait()
            except queue.Empty:
                pass
            self._thread.join(timeout=0.1)
        self._thread = None


class OverlappedPrepareIterator:
    """Same-thread batch preparation (reference ``_OverlappedHostPrepareIterator``
    ``src/train.py:4360-4440``): ``next`` returns the batch prepared ahead, or prepares one
    now; ``schedule_next`` prepares the following batch, and the training loop calls it
    right after launching a step, so the Parquet read and tensorisation run on the
    training thread while the device works through the step -- no second Python thread
    contending for the interpreter lock with the step's launches."""

    def __init__(self, batches) -> None:
        self._gen = iter(batches)
        self._ready = None
        self._done = False
        self.prepared_ahead = 0

    def __iter__(self) -> "OverlappedPrepareIterator":
        return self

    def __next__(self) -> PackedBatch:
        if self._ready is None:
            self._advance()
        else:
            self.prepared_ahead += 1
        if self._ready is None:
            raise StopIteration
        b, self._ready = self._ready, None
        return b

    def _advance(self) -> None:
        if self._done:
            return
        try:
            self._ready = next(self._gen)
        except StopIteration:
            self._done = True

    def schedule_next(self) -> None:
        if self._ready is None:
            self._advance()

    def close(self) -> None:
        close = getattr(self._gen, "close", None)
        if close is not None:
            close()


class DevicePrefetcher:
    """Copies batch k+1 host->device on a side CUDA stream while step k runs; the consumer's
    stream waits on an event and the tensors are recorded on it (no host sync)."""

    def __init__(self, batches, device: torch.device, stream: torch.cuda.Stream | None = None) -> None:
        """``stream``: the copy stream to use (reuse one across prefetchers: the caching
        allocator keeps its blocks per stream, so a fresh stream starts with none)."""

        self.it = iter(batches)
        self.device = torch.device(device)
        self.stream = stream if stream is not None else torch.cuda.Stream(device=self.device)
        self._next = None
        self._preload()

    def _preload(self) -> None:
        try:
            host = next(self.it)
        except StopIteration:
            self._next = None
            return
        with torch.cuda.stream(self.stream):
            dev = host.to(self.device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self._next = (dev, ev, host)

    def __iter__(self):
        return self

    def __next__(self) -> PackedBatch:
        if self._next is None:
            raise StopIteration
        dev, ev, _host = self._next
        cur = torch.cuda.current_stream(self.device)
        cur.wait_event(ev)
        for t in dev._flat:
            t.record_stream(cur)
        self._preload()
        return dev


def write_synthetic_parquet(path: str, batch: PackedBatch, batch_plan, config, rows_per_group: int = 1024) -> None:
    """Write a ``PackedBatch`` as a flat Parquet file (test data / mock inputs): one column per
    feature (scalar ids for single-valued, lists for bags, lists for dense), one per label,
    and the scene column when the config has one."""

    pa, pq = _pa()
    rows = batch.rows
    by_name = {f.name: f for f in config.features}
    cols: dict[str, Any] = {}
    offs = batch.offsets.numpy()
    ids = batch.ids.numpy()
    for fi, lf in enumerate(batch_plan.features):
        f = by_name[lf.name]
        if lf.table is None:
            d = batch.dense.numpy()[:, lf.dense_col:lf.dense_col + int(f.dimension)]
            cols[f.source or f.name] = pa.array([list(map(float, r)) for r in d], type=pa.list_(pa.float32()))
            continue
        seg = [ids[offs[fi * rows + i]:offs[fi * rows + i + 1]].tolist() for i in range(rows)]
        if f.pooling == "none" and all(len(s) == 1 for s in seg):
            cols[f.source or f.name] = pa.array([s[0] for s in seg], type=pa.int64())
        else:
            cols[f.source or f.name] = pa.array(seg, type=pa.list_(pa.int64()))
    # event sequences: one list column per categorical field, valid (non-padding) events
    # oldest to newest; request-level payloads are expanded to the candidate rows
    by_seq = {q.name: q for q in config.sequences}
    for name, seq in batch.sequences.items():
        q = by_seq[name]
        L = int(q.max_length)
        cats = [fl for fl in q.fields if fl.kind == "categorical"]
        R = seq["lengths"].numel()
        sid = seq["ids"].numpy().reshape(len(cats), R, L)
        lens = seq["lengths"].numpy()
        ri = seq["row_indices"].numpy() if "row_indices" in seq else np.arange(rows)
        for k, fl in enumerate(cats):
            cols[fl.source or fl.name] = pa.array([sid[k, r, L - lens[r]:].tolist() for r in ri],
                                                  type=pa.list_(pa.int64()))
    sp = config.data.train
    for t, task in enumerate(config.task_names):
        cols[sp.labels.get(task, task)] = pa.array(batch.labels.numpy()[:, t].astype(np.float32))
    if config.scenarios.source and config.scenarios.source not in cols:
        cols[config.scenarios.source] = pa.array(batch.scenario_id.numpy().astype(np.int64))
    pq.write_table(pa.table(cols), path, row_group_size=rows_per_group)
