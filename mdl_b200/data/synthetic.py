"""Seeded synthetic data in the shapes of the benchmark configs.

There is no network in the benchmark environment, so every benchmark and
parity run uses generated data of the configured shape:

* categorical ids: Zipf(s) over ``[1, vocab]`` (inverse-CDF of the continuous
  power law, then a fixed per-field multiplicative scramble so frequent ids do
  not cluster at small row numbers) or uniform;
* multi-hot bags with uniform lengths in ``[min_len, max_len]``;
* dense features ``N(0, 1)``;
* labels ``Bernoulli`` drawn from a hidden ground-truth logit (a fixed random
  score per (field, id), averaged over bags, plus a dense projection, plus for
  multi-scene specs a per-(scene, task) offset and gain), shifted per task so
  the positive rate matches the configured one. A model can therefore learn
  something, and AUC comparisons are meaningful.

Generation is vectorised numpy; ``BatchPool`` pre-generates a few distinct
batches in pinned host memory for the timed loops.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from hashlib import sha256

import numpy as np
import torch

from ..ops.embedding import LookupPlan
from .batch import PackedBatch


@dataclass
class FieldSpec:
    vocab: int             # ids drawn from [1, vocab]
    multi_hot: bool = False
    min_len: int = 1
    max_len: int = 1


@dataclass
class SequenceSpec:
    """A raw event sequence: per-event categorical fields (ids in [1, vocab]; the
    first field carries the label signal), lengths uniform in [min_len, max_len],
    left-padded to ``max_len`` with id 0."""

    fields: dict[str, FieldSpec]
    max_len: int
    min_len: int | None = None       # None: every row is full length
    dense_width: int = 0
    # request-level batching: consecutive groups of this many candidate rows share one
    # request's sequence, stored once per request with ``row_indices`` (candidate -> request)
    candidates_per_request: int = 1


@dataclass
class SyntheticSpec:
    fields: dict[str, FieldSpec]
    dense_width: int
    task_rates: list[float]
    zipf_s: float | None = 1.05      # None -> uniform ids
    num_scenarios: int = 1
    seed: int = 0
    scene_field: str | None = None   # categorical field whose id is the scene id + 1
    scene_effect: float = 0.0        # strength of the per-(scene, task) part of the ground truth
    sequences: dict[str, SequenceSpec] | None = None


def zipf_ids(rng: np.random.Generator, n: int, vocab: int, s: float | None, scramble: int) -> np.ndarray:
    if vocab <= 1:
        return np.ones(n, dtype=np.int64)
    if s is None:
        k = rng.integers(1, vocab + 1, size=n, dtype=np.int64)
    else:
        u = rng.random(n)
        if abs(s - 1.0) < 1e-9:
            x = np.exp(u * math.log(vocab + 1.0))
        else:
            a = 1.0 - s
            x = np.power(1.0 + u * (math.pow(vocab + 1.0, a) - 1.0), 1.0 / a)
        k = np.clip(np.floor(x).astype(np.int64), 1, vocab)
    # fixed bijection of [1, vocab]: (k-1)*scramble mod vocab + 1 (scramble coprime to vocab)
    return ((k - 1) * scramble) % vocab + 1


def _coprime(vocab: int, seed: int) -> int:
    cand = 1000003 + 2 * (seed % 1000)
    while math.gcd(cand, vocab) != 1:
        cand += 2
    return cand


def _id_score(ids: np.ndarray, salt: int) -> np.ndarray:
    """Deterministic pseudo-random score in [-1, 1) per id (hash of id and salt)."""

    h = (ids.astype(np.uint64) * np.uint64(0x9E3779B97F4A7C15) + np.uint64(salt & 0xFFFFFFFF)) & np.uint64(0xFFFFFFFFFFFF)
    h ^= h >> np.uint64(17)
    return (h % np.uint64(1 << 20)).astype(np.float64) / float(1 << 19) - 1.0


class SyntheticGenerator:
    """Draws ``PackedBatch``es for a lookup plan from a ``SyntheticSpec``."""

    def __init__(self, plan: LookupPlan, spec: SyntheticSpec, rank: int = 0) -> None:
        self.plan = plan
        self.spec = spec
        self.rng = np.random.default_rng([spec.seed, rank])
        self.truth_rng = np.random.default_rng([spec.seed, 999])
        self.scramble = {name: _coprime(fs.vocab, i) for i, (name, fs) in enumerate(spec.fields.items())}
        self.field_weight = {name: float(self.truth_rng.normal(0.0, 1.0)) for name in spec.fields}
        self.dense_proj = self.truth_rng.normal(0.0, 1.0, size=(max(spec.dense_width, 1), len(spec.task_rates)))
        self.task_mix = self.truth_rng.normal(0.0, 1.0, size=(len(spec.task_rates),))
        self.task_bias = None
        ns, nt = max(1, spec.num_scenarios), len(spec.task_rates)
        self.scene_offset = self.truth_rng.normal(0.0, 1.0, size=(ns, nt)) * spec.scene_effect
        self.scene_gain = 1.0 + 0.5 * spec.scene_effect * self.truth_rng.normal(0.0, 1.0, size=(ns, nt))

    def _truth_logits(self, per_field_scores: np.ndarray, dense: np.ndarray, scen: np.ndarray) -> np.ndarray:
        nf = max(1, per_field_scores.shape[1])
        base = per_field_scores.sum(axis=1, keepdims=True) * (2.0 / math.sqrt(nf))
        dense_part = dense @ self.dense_proj[: dense.shape[1]] * (0.5 / math.sqrt(max(1, dense.shape[1])))
        logits = base * (1.0 + 0.3 * self.task_mix[None, :]) + dense_part
        if self.spec.scene_effect:
            logits = logits * self.scene_gain[scen] + self.scene_offset[scen]
        return logits

    def _calibrate(self, logits: np.ndarray) -> np.ndarray:
        if self.task_bias is None:
            biases = []
            for t, rate in enumerate(self.spec.task_rates):
                lo, hi = -30.0, 30.0
                for _ in range(60):
                    mid = 0.5 * (lo + hi)
                    p = 1.0 / (1.0 + np.exp(-(logits[:, t] + mid)))
                    if p.mean() > rate:
                        hi = mid
                    else:
                        lo = mid
                biases.append(0.5 * (lo + hi))
            self.task_bias = np.array(biases)
        return logits + self.task_bias[None, :]

    def batch(self, rows: int, pin: bool = False) -> PackedBatch:
        rng = self.rng
        spec = self.spec
        ids_parts = []
        lengths_parts = []
        scores = []
        scen = rng.integers(0, max(1, spec.num_scenarios), size=rows, dtype=np.int64)
        for f in self.plan.features:
            if f.table is None:
                lengths_parts.append(np.zeros(rows, dtype=np.int64))
                continue
            if f.name == spec.scene_field:
                ids_parts.append(scen + 1)
                lengths_parts.append(np.ones(rows, dtype=np.int64))
                continue
            fs = spec.fields[f.name]
            if fs.multi_hot:
                lengths = rng.integers(fs.min_len, fs.max_len + 1, size=rows, dtype=np.int64)
            else:
                lengths = np.ones(rows, dtype=np.int64)
            n = int(lengths.sum())
            ids = zipf_ids(rng, n, fs.vocab, spec.zipf_s, self.scramble[f.name])
            ids_parts.append(ids)
            lengths_parts.append(lengths)
            s = _id_score(ids, int.from_bytes(sha256(f.name.encode()).digest()[:4], 'little')) * self.field_weight[f.name]
            bag = np.repeat(np.arange(rows), lengths)
            per_row = np.bincount(bag, weights=s, minlength=rows) / np.maximum(lengths, 1)
            scores.append(per_row)
        dense = rng.standard_normal((rows, spec.dense_width)).astype(np.float32) if spec.dense_width else \
            np.zeros((rows, 0), dtype=np.float32)
        sequences = {}
        for name, ss in (spec.sequences or {}).items():
            L = ss.max_len
            lo = ss.min_len if ss.min_len is not None else L
            cpr = max(1, int(ss.candidates_per_request))
            cand_rows = rows
            rows = (cand_rows + cpr - 1) // cpr        # request rows
            lengths = rng.integers(lo, L + 1, size=rows, dtype=np.int64) if lo < L else np.full(rows, L, np.int64)
            valid = np.arange(L)[None, :] >= (L - lengths)[:, None]          # prefix padding
            ids = np.zeros((len(ss.fields), rows, L), dtype=np.int64)
            for k, (fname, fs) in enumerate(ss.fields.items()):
                key = f"{name}.{fname}"
                if key not in self.scramble:
                    self.scramble[key] = _coprime(fs.vocab, 7919 + k)
                draw = zipf_ids(rng, rows * L, fs.vocab, spec.zipf_s, self.scramble[key]).reshape(rows, L)
                ids[k] = np.where(valid, draw, 0)
                if k == 0:  # mean score of the valid events of the first field
                    sc = _id_score(ids[k].reshape(-1), int.from_bytes(sha256(key.encode()).digest()[:4], "little"))
                    sc = (sc.reshape(rows, L) * valid).sum(1) / np.maximum(lengths, 1)
                    scores.append(np.repeat(sc, cpr)[:cand_rows] * 2.0)
            seq = {"ids": torch.from_numpy(ids.reshape(len(ss.fields), rows * L)),
                   "lengths": torch.from_numpy(lengths)}
            if ss.dense_width:
                seq["dense"] = torch.from_numpy(rng.standard_normal((rows * L, ss.dense_width)).astype(np.float32))
            if cpr > 1:
                seq["row_indices"] = torch.arange(cand_rows, dtype=torch.int64) // cpr
            sequences[name] = seq
            rows = cand_rows
        per_field = np.stack(scores, axis=1) if scores else np.zeros((rows, 0))
        logits = self._calibrate(self._truth_logits(per_field, dense.astype(np.float64), scen))
        probs = 1.0 / (1.0 + np.exp(-logits))
        labels = (rng.random(probs.shape) < probs).astype(np.float32)
        offsets = np.zeros(len(self.plan.features) * rows + 1, dtype=np.int64)
        np.cumsum(np.concatenate(lengths_parts), out=offsets[1:])
        ids_all = np.concatenate(ids_parts) if ids_parts else np.zeros(0, dtype=np.int64)
        return PackedBatch.pack(torch.from_numpy(ids_all), torch.from_numpy(offsets),
                                torch.from_numpy(dense) if spec.dense_width else None, torch.from_numpy(labels), None,
                                torch.from_numpy(scen), rows, sequences=sequences, pin=pin)


class BatchPool:
    """A fixed set of pre-generated pinned host batches, served round-robin."""

    def __init__(self, gen: SyntheticGenerator, rows: int, count: int, pin: bool = True) -> None:
        self.batches = [gen.batch(rows, pin=pin and torch.cuda.is_available()) for _ in range(count)]
        self.i = 0

    def next(self) -> PackedBatch:
        b = self.batches[self.i % len(self.batches)]
        self.i += 1
        return b


def synthetic_spec_from_config(config, batch_plan, *, zipf_s: float | None = 1.05, seed: int = 0,
                               task_rate: float = 0.1, sequences: list | None = None) -> SyntheticSpec:
    """A ``SyntheticSpec`` for any config: every categorical input of the batch layout draws
    ids over its table (``max_id`` / ``num_buckets``; ``vocab`` features over a
    1000-entry vocabulary), bags draw lengths in [1, max_length or 8]. ``sequences``
    (sequence configs, e.g. the model encoder's) get event sequences of lengths in
    [1, max_length] with their categorical fields and dense fields."""

    def vocab_of(enc) -> int:
        if enc is not None and enc.max_id:
            return int(enc.max_id)
        if enc is not None and enc.num_buckets:
            return int(enc.num_buckets)
        return 1000

    seq_specs = {}
    for seq in sequences or []:
        cats = {fl.name: FieldSpec(vocab=vocab_of(fl.encoding)) for fl in seq.fields if fl.kind == "categorical"}
        dense = sum(int(fl.dimension) for fl in seq.fields if fl.kind == "dense")
        seq_specs[seq.name] = SequenceSpec(fields=cats, max_len=int(seq.max_length), min_len=1, dense_width=dense)

    by_name = {f.name: f for f in config.features}
    fields = {}
    for lf in batch_plan.features:
        if lf.table is None:
            continue
        f = by_name[lf.name]
        enc = f.encoding
        vocab = 1000
        if enc is not None and enc.max_id:
            vocab = int(enc.max_id)
        elif enc is not None and enc.num_buckets:
            vocab = int(enc.num_buckets)
        multi = f.pooling != "none"
        fields[f.name] = FieldSpec(vocab=vocab, multi_hot=multi, min_len=1, max_len=(f.max_length or 8) if multi else 1)
    return SyntheticSpec(fields=fields, dense_width=batch_plan.dense_width,
                         task_rates=[task_rate] * len(config.task_names), zipf_s=zipf_s,
                         num_scenarios=len(config.scenarios.names), seed=seed, sequences=seq_specs or None)
