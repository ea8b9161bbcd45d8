"""Feature encoder bank: embedding tables, sharding plan and lookup plans.

Counterpart of the reference ``FeatureEncoderBank`` (``src/model.py:2299-4260``)
for the scalar inputs of a ranker: categorical features (single-valued or
bags with mean/sum pooling) and dense features, in tokenizer input order. All
tables of a model live in one ``EmbeddingStore``; shared embeddings
(``encoding.share_with`` + ``share_embedding``) map several inputs onto one table.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..config.schema import AppConfig, FeatureConfig
from ..ops.embedding import (HASH_NONE, HASH_PREHASHED, POOL_MEAN, POOL_NONE, POOL_SUM, EmbeddingStore,
                             LookupFeature, LookupPlan)
from ..parallel.sharding import EmbeddingTableSpec, plan_embedding_shards


def categorical_size(feature: FeatureConfig, vocab_sizes: dict[str, int] | None = None) -> int:
    """Rows of a feature's table including the padding row 0."""

    enc = feature.encoding
    if enc is not None and enc.num_buckets:
        return int(enc.num_buckets) + 1
    if enc is not None and enc.max_id:
        return int(enc.max_id) + 1
    if vocab_sizes and feature.name in vocab_sizes:
        return int(vocab_sizes[feature.name]) + 1
    raise ValueError(f"cannot size embedding table of {feature.name!r}: set encoding.num_buckets or a vocab")


def table_name_of(config: AppConfig, name: str) -> str:
    """Follow ``share_with`` chains to the owning table name."""

    by_name = {f.name: f for f in config.features}
    seen = set()
    cur = name
    while True:
        if cur in seen:
            raise ValueError(f"shared embedding cycle at {name!r}")
        seen.add(cur)
        f = by_name.get(cur)
        if f is None or f.encoding is None or not f.encoding.share_with or not f.encoding.share_embedding:
            return cur
        cur = f.encoding.share_with


@dataclass
class ScalarInputs:
    names: list[str]          # tokenizer input order
    widths: list[int]
    total_width: int
    dense_names: list[str]
    dense_width: int


class FeatureEncoder:
    """Builds the tables + lookup plan of a config's scalar token inputs."""

    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1,
                 process_group=None, vocab_sizes: dict[str, int] | None = None, input_names: list[str] | None = None,
                 slice_tokens: int = 0, base_seed: int | None = None) -> None:
        self.config = config
        by_name = {f.name: f for f in config.features}
        names = list(input_names if input_names is not None else config.resolved.tokenization.feature_token_inputs)
        names = [n for n in names if n in by_name]
        self.inputs = names
        tables: dict[str, tuple[int, int]] = {}
        features: list[LookupFeature] = []
        col = 0
        dense_col = 0
        dense_names = []
        for name in names:
            f = by_name[name]
            if f.kind == "dense":
                width = int(f.dimension) + (1 if f.presence else 0)
                features.append(LookupFeature(name, None, width=width, out_col=col, dense_col=dense_col))
                dense_names.append(name)
                dense_col += width
                col += width
                continue
            tname = table_name_of(config, name)
            owner = by_name.get(tname, f)
            dim = int(owner.embedding_dim or config.model.embedding_dim)
            rows = categorical_size(owner, vocab_sizes)
            if tname in tables and tables[tname] != (rows, dim):
                raise ValueError(f"shared table {tname!r} used with different shapes")
            tables[tname] = (rows, dim)
            pool = {"none": POOL_NONE, "mean": POOL_MEAN, "sum": POOL_SUM}[f.pooling]
            enc = f.encoding
            hmode = HASH_PREHASHED if (enc is not None and enc.type == "pre_hashed" and self._device_hash) else HASH_NONE
            buckets = int(enc.num_buckets or 0) if enc is not None else 0
            features.append(LookupFeature(name, tname, pooling=pool, hash_mode=hmode, buckets=buckets, width=dim,
                                          out_col=col))
            col += dim
        self.table_shapes = tables
        self.scalar = ScalarInputs(names, [f.width for f in features], col, dense_names, dense_col)
        slice_k = 0
        slice_stride = 0
        if slice_tokens:
            # per-token slices of the RankMixer tokenizer, padded to a multiple of 8 columns (16 bytes)
            slice_k = (col + slice_tokens - 1) // slice_tokens
            slice_stride = (slice_k + 7) // 8 * 8
        self.slice_tokens = slice_tokens
        self.plan = LookupPlan(features, out_width=col, slice_k=slice_k, slice_stride=slice_stride,
                               dense_width=dense_col)
        train = config.training
        specs = [EmbeddingTableSpec(n, r, d, 4 if train.embedding_weight_dtype == "fp32" else 2)
                 for n, (r, d) in sorted(tables.items())]
        self.shard_plan = plan_embedding_shards(
            specs, world_size=world, strategy=train.embedding_sharding.strategy,
            table_wise_max_rows=train.embedding_sharding.table_wise_max_rows,
            optimizer_state_layout="rowwise" if train.sparse_optimizer == "rowwise_adagrad" else "full")
        lr_sparse = train.lr_sparse if train.lr_sparse is not None else train.lr_dense
        self.store = EmbeddingStore(
            [(n, r, d) for n, (r, d) in sorted(tables.items())], self.shard_plan, rank=rank, world=world,
            device=device, init_std=config.model.init_std, lr=lr_sparse, eps=train.adagrad_eps,
            initial_accumulator_value=train.adagrad_initial_accumulator_value, process_group=process_group,
            base_seed=base_seed)

    # ids arrive already encoded (tensorization applies the encodings on the host)
    _device_hash = False

    @property
    def slice_k(self) -> int:
        return self.plan.slice_k

    @property
    def slice_stride(self) -> int:
        return self.plan.slice_stride
