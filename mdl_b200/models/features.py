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
    """Builds the tables + lookup plans of a config's scalar inputs.

    * ``plan``: the feature-token inputs, concatenated (optionally cut into
      per-token slices padded to 8 columns for the RankMixer tokenizer), or with
      ``token_groups`` one padded slice per token holding that token's inputs
      (``groupwise`` tokenizer);
    * ``domain_plan`` (when ``domain_tokens`` is given): the inputs of each MDL
      domain token, token ``t`` at columns ``[t * domain_k_pad, ...)`` of a
      ``[rows, n_tokens * domain_k_pad]`` matrix (an input read by several
      tokens is looked up once per token);
    * ``target_plan``: the ``target_inputs`` (and LONGER user-global inputs) of the
      summary sequences, one padded slice per group;
    * ``batch_plan``: the batch layout (CSR order of the ids and column order
      of the dense matrix) that all plans read: the feature-token inputs,
      then the inputs used only by domain tokens, then target-only inputs.

    An input that names a sequence with a summary encoder (``mean_pool``,
    ``attention_pool``, ``longer``, ``stca``) reserves ``summary_width`` columns
    in the matrix it appears in; ``summary_cols[plan]`` lists ``(sequence, physical
    columns)`` and the model adds each summary there after the lookup.
    """

    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1,
                 process_group=None, vocab_sizes: dict[str, int] | None = None, input_names: list[str] | None = None,
                 slice_tokens: int = 0, base_seed: int | None = None,
                 domain_tokens: list[list[str]] | None = None, sequences: list | None = None,
                 token_groups: list[list[str]] | None = None, peers=None) -> None:
        from .sequence_encoders import SUMMARY_ENCODERS, summary_width

        self.config = config
        by_name = {f.name: f for f in config.features}
        seq_by_name = {s.name: s for s in config.sequences}

        def is_summary(n: str) -> bool:
            return n in seq_by_name and seq_by_name[n].encoder in SUMMARY_ENCODERS

        if token_groups is not None:
            token_groups = [[n for n in g if n in by_name or is_summary(n)] for g in token_groups]
            names = [n for g in token_groups for n in g]
        else:
            names = list(input_names if input_names is not None
                         else config.resolved.tokenization.feature_token_inputs)
            names = [n for n in names if n in by_name or is_summary(n)]
        self.inputs = [n for n in names if n in by_name]
        domain_tokens = [list(t) for t in (domain_tokens or [])]
        for tok in domain_tokens:
            missing = [n for n in tok if n not in by_name and not is_summary(n)]
            if missing:
                raise ValueError(f"domain token inputs reference unknown features: {missing}")
        # summary sequences of this model (feature tokens, then domain tokens) and their
        # target / user-global input groups
        summary_names: list[str] = []
        for n in names + [n for tok in domain_tokens for n in tok]:
            if is_summary(n) and n not in summary_names:
                summary_names.append(n)
        self.summary_names = summary_names
        target_groups: list[list[str]] = []
        self.target_index: dict[tuple[str, str], int] = {}
        for n in summary_names:
            seq = seq_by_name[n]
            tgt = [t for t in seq.target_inputs if t in by_name]
            if tgt:
                self.target_index[(n, "target")] = len(target_groups)
                target_groups.append(tgt)
            user = ([u for u in seq.longer_user_global_inputs if u in by_name]
                    if seq.encoder == "longer" and seq.longer_user_global_tokens else [])
            if user:
                self.target_index[(n, "user")] = len(target_groups)
                target_groups.append(user)
        batch_names = list(self.inputs)
        for tok in domain_tokens + target_groups:
            for n in tok:
                if n in by_name and n not in batch_names:
                    batch_names.append(n)
        self.batch_names = batch_names
        src_of = {n: i for i, n in enumerate(batch_names)}
        tables: dict[str, tuple[int, int]] = {}
        dense_col_of: dict[str, int] = {}
        dense_names: list[str] = []
        dense_total = 0
        for name in batch_names:
            f = by_name[name]
            if f.kind == "dense":
                dense_col_of[name] = dense_total
                dense_names.append(name)
                dense_total += int(f.dimension) + (1 if f.presence else 0)

        def make(name: str, out_col: int) -> LookupFeature:
            f = by_name[name]
            if f.kind == "dense":
                width = int(f.dimension) + (1 if f.presence else 0)
                return LookupFeature(name, None, width=width, out_col=out_col, dense_col=dense_col_of[name],
                                     src=src_of[name])
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
            return LookupFeature(name, tname, pooling=pool, hash_mode=hmode, buckets=buckets, width=dim,
                                 out_col=out_col, src=src_of[name])

        def width_of(name: str) -> int:
            if is_summary(name):
                return summary_width(seq_by_name[name])
            f = by_name[name]
            if f.kind == "dense":
                return int(f.dimension) + (1 if f.presence else 0)
            owner = by_name.get(table_name_of(config, name), f)
            return int(owner.embedding_dim or config.model.embedding_dim)

        def slices(groups: list[list[str]]):
            """Per-group padded slices: lookup features, summary columns, widths, pad."""

            widths = [sum(width_of(n) for n in g) for g in groups]
            kp = (max(widths) + 7) // 8 * 8 if widths else 0
            feats, summ = [], []
            for t, g in enumerate(groups):
                c = t * kp
                for n in g:
                    w = width_of(n)
                    if is_summary(n):
                        summ.append((n, torch.arange(c, c + w, dtype=torch.long)))
                    else:
                        feats.append(make(n, c))
                    c += w
            return feats, summ, widths, kp

        self.summary_cols: dict[str, list[tuple[str, torch.Tensor]]] = {"plan": [], "domain": []}
        slice_k = slice_stride = 0
        if token_groups is not None:
            feats, summ, self.group_widths, kp = slices(token_groups)
            self.summary_cols["plan"] = summ
            col = kp * len(token_groups)
            self.group_k_pad = kp
            self.plan = LookupPlan(feats, out_width=col, dense_width=dense_total,
                                   zero_fill=bool(summ) or any(w != kp for w in self.group_widths))
            features = feats
        else:
            features = []
            spans: list[tuple[str, int, int]] = []
            col = 0
            for name in names:
                w = width_of(name)
                if is_summary(name):
                    spans.append((name, col, w))
                else:
                    features.append(make(name, col))
                col += w
            width = col
            if slice_tokens:
                # per-token slices of the RankMixer tokenizer: the inputs padded to slice_tokens x
                # slice_k logical columns (reference RankMixerSliceTokenizer), each slice padded
                # to a multiple of 8 columns (16-byte rows for TMA)
                slice_k = (col + slice_tokens - 1) // slice_tokens
                slice_stride = (slice_k + 7) // 8 * 8
                width = slice_k * slice_tokens
            self.plan = LookupPlan(features, out_width=width, slice_k=slice_k, slice_stride=slice_stride,
                                   dense_width=dense_total, zero_fill=bool(spans), written_width=col)
            self.summary_cols["plan"] = [
                (n, torch.tensor([self.plan.phys_col(c) for c in range(c0, c0 + w)], dtype=torch.long))
                for n, c0, w in spans]
            self.group_widths, self.group_k_pad = [], 0
        self.scalar = ScalarInputs(self.inputs, [f.width for f in features], col,
                                   [n for n in self.inputs if n in dense_col_of], dense_total)
        self.slice_tokens = slice_tokens
        # MDL domain-token inputs
        self.domain_plan = None
        self.domain_widths: list[int] = []
        self.domain_k_pad = 0
        if domain_tokens:
            feats, summ, self.domain_widths, kp = slices(domain_tokens)
            self.domain_k_pad = kp
            self.summary_cols["domain"] = summ
            self.domain_plan = LookupPlan(feats, out_width=len(domain_tokens) * kp, dense_width=dense_total,
                                          zero_fill=bool(summ) or any(w != kp for w in self.domain_widths))
        # target / user-global inputs of the summary sequences
        self.target_plan = None
        self.target_widths: list[int] = []
        self.target_k_pad = 0
        if target_groups:
            feats, _summ, self.target_widths, kp = slices(target_groups)
            self.target_k_pad = kp
            self.target_plan = LookupPlan(feats, out_width=len(target_groups) * kp, dense_width=dense_total,
                                          zero_fill=any(w != kp for w in self.target_widths))
        self.batch_plan = LookupPlan([make(n, 0) for n in batch_names], out_width=0, dense_width=dense_total)
        sequences = list(sequences or [])
        for n in summary_names:
            if all(s.name != n for s in sequences):
                sequences.append(seq_by_name[n])
        # Raw event sequences (OneTrans S tokens): one plan per sequence whose rows are the
        # events (rows * max_length), categorical fields first, then dense fields.
        self._seq_offsets: dict = {}  # per (sequence, rows) CSR offsets of the one-id-per-event lookups
        self.seq_plans: dict[str, LookupPlan] = {}
        self.seq_fields: dict[str, list[str]] = {}
        self.seq_dense_fields: dict[str, list[str]] = {}
        self.seq_widths: dict[str, int] = {}
        for seq in sequences:
            cats = [fl for fl in seq.fields if fl.kind == "categorical"]
            dens = [fl for fl in seq.fields if fl.kind == "dense"]
            lfs: list[LookupFeature] = []
            col = 0
            for i, fl in enumerate(cats):
                tname, owner = self._sequence_field_table(config, seq, fl, by_name)
                dim = int(owner.embedding_dim or config.model.embedding_dim)
                rows = categorical_size(owner, vocab_sizes)
                if tname in tables and tables[tname] != (rows, dim):
                    raise ValueError(f"shared table {tname!r} used with different shapes")
                tables[tname] = (rows, dim)
                lfs.append(LookupFeature(f"{seq.name}.{fl.name}", tname, pooling=POOL_NONE, width=dim, out_col=col,
                                         src=i))
                col += dim
            dcol = 0
            for j, fl in enumerate(dens):
                lfs.append(LookupFeature(f"{seq.name}.{fl.name}", None, width=int(fl.dimension), out_col=col,
                                         dense_col=dcol, src=len(cats) + j))
                col += int(fl.dimension)
                dcol += int(fl.dimension)
            pad = (col + 7) // 8 * 8  # 16-byte rows for the projection GEMM
            self.seq_plans[seq.name] = LookupPlan(lfs, out_width=col, slice_k=col if pad != col else 0,
                                                  slice_stride=pad if pad != col else 0, dense_width=dcol)
            self.seq_fields[seq.name] = [fl.name for fl in cats]
            self.seq_dense_fields[seq.name] = [fl.name for fl in dens]
            self.seq_widths[seq.name] = col
        train = config.training
        specs = [EmbeddingTableSpec(n, r, d, 4 if train.embedding_weight_dtype == "fp32" else 2)
                 for n, (r, d) in sorted(tables.items())]
        self.table_shapes = tables
        # replicated tables: every rank holds all rows (one shard) and trains them with
        # torch.optim.Adagrad semantics (reference src/train.py:6619-6629); sharded tables
        # use the configured row-wise or full Adagrad
        replicated = train.embedding_distribution == "replicated"
        shard_world = 1 if replicated else world
        layout = "full" if replicated or train.sparse_optimizer != "rowwise_adagrad" else "rowwise"
        self.shard_plan = plan_embedding_shards(
            specs, world_size=shard_world, strategy=train.embedding_sharding.strategy,
            table_wise_max_rows=train.embedding_sharding.table_wise_max_rows, optimizer_state_layout=layout)
        lr_sparse = train.lr_sparse if train.lr_sparse is not None else train.lr_dense
        self.store = EmbeddingStore(
            [(n, r, d) for n, (r, d) in sorted(tables.items())], self.shard_plan, rank=0 if replicated else rank,
            world=shard_world, device=device, init_std=config.model.init_std, lr=lr_sparse, eps=train.adagrad_eps,
            initial_accumulator_value=train.adagrad_initial_accumulator_value, process_group=process_group,
            base_seed=base_seed, optimizer=layout, lr_decay=train.adagrad_lr_decay,
            replicas=world if replicated else 1, replica_group=process_group, peers=peers)

    # ids arrive already encoded (tensorization applies the encodings on the host)
    _device_hash = False

    @staticmethod
    def _sequence_field_table(config: AppConfig, seq, fl, by_name):
        """(table name, config that sizes it) of a sequence field: its own table
        ``<sequence>.<field>``, or, with ``share_with`` + ``share_embedding``, the table of
        the scalar feature or the qualified sequence field it names (chains followed)."""

        qualified = {f"{s.name}.{f.name}": f for s in config.sequences for f in s.fields}
        seen = set()
        name, cur = f"{seq.name}.{fl.name}", fl
        while True:
            enc = cur.encoding
            if enc is None or not enc.share_with or not enc.share_embedding:
                return name, cur
            if name in seen:
                raise ValueError(f"shared embedding cycle at {seq.name}.{fl.name}")
            seen.add(name)
            target = enc.share_with
            if target in by_name:
                tname = table_name_of(config, target)
                return tname, by_name.get(tname, by_name[target])
            if target not in qualified:
                raise ValueError(f"sequence field {seq.name}.{fl.name} shares unknown table {target!r}")
            name, cur = target, qualified[target]

    @property
    def slice_k(self) -> int:
        return self.plan.slice_k

    @property
    def slice_stride(self) -> int:
        return self.plan.slice_stride


def lookup_sequence(encoder: FeatureEncoder, batch, name: str, rows: int, max_len: int, anchor: torch.Tensor,
                    expand: bool = True):
    """Event rows ``[rows * max_len, out_ld]`` of sequence ``name`` and its lengths ``[rows]``.

    With request-level batching (``row_indices`` in the sequence payload, reference
    ``_batch_gather_indexed_rows`` ``src/model.py:701-750``) the events are looked up
    once per request (``R * max_len`` rows) and each candidate row then takes its
    request's rows (``index_select``; its backward sums the candidates of a request).
    With ``expand=False`` the request-level rows come back as ``(rows [R * max_len, out_ld],
    lengths [R], row_indices or None)``, so request-only work (event projections) runs
    once per request before ``expand_requests`` hands each candidate its request's result
    (the training-time counterpart of the reference's request caches)."""

    from ..ops.embedding import fused_lookup

    seq = batch.sequences[name]
    ids = seq["ids"].reshape(-1)
    lengths = seq["lengths"]
    R = lengths.numel()
    nf = len(encoder.seq_fields[name])
    key = (name, R, max_len, str(ids.device))
    cache = encoder._seq_offsets
    if key not in cache:
        if len(cache) > 64:
            cache.clear()
        cache[key] = torch.arange(nf * R * max_len + 1, dtype=torch.int64, device=ids.device)
    x = fused_lookup(encoder.store, encoder.seq_plans[name], ids, cache[key], seq.get("dense"), R * max_len, anchor)
    ri = seq.get("row_indices")
    if not expand:
        return x, lengths, (None if ri is None else ri.to(x.device))
    if ri is None:
        return x, lengths
    ri = ri.to(x.device)
    x = x.view(R, max_len * x.shape[1]).index_select(0, ri).view(rows * max_len, x.shape[1])
    return x, lengths.index_select(0, ri.to(lengths.device))


def expand_requests(t: torch.Tensor, row_indices: torch.Tensor | None) -> torch.Tensor:
    """Request-level rows (leading axis) -> candidate rows (identity without request batching)."""

    if row_indices is None:
        return t
    return t.index_select(0, row_indices.to(t.device))
