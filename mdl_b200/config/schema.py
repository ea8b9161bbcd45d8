"""YAML config schema: frozen, deeply immutable dataclasses.

The section and key names follow the reference's config schema so its YAML
files load unchanged (``src/config.py:75-3379``: ``ReaderConfig`` :504,
``ParquetSplitConfig`` :865, ``FeatureConfig`` :1043, ``SequenceConfig``
:1217, ``ScenarioConfig`` :1645, ``TokenizationConfig`` :1907,
``RuntimeConfig`` :2269, ``ModelConfig`` :2451, ``TrainingConfig`` :3036,
``AppConfig`` :3298). Keys this framework adds are listed in
``SCHEMA_EXTENSIONS``; they default to the reference behaviour.

Construction goes through :func:`build_dataclass`, which converts nested
mappings and lists by the field annotations, validates ``Literal`` values and
rejects unknown keys with the full dotted path in the message.
"""

from __future__ import annotations

import dataclasses
import types
import typing
from collections.abc import Mapping
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any, Literal

# Keys added beyond the reference schema (additive, back-compatible).
SCHEMA_EXTENSIONS = {
    "features[].pooling": "adds 'sum' pooling next to 'none'/'mean'",
    "training.dense_optimizer": "adds 'adam' next to 'rmsprop'",
    "training.adam_beta1/adam_beta2/adam_eps/weight_decay": "Adam hyper-parameters",
    "model.tokens_per_scenario": "N domain tokens per scene (pooled by DomainFused)",
    "model.pyramid_schedule/pyramid_halve_every": "OneTrans pyramid: linear or halve every k layers",
    "model.sequence_head": "LONGER sequence encoder feeding a MixFormer-style head",
    "runtime.kernel_backend": "'native' (sm_100a kernels, mandatory on CUDA) or 'torch' (CPU oracle)",
    "training.comm": "fused NVLink collectives ('fused') or NCCL baseline ('nccl')",
}


class ConfigError(ValueError):
    """Raised when a config mapping does not match the schema."""


def freeze(value: Any) -> Any:
    """Recursively convert dicts to read-only mappings and lists to tuples."""

    if isinstance(value, Mapping) and not isinstance(value, MappingProxyType):
        return MappingProxyType({k: freeze(v) for k, v in value.items()})
    if isinstance(value, (list, tuple)):
        return tuple(freeze(v) for v in value)
    return value


def thaw(value: Any) -> Any:
    """Inverse of :func:`freeze` (plain dicts and lists), for YAML round trips."""

    if dataclasses.is_dataclass(value) and not isinstance(value, type):
        return {f.name: thaw(getattr(value, f.name)) for f in dataclasses.fields(value) if not f.name.startswith("_")}
    if isinstance(value, Mapping):
        return {k: thaw(v) for k, v in value.items()}
    if isinstance(value, tuple):
        return [thaw(v) for v in value]
    return value


def _convert(tp: Any, value: Any, path: str) -> Any:
    origin = typing.get_origin(tp)
    args = typing.get_args(tp)
    if tp is Any:
        return freeze(value)
    if origin in (typing.Union, types.UnionType):
        if value is None and type(None) in args:
            return None
        errors = []
        for arg in args:
            if arg is type(None):
                continue
            try:
                return _convert(arg, value, path)
            except ConfigError as error:
                errors.append(str(error))
        raise ConfigError(f"{path}: value {value!r} matches none of {args}: {errors}")
    if origin is Literal:
        if value not in args:
            raise ConfigError(f"{path}: {value!r} is not one of {list(args)}")
        return value
    if origin in (tuple, list):
        if value is None:
            return ()
        if isinstance(value, (str, bytes)) or not isinstance(value, (list, tuple)):
            raise ConfigError(f"{path}: expected a list, got {type(value).__name__}")
        item_tp = args[0] if args else Any
        return tuple(_convert(item_tp, v, f"{path}[{i}]") for i, v in enumerate(value))
    if origin in (dict, Mapping) or tp in (dict, Mapping) or origin is typing.Mapping:
        if value is None:
            return MappingProxyType({})
        if not isinstance(value, Mapping):
            raise ConfigError(f"{path}: expected a mapping, got {type(value).__name__}")
        val_tp = args[1] if len(args) == 2 else Any
        return MappingProxyType({str(k): _convert(val_tp, v, f"{path}.{k}") for k, v in value.items()})
    if dataclasses.is_dataclass(tp):
        if isinstance(value, tp):
            return value
        if not isinstance(value, Mapping):
            raise ConfigError(f"{path}: expected a mapping for {tp.__name__}, got {type(value).__name__}")
        return build_dataclass(tp, value, path)
    if tp is bool:
        if not isinstance(value, bool):
            raise ConfigError(f"{path}: expected a bool, got {value!r}")
        return value
    if tp is int:
        if isinstance(value, bool) or not isinstance(value, int):
            raise ConfigError(f"{path}: expected an int, got {value!r}")
        return value
    if tp is float:
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise ConfigError(f"{path}: expected a number, got {value!r}")
        return float(value)
    if tp is str:
        if not isinstance(value, str):
            raise ConfigError(f"{path}: expected a string, got {value!r}")
        return value
    return freeze(value)


_HINTS: dict[type, dict[str, Any]] = {}


def build_dataclass(cls: type, mapping: Mapping[str, Any], path: str = "") -> Any:
    """Build a frozen config dataclass from a (YAML) mapping, strictly."""

    hints = _HINTS.get(cls)
    if hints is None:
        hints = typing.get_type_hints(cls)
        _HINTS[cls] = hints
    names = {f.name for f in dataclasses.fields(cls) if f.init}
    unknown = sorted(set(mapping) - names)
    if unknown:
        raise ConfigError(f"{path or cls.__name__}: unknown key(s) {unknown}")
    legacy = getattr(cls, "_legacy_values", {})
    kwargs = {}
    for key, value in mapping.items():
        if key in legacy and isinstance(value, str):
            value = legacy[key].get(value, value)
        kwargs[key] = _convert(hints[key], value, f"{path}.{key}" if path else key)
    try:
        return cls(**kwargs)
    except TypeError as error:
        raise ConfigError(f"{path or cls.__name__}: {error}") from error


def _frozen(cls):
    return dataclass(frozen=True)(cls)


# --------------------------------------------------------------------- data
@_frozen
class LengthBucketConfig:
    batch_size: int
    max_length: int | None = None


@_frozen
class PartitionConfig:
    mode: str = "none"
    base_dir: str | None = None
    start_hour: str | None = None
    end_hour: str | None = None
    tz_offset: str | int | None = None


@_frozen
class ReaderConfig:
    engine: str = "pyarrow_dataset"
    columns_pruning: bool = True
    num_workers: int = 0
    adapter_workers: int = 0
    prefetch_batches: int = 2
    max_prefetch_bytes: int = 512 * 1024 * 1024
    pin_memory: bool = False
    coalesce_pinned_tensors: bool = False
    device_prefetch_batches: int = 0
    overlap_host_prepare: bool = True
    host_prepare_prefetch: int = 0
    host_prepare_startup_timeout_sec: float | None = 300.0
    host_prepare_idle_timeout_sec: float | None = 900.0
    step_batch_budget_sec: float | None = 30.0
    deduplicate_request_features: bool = False
    validate_prehashed_nonzero: bool = True
    trusted_input: bool = False
    cardinality_audit_raw_rows: int | None = None
    shard_unit: Literal["file", "row_group", "record_batch"] = "row_group"
    shard_strategy: str = "lpt"
    scanner_batch_rows: int | None = None
    batch_size_rows: int | None = None
    batch_size_candidates: int | None = None
    shuffle_buffer_rows: int = 0
    shuffle_seed: int = 0
    eager_schema_validation: Literal["all", "sample"] = "all"
    schema_validation_samples: int = 64
    length_buckets: tuple[LengthBucketConfig, ...] = ()
    length_bucket_metric: Literal["max", "sum"] = "max"
    agg_direct_mode: Literal["legacy", "direct", "direct_arrow", "compare"] = "legacy"
    from_hdfs: bool = False
    hdfs_close_timeout: float | None = None
    hdfs_file_lock: bool = False
    hdfs_op_timeout: float | None = None
    hdfs_open_timeout: float | None = None
    hdfs_pre_buffer: bool = False
    hdfs_retry_base_sec: float = 1.0
    hdfs_retry_count: int = 3
    on_hdfs_failure: Literal["error", "skip"] = "error"
    worker_stagger_sec: float = 0.0
    partition: PartitionConfig | None = None


@_frozen
class AdapterConfig:
    callable: str
    input_columns: tuple[str, ...] | None = None
    optional_input_columns: tuple[str, ...] = ()
    options: Mapping[str, Any] = field(default_factory=dict)


@_frozen
class ParquetSplitConfig:
    format: Literal["flat_parquet", "adapter_parquet", "agg_parquet"] = "flat_parquet"
    inputs: tuple[str, ...] = ()
    reader: ReaderConfig = field(default_factory=ReaderConfig)
    adapter: AdapterConfig | None = None
    agg_layout: Mapping[str, Any] | None = None
    request_id: str | None = None
    group_id: str | None = None
    labels: Mapping[str, str] = field(default_factory=dict)
    label_masks: Mapping[str, str] = field(default_factory=dict)
    prediction_keys: Mapping[str, str] = field(default_factory=dict)
    prediction_score_suffix: str = ""


@_frozen
class SchemaPolicy:
    allow_missing_nullable_columns: bool = False
    require_same_schema: bool = True
    validate_before_train: bool = True


@_frozen
class DataConfig:
    train: ParquetSplitConfig = field(default_factory=ParquetSplitConfig)
    test: ParquetSplitConfig | None = None
    schema_policy: SchemaPolicy = field(default_factory=SchemaPolicy)


# ----------------------------------------------------------------- features
EncodingType = Literal["vocab", "hash", "pre_hashed", "identity", "shared_vocab"]
EmbeddingScope = Literal["feature", "scenario", "task", "shared"]


@_frozen
class CategoricalEncodingConfig:
    type: EncodingType = "vocab"
    min_count: int | None = None
    max_size: int | None = None
    artifact: str | None = None
    num_buckets: int | None = None
    salt: str | None = None
    max_id: int | None = None
    padding_id: int = 0
    out_of_range: Literal["error", "clip", "zero"] = "error"
    share_with: str | None = None
    share_embedding: bool = False


@_frozen
class FeatureConfig:
    name: str
    kind: Literal["categorical", "dense"]
    source: str = ""
    dtype: str | None = None
    embedding_scope: EmbeddingScope = "feature"
    dimension: int = 1
    embedding_dim: int | None = None
    encoding: CategoricalEncodingConfig | None = None
    pooling: Literal["none", "mean", "sum"] = "none"
    pooling_null_policy: Literal["exclude", "include", "include_as_padding"] = "exclude"
    max_length: int | None = None
    truncation: Literal["head", "tail"] = "tail"
    presence: bool = True


@_frozen
class SequenceFieldConfig:
    name: str
    kind: Literal["categorical", "dense"]
    source: str = ""
    dtype: str | None = None
    dimension: int = 1
    embedding_dim: int | None = None
    encoding: CategoricalEncodingConfig | None = None


SequenceEncoderType = Literal["raw", "attention_pool", "mean_pool", "longer", "stca"]


@_frozen
class SequenceConfig:
    name: str
    fields: tuple[SequenceFieldConfig, ...] = ()
    embedding_scope: EmbeddingScope = "feature"
    layout: str | None = None
    max_length: int | None = None
    truncation: Literal["head", "tail"] = "tail"
    sequence_order: Literal["oldest_to_newest", "newest_to_oldest"] = "oldest_to_newest"
    encoder: SequenceEncoderType = "attention_pool"
    target_inputs: tuple[str, ...] = ()
    rankmixer_summary_tokens: int = 1
    pool_dim: int = 32
    stca_dim: int = 256
    stca_layers: int = 4
    stca_num_heads: int | None = None
    stca_expansion_ratio: int = 4
    stca_parameter_group: str | None = None
    stca_history_group: str | None = None
    longer_dim: int = 32
    longer_num_heads: int | None = None
    longer_hidden_dim: int | None = None
    longer_query_tokens: int = 32
    longer_self_layers: int = 1
    longer_token_merge: int = 1
    longer_inner_layers: int = 0
    longer_output: Literal["full", "summary"] = "full"
    longer_user_global_inputs: tuple[str, ...] = ()
    longer_user_global_tokens: int = 0
    longer_cls_tokens: int = 0
    longer_candidate_global_tokens: int | None = None
    timestamp_field: str | None = None
    time_delta_field: str | None = None
    null_anchor_field: str | None = None


@_frozen
class ScenarioConfig:
    names: tuple[str, ...] = ("default",)
    source: str | None = None
    source_encoding: Literal["auto", "raw", "index"] = "auto"
    auto_discover: bool = False
    max_discovered: int = 256
    discovery_cache_path: str | None = None


@_frozen
class TokenGroupConfig:
    name: str
    inputs: tuple[str, ...] = ()


@_frozen
class DomainTokenConfig:
    name: str
    inputs: tuple[str, ...] = ()
    important_inputs: tuple[str, ...] = ()
    prior_inputs: tuple[str, ...] = ()


@_frozen
class TokenizationConfig:
    feature_tokenizer: Literal["groupwise", "rankmixer", "auto_split"] = "groupwise"
    num_feature_tokens: int | None = None
    feature_token_inputs: tuple[str, ...] = ()
    omit_scene_features: bool = True
    feature_tokens: tuple[TokenGroupConfig, ...] = ()
    sequence_tokens: tuple[TokenGroupConfig, ...] = ()
    ns_tokens: tuple[TokenGroupConfig, ...] = ()
    scenario_tokens: tuple[DomainTokenConfig, ...] = ()
    task_tokens: tuple[DomainTokenConfig, ...] = ()
    scenario_token_inputs: tuple[str, ...] = ()
    task_token_inputs: tuple[str, ...] = ()


@_frozen
class VocabStrategy:
    defaults: Mapping[str, Any] = field(default_factory=dict)
    features: Mapping[str, Any] = field(default_factory=dict)


# ------------------------------------------------------------------ runtime
@_frozen
class RuntimeConfig:
    device: str = "cpu"
    precision: Literal["fp32", "bf16", "fp16"] = "fp32"
    allow_tf32: bool = True
    compile: bool = False
    compile_mode: Literal["default", "reduce-overhead"] = "default"
    cuda_graph_backbone: bool = False
    require_compact_sequence_batches: bool = False
    trim_all_invalid_sequence_prefix: bool = True
    validate_scenario_ids: bool = True
    activation_checkpoint: Literal["none", "selective", "full"] | bool = "none"
    attention_backend: Literal["auto", "sdpa", "flash"] = "flash"
    varlen_packing: Literal["fixed", "compact"] = "fixed"
    domain_varlen_packing: Literal["fixed", "compact"] | None = None
    checkpoint_domain_blocks: bool = False
    sequence_projection_chunk_tokens: int = 0
    sequence_encoder_chunk_rows: int = 0
    sequence_encoder_chunk_tokens: int = 0
    onetrans_batched_ns: bool = True
    distributed: Literal["none", "ddp"] = "none"
    nproc_per_node: int | None = 1
    master_addr: str = "127.0.0.1"
    master_port: int = 29500
    kernel_backend: Literal["native", "torch"] = "native"

    def __post_init__(self) -> None:
        # YAML booleans are accepted as the reference does: true -> full, false -> none.
        if isinstance(self.activation_checkpoint, bool):
            object.__setattr__(self, "activation_checkpoint", "full" if self.activation_checkpoint else "none")


# -------------------------------------------------------------------- model
@_frozen
class ModelConfig:
    # old spellings accepted by the reference loader (src/config.py:2558-2564)
    _legacy_values = {"mdl_feature_interaction": {"paper": "direct_ffn", "rankmixer_full": "residual_ffn"}}

    name: Literal["rankmixer", "mdl_rankmixer", "onetrans", "mdl_onetrans", "mixformer", "mdl_mixformer", "longer"]
    embedding_dim: int = 32
    token_dim: int = 768
    num_layers: int = 6
    num_heads: int = 12
    hidden_dim: int = 1536
    init_std: float = 0.02
    ffn_activation: Literal["gelu", "relu"] = "gelu"
    task_head_hidden_dim: int | None = None
    task_head_dropout: float = 0.0
    task_head_activation: Literal["gelu", "relu"] = "gelu"
    readout: Literal["default", "task_query"] = "default"
    use_task_tokens: bool = True
    use_scenario_tokens: bool = True
    use_global_scenario_token: bool = True
    use_task_feature_interaction: bool = True
    use_scenario_feature_interaction: bool = True
    mdl_feature_interaction: Literal["direct_ffn", "residual_ffn"] = "residual_ffn"
    mdl_token_state: Literal["coupled", "split"] = "coupled"
    scene_feature_bias: Literal["none", "additive", "film"] = "none"
    tokens_per_scenario: int = 1
    use_request_cache: bool = False
    first_domain_sequence_layer: int | None = None
    use_pyramid: bool = True
    pyramid_round_to: int = 32
    pyramid_schedule: Literal["linear", "halve"] = "linear"
    pyramid_halve_every: int = 2
    ns_tokenizer: Literal["auto_split", "groupwise", "dcnv2"] = "auto_split"
    num_ns_tokens: int | None = None
    ns_dcn_cross_layers: int = 3
    ns_dcn_deep_layers: int = 2
    ns_dcn_projection_dim: int | None = None
    ns_dcn_low_rank: int | None = None
    ns_dcn_deep_dim: int | None = None
    max_position_embeddings: int | None = None
    use_sep_tokens: bool = True
    final_s_tokens: int | None = None
    sequence_fusion: Literal["intent_ordered", "timestamp_aware"] = "intent_ordered"
    global_sequence_max_length: int | None = None
    mixformer_user_head_count: int | None = None
    mdl_mixformer_query_conditioning: bool = True
    sequence_head: Literal["none", "mixformer"] = "none"
    rankmixer_ffn_type: Literal["dense", "sparse_moe"] = "dense"
    sparse_moe_num_experts: int = 4
    sparse_moe_use_dtsi: bool = True
    sparse_moe_inference_threshold: float = 0.0
    sparse_moe_target_active_ratio: float = 0.25
    sparse_moe_regularization_initial: float = 1.0e-8
    sparse_moe_regularization_multiplier: float = 1.2
    sparse_moe_loss_weight: float = 1.0
    sparse_moe_dtsi_training_output: Literal["dense_router", "mean"] | None = None
    experimental_model_acknowledged: bool = False


# ----------------------------------------------------------------- training
@_frozen
class EmbeddingShardingConfig:
    strategy: Literal["auto", "row_wise", "table_wise"] = "auto"
    local_dedup: bool = True
    table_wise_max_rows: int = 65536


@_frozen
class DDPConfig:
    static_graph: bool = False
    find_unused_parameters: bool = True
    gradient_as_bucket_view: bool = True
    bucket_cap_mb: float = 25.0
    audit_steps: int = 10
    validated_no_unused_parameters: bool = False
    validated_static_graph: bool = False


@_frozen
class FixedTestEvalConfig:
    enabled: bool = True
    every_steps: int = 5000
    files_per_rank: int = 4
    auc_bins: int = 4096


@_frozen
class CheckpointConfig:
    dir: str | None = None
    run_name: str | None = None
    every_steps: int = 0
    keep_last: int = 3
    save_on_exit: bool = True
    resume: str | None = None
    # stage each step on local disk and publish it to the run directory from a
    # background thread (training does not wait for the run directory)
    async_upload: bool = True
    staging_dir: str | None = None
    shard_chunk_bytes: int = 2 * 1024 ** 3
    # refuse to start when the staging filesystem cannot hold this node's ranks' files
    preflight_staging: bool = True
    # rank 0 waits this long for every rank's READY marker before committing a step
    ready_timeout_sec: float = 1800.0
    data_resume: bool = True
    data_resume_rewind: int = 1


@_frozen
class TrainingConfig:
    batch_size: int = 2048
    gradient_accumulation_steps: int = 1
    lr_dense: float = 1.0e-4
    lr_sparse: float | None = None
    lr_schedule: Literal["constant", "cosine"] = "constant"
    lr_warmup_steps: int = 5000
    warmup_steps: int | None = None
    lr_decay_steps: int | None = None
    lr_min_ratio: float = 0.0
    dense_optimizer: Literal["rmsprop", "adam"] = "rmsprop"
    fused_dense_optimizer: bool = True
    dense_optimizer_foreach_bucket_mb: int = 0
    rmsprop_alpha: float = 0.99999
    rmsprop_momentum: float = 0.0
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    adam_eps: float = 1.0e-8
    weight_decay: float = 0.0
    sparse_optimizer: Literal["adagrad", "rowwise_adagrad"] = "adagrad"
    adagrad_lr_decay: float = 0.0
    adagrad_weight_decay: float = 0.0
    adagrad_initial_accumulator_value: float = 0.1
    adagrad_eps: float = 1.0e-10
    embedding_distribution: Literal["replicated", "sharded"] = "replicated"
    dense_distribution: Literal["ddp"] = "ddp"
    embedding_sharding: EmbeddingShardingConfig = field(default_factory=EmbeddingShardingConfig)
    ddp: DDPConfig = field(default_factory=DDPConfig)
    embedding_sparse_gradients: bool = True
    embedding_weight_dtype: Literal["fp32", "bf16"] = "fp32"
    embedding_collect_stats: bool = False
    embedding_validate_indices: bool = True
    sparse_embedding_size_threshold_gb: float | None = None
    sparse_update_mode: Literal["ddp_synced_adagrad", "external_parameter_server"] = "ddp_synced_adagrad"
    sparse_parameter_server_adapter: str | None = None
    dense_clip_norm: float | None = None
    sparse_clip_norm: float | None = None
    loss_reduction: Literal["sum", "mean_per_task", "mean_per_request_per_task"] = "sum"
    task_loss_weights: Mapping[str, float] = field(default_factory=dict)
    log_every_steps: int = 100
    step_watchdog_sec: float | None = 600.0
    fixed_test_eval: FixedTestEvalConfig = field(default_factory=FixedTestEvalConfig)
    eval_interval: int | None = None
    eval_batches: int | None = None
    checkpoint_path: str | None = None
    save_checkpoint: bool = True
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    comm: Literal["fused", "nccl"] = "fused"


# ---------------------------------------------------------------------- app
@_frozen
class AppConfig:
    data: DataConfig = field(default_factory=DataConfig)
    features: tuple[FeatureConfig, ...] = ()
    sequences: tuple[SequenceConfig, ...] = ()
    vocab_strategy: VocabStrategy = field(default_factory=VocabStrategy)
    model: ModelConfig = field(default_factory=lambda: ModelConfig(name="rankmixer"))
    scenarios: ScenarioConfig = field(default_factory=ScenarioConfig)
    tokenization: TokenizationConfig = field(default_factory=TokenizationConfig)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)
    training: TrainingConfig = field(default_factory=TrainingConfig)
    extends: str | None = None

    @property
    def task_names(self) -> tuple[str, ...]:
        """Task (label) names in config order (``data.train.labels``)."""

        return tuple(self.data.train.labels.keys()) or ("label",)

    @property
    def resolved(self):
        from .resolve import resolve_app_config

        cached = self.__dict__.get("_resolved_cache")
        if cached is None:
            cached = resolve_app_config(self)
            object.__setattr__(self, "_resolved_cache", cached)
        return cached

    def replace(self, **changes: Any) -> "AppConfig":
        new = dataclasses.replace(self, **changes)
        new.__dict__.pop("_resolved_cache", None)
        return new
