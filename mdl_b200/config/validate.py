"""Cross-field validation of an :class:`AppConfig`.

Covers the checks of the reference's ``validate_app_config``
(``src/config.py:4819-5410``) that this framework relies on: unique names,
token references that exist, divisibility rules of each model family,
encoding parameters and optimizer/loss settings.
"""

from __future__ import annotations

from .schema import AppConfig, ConfigError


def _require(cond: bool, message: str) -> None:
    if not cond:
        raise ConfigError(message)


def validate_app_config(config: AppConfig) -> None:
    names = [f.name for f in config.features] + [s.name for s in config.sequences]
    dupes = sorted({n for n in names if names.count(n) > 1})
    _require(not dupes, f"duplicate feature/sequence names: {dupes}")
    known = set(names)
    for feature in config.features:
        if feature.kind == "categorical":
            enc = feature.encoding
            if enc is not None and enc.type in ("hash", "pre_hashed"):
                _require(bool(enc.num_buckets) and enc.num_buckets > 0,
                         f"feature {feature.name}: {enc.type} encoding needs num_buckets > 0")
            if enc is not None and enc.type == "pre_hashed":
                n = int(enc.num_buckets or 0)
                _require(n & (n - 1) == 0, f"feature {feature.name}: pre_hashed num_buckets must be a power of two")
            if enc is not None and enc.share_with is not None:
                _require(enc.share_with in known or any(
                    f"{s.name}.{fl.name}" == enc.share_with for s in config.sequences for fl in s.fields),
                    f"feature {feature.name}: share_with {enc.share_with!r} is unknown")
        else:
            _require(feature.pooling == "none", f"dense feature {feature.name} cannot be pooled")
            _require(feature.dimension > 0, f"dense feature {feature.name}: dimension must be positive")
    for sequence in config.sequences:
        _require(len(sequence.fields) > 0 or sequence.encoder == "raw",
                 f"sequence {sequence.name} has no fields")
    tok = config.tokenization
    for group in (*tok.feature_tokens, *tok.sequence_tokens):
        for item in group.inputs:
            _require(item in known, f"token group {group.name}: unknown input {item!r}")
    for item in tok.feature_token_inputs:
        _require(item in known, f"tokenization.feature_token_inputs: unknown input {item!r}")

    # options this framework implements differently or not at all are rejected, never
    # silently changed into something else
    rt = config.runtime
    _require(rt.precision != "fp16", "runtime.precision fp16 (autocast with a GradScaler) is not implemented; use bf16")
    if rt.device == "cuda" and rt.kernel_backend == "native":
        _require(rt.precision == "bf16", f"runtime.precision {rt.precision!r} on CUDA: the sm_100a kernels compute in "
                                         "bf16 (use precision bf16, or kernel_backend torch for fp32 math)")
    seq_by_name = {s.name: s for s in config.sequences}
    for sequence in config.sequences:
        if sequence.encoder == "longer":
            _require(int(sequence.longer_token_merge) >= 1 and int(sequence.longer_inner_layers) >= 0,
                     f"sequence {sequence.name!r}: longer_token_merge must be >= 1 and longer_inner_layers >= 0")
    model = config.model
    if model.name in ("rankmixer", "mdl_rankmixer"):
        raw = [n for n in config.resolved.tokenization.feature_token_inputs
               if n in seq_by_name and seq_by_name[n].encoder == "raw"]
        _require(not raw, f"{model.name} feature tokens cannot read raw sequences {raw}: give them a summary encoder "
                          "(mean_pool, attention_pool, longer or stca)")
    _require(model.sequence_fusion in ("intent_ordered", "timestamp_aware"),
             f"model.sequence_fusion {model.sequence_fusion!r}")
    _require(model.token_dim > 0 and model.num_layers >= 0 and model.hidden_dim > 0, "model dims must be positive")
    if model.name in ("rankmixer", "mdl_rankmixer"):
        count = config.resolved.tokenization.feature_token_count
        _require(count > 0, "rankmixer needs at least one feature token")
        _require(model.token_dim % count == 0,
                 f"rankmixer requires token_dim ({model.token_dim}) divisible by the feature token count ({count})")
    if model.name in ("onetrans", "mdl_onetrans", "mixformer", "mdl_mixformer", "longer"):
        _require(model.token_dim % model.num_heads == 0, "token_dim must be divisible by num_heads")
    if model.name.startswith("mdl_"):
        _require(model.tokens_per_scenario >= 1, "tokens_per_scenario must be >= 1")
    if model.name in ("mdl_onetrans", "mdl_mixformer"):
        # experimental compositions (reference ``ModelConfig`` validation, src/config.py:2826-2833)
        _require(model.experimental_model_acknowledged,
                 f"{model.name} is an experimental composition: set model.experimental_model_acknowledged: true")
    _require(model.readout != "task_query" or model.name in ("onetrans", "mixformer"),
             "model.readout=task_query is the equal-readout control of the onetrans and mixformer baselines")
    if model.first_domain_sequence_layer is not None:
        _require(0 <= model.first_domain_sequence_layer < model.num_layers,
                 "model.first_domain_sequence_layer must be in [0, model.num_layers)")
    if model.rankmixer_ffn_type == "sparse_moe":
        _require(model.sparse_moe_num_experts > 0, "model.sparse_moe_num_experts must be positive")
        _require(0.0 < model.sparse_moe_target_active_ratio <= 1.0,
                 "model.sparse_moe_target_active_ratio must be in (0, 1]")
        _require(model.sparse_moe_regularization_initial > 0.0,
                 "model.sparse_moe_regularization_initial must be positive")
        _require(model.sparse_moe_regularization_multiplier > 1.0,
                 "model.sparse_moe_regularization_multiplier must be greater than 1")
        _require(model.sparse_moe_loss_weight >= 0.0, "model.sparse_moe_loss_weight must be non-negative")
        _require(not model.sparse_moe_use_dtsi or model.sparse_moe_dtsi_training_output is not None,
                 "DTSI needs model.sparse_moe_dtsi_training_output (dense_router or mean)")
    train = config.training
    _require(train.batch_size > 0, "training.batch_size must be positive")
    _require(not train.rmsprop_momentum, "training.rmsprop_momentum: RMSprop with momentum is not implemented")
    _require(train.gradient_accumulation_steps >= 1, "gradient_accumulation_steps must be >= 1")
    _require(train.lr_dense > 0, "lr_dense must be positive")
    for task in train.task_loss_weights:
        _require(task in config.task_names, f"task_loss_weights names unknown task {task!r}")
    if train.sparse_update_mode == "external_parameter_server":
        _require(bool(train.sparse_parameter_server_adapter),
                 "external_parameter_server needs sparse_parameter_server_adapter")
    if config.scenarios.source_encoding == "index":
        _require(len(config.scenarios.names) > 0, "index scenario encoding needs scenario names")
