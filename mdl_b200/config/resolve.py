"""Resolved (derived) config: token layouts, embedding dims, scene filtering.

Mirrors the reference's ``resolve_app_config`` (``src/config.py:4424``),
``resolve_tokenization`` (:4189), ``resolve_categorical_embedding_dims``
(:4344) and ``resolve_onetrans_max_position_embeddings`` (:4763): the
derived values every model constructor needs, computed once per config.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import MappingProxyType
from typing import Mapping

from .schema import AppConfig, FeatureConfig, SequenceConfig


@dataclass(frozen=True)
class ResolvedTokenGroup:
    name: str
    inputs: tuple[str, ...]


@dataclass(frozen=True)
class ResolvedDomainToken:
    name: str
    kind: str  # "scenario", "global" or "task"
    scenario_index: int | None
    important_inputs: tuple[str, ...]
    prior_inputs: tuple[str, ...]
    inputs: tuple[str, ...] = ()

    def resolved_inputs(self) -> list[str]:
        """Projector inputs in order: direct, important, prior (duplicates dropped)."""

        return list(dict.fromkeys((*self.inputs, *self.important_inputs, *self.prior_inputs)))


@dataclass(frozen=True)
class ResolvedTokenization:
    feature_tokenizer: str
    feature_token_inputs: tuple[str, ...]
    feature_token_count: int
    feature_token_groups: tuple[ResolvedTokenGroup, ...]
    sequence_token_groups: tuple[ResolvedTokenGroup, ...]
    scenario_token_specs: tuple[ResolvedDomainToken, ...]
    task_token_specs: tuple[ResolvedDomainToken, ...]
    sequence_names: tuple[str, ...]
    ns_token_groups: tuple[ResolvedTokenGroup, ...] = ()


@dataclass(frozen=True)
class ResolvedConfig:
    tokenization: ResolvedTokenization
    categorical_embedding_dims: Mapping[str, int]
    scalar_input_dims: Mapping[str, int]
    scene_feature_names: tuple[str, ...]
    onetrans_max_position_embeddings: int


def scene_feature_names(config: AppConfig) -> tuple[str, ...]:
    """Scalar features that carry the scenario id itself (omitted from tokens)."""

    source = config.scenarios.source
    if not source:
        return ()
    return tuple(f.name for f in config.features if f.source == source or f.name == source)


def categorical_embedding_dim(config: AppConfig, feature: FeatureConfig) -> int:
    return int(feature.embedding_dim or config.model.embedding_dim)


def scalar_input_dim(config: AppConfig, feature: FeatureConfig) -> int:
    """Width of the encoded (pooled) value of one scalar feature."""

    if feature.kind == "dense":
        return int(feature.dimension) + (1 if feature.presence else 0)
    return categorical_embedding_dim(config, feature)


def sequence_output_dim(config: AppConfig, sequence: SequenceConfig) -> int:
    """Width of a pooled sequence summary as a token input."""

    if sequence.encoder == "longer":
        return int(sequence.longer_dim)
    if sequence.encoder == "stca":
        return int(sequence.stca_dim)
    return int(sequence.pool_dim)


def tokenizable_input_names(config: AppConfig) -> tuple[str, ...]:
    """Inputs that become feature tokens by default: embedding scope ``feature`` or ``shared``
    (scenario/task-scope inputs only feed MDL domain tokens; reference ``src/config.py:3730-3744``)."""

    keep = ("feature", "shared")
    names = [f.name for f in config.features if f.embedding_scope in keep]
    names += [s.name for s in config.sequences if s.encoder != "raw" and s.embedding_scope in keep]
    return tuple(names)


def resolve_tokenization(config: AppConfig) -> ResolvedTokenization:
    tok = config.tokenization
    omit = set(scene_feature_names(config)) if tok.omit_scene_features else set()
    inputs = tuple(n for n in (tok.feature_token_inputs or tokenizable_input_names(config)) if n not in omit)
    if tok.feature_tokens:
        groups = []
        for group in tok.feature_tokens:
            kept = tuple(n for n in group.inputs if n not in omit)
            if kept:
                groups.append(ResolvedTokenGroup(group.name, kept))
        groups = tuple(groups)
    else:
        groups = tuple(ResolvedTokenGroup(n, (n,)) for n in inputs)
    if tok.feature_tokenizer == "groupwise":
        if tok.feature_tokens and not tok.feature_token_inputs:
            inputs = tuple(n for g in groups for n in g.inputs)
        count = len(groups)
    else:
        count = int(tok.num_feature_tokens or len(inputs))
    seq_groups = tuple(ResolvedTokenGroup(g.name, tuple(g.inputs)) for g in tok.sequence_tokens)
    # OneTrans groupwise NS tokens (reference ``_scalar_token_groups`` src/config.py:4083-4106):
    # tokenization.ns_tokens, else the all-scalar feature_tokens groups, else one per feature
    seq_names = {s.name for s in config.sequences}
    feat_names = {f.name for f in config.features}
    if tok.ns_tokens:
        ns_groups = tuple(ResolvedTokenGroup(g.name, tuple(g.inputs)) for g in tok.ns_tokens)
    elif tok.feature_tokens:
        ns_groups = tuple(ResolvedTokenGroup(g.name, tuple(g.inputs)) for g in tok.feature_tokens
                          if all(n in feat_names and n not in seq_names for n in g.inputs))
    else:
        ns_groups = tuple(ResolvedTokenGroup(f.name, (f.name,)) for f in config.features
                          if f.embedding_scope in ("feature", "shared"))

    scenario_specs: list[ResolvedDomainToken] = []
    by_name = {t.name: t for t in tok.scenario_tokens}
    per_scene = max(1, int(config.model.tokens_per_scenario))
    for index, scene in enumerate(config.scenarios.names):
        spec = by_name.get(scene)
        for k in range(per_scene):
            name = scene if per_scene == 1 else f"{scene}#{k}"
            scenario_specs.append(
                ResolvedDomainToken(
                    name=name,
                    kind="scenario",
                    scenario_index=index,
                    important_inputs=tuple(spec.important_inputs) if spec else tuple(tok.scenario_token_inputs),
                    prior_inputs=tuple(spec.prior_inputs) if spec else (),
                    inputs=tuple(spec.inputs) if spec else (),
                )
            )
    if config.model.use_global_scenario_token:
        spec = by_name.get("global")
        scenario_specs.append(
            ResolvedDomainToken(
                name="global",
                kind="global",
                scenario_index=None,
                important_inputs=tuple(spec.important_inputs) if spec else tuple(tok.scenario_token_inputs),
                prior_inputs=tuple(spec.prior_inputs) if spec else (),
                inputs=tuple(spec.inputs) if spec else (),
            )
        )
    task_by_name = {t.name: t for t in tok.task_tokens}
    task_specs = tuple(
        ResolvedDomainToken(
            name=task,
            kind="task",
            scenario_index=None,
            important_inputs=tuple(task_by_name[task].important_inputs) if task in task_by_name
            else tuple(tok.task_token_inputs),
            prior_inputs=tuple(task_by_name[task].prior_inputs) if task in task_by_name else (),
            inputs=tuple(task_by_name[task].inputs) if task in task_by_name else (),
        )
        for task in config.task_names
    )
    return ResolvedTokenization(
        feature_tokenizer=tok.feature_tokenizer,
        feature_token_inputs=inputs,
        feature_token_count=count,
        feature_token_groups=groups,
        sequence_token_groups=seq_groups,
        scenario_token_specs=tuple(scenario_specs),
        task_token_specs=task_specs,
        sequence_names=tuple(s.name for s in config.sequences),
        ns_token_groups=ns_groups,
    )


def resolve_onetrans_max_position_embeddings(config: AppConfig) -> int:
    if config.model.max_position_embeddings:
        return int(config.model.max_position_embeddings)
    total = 0
    for sequence in config.sequences:
        total += int(sequence.max_length or 0) + (1 if config.model.use_sep_tokens else 0)
    if config.model.global_sequence_max_length:
        total = max(total, int(config.model.global_sequence_max_length))
    ns = int(config.model.num_ns_tokens or 0)
    return max(1, total + ns)


def resolve_app_config(config: AppConfig) -> ResolvedConfig:
    dims = {}
    scalar_dims = {}
    for feature in config.features:
        if feature.kind == "categorical":
            dims[feature.name] = categorical_embedding_dim(config, feature)
        scalar_dims[feature.name] = scalar_input_dim(config, feature)
    for sequence in config.sequences:
        scalar_dims[sequence.name] = sequence_output_dim(config, sequence)
        for fld in sequence.fields:
            if fld.kind == "categorical":
                dims[f"{sequence.name}.{fld.name}"] = int(fld.embedding_dim or config.model.embedding_dim)
    return ResolvedConfig(
        tokenization=resolve_tokenization(config),
        categorical_embedding_dims=MappingProxyType(dims),
        scalar_input_dims=MappingProxyType(scalar_dims),
        scene_feature_names=scene_feature_names(config),
        onetrans_max_position_embeddings=resolve_onetrans_max_position_embeddings(config),
    )
