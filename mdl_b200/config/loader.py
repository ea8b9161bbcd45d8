"""YAML loading with ``extends:`` inheritance (reference ``src/config.py:5413-5461``).

A config file may name a parent with ``extends: parent.yaml`` (relative to the
child). Mappings are deep-merged child-over-parent; lists and scalars in the
child replace the parent's. Cycles are detected and reported with the chain.
"""

from __future__ import annotations

from collections.abc import Mapping
from pathlib import Path
from typing import Any

import yaml

from .schema import AppConfig, ConfigError, build_dataclass


def merge_config_mappings(parent: Mapping[str, Any], child: Mapping[str, Any]) -> dict[str, Any]:
    """Deep merge: nested mappings merge key by key; anything else is replaced."""

    merged: dict[str, Any] = dict(parent)
    for key, value in child.items():
        base = merged.get(key)
        if isinstance(base, Mapping) and isinstance(value, Mapping):
            merged[key] = merge_config_mappings(base, value)
        else:
            merged[key] = value
    return merged


def load_config_mapping(path: str | Path, _chain: tuple[Path, ...] = ()) -> dict[str, Any]:
    """Read a YAML file and resolve its ``extends`` chain into one mapping."""

    resolved = Path(path).expanduser().resolve()
    if resolved in _chain:
        chain = " -> ".join(str(p) for p in (*_chain, resolved))
        raise ConfigError(f"config extends cycle: {chain}")
    with resolved.open("r", encoding="utf-8") as handle:
        data = yaml.safe_load(handle) or {}
    if not isinstance(data, Mapping):
        raise ConfigError(f"{resolved}: top level must be a mapping")
    data = dict(data)
    parent_ref = data.pop("extends", None)
    if parent_ref is None:
        return data
    if not isinstance(parent_ref, str):
        raise ConfigError(f"{resolved}: extends must be a path string")
    parent_path = (resolved.parent / parent_ref).resolve()
    parent = load_config_mapping(parent_path, (*_chain, resolved))
    return merge_config_mappings(parent, data)


def app_config_from_mapping(mapping: Mapping[str, Any], *, validate: bool = True) -> AppConfig:
    """Build (and by default validate) an :class:`AppConfig` from a mapping."""

    if "model" not in mapping:
        raise ConfigError("config is missing the 'model' section")
    config = build_dataclass(AppConfig, mapping)
    if validate:
        from .validate import validate_app_config

        validate_app_config(config)
    return config


def load_app_config(path: str | Path, *, validate: bool = True) -> AppConfig:
    """Load a YAML config file (with ``extends``) into a frozen :class:`AppConfig`."""

    return app_config_from_mapping(load_config_mapping(path), validate=validate)


def dump_app_config(config: AppConfig) -> str:
    """Serialise a config back to YAML (round-trips through :func:`load_app_config`)."""

    from .schema import thaw

    data = thaw(config)
    data.pop("extends", None)
    return yaml.safe_dump(data, sort_keys=False)
