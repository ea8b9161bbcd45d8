"""Config system: YAML schema, ``extends`` loader, resolution and validation."""

from .loader import app_config_from_mapping, dump_app_config, load_app_config, load_config_mapping, merge_config_mappings
from .schema import AppConfig, ConfigError, freeze, thaw

__all__ = [
    "AppConfig",
    "ConfigError",
    "app_config_from_mapping",
    "dump_app_config",
    "freeze",
    "load_app_config",
    "load_config_mapping",
    "merge_config_mappings",
    "thaw",
]
