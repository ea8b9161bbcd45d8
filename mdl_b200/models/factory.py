"""Model factory: ``model.name`` -> model class (reference ``build_model`` ``src/model.py:8953-9001``)."""

from __future__ import annotations

import torch

from ..config.schema import AppConfig


def build_model(config: AppConfig, *, device: torch.device | str = "cpu", rank: int = 0, world: int = 1,
                process_group=None, vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None):
    name = config.model.name
    kw = dict(device=torch.device(device), rank=rank, world=world, process_group=process_group,
              vocab_sizes=vocab_sizes, base_seed=base_seed)
    if name == "rankmixer":
        from .rankmixer import RankMixerModel

        return RankMixerModel(config, **kw)
    if name == "mdl_rankmixer":
        from .mdl import MDLRankMixerModel

        return MDLRankMixerModel(config, **kw)
    if name in ("onetrans", "mdl_onetrans"):
        from .onetrans import build_onetrans

        return build_onetrans(config, **kw)
    if name in ("mixformer", "mdl_mixformer"):
        from .mixformer import build_mixformer

        return build_mixformer(config, **kw)
    if name == "longer":
        from .longer import LongerModel

        return LongerModel(config, **kw)
    raise ValueError(f"unknown model.name {name!r}")
