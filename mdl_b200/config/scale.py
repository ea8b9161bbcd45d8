"""Smoke-sized copies of production configs.

``shrink_mapping`` keeps a config's architecture (features, sequences, token layout,
model family and widths) and caps what only costs memory or time: embedding table
rows (``num_buckets`` / ``max_id``), sequence lengths, LONGER query windows and the
batch size. Used to build and train every shipped reference config on a CPU in
tests, and for quick local runs of production configs.
"""

from __future__ import annotations

import copy
from typing import Any


def _cap_encoding(enc: dict | None, max_rows: int) -> None:
    if not isinstance(enc, dict):
        return
    if enc.get("num_buckets"):
        n = min(int(enc["num_buckets"]), max_rows)
        if enc.get("type") == "pre_hashed":  # keep a power of two
            n = 1 << max(0, n.bit_length() - 1)
        enc["num_buckets"] = n
    if enc.get("max_id"):
        enc["max_id"] = min(int(enc["max_id"]), max_rows)


def shrink_mapping(mapping: dict[str, Any], *, max_rows: int = 512, max_length: int = 16, batch: int = 16,
                   device: str = "cpu", max_hidden: int | None = None) -> dict[str, Any]:
    """``max_hidden`` also caps the FFN / head hidden widths (token widths, token counts
    and head counts stay as configured)."""

    m = copy.deepcopy(mapping)
    for f in m.get("features", []):
        _cap_encoding(f.get("encoding"), max_rows)
        if f.get("max_length"):
            f["max_length"] = min(int(f["max_length"]), max_length)
    for strat in (m.get("vocab_strategy") or {}).get("features", {}).values():
        _cap_encoding(strat, max_rows)
    for s in m.get("sequences", []):
        for fl in s.get("fields", []):
            _cap_encoding(fl.get("encoding"), max_rows)
        if s.get("max_length"):
            s["max_length"] = min(int(s["max_length"]), max_length)
        if s.get("longer_query_tokens"):
            s["longer_query_tokens"] = min(int(s["longer_query_tokens"]), max(1, max_length // 2))
    model = m.setdefault("model", {})
    if max_hidden:
        for key in ("hidden_dim", "task_head_hidden_dim"):
            if model.get(key):
                model[key] = min(int(model[key]), int(max_hidden))
        for s in m.get("sequences", []):
            if s.get("longer_hidden_dim"):
                s["longer_hidden_dim"] = min(int(s["longer_hidden_dim"]), int(max_hidden))
    if model.get("max_position_embeddings"):
        model["max_position_embeddings"] = min(int(model["max_position_embeddings"]), 64 * max_length)
    runtime = m.setdefault("runtime", {})
    runtime["device"] = device
    if device == "cpu":
        runtime["precision"] = "fp32"
        runtime["attention_backend"] = "sdpa"
    training = m.setdefault("training", {})
    training["batch_size"] = batch
    training["save_checkpoint"] = False
    training.setdefault("fixed_test_eval", {})["enabled"] = False
    return m
