"""Embedding model-parallel sharding plan.

Ownership rules are part of the on-disk checkpoint format, so they are kept
identical to the reference (``src/embeddings.py:163-353``):

* ``row_wise``: ``owner(id) = (id + offset) % W`` and ``local_row = id // W``,
  where ``offset = int.from_bytes(sha256(name)[:8], 'little') % W``.
* ``table_wise``: the whole table lives on one rank, chosen by a
  longest-processing-time pass over the per-rank memory load (weights plus
  optimizer state), largest tables first, ties to the lowest rank.
* ``auto``: table-wise when ``rows <= table_wise_max_rows``, else row-wise.

The plan fingerprint (sha256 over a canonical JSON payload) lets ranks and
checkpoints verify they agree on the layout.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from hashlib import sha256
from typing import Iterable, Literal

import torch

OptimizerStateLayout = Literal["full", "rowwise"]


def embedding_local_bytes(*, rows: int, embedding_dim: int, weight_element_size: int,
                          optimizer_state_layout: OptimizerStateLayout = "full") -> int:
    """Bytes of one local shard: weights plus sparse Adagrad state."""

    if rows < 0 or embedding_dim < 0 or weight_element_size <= 0:
        raise ValueError("rows, embedding_dim and weight_element_size must be valid")
    state = rows * embedding_dim * 4 if optimizer_state_layout == "full" else rows * 4
    return rows * embedding_dim * weight_element_size + state


@dataclass(frozen=True)
class EmbeddingTableSpec:
    name: str
    num_embeddings: int
    embedding_dim: int
    element_size: int = 4

    @property
    def weight_bytes(self) -> int:
        return self.num_embeddings * self.embedding_dim * self.element_size


@dataclass(frozen=True)
class EmbeddingShardSpec:
    table_name: str
    strategy: Literal["row_wise", "table_wise"]
    world_size: int
    cyclic_offset: int = 0
    table_owner: int | None = None

    def owner(self, ids: torch.Tensor) -> torch.Tensor:
        if self.strategy == "row_wise":
            return torch.remainder(ids + self.cyclic_offset, self.world_size)
        if self.table_owner is None:
            raise RuntimeError("table-wise shard is missing its owner")
        return torch.full_like(ids, self.table_owner)

    def owner_of(self, index: int) -> int:
        if self.strategy == "row_wise":
            return (index + self.cyclic_offset) % self.world_size
        return int(self.table_owner)

    def local_rows(self, num_embeddings: int, rank: int) -> int:
        if self.strategy == "table_wise":
            return num_embeddings if rank == self.table_owner else 0
        residue = (rank - self.cyclic_offset) % self.world_size
        if residue >= num_embeddings:
            return 0
        return (num_embeddings - 1 - residue) // self.world_size + 1

    def local_row_ids(self, global_ids: torch.Tensor) -> torch.Tensor:
        if self.strategy == "table_wise":
            return global_ids
        return torch.div(global_ids, self.world_size, rounding_mode="floor")

    def global_ids(self, num_embeddings: int, rank: int) -> torch.Tensor:
        """Global ids of this rank's local rows, in local-row order."""

        if self.strategy == "table_wise":
            if rank != self.table_owner:
                return torch.empty(0, dtype=torch.long)
            return torch.arange(num_embeddings, dtype=torch.long)
        n_local = self.local_rows(num_embeddings, rank)
        local = torch.arange(n_local, dtype=torch.long)
        residue = (rank - self.cyclic_offset) % self.world_size
        # row r holds the id with id // W == r and (id + offset) % W == rank
        return local * self.world_size + residue


@dataclass(frozen=True)
class EmbeddingShardingPlan:
    world_size: int
    tables: dict[str, EmbeddingShardSpec]
    fingerprint: str


def stable_offset(table_name: str, world_size: int) -> int:
    if world_size <= 1:
        return 0
    return int.from_bytes(sha256(table_name.encode("utf-8")).digest()[:8], "little") % world_size


def plan_embedding_shards(table_specs: Iterable[EmbeddingTableSpec], *, world_size: int,
                          strategy: Literal["auto", "row_wise", "table_wise"] = "auto",
                          table_wise_max_rows: int = 65536,
                          optimizer_state_layout: OptimizerStateLayout = "full") -> EmbeddingShardingPlan:
    """Deterministic plan shared by every rank (same inputs -> same plan)."""

    if world_size <= 0:
        raise ValueError("world_size must be positive")
    if strategy not in {"auto", "row_wise", "table_wise"}:
        raise ValueError("strategy must be auto, row_wise or table_wise")
    specs = sorted(table_specs, key=lambda item: item.name)
    if len({s.name for s in specs}) != len(specs):
        raise ValueError("embedding table names must be unique")
    loads = [0] * world_size
    planned: dict[str, EmbeddingShardSpec] = {}
    deferred: list[EmbeddingTableSpec] = []
    for table in specs:
        if strategy == "table_wise" or (strategy == "auto" and table.num_embeddings <= table_wise_max_rows):
            deferred.append(table)
            continue
        shard = EmbeddingShardSpec(table.name, "row_wise", world_size, cyclic_offset=stable_offset(table.name, world_size))
        planned[table.name] = shard
        for rank in range(world_size):
            loads[rank] += embedding_local_bytes(
                rows=shard.local_rows(table.num_embeddings, rank), embedding_dim=table.embedding_dim,
                weight_element_size=table.element_size, optimizer_state_layout=optimizer_state_layout)
    for table in sorted(deferred, key=lambda item: (-item.weight_bytes, item.name)):
        owner = min(range(world_size), key=lambda rank: (loads[rank], rank))
        planned[table.name] = EmbeddingShardSpec(table.name, "table_wise", world_size, table_owner=owner)
        loads[owner] += embedding_local_bytes(
            rows=table.num_embeddings, embedding_dim=table.embedding_dim, weight_element_size=table.element_size,
            optimizer_state_layout=optimizer_state_layout)
    payload = {
        "world_size": world_size,
        "optimizer_state_layout": optimizer_state_layout,
        "cost_model_version": 2,
        "tables": {name: asdict(planned[name]) for name in sorted(planned)},
    }
    fingerprint = sha256(json.dumps(payload, sort_keys=True, separators=(",", ":")).encode("utf-8")).hexdigest()
    return EmbeddingShardingPlan(world_size=world_size, tables=planned, fingerprint=fingerprint)
