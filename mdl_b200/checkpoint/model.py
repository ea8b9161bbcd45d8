"""Sharded, reshardable model checkpoints.

Layout (kept alike with the reference's ``save_model_checkpoint``
``src/checkpoint.py:466-602`` so run directories look the same):

* ``manifest.json`` (rank 0, written last): format ``mdl_sharded_embedding_v2``,
  ``world_size``, ``dense_file``, ``chunks`` (per chunk: its tables and one file
  name per rank), per-table ``num_embeddings`` / ``embedding_dim`` /
  ``padding_idx``, the sparse optimizer name, model name, task names;
* ``dense.pt`` (rank 0): ``model_state_dict`` of every dense parameter (fp32, the
  authoritative values gathered from their owners when the update is sharded);
* ``shard-CCCC-rank-RRRRR-of-WWWWW.pt`` (every rank): the rank's local rows of
  each table of chunk CCCC with its ``shard_spec`` and row-wise Adagrad state
  (``sum`` per row, ``step``); chunks hold tables up to 2 GiB per file.

Loading at the saved world size reads only the rank's own files; at another
world size every rank reads all saved shards one file at a time and keeps the
rows it owns under the new plan (global id of a saved local row: row-wise
``residue + row * W_old`` with ``residue = (rank_old - offset) % W_old``;
table-wise: the row itself).
"""

from __future__ import annotations

from dataclasses import asdict
from typing import Any

import torch
import torch.distributed as dist

from ..parallel.sharding import EmbeddingShardSpec
from .store import CheckpointStore

SHARDED_FORMAT = "mdl_sharded_embedding_v2"
DENSE_FILE = "dense.pt"
MANIFEST = "manifest.json"
DEFAULT_CHUNK_BYTES = 2 * 1024 ** 3


def shard_chunk_file(index: int, rank: int, world_size: int) -> str:
    return f"shard-{int(index):04d}-rank-{int(rank):05d}-of-{int(world_size):05d}.pt"


def checkpoint_metadata(config) -> dict[str, Any]:
    return {"model_name": config.model.name, "task_names": list(config.task_names)}


def _barrier(world: int, group) -> None:
    if world > 1 and dist.is_initialized():
        dist.barrier(group=group)


def plan_chunks(store, chunk_bytes: int) -> list[list[str]]:
    """Group tables (sorted by name) into files of at most ``chunk_bytes`` (per rank,
    sized by the largest shard of any rank; a larger table gets its own file)."""

    chunks: list[list[str]] = [[]]
    used = 0
    for t in sorted(store.layouts, key=lambda t: t.name):
        rows = max(t.spec.local_rows(t.num_embeddings, r) for r in range(store.world))
        size = rows * t.dim * 4 + rows * 4
        if chunks[-1] and used + size > chunk_bytes:
            chunks.append([])
            used = 0
        chunks[-1].append(t.name)
        used += size
    return [c for c in chunks if c]


def dense_state(trainer) -> dict[str, torch.Tensor]:
    """Every dense parameter at full fp32 precision (gathered from its owner)."""

    dp = trainer.dense
    master = dp.gather_master().detach().float().cpu()
    return {n: master[dp.offsets[n]:dp.offsets[n] + p.numel()].view_as(p).clone() for n, p in dp.params.items()}


@torch.no_grad()
def save_model_checkpoint(config, trainer, store: CheckpointStore, *, chunk_bytes: int = DEFAULT_CHUNK_BYTES,
                          sparse_step: int = 0) -> list[str]:
    """Write this rank's shard files (and, on rank 0, ``dense.pt`` and the manifest)."""

    emb = trainer.store
    rank, world, group = trainer.rank, trainer.world, trainer.group
    # table shards are laid out over emb.world ranks (1 for replicated tables, whose
    # identical copies only rank 0 writes)
    emb_rank, emb_world = emb.rank, emb.world
    writes_tables = emb.replicas == 1 or rank == 0
    written: list[str] = []
    store.makedirs()
    chunks = plan_chunks(emb, chunk_bytes)
    for index, names in enumerate(chunks):
        if not writes_tables:
            break
        tables = {}
        for name in names:
            t = emb.layouts[emb.index[name]]
            tables[name] = {
                "weight": emb.weight(name).detach().cpu().clone(),
                "num_embeddings": t.num_embeddings,
                "embedding_dim": t.dim,
                "padding_idx": 0,
                "shard_spec": asdict(t.spec),
                "optimizer_state": {"sum": emb.accumulator(name).detach().cpu().clone(),
                                    "step": torch.tensor(float(sparse_step), dtype=torch.float64)},
            }
        name = shard_chunk_file(index, emb_rank, emb_world)
        store.write_torch({"format": SHARDED_FORMAT, "rank": emb_rank, "world_size": emb_world, "chunk": index,
                           "tables": tables}, name)
        written.append(name)
    state = dense_state(trainer)  # collective (all ranks) when the dense update is sharded
    if rank == 0:
        store.write_torch({"model_state_dict": state, **checkpoint_metadata(config)}, DENSE_FILE)
        written.append(DENSE_FILE)
    _barrier(world, group)
    if rank == 0:
        store.write_json({
            "format": SHARDED_FORMAT,
            "version": 2,
            "world_size": world,
            "embedding_world_size": emb_world,
            "dense_file": DENSE_FILE,
            "chunks": [{"index": i, "tables": names,
                        "rank_files": [shard_chunk_file(i, r, emb_world) for r in range(emb_world)]}
                       for i, names in enumerate(chunks)],
            "tables": {t.name: {"num_embeddings": t.num_embeddings, "embedding_dim": t.dim, "padding_idx": 0}
                       for t in emb.layouts},
            "training_metadata": {"sparse_optimizer": config.training.sparse_optimizer},
            **checkpoint_metadata(config),
        }, MANIFEST)
        written.append(MANIFEST)
    _barrier(world, group)
    return written


def _saved_ids(spec: dict, rows: int, saved_rank: int, num_embeddings: int) -> torch.Tensor:
    s = EmbeddingShardSpec(**spec)
    if s.strategy == "table_wise":
        return torch.arange(rows, dtype=torch.int64)
    residue = (saved_rank - s.cyclic_offset) % s.world_size
    ids = residue + torch.arange(rows, dtype=torch.int64) * s.world_size
    return ids[ids < num_embeddings]


def _restore_rows(emb, name: str, t, tab: dict, saved_rank: int, rank: int, filled: torch.Tensor) -> None:
    """Copy the rows of one saved shard that this rank owns into its local table and
    mark them in ``filled``. A shard saved by this rank under the same shard spec is
    copied as a whole; anything else is remapped through global ids."""

    w = tab["weight"]
    acc = (tab.get("optimizer_state") or {}).get("sum")
    dst_w = emb.weight(name)
    dst_a = emb.accumulator(name)
    if saved_rank == rank and tab.get("shard_spec") == asdict(t.spec):
        if w.shape[0] != t.local_rows:
            raise ValueError(f"table {name!r}: {w.shape[0]} saved rows, {t.local_rows} local rows")
        dst_w.copy_(w.to(dst_w.device, dst_w.dtype))
        if acc is not None:
            dst_a.copy_(acc.to(dst_a.device, dst_a.dtype))
        filled.fill_(True)
        return
    ids = _saved_ids(tab["shard_spec"], w.shape[0], saved_rank, t.num_embeddings)
    if ids.numel() != w.shape[0]:
        raise ValueError(f"table {name!r}: shard of rank {saved_rank} holds {w.shape[0]} rows, its spec "
                         f"owns {ids.numel()}")
    mine = t.spec.owner(ids) == rank
    if not bool(mine.any()):
        return
    local = t.spec.local_row_ids(ids[mine])
    sel = mine.nonzero().flatten()
    dst_w[local.to(dst_w.device)] = w[sel].to(dst_w.device, dst_w.dtype)
    if acc is not None:
        dst_a[local.to(dst_a.device)] = acc[sel].to(dst_a.device, dst_a.dtype)
    filled[local] = True


@torch.no_grad()
def load_model_checkpoint(config, trainer, store: CheckpointStore, *, strict: bool = True) -> dict[str, Any]:
    """Restore dense parameters and every table shard (resharding when the world size
    or a table's shard spec changed).

    Every local row of every model table must be restored: like the reference
    (``src/checkpoint.py:722-790``) a per-table mask records the rows written and a
    table with any row left out (a table missing from the checkpoint, or shard files
    that do not cover it) raises. At the saved world size a rank first reads only its
    own files; tables whose saved shard spec differs from the current one are then
    completed from the other ranks' files."""

    manifest = store.read_json(MANIFEST)
    if manifest.get("format") != SHARDED_FORMAT:
        raise ValueError(f"unsupported checkpoint format {manifest.get('format')!r}")
    if strict and manifest.get("model_name") != config.model.name:
        raise ValueError(f"checkpoint is a {manifest.get('model_name')!r} model, config builds {config.model.name!r}")
    saved_opt = manifest.get("training_metadata", {}).get("sparse_optimizer")
    if saved_opt not in (None, config.training.sparse_optimizer):
        raise ValueError(f"checkpoint sparse_optimizer {saved_opt!r} != config {config.training.sparse_optimizer!r}")
    emb = trainer.store
    rank = emb.rank  # shard coordinates of the tables (0 of 1 for replicated tables)
    saved_world = int(manifest.get("embedding_world_size", manifest["world_size"]))
    dense = store.read_torch(manifest.get("dense_file", DENSE_FILE))["model_state_dict"]
    dp = trainer.dense
    missing = [n for n in dp.params if n not in dense]
    if strict and missing:
        raise KeyError(f"dense parameters missing from the checkpoint: {missing[:5]}")
    dp.load_state_dict({"params": {n: v for n, v in dense.items() if n in dp.params}})
    filled = {t.name: torch.zeros(t.local_rows, dtype=torch.bool) for t in emb.layouts}

    def read(fname: str, only: set[str] | None) -> None:
        payload = store.read_torch(fname)
        saved_rank = int(payload["rank"])
        if int(payload.get("world_size", saved_world)) != saved_world:
            raise ValueError(f"{fname}: world size {payload.get('world_size')} != manifest {saved_world}")
        for name, tab in payload["tables"].items():
            if name not in emb.index:
                if strict:
                    raise KeyError(f"checkpoint table {name!r} is not in the model")
                continue
            if only is not None and name not in only:
                continue
            t = emb.layouts[emb.index[name]]
            if (tab["num_embeddings"] != t.num_embeddings or tab["embedding_dim"] != t.dim
                    or int(tab.get("padding_idx", 0)) != 0):
                raise ValueError(f"table {name!r}: checkpoint (rows {tab['num_embeddings']}, dim "
                                 f"{tab['embedding_dim']}, padding_idx {tab.get('padding_idx', 0)}) != model "
                                 f"(rows {t.num_embeddings}, dim {t.dim}, padding_idx 0)")
            _restore_rows(emb, name, t, tab, saved_rank, rank, filled[name])

    same_world = saved_world == emb.world
    for chunk in manifest["chunks"]:
        for fname in ([chunk["rank_files"][rank]] if same_world else chunk["rank_files"]):
            read(fname, None)
    if same_world:
        # tables saved under another shard spec: their rows live in other ranks' files
        saved_tables = {n for chunk in manifest["chunks"] for n in chunk["tables"]}
        pending = {n for n, m in filled.items() if n in saved_tables and not bool(m.all())}
        if pending:
            for chunk in manifest["chunks"]:
                if pending & set(chunk["tables"]):
                    for r, fname in enumerate(chunk["rank_files"]):
                        if r != rank:
                            read(fname, pending)
    incomplete = sorted(n for n, m in filled.items() if not bool(m.all()))
    if incomplete:
        raise ValueError("checkpoint did not cover all local rows for tables: " + ", ".join(incomplete))
    emb.sync_peers()
    return manifest
