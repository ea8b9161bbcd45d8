"""Training checkpoints, commit protocol, resume and retention.

Run-directory layout (kept alike with the reference ``src/checkpoint.py:825-1170``):

    <run>/step-000001200/model/            sharded model checkpoint (``model.py``)
    <run>/step-000001200/train_state.pt    dense optimizer state by name, step counters, RNG
    <run>/step-000001200/progress-rank-RRRRR.json   where each rank's input stood
    <run>/step-000001200/_READY-rank-RRRRR   a rank's files are complete
    <run>/step-000001200/checkpoint.json   step, world size, time (rank 0)
    <run>/step-000001200/_COMMIT           the step is resumable (rank 0, last)
    <run>/_latest.json                     newest committed step

Only directories with ``_COMMIT`` are resumed from; ``keep_last`` prunes older
committed steps and removes uncommitted remnants older than the newest commit.
"""

from __future__ import annotations

import time
from dataclasses import asdict, dataclass, field
from typing import Any

import torch
import torch.distributed as dist

from .model import load_model_checkpoint, save_model_checkpoint
from .store import CheckpointStore

STEP_DIR_PREFIX = "step-"
MODEL_SUBDIR = "model"
TRAIN_STATE_FILE = "train_state.pt"
CHECKPOINT_MANIFEST = "checkpoint.json"
COMMIT_MARKER = "_COMMIT"
LATEST_POINTER = "_latest.json"
TRAINING_FORMAT = "mdl_training_checkpoint_v1"


def step_directory_name(step: int) -> str:
    return f"{STEP_DIR_PREFIX}{int(step):09d}"


def parse_step_directory(name: str) -> int | None:
    if not name.startswith(STEP_DIR_PREFIX):
        return None
    suffix = name[len(STEP_DIR_PREFIX):]
    return int(suffix) if suffix.isdigit() else None


def rank_ready_marker(rank: int) -> str:
    return f"_READY-rank-{int(rank):05d}"


def rank_progress_file(rank: int) -> str:
    return f"progress-rank-{int(rank):05d}.json"


@dataclass(frozen=True)
class DataCursor:
    """Where one rank's input stood: ``position`` in its deterministic work list,
    rows trained so far, and how many items a restart must rewind."""

    work_unit: str = "batch"
    position: int = 0
    rank: int = 0
    world_size: int = 1
    rewind: int = 0
    rows_trained: int = 0
    extra: dict = field(default_factory=dict)


@dataclass(frozen=True)
class CommittedCheckpoint:
    step: int
    directory: str
    uri: str
    world_size: int = 0
    saved_at: float = 0.0


def _barrier(trainer) -> None:
    if trainer.world > 1 and dist.is_initialized():
        dist.barrier(group=trainer.group)


def _step_entries(store: CheckpointStore) -> list[tuple[int, str]]:
    out = []
    for entry in store.list_entries():
        if entry.is_dir:
            step = parse_step_directory(entry.name)
            if step is not None:
                out.append((step, entry.name))
    return sorted(out)


def list_committed_checkpoints(store: CheckpointStore) -> list[CommittedCheckpoint]:
    found = []
    for step, name in _step_entries(store):
        if not store.exists(name, COMMIT_MARKER):
            continue
        world, saved_at = 0, 0.0
        try:
            meta = store.read_json(name, CHECKPOINT_MANIFEST)
            world, saved_at = int(meta.get("world_size", 0)), float(meta.get("saved_at", 0.0))
        except Exception:  # a commit marker alone is enough to resume
            pass
        found.append(CommittedCheckpoint(step, name, store.uri(name), world, saved_at))
    return found


def latest_committed_checkpoint(store: CheckpointStore) -> CommittedCheckpoint | None:
    found = list_committed_checkpoints(store)
    return found[-1] if found else None


def resolve_resume_checkpoint(store: CheckpointStore, spec: str | int | None) -> CommittedCheckpoint | None:
    """``auto`` / ``latest``: newest committed step; ``none``: no resume; a step number
    or ``step-NNNNNNNNN``: exactly that (committed) step."""

    text = str(spec if spec is not None else "auto").strip()
    if text.lower() in {"none", "off", "false", ""}:
        return None
    if text.lower() in {"auto", "latest"}:
        return latest_committed_checkpoint(store)
    step = parse_step_directory(text)
    if step is None and text.isdigit():
        step = int(text)
    if step is None:
        raise ValueError(f"resume must be auto, latest, none, a step number or a step directory; got {spec!r}")
    name = step_directory_name(step)
    if not store.exists(name, COMMIT_MARKER):
        raise FileNotFoundError(f"step {step} is not committed under {store.root_uri}")
    return CommittedCheckpoint(step, name, store.uri(name))


def prune_run_directory(store: CheckpointStore, keep_last: int) -> list[str]:
    entries = _step_entries(store)
    committed = [(s, n) for s, n in entries if store.exists(n, COMMIT_MARKER)]
    newest = committed[-1][0] if committed else -1
    doomed = []
    if keep_last > 0 and len(committed) > keep_last:
        doomed += [n for _, n in committed[:len(committed) - keep_last]]
    names = {n for _, n in committed}
    doomed += [n for s, n in entries if n not in names and s < newest]
    removed = []
    for name in doomed:
        try:
            store.remove_tree(name)
            removed.append(name)
        except Exception:  # retention must never fail a training run
            pass
    return removed


def _rng_state() -> dict[str, Any]:
    state = {"torch": torch.get_rng_state()}
    if torch.cuda.is_available():
        state["cuda"] = torch.cuda.get_rng_state_all()
    return state


def _commit_step(run: CheckpointStore, step: int, name: str, manifest: dict, keep_last: int) -> None:
    """Rank 0, after every rank's READY marker: manifest, ``_COMMIT``, latest pointer,
    retention."""

    run.write_json(manifest, name, CHECKPOINT_MANIFEST)
    run.write_bytes(b"", name, COMMIT_MARKER)
    run.write_json({"step": step, "directory": name}, LATEST_POINTER)
    if keep_last > 0:
        prune_run_directory(run, keep_last)


def save_training_checkpoint(config, trainer, run: CheckpointStore, step: int, *,
                             cursor: DataCursor | None = None, keep_last: int = 0,
                             extra: dict | None = None, uploader=None,
                             chunk_bytes: int | None = None) -> CommittedCheckpoint:
    """Collective: every rank writes its files, rank 0 commits after all are READY.

    With an ``uploader`` (``checkpoint.uploader.CheckpointUploader``) the files go to the
    rank's local staging directory and the uploader's thread publishes and commits them;
    the call returns once the step is staged (the returned record is committed when the
    uploader reports the step in ``published_steps``)."""

    name = step_directory_name(step)
    target = run
    if uploader is not None:
        target = uploader.stage_store(name)
    else:
        run.makedirs(name)
    model_store = target.child(MODEL_SUBDIR) if uploader is not None else run.child(name, MODEL_SUBDIR)
    kw = {} if chunk_bytes is None else {"chunk_bytes": int(chunk_bytes)}
    save_model_checkpoint(config, trainer, model_store, sparse_step=trainer.step_index, **kw)
    dense_state = trainer.dense.state_dict()  # collective under the sharded update
    parts = (name,) if uploader is None else ()
    if trainer.rank == 0:
        target.write_torch({
            "format": TRAINING_FORMAT,
            "dense_optimizer": dense_state,
            "step_index": trainer.step_index,
            "micro_index": trainer.micro_index,
            "rng": _rng_state(),
            "extra": extra or {},
        }, *parts, TRAIN_STATE_FILE)
    cur = cursor or DataCursor(position=trainer.step_index, rank=trainer.rank, world_size=trainer.world)
    target.write_json(asdict(cur), *parts, rank_progress_file(trainer.rank))
    saved_at = time.time()
    manifest = {"format": TRAINING_FORMAT, "step": step, "world_size": trainer.world,
                "saved_at": saved_at, "model_name": config.model.name}
    if uploader is not None:
        uploader.submit(step, name, manifest if trainer.rank == 0 else None)
        return CommittedCheckpoint(step, name, run.uri(name), trainer.world, saved_at)
    run.write_bytes(b"", name, rank_ready_marker(trainer.rank))
    _barrier(trainer)
    if trainer.rank == 0:
        missing = [r for r in range(trainer.world) if not run.exists(name, rank_ready_marker(r))]
        if missing:
            raise RuntimeError(f"checkpoint {name}: ranks {missing} did not finish writing")
        _commit_step(run, step, name, manifest, keep_last)
    _barrier(trainer)
    return CommittedCheckpoint(step, name, run.uri(name), trainer.world, saved_at)


def make_uploader(config, trainer, run: CheckpointStore, *, keep_last: int | None = None,
                  local_ranks: int = 1, asynchronous: bool | None = None):
    """The uploader a run's checkpoint settings ask for (``training.checkpoint``), after
    the staging-space preflight; None for synchronous saves."""

    from .uploader import CheckpointUploader, check_staging_space, estimate_staging_bytes

    ck = config.training.checkpoint
    use_async = ck.async_upload if asynchronous is None else asynchronous
    if not use_async:
        return None
    uploader = CheckpointUploader(run, rank=trainer.rank, world=trainer.world, staging_dir=ck.staging_dir,
                                  keep_last=ck.keep_last if keep_last is None else keep_last,
                                  ready_timeout_sec=ck.ready_timeout_sec, commit_fn=_commit_step)
    if ck.preflight_staging:
        try:
            check_staging_space(uploader.staging_root, estimate_staging_bytes(trainer, ck.shard_chunk_bytes),
                                local_ranks=local_ranks)
        except Exception:
            uploader.close()
            raise
    return uploader


@dataclass
class ResumedTrainingState:
    step: int
    cursor: DataCursor | None
    extra: dict


def load_training_checkpoint(config, trainer, run: CheckpointStore, spec: str | int | None = "auto",
                             *, restore_rng: bool = True) -> ResumedTrainingState | None:
    """Restore model, dense optimizer state, counters and (same world size) RNG; returns
    where to continue, or None when there is nothing to resume."""

    ck = resolve_resume_checkpoint(run, spec)
    if ck is None:
        return None
    load_model_checkpoint(config, trainer, run.child(ck.directory, MODEL_SUBDIR))
    state = run.read_torch(ck.directory, TRAIN_STATE_FILE)
    if state.get("format") != TRAINING_FORMAT:
        raise ValueError(f"unsupported training checkpoint format {state.get('format')!r}")
    trainer.dense.load_state_dict(state["dense_optimizer"])
    trainer.step_index = int(state["step_index"])
    trainer.micro_index = int(state.get("micro_index", 0))
    meta = run.read_json(ck.directory, CHECKPOINT_MANIFEST)
    if restore_rng and int(meta.get("world_size", 0)) == trainer.world:
        rng = state.get("rng") or {}
        if "torch" in rng:
            torch.set_rng_state(rng["torch"])
        if "cuda" in rng and torch.cuda.is_available():
            try:
                torch.cuda.set_rng_state_all(rng["cuda"])
            except RuntimeError:  # a different device count
                pass
    cursor = None
    if run.exists(ck.directory, rank_progress_file(trainer.rank)):
        payload = run.read_json(ck.directory, rank_progress_file(trainer.rank))
        cursor = DataCursor(**{k: v for k, v in payload.items() if k in DataCursor.__dataclass_fields__})
    return ResumedTrainingState(step=trainer.step_index, cursor=cursor, extra=state.get("extra", {}))
