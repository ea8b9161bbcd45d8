"""Asynchronous checkpoint publication and the staging-space preflight.

Counterpart of the reference's ``CheckpointUploader`` (``src/checkpoint.py:1178-1485``)
and ``estimate_staging_space`` / ``check_staging_space`` (``src/checkpoint.py:270-397``).

A save with an uploader writes the step's files to a local staging directory on the
training thread (the device-to-host copies and the collectives of the save must run
there) and hands the staged step to a background thread. That thread copies every
staged file to the run directory, deletes the staged copy, and then writes the rank's
``_READY`` marker, so the marker always lands after the rank's last byte. On rank 0 it
then waits (``ready_timeout_sec``) for every rank's marker and only then writes the
manifest, ``_COMMIT``, the ``_latest.json`` pointer and the retention pass. A step that
misses a marker is never committed, so a crash in the middle of an upload leaves
nothing that a resume would pick up. Training waits for the thread only when
``max_pending`` staged steps are already queued (back pressure), at ``flush()`` and at
``close()``.

The preflight sizes one rank's staged files from the live tables and dense state
(shard chunks as the model checkpoint plans them, plus the dense parameters and
optimizer state on rank 0) and refuses to start when the staging filesystem cannot
hold every local rank's files with 10% headroom.
"""

from __future__ import annotations

import os
import queue
import shutil
import tempfile
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path

from .model import plan_chunks
from .store import CheckpointStore


class CheckpointStagingSpaceError(RuntimeError):
    pass


def _fmt(n: int | None) -> str:
    if n is None:
        return "unknown"
    for unit in ("B", "KiB", "MiB", "GiB", "TiB"):
        if n < 1024 or unit == "TiB":
            return f"{n:.1f} {unit}" if unit != "B" else f"{n} B"
        n /= 1024.0
    return str(n)


@dataclass(frozen=True)
class StagingEstimate:
    """One rank's staged files of one checkpoint step."""

    total_bytes: int
    largest_file_bytes: int
    files: int

    def describe(self) -> str:
        return f"total={_fmt(self.total_bytes)} largest={_fmt(self.largest_file_bytes)} files={self.files}"


def estimate_staging_bytes(trainer, chunk_bytes: int) -> StagingEstimate:
    """Bytes this rank stages per checkpoint: its table shard chunks (weights and the
    Adagrad accumulator, as ``save_model_checkpoint`` packs them) and, on rank 0, the
    dense parameters twice (``dense.pt`` and the training state) plus the dense
    optimizer's state vectors."""

    emb = trainer.store
    sizes: list[int] = []
    if emb.replicas == 1 or trainer.rank == 0:
        for names in plan_chunks(emb, chunk_bytes):
            b = 0
            for n in names:
                b += emb.weight(n).numel() * 4 + emb.accumulator(n).numel() * 4
            sizes.append(b)
    if trainer.rank == 0:
        dense = sum(p.numel() for p in trainer.dense.params.values()) * 4
        states = 2 if getattr(trainer.dense, "optimizer", "rmsprop") == "adam" else 1
        sizes.append(dense)                  # dense.pt
        sizes.append(dense * (1 + states))   # train_state.pt (params + optimizer state)
    return StagingEstimate(sum(sizes), max(sizes, default=0), len(sizes))


def free_bytes(path: str | os.PathLike[str]) -> int | None:
    p = Path(path)
    while not p.exists() and p != p.parent:
        p = p.parent
    try:
        return shutil.disk_usage(p).free
    except OSError:
        return None


def check_staging_space(staging_dir: str | os.PathLike[str], estimate: StagingEstimate, *, local_ranks: int = 1,
                        headroom: float = 1.1, enforce: bool = True, free: int | None = None) -> str:
    """Raise ``CheckpointStagingSpaceError`` when ``staging_dir`` cannot hold the staged
    files of every rank of this node (they share the filesystem). Returns a summary."""

    have = free_bytes(staging_dir) if free is None else free
    need = int(estimate.total_bytes * max(1, int(local_ranks)) * max(1.0, float(headroom)))
    summary = (f"staging_dir={staging_dir} free={_fmt(have)} needed={_fmt(need)} "
               f"(local_ranks={local_ranks} {estimate.describe()})")
    if have is not None and have < need:
        msg = (f"checkpoint staging has too little room: {summary}; set training.checkpoint.staging_dir "
               "to a filesystem with more space (the system temp directory is often a small tmpfs)")
        if enforce:
            raise CheckpointStagingSpaceError(msg)
    return summary


@dataclass
class _StagedStep:
    step: int
    directory: str                      # step directory name in the run store
    source: Path                        # staged copy of the step directory
    commit: dict | None                 # manifest payload (rank 0), None elsewhere
    done: threading.Event = field(default_factory=threading.Event)
    ok: bool = False


class CheckpointUploader:
    """Publishes staged checkpoint steps of one rank to the run directory.

    ``asynchronous=False`` runs every publication on the caller's thread (tests, and
    runs whose run directory is as fast as the staging disk)."""

    def __init__(self, run: CheckpointStore, *, rank: int = 0, world: int = 1, staging_dir: str | None = None,
                 keep_last: int = 0, ready_timeout_sec: float = 1800.0, poll_sec: float = 0.25,
                 asynchronous: bool = True, max_pending: int = 1, ready_marker=None, commit_fn=None) -> None:
        from .training import rank_ready_marker

        self.run = run
        self.rank, self.world = int(rank), max(1, int(world))
        root = Path(staging_dir) if staging_dir else Path(tempfile.gettempdir()) / "mdl_b200_ckpt_staging"
        self.staging_root = root / f"rank-{self.rank:05d}-{os.getpid()}"
        self.staging_root.mkdir(parents=True, exist_ok=True)
        self.keep_last = int(keep_last)
        self.ready_timeout_sec = float(ready_timeout_sec)
        self.poll_sec = float(poll_sec)
        self.asynchronous = bool(asynchronous)
        self._ready_marker = ready_marker or rank_ready_marker
        self._commit_fn = commit_fn
        self._queue: queue.Queue = queue.Queue(maxsize=max(1, int(max_pending)))
        self._thread: threading.Thread | None = None
        self.published_steps: list[int] = []
        self.failed_steps: list[tuple[int, str]] = []
        self.uploaded_bytes = 0
        if self.asynchronous:
            self._thread = threading.Thread(target=self._loop, name=f"mdl-ckpt-upload-rank{self.rank}", daemon=True)
            self._thread.start()

    # ----------------------------------------------------------------- staging
    def stage_store(self, directory: str) -> CheckpointStore:
        """A fresh local store for one step's files."""

        path = self.staging_root / directory
        if path.exists():
            shutil.rmtree(path)
        path.mkdir(parents=True)
        return CheckpointStore(str(path))

    def submit(self, step: int, directory: str, commit: dict | None = None) -> _StagedStep:
        """Queue a staged step for publication (blocks while ``max_pending`` steps wait)."""

        item = _StagedStep(int(step), directory, self.staging_root / directory, commit)
        if self._thread is None:
            self._publish(item)
        else:
            if not self._thread.is_alive():
                raise RuntimeError("checkpoint upload thread is not running")
            self._queue.put(item)
        return item

    def flush(self, timeout: float | None = None) -> bool:
        """Wait until every queued step is published (or failed); False on timeout."""

        if self._thread is None:
            return True
        deadline = None if timeout is None else time.monotonic() + timeout
        while self._queue.unfinished_tasks:
            if deadline is not None and time.monotonic() > deadline:
                return False
            time.sleep(0.01)
        return True

    def close(self, timeout: float | None = None) -> None:
        if self._thread is not None:
            self.flush(timeout)
            self._queue.put(None)
            self._thread.join(timeout=5.0)
            self._thread = None
        shutil.rmtree(self.staging_root, ignore_errors=True)

    # ----------------------------------------------------------------- worker
    def _loop(self) -> None:
        while True:
            item = self._queue.get()
            try:
                if item is None:
                    return
                self._publish(item)
            finally:
                self._queue.task_done()

    def _publish(self, item: _StagedStep) -> None:
        try:
            files = sorted(p for p in item.source.rglob("*") if p.is_file())
            for f in files:
                rel = f.relative_to(item.source).as_posix()
                self.uploaded_bytes += self.run.upload_file(f, item.directory, *rel.split("/"))
                f.unlink()
            self.run.write_bytes(b"", item.directory, self._ready_marker(self.rank))
            if self.rank == 0:
                self._commit(item)
            item.ok = True
            self.published_steps.append(item.step)
        except Exception as error:  # noqa: BLE001 - a failed upload must not kill training
            self.failed_steps.append((item.step, f"{type(error).__name__}: {error}"))
        finally:
            shutil.rmtree(item.source, ignore_errors=True)
            item.done.set()

    def _commit(self, item: _StagedStep) -> None:
        deadline = time.monotonic() + self.ready_timeout_sec
        while True:
            missing = [r for r in range(self.world) if not self.run.exists(item.directory, self._ready_marker(r))]
            if not missing:
                break
            if time.monotonic() > deadline:
                raise TimeoutError(f"checkpoint {item.directory}: ranks {missing} not READY after "
                                   f"{self.ready_timeout_sec:.0f}s; the step stays uncommitted")
            time.sleep(self.poll_sec)
        if self._commit_fn is not None:
            self._commit_fn(self.run, item.step, item.directory, item.commit or {}, self.keep_last)
