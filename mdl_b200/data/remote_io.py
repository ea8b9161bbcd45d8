"""Resilient reads of remote (HDFS / object-store) Parquet inputs.

Reference: ``RemoteIoPolicy`` / ``call_with_timeout`` / ``retry_with_backoff`` /
``apply_worker_stagger`` / ``PerFileLock`` / ``RemoteSkipTracker`` /
``RemoteIoStallError`` (``src/dataloader.py:352-1130``).

* every open / read runs under ``hdfs_op_timeout`` (``hdfs_open_timeout`` for
  opens) on a worker thread; a call that overruns is abandoned (its thread is
  left to finish on its own) and counts as a failure;
* failures (``OSError``, timeouts) are retried ``hdfs_retry_count`` times with
  exponential backoff from ``hdfs_retry_base_sec``;
* a unit that still fails either raises ``RemoteIoStallError`` (exit code 70,
  so a launcher can restart the job) or, with ``on_hdfs_failure: skip``, is
  skipped and counted;
* ``worker_stagger_sec`` delays the first open of rank ``r`` by ``r`` times
  that, so many ranks do not hit the name node at once;
* ``hdfs_file_lock`` serialises opens of one file across the processes of a
  host with an advisory lock file.
"""

from __future__ import annotations

import fcntl
import hashlib
import os
import threading
import time
from dataclasses import dataclass

EXIT_REMOTE_STALL = 70


class RemoteIoStallError(RuntimeError):
    exit_code = EXIT_REMOTE_STALL


def call_with_timeout(fn, timeout_s: float | None, what: str = "remote call"):
    if not timeout_s:
        return fn()
    box: dict = {}

    def run():
        try:
            box["value"] = fn()
        except BaseException as error:  # handed to the caller
            box["error"] = error

    t = threading.Thread(target=run, daemon=True)
    t.start()
    t.join(timeout_s)
    if t.is_alive():
        raise TimeoutError(f"{what} did not finish within {timeout_s} s")
    if "error" in box:
        raise box["error"]
    return box.get("value")


def retry_with_backoff(fn, retries: int, base_s: float, what: str = "remote call", sleep=time.sleep,
                       max_backoff_s: float = 60.0):
    attempt = 0
    while True:
        try:
            return fn()
        except (OSError, TimeoutError) as error:
            if attempt >= retries:
                raise RemoteIoStallError(f"{what} failed after {attempt + 1} attempts: {error}") from error
            sleep(min(max_backoff_s, base_s * (2 ** attempt)))
            attempt += 1


class PerFileLock:
    """Advisory lock on ``<lock_dir>/<sha1(path)>.lock`` (one holder per host at a time)."""

    def __init__(self, path: str, lock_dir: str | None = None) -> None:
        d = lock_dir or os.path.join(os.environ.get("TMPDIR", "/tmp"), "mdl_b200_file_locks")
        os.makedirs(d, exist_ok=True)
        self.file = os.path.join(d, hashlib.sha1(path.encode()).hexdigest() + ".lock")
        self._fh = None

    def __enter__(self):
        self._fh = open(self.file, "a")
        fcntl.flock(self._fh, fcntl.LOCK_EX)
        return self

    def __exit__(self, *exc):
        fcntl.flock(self._fh, fcntl.LOCK_UN)
        self._fh.close()
        self._fh = None


@dataclass
class RemoteIoPolicy:
    op_timeout_s: float | None = None
    open_timeout_s: float | None = None
    retries: int = 3
    retry_base_s: float = 1.0
    skip_failures: bool = False
    file_lock: bool = False
    stagger_s: float = 0.0
    lock_dir: str | None = None
    skipped: int = 0

    @classmethod
    def from_reader(cls, reader) -> "RemoteIoPolicy":
        return cls(op_timeout_s=reader.hdfs_op_timeout, open_timeout_s=reader.hdfs_open_timeout or reader.hdfs_op_timeout,
                   retries=int(reader.hdfs_retry_count), retry_base_s=float(reader.hdfs_retry_base_sec),
                   skip_failures=reader.on_hdfs_failure == "skip", file_lock=bool(reader.hdfs_file_lock),
                   stagger_s=float(reader.worker_stagger_sec))

    def stagger(self, rank: int, sleep=time.sleep) -> None:
        if self.stagger_s > 0 and rank > 0:
            sleep(self.stagger_s * rank)

    def run(self, fn, what: str, *, opening: bool = False, path: str | None = None):
        """``fn()`` under the timeout / retry rules; ``None`` when the unit is skipped."""

        timeout = self.open_timeout_s if opening else self.op_timeout_s

        def once():
            if opening and self.file_lock and path is not None:
                with PerFileLock(path, self.lock_dir):
                    return call_with_timeout(fn, timeout, what)
            return call_with_timeout(fn, timeout, what)

        try:
            return retry_with_backoff(once, self.retries, self.retry_base_s, what)
        except RemoteIoStallError:
            if not self.skip_failures:
                raise
            self.skipped += 1
            return None
