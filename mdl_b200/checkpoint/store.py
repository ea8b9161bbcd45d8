"""Checkpoint storage: a local directory or any ``pyarrow.fs`` filesystem URI.

Counterpart of the reference's ``CheckpointStore`` (``src/checkpoint_store.py:94-147``,
local ``:150``, HDFS ``:225``, ``open_checkpoint_store`` ``:382``): every run
directory is reached through one object with atomic writes (write to a
temporary name, then rename), JSON helpers, listing, recursive removal, and a
retry with exponential backoff around remote operations.
"""

from __future__ import annotations

import io
import json
import os
import shutil
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, TypeVar

T = TypeVar("T")


class CheckpointStoreError(RuntimeError):
    pass


@dataclass(frozen=True)
class StoredEntry:
    name: str
    is_dir: bool


def _retry(fn: Callable[[], T], *, attempts: int, base_sec: float, what: str) -> T:
    last: BaseException | None = None
    for i in range(max(1, attempts)):
        try:
            return fn()
        except FileNotFoundError:
            raise
        except OSError as error:  # transient filesystem / network failure
            last = error
            if i + 1 < attempts:
                time.sleep(base_sec * (2 ** i))
    raise CheckpointStoreError(f"{what} failed after {attempts} attempts: {last}") from last


class CheckpointStore:
    """A directory tree addressed by relative path parts."""

    def __init__(self, root: str, *, retries: int = 3, retry_base_sec: float = 0.5) -> None:
        self.root_uri = root
        self.retries = retries
        self.retry_base_sec = retry_base_sec
        self._fs = None
        self._root = root
        if "://" in root and not root.startswith("file://"):
            from pyarrow import fs as pafs

            self._fs, self._root = pafs.FileSystem.from_uri(root)
        elif root.startswith("file://"):
            self._root = root[len("file://"):]

    # -------------------------------------------------------------- paths
    @property
    def remote(self) -> bool:
        return self._fs is not None

    def path(self, *parts: str) -> str:
        return "/".join([self._root.rstrip("/"), *[p.strip("/") for p in parts if p]])

    def uri(self, *parts: str) -> str:
        if not self.remote:
            return self.path(*parts)
        return "/".join([self.root_uri.rstrip("/"), *[p.strip("/") for p in parts if p]])

    def local_path(self, *parts: str) -> Path:
        if self.remote:
            raise CheckpointStoreError("local_path() on a remote store")
        return Path(self.path(*parts))

    def _do(self, fn: Callable[[], T], what: str) -> T:
        if not self.remote:
            return fn()
        return _retry(fn, attempts=self.retries, base_sec=self.retry_base_sec, what=what)

    # -------------------------------------------------------------- queries
    def exists(self, *parts: str) -> bool:
        p = self.path(*parts)
        if not self.remote:
            return os.path.exists(p)
        from pyarrow import fs as pafs

        return self._do(lambda: self._fs.get_file_info(p).type != pafs.FileType.NotFound, f"stat {p}")

    def list_entries(self, *parts: str) -> list[StoredEntry]:
        p = self.path(*parts)
        if not self.remote:
            if not os.path.isdir(p):
                return []
            return [StoredEntry(e.name, e.is_dir()) for e in sorted(os.scandir(p), key=lambda e: e.name)]
        from pyarrow import fs as pafs

        infos = self._do(lambda: self._fs.get_file_info(pafs.FileSelector(p, allow_not_found=True)), f"list {p}")
        return sorted((StoredEntry(i.base_name, i.type == pafs.FileType.Directory) for i in infos),
                      key=lambda e: e.name)

    # -------------------------------------------------------------- writes
    def makedirs(self, *parts: str) -> None:
        p = self.path(*parts)
        if not self.remote:
            os.makedirs(p, exist_ok=True)
        else:
            self._do(lambda: self._fs.create_dir(p, recursive=True), f"mkdir {p}")

    def write_bytes(self, data: bytes, *parts: str) -> None:
        """Atomic write: a reader sees the old file, no file, or the complete new file."""

        p = self.path(*parts)
        tmp = p + f".tmp-{os.getpid()}"
        if not self.remote:
            os.makedirs(os.path.dirname(p), exist_ok=True)
            with open(tmp, "wb") as fh:
                fh.write(data)
                fh.flush()
                os.fsync(fh.fileno())
            os.replace(tmp, p)
            return

        def put():
            with self._fs.open_output_stream(tmp) as out:
                out.write(data)
            self._fs.move(tmp, p)

        self._do(put, f"write {p}")

    def upload_file(self, source: str | os.PathLike[str], *parts: str, chunk_bytes: int = 64 << 20) -> int:
        """Copy a local file to ``parts`` (atomic like ``write_bytes``) without holding it
        in memory; returns the bytes copied."""

        p = self.path(*parts)
        tmp = p + f".tmp-{os.getpid()}"
        if not self.remote:
            os.makedirs(os.path.dirname(p), exist_ok=True)
            shutil.copyfile(source, tmp)
            with open(tmp, "rb+") as fh:
                os.fsync(fh.fileno())
            os.replace(tmp, p)
            return os.path.getsize(p)

        def put():
            n = 0
            with open(source, "rb") as inp, self._fs.open_output_stream(tmp) as out:
                while True:
                    block = inp.read(chunk_bytes)
                    if not block:
                        break
                    out.write(block)
                    n += len(block)
            self._fs.move(tmp, p)
            return n

        return self._do(put, f"upload {p}")

    def read_bytes(self, *parts: str) -> bytes:
        p = self.path(*parts)
        if not self.remote:
            with open(p, "rb") as fh:
                return fh.read()

        def get():
            with self._fs.open_input_stream(p) as inp:
                return inp.read()

        return self._do(get, f"read {p}")

    def write_json(self, payload: dict[str, Any], *parts: str) -> None:
        self.write_bytes(json.dumps(payload, indent=2, sort_keys=True).encode("utf-8"), *parts)

    def read_json(self, *parts: str) -> dict[str, Any]:
        return json.loads(self.read_bytes(*parts).decode("utf-8"))

    def write_torch(self, payload: Any, *parts: str) -> None:
        import torch

        buf = io.BytesIO()
        torch.save(payload, buf)
        self.write_bytes(buf.getvalue(), *parts)

    def read_torch(self, *parts: str) -> Any:
        import torch

        return torch.load(io.BytesIO(self.read_bytes(*parts)), map_location="cpu", weights_only=False)

    def remove_tree(self, *parts: str) -> None:
        p = self.path(*parts)
        if not self.remote:
            if os.path.isdir(p):
                shutil.rmtree(p)
            elif os.path.exists(p):
                os.remove(p)
            return
        self._do(lambda: self._fs.delete_dir(p), f"rmtree {p}")

    def child(self, *parts: str) -> "CheckpointStore":
        return CheckpointStore(self.uri(*parts), retries=self.retries, retry_base_sec=self.retry_base_sec)


def open_checkpoint_store(uri: str | os.PathLike[str], **kw) -> CheckpointStore:
    return CheckpointStore(str(uri), **kw)
