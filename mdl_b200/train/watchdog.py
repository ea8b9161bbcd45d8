"""Step watchdog and CUDA out-of-memory abort (reference ``_StepWatchdog``
``src/train.py:136-233`` and ``_abort_rank_for_cuda_oom`` ``:264-295``).

A daemon thread expects ``beat(phase)`` at least every ``timeout_sec``; when no
optimizer step completes in time it logs the last phase, the step and the
device memory in use, then ends the process with exit code 70 so the launcher
(torchrun) tears the job down and a supervisor can restart it from the last
committed checkpoint. ``abort_on_cuda_oom`` does the same for an out-of-memory
error raised by a step. Both act on the host only.
"""

from __future__ import annotations

import logging
import os
import sys
import threading
import time
from typing import Callable

EXIT_CODE = 70
log = logging.getLogger(__name__)


class StepWatchdog:
    def __init__(self, timeout_sec: float, *, on_expire: Callable[[str], None] | None = None,
                 poll_sec: float | None = None) -> None:
        self.timeout = float(timeout_sec)
        self.poll = poll_sec if poll_sec is not None else max(0.05, min(5.0, self.timeout / 10))
        self._last = time.monotonic()
        self._phase = "start"
        self._step = 0
        self._stop = threading.Event()
        self._on_expire = on_expire or self._exit
        self._thread: threading.Thread | None = None
        self.expired = False

    def start(self) -> "StepWatchdog":
        if self.timeout > 0 and self._thread is None:
            self._thread = threading.Thread(target=self._run, name="step-watchdog", daemon=True)
            self._thread.start()
        return self

    def beat(self, phase: str = "step", step: int | None = None) -> None:
        self._last = time.monotonic()
        self._phase = phase
        if step is not None:
            self._step = step

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.poll + 1)
            self._thread = None

    def _report(self) -> str:
        mem = ""
        try:
            import torch

            if torch.cuda.is_available() and torch.cuda.is_initialized():
                mem = f", device memory in use {torch.cuda.memory_allocated() / 2**30:.2f} GiB"
        except Exception:
            pass
        idle = time.monotonic() - self._last
        return (f"no training progress for {idle:.1f} s (limit {self.timeout:.1f} s); last phase "
                f"{self._phase!r} at step {self._step}{mem}")

    def _run(self) -> None:
        while not self._stop.wait(self.poll):
            if time.monotonic() - self._last > self.timeout:
                self.expired = True
                msg = self._report()
                log.error("step watchdog: %s", msg)
                self._on_expire(msg)
                return

    @staticmethod
    def _exit(msg: str) -> None:
        print(f"step watchdog: {msg}; exiting with {EXIT_CODE}", file=sys.stderr, flush=True)
        os._exit(EXIT_CODE)


def is_cuda_oom(error: BaseException) -> bool:
    try:
        import torch

        if isinstance(error, torch.cuda.OutOfMemoryError):
            return True
    except Exception:
        pass
    return "out of memory" in str(error).lower() and "cuda" in str(error).lower()


def abort_on_cuda_oom(fn: Callable, *args, exit_fn: Callable[[int], None] = os._exit, **kw):
    """Run ``fn``; on a CUDA out-of-memory error log it and exit with code 70."""

    try:
        return fn(*args, **kw)
    except BaseException as error:
        if is_cuda_oom(error):
            print(f"CUDA out of memory: {error}; exiting with {EXIT_CODE}", file=sys.stderr, flush=True)
            exit_fn(EXIT_CODE)
            return None  # only reached when exit_fn returns (tests)
        raise
