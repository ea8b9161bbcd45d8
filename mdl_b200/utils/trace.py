"""Named ranges for profilers.

Counterpart of the reference's ``record_function`` ranges around its embedding exchange
and attention (``src/embeddings.py:532-534``, ``src/model.py:1209, 5677``). ``trace_range``
opens a ``torch.profiler.record_function`` range (shown by ``torch.profiler`` and in its
Chrome traces) and an NVTX range (shown by Nsight tools) around a block, but only while a
``torch.profiler`` session is recording or ``MDL_B200_TRACE=1`` is set: the unprofiled
step pays one boolean check per range.

Ranges in the framework: ``mdl.forward`` / ``mdl.backward`` / ``mdl.dense_update`` /
``mdl.sparse_update`` (trainer), ``mdl.embedding.*`` (lookup and its exchange phases),
``mdl.attention.*`` (the attention kernels).
"""

from __future__ import annotations

import contextlib
import os

import torch

_FORCE = os.environ.get("MDL_B200_TRACE", "0") == "1"


def tracing() -> bool:
    if _FORCE:
        return True
    try:
        return bool(torch.autograd.profiler._is_profiler_enabled)
    except AttributeError:  # pragma: no cover - older torch
        return False


@contextlib.contextmanager
def _range(name: str):
    nvtx = torch.cuda.is_available()
    with torch.profiler.record_function(name):
        if nvtx:
            torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            if nvtx:
                torch.cuda.nvtx.range_pop()


def trace_range(name: str):
    """Context manager: a profiler range named ``name`` when tracing, else nothing."""

    return _range(name) if tracing() else contextlib.nullcontext()


def set_tracing(on: bool) -> None:
    """Force ranges on (or back to profiler-driven) for this process."""

    global _FORCE
    _FORCE = bool(on)
