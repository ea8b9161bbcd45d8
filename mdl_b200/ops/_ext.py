"""Loader of the native sm_100a extension (``mdl_b200/_mdl_C.so``).

On a machine with a CUDA device the extension is mandatory: every op that has
a CUDA kernel calls :func:`ext` and raises if the library cannot be built or
loaded, so a GPU run never silently falls back to PyTorch. On CPU-only hosts
the ops use their PyTorch definitions (which double as the numerics oracle in
the tests).
"""

from __future__ import annotations

import importlib.util
import os
import threading
from pathlib import Path
from types import ModuleType

import torch

_LOCK = threading.Lock()
_MODULE: ModuleType | None = None
_ERROR_WORDS: dict[int, torch.Tensor] = {}


def _lib_path() -> Path:
    return Path(__file__).resolve().parent.parent / "_mdl_C.so"


def ext() -> ModuleType:
    """Return the loaded native module, building it first if needed."""

    global _MODULE
    if _MODULE is not None:
        return _MODULE
    with _LOCK:
        if _MODULE is not None:
            return _MODULE
        from ..csrc import build as _build

        path = _lib_path()
        if not _build.is_up_to_date():
            if os.environ.get("MDL_B200_NO_BUILD") == "1":
                if not path.exists():
                    raise RuntimeError(f"mdl_b200 native extension missing at {path}")
            else:
                _build.build()
        spec = importlib.util.spec_from_file_location("mdl_b200._mdl_C", path)
        if spec is None or spec.loader is None:
            raise RuntimeError(f"cannot load mdl_b200 native extension from {path}")
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
        _MODULE = module
        return module


def use_cuda_kernels(*tensors: torch.Tensor) -> bool:
    """True when the tensors live on a CUDA device (the native path is then mandatory)."""

    return any(isinstance(t, torch.Tensor) and t.is_cuda for t in tensors)


def error_word(device: torch.device | int) -> torch.Tensor:
    """Per-device int32 word that kernels OR their error codes into."""

    index = torch.device(device).index if not isinstance(device, int) else device
    if index is None:
        index = torch.cuda.current_device()
    word = _ERROR_WORDS.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _ERROR_WORDS[index] = word
    return word


ERROR_NAMES = {
    1: "mbarrier wait timed out",
    2: "peer flag wait timed out",
    4: "fixed-capacity buffer overflow",
    8: "id outside its embedding table",
    16: "bad kernel argument",
}


def check_error_word(device: torch.device | int) -> None:
    """Raise if any kernel on ``device`` recorded an error (one device->host read)."""

    word = error_word(device)
    value = int(word.item())
    if value:
        names = [name for bit, name in ERROR_NAMES.items() if value & bit]
        word.zero_()
        raise RuntimeError(f"mdl_b200 kernel error 0x{value:x}: {', '.join(names)}")
