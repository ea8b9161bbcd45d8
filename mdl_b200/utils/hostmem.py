"""Host memory tools (reference ``limit_malloc_arenas`` / ``trim_process_heap`` /
``process_resident_bytes``, ``src/dataloader.py:204-260``).

Data threads that allocate and free large Arrow / NumPy buffers make glibc grow
one malloc arena per thread and keep freed pages. ``limit_malloc_arenas`` caps
the arena count (``mallopt(M_ARENA_MAX)``), ``trim_process_heap`` returns free
heap pages to the OS (``malloc_trim(0)``), ``process_resident_bytes`` reads the
resident set size from ``/proc/self/statm``.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import os

_M_ARENA_MAX = -8  # glibc mallopt parameter number


def _libc():
    name = ctypes.util.find_library("c")
    if name is None:
        return None
    try:
        return ctypes.CDLL(name)
    except OSError:
        return None


def limit_malloc_arenas(count: int) -> bool:
    libc = _libc()
    if libc is None or not hasattr(libc, "mallopt") or count <= 0:
        return False
    return bool(libc.mallopt(ctypes.c_int(_M_ARENA_MAX), ctypes.c_int(int(count))))


def trim_process_heap() -> bool:
    libc = _libc()
    if libc is None or not hasattr(libc, "malloc_trim"):
        return False
    return bool(libc.malloc_trim(ctypes.c_size_t(0)))


def process_resident_bytes() -> int:
    try:
        with open("/proc/self/statm") as fh:
            pages = int(fh.read().split()[1])
    except (OSError, ValueError, IndexError):
        return 0
    return pages * os.sysconf("SC_PAGE_SIZE")


def arrow_pool_bytes() -> int:
    try:
        import pyarrow as pa
    except ImportError:
        return 0
    return int(pa.total_allocated_bytes())
