"""Pinned host buffer pool for packed batches.

Counterpart of the reference's ``_PinnedHostBufferPool`` / ``_PinnedPoolLease``
(``src/train.py:2923-3108``). A fresh ``pin_memory=True`` allocation per batch makes the
host allocator keep one cached slab per size class it has ever seen, so resident memory
ratchets up with variable batch sizes. The pool instead lends a batch one *slot* (one
pinned slab per dtype: the int64 and fp32 flat buffers of ``PackedBatch``) for its lifetime:

* ``checkout`` reuses a free slot whose slabs are large enough (growing a slab by 1/8
  headroom when not), or pins a new one;
* the lease returns the slot when the batch is released or collected; if the batch was
  copied to the device, the slot waits for the copy's CUDA event before it can be lent
  again (the copy reads the pinned memory asynchronously);
* on return, a slab larger than ``shrink_factor`` times the largest request of the recent
  window is dropped, so one unusually long batch does not keep its slab pinned forever;
  at most ``max_free`` slots are kept.
"""

from __future__ import annotations

import threading
from collections import deque

import torch


class PinnedLease:
    """A batch's claim on one slot; returned on ``release`` or when collected."""

    __slots__ = ("_pool", "_slot", "_event", "__weakref__")

    def __init__(self, pool: "PinnedPool", slot: dict) -> None:
        self._pool, self._slot, self._event = pool, slot, None

    def fence(self, event) -> None:
        """The slot's memory is read by work that completes with ``event``."""

        self._event = event

    def release(self) -> None:
        pool, slot = self._pool, self._slot
        self._pool, self._slot = None, None
        if pool is not None and slot is not None:
            pool._give_back(slot, self._event)

    def __del__(self) -> None:
        try:
            self.release()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class PinnedPool:
    def __init__(self, *, max_free: int = 4, recent_window: int = 256, shrink_factor: float = 2.0) -> None:
        self.max_free = max(1, int(max_free))
        self.shrink_factor = max(1.0, float(shrink_factor))
        self._free: list[dict] = []
        self._pending: list[tuple[dict, object]] = []   # (slot, CUDA event) awaiting a copy
        self._recent: dict[torch.dtype, deque] = {}
        self._window = max(8, int(recent_window))
        self._lock = threading.Lock()
        self.checkouts = self.reuses = self.grows = self.shrinks = self.allocs = 0

    # ------------------------------------------------------------------ lending
    def checkout(self, specs: list[tuple[torch.dtype, int]]) -> tuple[list[torch.Tensor], PinnedLease]:
        with self._lock:
            self._collect_pending()
            self.checkouts += 1
            for dt, n in specs:
                self._recent.setdefault(dt, deque(maxlen=self._window)).append(int(n))
            slot = self._free.pop() if self._free else {}
            if slot:
                self.reuses += 1
        views = []
        for dt, n in specs:
            n = max(1, int(n))
            buf = slot.get(dt)
            if buf is None or buf.numel() < n:
                if buf is not None:
                    self.grows += 1
                buf = torch.empty(n + n // 8, dtype=dt, pin_memory=torch.cuda.is_available())
                self.allocs += 1
                slot[dt] = buf
            views.append(buf[:n])
        return views, PinnedLease(self, slot)

    def _collect_pending(self) -> None:
        keep = []
        for slot, ev in self._pending:
            if ev is None or ev.query():
                self._admit(slot)
            else:
                keep.append((slot, ev))
        self._pending = keep

    def _admit(self, slot: dict) -> None:
        for dt in list(slot):
            recent = self._recent.get(dt)
            hw = max(recent) if recent else 0
            if hw and slot[dt].numel() > self.shrink_factor * (hw + hw // 8):
                del slot[dt]
                self.shrinks += 1
        if slot and len(self._free) < self.max_free:
            self._free.append(slot)

    def _give_back(self, slot: dict, event) -> None:
        with self._lock:
            if event is None:
                self._admit(slot)
            else:
                self._pending.append((slot, event))

    def stats(self) -> dict:
        with self._lock:
            pinned = sum(b.numel() * b.element_size() for s in self._free for b in s.values())
            return {"checkouts": self.checkouts, "reuses": self.reuses, "grows": self.grows,
                    "shrinks": self.shrinks, "allocs": self.allocs, "free_slots": len(self._free),
                    "pending_slots": len(self._pending), "free_pinned_bytes": pinned}


_DEFAULT: PinnedPool | None = None


def default_pool() -> PinnedPool:
    global _DEFAULT
    if _DEFAULT is None:
        _DEFAULT = PinnedPool()
    return _DEFAULT
