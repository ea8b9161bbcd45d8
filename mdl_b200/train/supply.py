"""Batch supply protocol for several ranks (reference ``_next_batch_within``,
``_RankSupply`` / ``_supply_verdict`` / ``_start_rank_supply_count``,
``src/train.py:4532-4545, 5542-5616``).

Every step each rank reads its next batch within a time budget and reports one
of three states: it has a batch (*active*), its shard is finished
(*exhausted*), or the reader is late (neither). The counts are summed over the
gloo control group (host memory, no device sync), and every rank acts on the
same verdict:

* ``train``  -- this rank has a batch;
* ``replay`` -- this rank has none but peers are training: it runs a step on its
  last batch with a zero label mask, so the collective lookups and the dense
  gradient exchange stay aligned and its loss contributes nothing;
* ``retry``  -- nobody has data but not everybody is exhausted (a world-wide
  reader stall is not the end of the data);
* ``stop``   -- every rank is exhausted.
"""

from __future__ import annotations

import queue
import threading

import torch
import torch.distributed as dist

from ..data.batch import PackedBatch

BATCH_NOT_READY = object()
_END = object()


class BudgetedIterator:
    """Pulls an iterator on a background thread; ``next_within`` waits at most ``timeout_s``."""

    def __init__(self, iterable, depth: int = 2) -> None:
        self._it = iter(iterable)
        self._q: queue.Queue = queue.Queue(maxsize=max(1, depth))
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _run(self) -> None:
        try:
            for item in self._it:
                while not self._stop.is_set():
                    try:
                        self._q.put(item, timeout=0.1)
                        break
                    except queue.Full:
                        continue
                if self._stop.is_set():
                    return
            self._q.put(_END)
        except BaseException as error:  # surfaced to the consumer
            self._q.put(error)

    def next_within(self, timeout_s: float | None):
        """A batch, ``BATCH_NOT_READY``, or ``StopIteration`` raised at the end."""

        try:
            item = self._q.get(timeout=timeout_s)
        except queue.Empty:
            return BATCH_NOT_READY
        if item is _END:
            self._q.put(_END)  # stay exhausted on later calls
            raise StopIteration
        if isinstance(item, BaseException):
            raise item
        return item

    def close(self) -> None:
        self._stop.set()


def start_supply_count(active: bool, exhausted: bool, world: int, group=None):
    """Asynchronous sum of (active, exhausted) over the ranks; ``wait()`` gives the pair."""

    value = torch.tensor([int(active), int(exhausted)], dtype=torch.long)
    work = None
    if world > 1 and dist.is_initialized():
        work = dist.all_reduce(value, op=dist.ReduceOp.SUM, group=group, async_op=True)

    class _Handle:
        def wait(self):
            if work is not None:
                work.wait()
            a, e = value.tolist()
            return int(a), int(e)

    return _Handle()


def supply_verdict(has_batch: bool, active: int, exhausted: int, world: int) -> str:
    if has_batch:
        return "train"
    if exhausted >= world:
        return "stop"
    if active == 0:
        return "retry"
    return "replay"


def zero_weight(batch: PackedBatch) -> PackedBatch:
    """The same rows with a zero label mask (a step that contributes no loss)."""

    mask = torch.zeros_like(batch.labels) if batch.labels is not None else None
    return PackedBatch(batch.ids, batch.offsets, batch.dense, batch.labels, mask, batch.scenario_id, batch.rows,
                       batch.sequences, group_key=batch.group_key)
