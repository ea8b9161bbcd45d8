"""Host-prepare child process (reference ``_ProcessHostPrepareIterator`` /
``_host_prepare_process_main``, ``src/train.py:3465-4357``).

Parquet reading, batch cutting and tensorisation run in a spawned child process
so they do not compete with the training loop for the interpreter. The child
builds each ``PackedBatch`` as two flat buffers (int64 and fp32) and sends them
through a ``torch.multiprocessing`` queue, which moves tensors through shared
memory; the parent rebuilds the batch views around the shared buffers (and,
with ``pin``, copies them into page-locked memory for asynchronous H2D).

A thread of the child sends a heartbeat every ``beat_s``; the parent raises
when the child exits or fails, when nothing (heartbeat or batch) arrives for
``startup_timeout_s`` before the first batch, or when no batch arrives for
``idle_timeout_s`` after it (heartbeats do not extend that one). The child
stays alive after its last item until the parent's ``close`` (shared tensors
travel as file descriptors of the sender), which then joins it. The child never
touches CUDA.
"""

from __future__ import annotations

import queue
import time

import torch
import torch.multiprocessing as mp

from .batch import PackedBatch

_BATCH, _END, _ERROR, _BEAT = 0, 1, 2, 3


def parquet_batches(config_mapping: dict, batch_plan, paths: list[str], batch_size: int, rank: int, world: int,
                    split: str, loop: bool, shuffle_rows: int, seed: int, seq_names=None):
    """Child-side factory: the rank's Parquet batches (no pinning in the child)."""

    from ..config.loader import app_config_from_mapping
    from .parquet import ParquetBatchIterator, Tensorizer

    cfg = app_config_from_mapping(config_mapping)
    tz = Tensorizer(cfg, batch_plan, split=split, seq_names=seq_names)
    sp = getattr(cfg.data, split) or cfg.data.train
    r = sp.reader
    adapter = None
    if sp.format in ("adapter_parquet", "agg_parquet"):
        from .agg import AggAdapter, AggPlan

        adapter = AggAdapter(AggPlan.from_config(cfg, split))
    it = ParquetBatchIterator(paths, tz, batch_size, rank=rank, world=world, shuffle_rows=shuffle_rows, seed=seed,
                              loop=loop, prefetch=2, pin=False, adapter=adapter,
                              length_buckets=[(b.max_length, b.batch_size) for b in r.length_buckets],
                              length_bucket_metric=r.length_bucket_metric, agg_direct_mode=r.agg_direct_mode)
    return iter(it)


def _child(factory, args, q, stop, beat_s: float) -> None:
    import threading

    torch.set_num_threads(1)
    done = threading.Event()

    def beat():
        while not done.wait(beat_s) and not stop.is_set():
            try:
                q.put((_BEAT, time.monotonic()), timeout=beat_s)
            except queue.Full:
                pass

    threading.Thread(target=beat, daemon=True).start()
    try:
        for batch in factory(*args):
            if stop.is_set():
                return
            if not batch._flat:
                batch = PackedBatch.pack(batch.ids, batch.offsets, batch.dense, batch.labels, batch.label_mask,
                                         batch.scenario_id, batch.rows, batch.sequences, group_key=batch.group_key)
            b64, b32 = batch._flat
            q.put((_BATCH, (b64, batch._views[0], b32, batch._views[1], batch.rows)))
        done.set()
        q.put((_END, None))
    except BaseException as error:  # reported to the parent
        done.set()
        q.put((_ERROR, repr(error)))
    # shared-memory tensors are handed over by file descriptor: stay alive until the
    # parent has received everything (it sets ``stop`` on close)
    stop.wait(3600.0)


class ProcessBatchIterator:
    def __init__(self, factory, args: tuple, *, depth: int = 4, pin: bool = False,
                 startup_timeout_s: float = 300.0, idle_timeout_s: float = 600.0, beat_s: float = 5.0) -> None:
        ctx = mp.get_context("spawn")
        self._q = ctx.Queue(maxsize=max(1, depth))
        self._stop = ctx.Event()
        self._proc = ctx.Process(target=_child, args=(factory, args, self._q, self._stop, beat_s), daemon=True)
        self._proc.start()
        self.pin = pin
        self.startup_timeout_s = float(startup_timeout_s or 1e9)
        self.idle_timeout_s = float(idle_timeout_s or 1e9)

    def _get(self, deadline: float, what: str):
        while True:
            try:
                return self._q.get(timeout=min(1.0, max(0.01, deadline - time.monotonic())))
            except queue.Empty:
                if not self._proc.is_alive():
                    raise RuntimeError(f"host-prepare process exited with code {self._proc.exitcode}")
                if time.monotonic() > deadline:
                    raise TimeoutError(f"host-prepare process: {what}")

    def __iter__(self):
        # before the first batch any message (heartbeat included) shows progress; after it
        # only delivered batches count, so a child that is alive but stuck is caught
        last_batch = None
        since = time.monotonic()
        while True:
            if last_batch is None:
                deadline = since + self.startup_timeout_s
                what = f"no message within {self.startup_timeout_s:.0f} s before the first batch"
            else:
                deadline = last_batch + self.idle_timeout_s
                what = f"no batch within {self.idle_timeout_s:.0f} s"
            kind, payload = self._get(deadline, what)
            if kind == _BEAT:
                since = time.monotonic()
                continue
            if kind == _END:
                return
            if kind == _ERROR:
                raise RuntimeError(f"host-prepare process failed: {payload}")
            last_batch = time.monotonic()
            b64, v64, b32, v32, rows = payload
            if self.pin:
                b64, b32 = b64.pin_memory(), b32.pin_memory()
            yield PackedBatch._from_flat(b64, v64, b32, v32, rows)

    def close(self, join_timeout_s: float = 10.0) -> None:
        self._stop.set()
        try:
            while True:
                self._q.get_nowait()
        except Exception:
            pass
        self._proc.join(join_timeout_s)
        if self._proc.is_alive():
            self._proc.terminate()
            self._proc.join(join_timeout_s)
