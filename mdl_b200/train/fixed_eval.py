"""Fixed-test evaluation during training (``training.fixed_test_eval``).

Reference: ``_prepare_fixed_test_eval`` (``src/train.py:1361-1460``),
``_run_fixed_test_eval`` (``:7781-7960``) and ``_reduce_evaluation_histograms``
(``:7756``).

* Rank 0 lists ``data.test`` once, keeps the first ``files_per_rank * W`` files
  (sorted) and broadcasts that manifest, so every evaluation during the run sees
  the same rows.
* Every ``every_steps`` optimizer steps each rank streams its row groups of the
  manifest (``plan_row_groups``) without gradients. The lookup is collective,
  so all ranks run the same number of batches: the count is the maximum over
  ranks of each rank's ``ceil(rows / batch)`` (known from the Parquet metadata),
  and a rank that runs out replays its last batch with a zero label mask.
* Per-task histograms (``auc_bins``) and loss sums are reduced across ranks;
  the result is AUC, log-loss, mean prediction and label rate per task.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..metrics.auc import TaskMonitor
from .evaluate import predict_logits


class FixedTestEval:
    def __init__(self, config, trainer, *, rank: int = 0, world: int = 1, group=None) -> None:
        ev = config.training.fixed_test_eval
        self.config, self.trainer = config, trainer
        self.rank, self.world, self.group = rank, world, group
        self.every = int(ev.every_steps)
        self.bins = int(ev.auc_bins)
        self.files: list[str] = []
        test = config.data.test
        self.enabled = bool(ev.enabled) and test is not None and bool(test.inputs)
        if not self.enabled:
            return
        payload = [None]
        if rank == 0:
            from ..data.parquet import discover_parquet_inputs

            paths = sorted(discover_parquet_inputs(test.inputs))
            payload = [paths[:int(ev.files_per_rank) * max(1, world)]]
        if world > 1 and dist.is_initialized():
            dist.broadcast_object_list(payload, src=0, group=group)
        self.files = list(payload[0] or [])
        self.enabled = bool(self.files)

    def due(self, step: int) -> bool:
        return self.enabled and step > 0 and step % self.every == 0

    def _local_batches(self, model, batch_size: int):
        from ..data.parquet import ParquetBatchIterator, Tensorizer

        test = self.config.data.test
        it = ParquetBatchIterator(self.files, Tensorizer(self.config, model.encoder.batch_plan, split="test",
                                                         seq_names=list(model.encoder.seq_plans)),
                                  batch_size, rank=self.rank, world=self.world, shard_unit=test.reader.shard_unit,
                                  drop_last=False, prefetch=2, loop=False)
        rows = sum(ref.rows for ref in it.refs)
        return it, math.ceil(rows / batch_size) if rows else 0

    @torch.no_grad()
    def run(self, model) -> dict:
        batch_size = self.config.training.batch_size
        it, local = self._local_batches(model, batch_size)
        count = torch.tensor([local], dtype=torch.int64, device=self.trainer.device)
        if self.world > 1 and dist.is_initialized():
            dist.all_reduce(count, op=dist.ReduceOp.MAX, group=self.group)
        total = int(count.item())
        tasks = list(self.config.task_names)
        monitor = TaskMonitor(tasks, bins=self.bins, device=self.trainer.device)
        last = None
        done = 0
        was_training = model.training
        model.eval()
        try:
            for batch in it:
                if done == total:
                    break
                logits = predict_logits(self.trainer, batch)
                mask = None if batch.label_mask is None else batch.label_mask.to(logits.device)
                monitor.update(logits, batch.labels.to(logits.device), mask)
                last = batch
                done += 1
        finally:
            it.close()
        try:
            while done < total:  # this rank ran out: keep the collective lookups in step
                if last is None:
                    raise RuntimeError("fixed-test evaluation: a rank has no test rows while others do")
                predict_logits(self.trainer, last)   # result discarded: zero weight
                done += 1
        finally:
            model.train(was_training)
        monitor.all_reduce(self.group)
        return {"batches": total, "tasks": monitor.summary()}
