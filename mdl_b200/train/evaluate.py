"""Evaluation and prediction (reference ``evaluate_mdl`` / ``predict_mdl``,
``src/train.py:8168-8496``).

``evaluate`` streams every batch through the model without gradients, keeps
per-task (and per-scenario) histograms / loss sums on the device, reduces them
across ranks and returns AUC, log-loss, mean prediction and label rate.
``predict`` returns the per-row probabilities and can write them to Parquet
together with the row index and scenario id. With several ranks every rank
must pass the same number of batches (the lookup is collective).
"""

from __future__ import annotations

from typing import Iterable

import torch

from ..data.batch import PackedBatch
from ..metrics.auc import TaskMonitor


@torch.no_grad()
def predict_logits(trainer, batch: PackedBatch) -> torch.Tensor:
    """Logits ``[rows, tasks]``; batches without labels get zero labels under a zero mask."""

    if trainer.device.type == "cuda" and batch.ids.device.type != "cuda":
        batch = batch.to(trainer.device)
    if batch.labels is None:
        nt = len(trainer.config.task_names)
        z = torch.zeros(batch.rows, nt, dtype=torch.float32, device=batch.ids.device)
        batch = PackedBatch(batch.ids, batch.offsets, batch.dense, z, z.clone(), batch.scenario_id, batch.rows,
                            batch.sequences, group_key=batch.group_key)
    return trainer.predict_logits(batch).float()


@torch.no_grad()
def evaluate(trainer, batches: Iterable[PackedBatch], *, bins: int = 4096, per_scenario: bool = True,
             group_metric: str | None = None, group_dir: str | None = None) -> dict:
    """``group_metric`` (``qauc`` / ``uauc``) adds the mean per-group AUC over the batches'
    ``group_key`` (the split's ``group_id`` column), overall and per scenario, through
    the disk-backed accumulator (one process: groups are not exchanged across ranks)."""

    tasks = list(trainer.config.task_names)
    dev = trainer.device
    grouped = None
    if group_metric is not None:
        if group_metric not in ("qauc", "uauc"):
            raise ValueError("group_metric must be None, 'qauc' or 'uauc'")
        if trainer.world > 1:
            raise ValueError("qauc / uauc evaluation runs in a single process (groups are not exchanged "
                             "across ranks)")
        from ..metrics.group_auc_disk import DiskGroupAUC

        grouped = DiskGroupAUC(bins, directory=group_dir)
    overall = TaskMonitor(tasks, bins=bins, device=dev)
    scenes = list(trainer.config.scenarios.names)
    by_scene = {s: TaskMonitor(tasks, bins=bins, device=dev) for s in scenes} if per_scenario and len(scenes) > 1 \
        else {}
    n_batches = 0
    for batch in batches:
        logits = predict_logits(trainer, batch)
        labels = batch.labels.to(logits.device)
        mask = None if batch.label_mask is None else batch.label_mask.to(logits.device)
        overall.update(logits, labels, mask)
        if by_scene:
            sid = batch.scenario_id.to(logits.device)
            for i, s in enumerate(scenes):
                sel = sid == i
                if bool(sel.any()):
                    by_scene[s].update(logits[sel], labels[sel], None if mask is None else mask[sel])
        if grouped is not None:
            if batch.group_key is None:
                raise ValueError(f"{group_metric} needs the split's group_id column in every batch")
            gk = batch.group_key.cpu()
            member = torch.nn.functional.one_hot(batch.scenario_id.cpu().long(), num_classes=max(1, len(scenes)))
            lc, yc = logits.cpu(), labels.cpu()
            for t in range(len(tasks)):
                keep = torch.ones(batch.rows, dtype=torch.bool) if mask is None else mask[:, t].cpu() > 0
                grouped.add(t, gk[keep], lc[keep, t], yc[keep, t], member[keep] if len(scenes) > 1 else None)
        n_batches += 1
    group = trainer.group
    overall.all_reduce(group)
    for m in by_scene.values():
        m.all_reduce(group)
    res = {"batches": n_batches, "tasks": overall.summary(),
           "scenarios": {s: m.summary() for s, m in by_scene.items()}}
    if grouped is not None:
        try:
            vals = grouped.compute_all()
            res[group_metric] = {
                task: {"all": vals.get((t, -1)), **({s: vals.get((t, i)) for i, s in enumerate(scenes)}
                                                   if len(scenes) > 1 else {})}
                for t, task in enumerate(tasks)}
            res[f"{group_metric}_records"] = grouped.records
        finally:
            grouped.close()
    return res


@torch.no_grad()
def predict(trainer, batches: Iterable[PackedBatch], out_path: str | None = None) -> torch.Tensor:
    outs, scen = [], []
    for batch in batches:
        outs.append(torch.sigmoid(predict_logits(trainer, batch)).cpu())
        scen.append(batch.scenario_id.cpu())
    probs = torch.cat(outs) if outs else torch.zeros(0, len(trainer.config.task_names))
    if out_path is not None:
        import pyarrow as pa
        import pyarrow.parquet as pq

        cols = {"row": pa.array(list(range(probs.shape[0])), type=pa.int64()),
                "scenario_id": pa.array(torch.cat(scen).tolist() if scen else [], type=pa.int64())}
        suffix = trainer.config.data.train.prediction_score_suffix or ""
        for t, name in enumerate(trainer.config.task_names):
            cols[f"pred_{name}{suffix}"] = pa.array(probs[:, t].numpy())
        pq.write_table(pa.table(cols), out_path)
    return probs
