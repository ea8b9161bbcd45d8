"""Group AUC (QAUC / UAUC) over an evaluation set larger than host memory.

Counterpart of the reference's ``_DiskBackedGroupAUC`` (``src/train.py:8020-8134``):
per (task, scenario, group, score bin) positive and negative counts, then the mean over
groups holding both classes of each group's AUC on the binned scores (pairs in one bin
count one half), which is what the reference reports. Its store is an SQLite table
updated row by row; this one is a set of append-only binary partition files:

* ``add`` bins the probabilities on the device-independent grid of the streaming
  histogram AUC (``ceil(p * (bins - 1)) - 1``), pre-aggregates the batch's records by
  (task, scenario, group, bin) with numpy, and appends them to the partition
  ``group mod P`` (``P`` files, 24 bytes per aggregated record). Scenario ``-1`` is the
  overall population; every scenario a row belongs to gets its own record.
* ``compute_all`` reads one partition at a time (a group lives in exactly one), merges
  its records by (task, scenario, group, bin) and evaluates every group's AUC with
  vectorised cumulative sums; memory is bounded by the largest partition.
"""

from __future__ import annotations

import os
import shutil
import tempfile

import numpy as np
import torch

RECORD = np.dtype([("ts", "<i4"), ("bin", "<i4"), ("group", "<i8"), ("pos", "<i4"), ("neg", "<i4")])


def probability_bins(logits: torch.Tensor, bins: int) -> np.ndarray:
    p = torch.sigmoid(logits.detach().double().flatten().cpu())
    return torch.clamp(torch.ceil(p * (bins - 1)).long() - 1, 0, bins - 1).numpy().astype(np.int32)


class DiskGroupAUC:
    def __init__(self, bins: int = 4096, *, partitions: int = 64, directory: str | None = None) -> None:
        if bins < 2:
            raise ValueError("group AUC needs at least two score bins")
        self.bins = int(bins)
        self.partitions = max(1, int(partitions))
        self._own_dir = directory is None
        self.dir = directory or tempfile.mkdtemp(prefix="mdl-group-auc-")
        os.makedirs(self.dir, exist_ok=True)
        self._files = [open(os.path.join(self.dir, f"part-{i:04d}.bin"), "ab") for i in range(self.partitions)]
        self.records = 0
        self.rows = 0

    @staticmethod
    def _ts(task: int, scenario: int) -> int:
        return task * 65536 + (scenario + 1)

    def add(self, task: int, groups, logits: torch.Tensor, labels: torch.Tensor,
            scenario_membership: torch.Tensor | None = None) -> None:
        """One task's rows: ``groups`` int64 keys, ``labels`` 0/1, ``scenario_membership``
        ``[rows, S]`` booleans (or None: the overall population only)."""

        g = np.asarray(groups.cpu().numpy() if isinstance(groups, torch.Tensor) else groups, dtype=np.int64)
        y = labels.detach().flatten().cpu().numpy()
        n = g.shape[0]
        if y.shape[0] != n or logits.numel() != n:
            raise ValueError("group AUC batch inputs must have matching rows")
        if n == 0:
            return
        b = probability_bins(logits, self.bins)
        pos = (y == 1).astype(np.int32)
        ts_parts = [np.full(n, self._ts(task, -1), np.int32)]
        idx_parts = [np.arange(n)]
        if scenario_membership is not None:
            m = scenario_membership.detach().bool().cpu().numpy()
            rows, scen = np.nonzero(m)
            ts_parts.append((task * 65536 + scen + 1).astype(np.int32))
            idx_parts.append(rows)
        idx = np.concatenate(idx_parts)
        rec = np.empty(idx.shape[0], RECORD)
        rec["ts"] = np.concatenate(ts_parts)
        rec["bin"] = b[idx]
        rec["group"] = g[idx]
        rec["pos"] = pos[idx]
        rec["neg"] = 1 - pos[idx]
        rec = _merge(rec)
        part = (rec["group"] % self.partitions).astype(np.int64)
        order = np.argsort(part, kind="stable")
        rec, part = rec[order], part[order]
        cuts = np.searchsorted(part, np.arange(self.partitions + 1))
        for p in range(self.partitions):
            lo, hi = cuts[p], cuts[p + 1]
            if hi > lo:
                self._files[p].write(rec[lo:hi].tobytes())
        self.records += rec.shape[0]
        self.rows += n

    def compute_all(self) -> dict[tuple[int, int], float | None]:
        """``{(task, scenario): mean group AUC}`` (scenario ``-1`` = all rows)."""

        for f in self._files:
            f.flush()
        sums: dict[int, float] = {}
        counts: dict[int, int] = {}
        seen: set[int] = set()
        for p in range(self.partitions):
            path = os.path.join(self.dir, f"part-{p:04d}.bin")
            if os.path.getsize(path) == 0:
                continue
            rec = _merge(np.fromfile(path, dtype=RECORD))
            seen.update(np.unique(rec["ts"]).tolist())
            ts, auc = _group_aucs(rec)
            for t in np.unique(ts):
                sel = ts == t
                sums[int(t)] = sums.get(int(t), 0.0) + float(auc[sel].sum())
                counts[int(t)] = counts.get(int(t), 0) + int(sel.sum())
        out = {}
        for t in seen:
            key = (t // 65536, t % 65536 - 1)
            out[key] = sums[t] / counts[t] if counts.get(t) else None
        return out

    def compute(self, task: int, scenario: int = -1) -> float | None:
        return self.compute_all().get((task, scenario))

    def close(self) -> None:
        for f in self._files:
            f.close()
        if self._own_dir:
            shutil.rmtree(self.dir, ignore_errors=True)

    def __enter__(self) -> "DiskGroupAUC":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def _merge(rec: np.ndarray) -> np.ndarray:
    """Sum the counts of records with equal (task-scenario, group, bin), sorted by them."""

    if rec.shape[0] == 0:
        return rec
    order = np.lexsort((rec["bin"], rec["group"], rec["ts"]))
    r = rec[order]
    new = np.ones(r.shape[0], dtype=bool)
    new[1:] = (r["ts"][1:] != r["ts"][:-1]) | (r["group"][1:] != r["group"][:-1]) | (r["bin"][1:] != r["bin"][:-1])
    starts = np.flatnonzero(new)
    out = r[starts].copy()
    out["pos"] = np.add.reduceat(r["pos"], starts)
    out["neg"] = np.add.reduceat(r["neg"], starts)
    return out


def _group_aucs(rec: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per (task-scenario, group) AUC of merged, sorted records; only groups with both
    classes. AUC = sum_b pos_b * (neg below b + neg_b / 2) / (P * N)."""

    new = np.ones(rec.shape[0], dtype=bool)
    new[1:] = (rec["ts"][1:] != rec["ts"][:-1]) | (rec["group"][1:] != rec["group"][:-1])
    starts = np.flatnonzero(new)
    seg = np.cumsum(new) - 1
    pos = rec["pos"].astype(np.float64)
    neg = rec["neg"].astype(np.float64)
    cum_neg = np.cumsum(neg)
    before = np.concatenate([[0.0], cum_neg])[starts]   # negatives of earlier groups
    neg_below = cum_neg - neg - before[seg]              # negatives in lower bins of this group
    conc = np.add.reduceat(pos * (neg_below + 0.5 * neg), starts)
    P = np.add.reduceat(pos, starts)
    N = np.add.reduceat(neg, starts)
    ok = (P > 0) & (N > 0)
    return rec["ts"][starts][ok], conc[ok] / (P[ok] * N[ok])
