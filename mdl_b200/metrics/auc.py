"""AUC family: exact rank AUC, group AUC, streaming histogram AUC, task monitor.

Semantics kept alike with the reference (``src/train.py:7452-7700``) so numbers
are comparable between the frameworks:

* ``binary_auc``: exact Mann-Whitney AUC with average ranks for ties; ``None``
  when a class is missing.
* ``group_auc``: unweighted mean of per-group AUCs over groups holding both
  classes (QAUC / UAUC with query or user ids as groups).
* ``StreamingHistogramAUC``: positive / negative counts per probability bucket
  of an N-point threshold grid (bucket ``ceil(p * (N - 1)) - 1``, which gives
  the confusion counts of the online evaluator's ``p > threshold`` rule at each
  threshold), ROC by reversed cumulative sums, trapezoid integration. The
  log-odds variant buckets logits uniformly on [-20, 20] (a diagnostic for
  predictions that crowd one end of the probability grid). Histograms reduce
  across ranks by a plain sum (``all_reduce``).
* ``TaskMonitor``: streaming per-task BCE, mean probability, label rate and
  AUC with collapse warnings (mean probability above 0.9, AUC below 0.55).

Updates bucket on the tensor's device (one ``bincount``); only the final
integration runs on the host.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

LOGIT_LIMIT = 20.0


def binary_auc(scores: torch.Tensor, labels: torch.Tensor) -> float | None:
    scores = scores.detach().double().flatten().cpu()
    labels = labels.detach().double().flatten().cpu()
    if scores.numel() != labels.numel():
        raise ValueError("AUC scores and labels must have the same length")
    if scores.numel() == 0:
        return None
    if not bool(torch.isfinite(scores).all()):
        raise ValueError("AUC scores must be finite")
    if not bool(((labels == 0) | (labels == 1)).all()):
        raise ValueError("AUC labels must be binary")
    n_pos = int((labels == 1).sum())
    n_neg = labels.numel() - n_pos
    if n_pos == 0 or n_neg == 0:
        return None
    order = torch.argsort(scores, stable=True)
    s, y = scores[order], labels[order]
    _, inverse, counts = torch.unique_consecutive(s, return_inverse=True, return_counts=True)
    ranks = torch.arange(1, s.numel() + 1, dtype=torch.float64)
    tie_rank = torch.zeros(counts.numel(), dtype=torch.float64).scatter_add_(0, inverse, ranks) / counts
    pos_rank_sum = tie_rank[inverse][y == 1].sum()
    return float((pos_rank_sum - n_pos * (n_pos + 1) / 2.0) / (n_pos * n_neg))


def group_auc(scores: torch.Tensor, labels: torch.Tensor, groups) -> float | None:
    groups = list(groups)
    if len(groups) != scores.numel() or len(groups) != labels.numel():
        raise ValueError("group AUC inputs must have matching lengths")
    by_group: dict = {}
    for i, g in enumerate(groups):
        by_group.setdefault(g, []).append(i)
    vals = []
    s, y = scores.flatten(), labels.flatten()
    for idx in by_group.values():
        it = torch.tensor(idx, dtype=torch.long)
        v = binary_auc(s[it], y[it])
        if v is not None:
            vals.append(v)
    return sum(vals) / len(vals) if vals else None


def trapezoid_auc(positives: torch.Tensor, negatives: torch.Tensor) -> float | None:
    pos, neg = positives.double().cpu(), negatives.double().cpu()
    p_tot, n_tot = float(pos.sum()), float(neg.sum())
    if p_tot == 0 or n_tot == 0:
        return None
    # counts at threshold j = everything in bucket j and above (reversed cumulative sum)
    tpr = torch.cat([pos.flip(0).cumsum(0).flip(0), pos.new_zeros(1)]) / p_tot
    fpr = torch.cat([neg.flip(0).cumsum(0).flip(0), neg.new_zeros(1)]) / n_tot
    return float(((fpr[:-1] - fpr[1:]) * (tpr[:-1] + tpr[1:]) * 0.5).sum())


class StreamingHistogramAUC:
    def __init__(self, bins: int = 4096, *, logit_grid: bool = False, device=None) -> None:
        if bins < 2:
            raise ValueError("AUC histogram requires at least two bins")
        self.bins = bins
        self.logit_grid = logit_grid
        self.hist = torch.zeros(2, bins, dtype=torch.float64, device=device)

    def _buckets(self, logits: torch.Tensor) -> torch.Tensor:
        if self.logit_grid:
            z = (logits.double().clamp(-LOGIT_LIMIT, LOGIT_LIMIT) + LOGIT_LIMIT) / (2 * LOGIT_LIMIT)
            return torch.clamp(torch.floor(z * self.bins).long(), 0, self.bins - 1)
        p = torch.sigmoid(logits.double())
        return torch.clamp(torch.ceil(p * (self.bins - 1)).long() - 1, 0, self.bins - 1)

    @torch.no_grad()
    def update(self, logits: torch.Tensor, labels: torch.Tensor, weight: torch.Tensor | None = None) -> None:
        logits = logits.detach().flatten()
        labels = labels.detach().flatten().to(logits.device)
        if logits.numel() != labels.numel():
            raise ValueError("AUC logits and labels must have the same length")
        if logits.numel() == 0:
            return
        keep = torch.ones_like(labels, dtype=torch.bool) if weight is None else weight.flatten().to(logits.device) > 0
        if self.hist.device != logits.device:
            self.hist = self.hist.to(logits.device)
        b = self._buckets(logits)
        pos = keep & (labels == 1)
        neg = keep & (labels == 0)
        self.hist[0] += torch.bincount(b[pos], minlength=self.bins).double()
        self.hist[1] += torch.bincount(b[neg], minlength=self.bins).double()

    def all_reduce(self, group=None) -> None:
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.hist, group=group)

    def compute(self) -> float | None:
        return trapezoid_auc(self.hist[0], self.hist[1])

    def counts(self) -> tuple[int, int, int]:
        p, n = int(self.hist[0].sum()), int(self.hist[1].sum())
        return p + n, p, n

    def occupied_bins(self) -> int:
        return int(((self.hist[0] + self.hist[1]) > 0).sum())


class TaskMonitor:
    """Streaming per-task loss / calibration / AUC for a few tasks."""

    PROB_MEAN_WARN = 0.9
    AUC_WARN = 0.55

    def __init__(self, tasks: list[str], bins: int = 4096, device=None) -> None:
        self.tasks = list(tasks)
        self.auc = [StreamingHistogramAUC(bins, device=device) for _ in tasks]
        self.sums = torch.zeros(len(tasks), 4, dtype=torch.float64, device=device)  # n, bce, prob, label

    @torch.no_grad()
    def update(self, logits: torch.Tensor, labels: torch.Tensor, mask: torch.Tensor | None = None) -> None:
        logits = logits.detach().double()
        labels = labels.detach().double().to(logits.device)
        m = torch.ones_like(labels) if mask is None else mask.detach().double().to(logits.device)
        if self.sums.device != logits.device:
            self.sums = self.sums.to(logits.device)
        bce = torch.nn.functional.binary_cross_entropy_with_logits(logits, labels, reduction="none")
        self.sums[:, 0] += m.sum(0)
        self.sums[:, 1] += (bce * m).sum(0)
        self.sums[:, 2] += (torch.sigmoid(logits) * m).sum(0)
        self.sums[:, 3] += (labels * m).sum(0)
        for t, a in enumerate(self.auc):
            a.update(logits[:, t], labels[:, t], m[:, t])

    def all_reduce(self, group=None) -> None:
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.sums, group=group)
            for a in self.auc:
                a.all_reduce(group)

    def summary(self) -> dict[str, dict]:
        out = {}
        s = self.sums.cpu()
        for t, name in enumerate(self.tasks):
            n = float(s[t, 0])
            auc = self.auc[t].compute()
            prob = float(s[t, 2]) / n if n else math.nan
            warn = []
            if n and prob > self.PROB_MEAN_WARN:
                warn.append("mean probability above 0.9")
            if auc is not None and auc < self.AUC_WARN:
                warn.append("AUC below 0.55")
            out[name] = {"count": n, "logloss": float(s[t, 1]) / n if n else math.nan, "mean_prob": prob,
                         "label_rate": float(s[t, 3]) / n if n else math.nan, "auc": auc, "warnings": warn}
        return out
