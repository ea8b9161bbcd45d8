"""Human-readable training log lines and the run environment.

Counterpart of the reference's stable stdout prefixes (``src/train.py:7270-7320``: ``Train
step | ...``, ``Train task | ...``, ``Train task warning | ...``; platform job logs often keep
stdout only, so these lines are what operators grep) and of its environment record
(``_environment``, ``src/benchmark.py:562-610``). The values are this framework's: per log
window the loss of the last step, rows, the host time spent waiting for batches and its
share of the window, the sparse rows touched, and per task the window's log-loss, mean
probability and logit moments, accumulated on the device (no host sync per step).
"""

from __future__ import annotations

import json
import math
import platform
import subprocess
import time

import torch


def environment(config, *, world: int, device: torch.device) -> dict:
    try:
        rev = subprocess.run(["git", "rev-parse", "HEAD"], capture_output=True, text=True, timeout=2.0,
                             check=False).stdout.strip()
    except (OSError, subprocess.SubprocessError):
        rev = ""
    name = torch.cuda.get_device_name(device) if device.type == "cuda" else None
    from ..ops._ext import ext  # noqa: F401 - the native library path is part of the record

    lib = None
    try:
        import mdl_b200

        lib = str(__import__("pathlib").Path(mdl_b200.__file__).parent / "_mdl_C.so")
    except Exception:  # noqa: BLE001
        pass
    return {
        "git_revision": rev or None, "python": platform.python_version(), "platform": platform.platform(),
        "torch": torch.__version__, "cuda_runtime": torch.version.cuda,
        "nccl": ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None,
        "device": str(device), "device_name": name, "world_size": world, "native_library": lib,
        "precision": config.runtime.precision, "kernel_backend": config.runtime.kernel_backend,
        "model": config.model.name, "batch_size": config.training.batch_size,
        "gradient_accumulation_steps": config.training.gradient_accumulation_steps,
    }


def _fmt(x: float | None) -> str:
    return "none" if x is None or (isinstance(x, float) and math.isnan(x)) else f"{x:.6f}"


class TrainLog:
    """Window statistics between log lines. ``step`` accumulates on the device; ``emit``
    (rank 0 prints, every rank reduces nothing: the lines describe rank 0's shard, as the
    reference's window stats do) reads them once per window."""

    PROB_MEAN_WARN = 0.9

    def __init__(self, tasks, *, world: int, micro_batches: int, checkpoint_every: int = 0) -> None:
        self.tasks = list(tasks)
        self.world, self.micro = world, micro_batches
        self.ckpt = checkpoint_every
        self._reset()

    def _reset(self) -> None:
        self.sums = None          # [tasks, 6]: n, bce, prob, logit, logit^2, label
        self.rows = 0
        self.wait_s = 0.0
        self.t0 = time.perf_counter()
        self.starved = 0

    @torch.no_grad()
    def step(self, result, batch, wait_s: float = 0.0, starved: bool = False) -> None:
        self.rows += int(batch.rows)
        self.wait_s += wait_s
        self.starved += int(starved)
        logits = result.logits
        if logits is None or batch.labels is None:
            return
        lg = logits.detach().float()
        if lg.dim() == 1:
            lg = lg.unsqueeze(1)
        y = batch.labels.to(lg.device).float()
        m = torch.ones_like(y) if batch.label_mask is None else batch.label_mask.to(lg.device).float()
        bce = torch.nn.functional.binary_cross_entropy_with_logits(lg, y, reduction="none")
        s = torch.stack([m.sum(0), (bce * m).sum(0), (torch.sigmoid(lg) * m).sum(0), (lg * m).sum(0),
                         (lg * lg * m).sum(0), (y * m).sum(0)], dim=1).double()
        self.sums = s if self.sums is None else self.sums + s

    def lines(self, step: int, loss: float | None, sparse_rows: int | None = None) -> list[str]:
        span = max(time.perf_counter() - self.t0, 1e-9)
        out = [f"Train step | step={step} | logloss={_fmt(loss)} active_ranks={self.world}/{self.world} "
               f"micro_batches={self.micro} local_rows={self.rows} dataloader_wait_s={self.wait_s:.4f} "
               f"dataloader_wait_ratio={self.wait_s / span:.4f}"
               + (f" sparse_local_rows={sparse_rows}" if sparse_rows is not None else "")
               + (f" starved_steps={self.starved}" if self.starved else "")
               + (f" checkpoint=on(every={self.ckpt})" if self.ckpt else " checkpoint=off")]
        if self.sums is not None:
            s = self.sums.cpu()
            for t, name in enumerate(self.tasks):
                n = float(s[t, 0])
                if n <= 0:
                    out.append(f"Train task | step={step} task={name} logloss=none prob_mean=none "
                               "logit_mean=none logit_std=none")
                    continue
                mean = float(s[t, 3]) / n
                var = max(0.0, float(s[t, 4]) / n - mean * mean)
                prob = float(s[t, 2]) / n
                out.append(f"Train task | step={step} task={name} logloss={float(s[t, 1]) / n:.6f} "
                           f"prob_mean={prob:.6f} logit_mean={mean:.6f} logit_std={math.sqrt(var):.6f}")
                if prob > self.PROB_MEAN_WARN:
                    out.append(f"Train task warning | step={step} task={name} prob_mean={prob:.4f} "
                               f"> {self.PROB_MEAN_WARN} (predictions collapsing to positive)")
        self._reset()
        return out


def environment_line(env: dict) -> str:
    return "Environment | " + json.dumps(env, sort_keys=True)
