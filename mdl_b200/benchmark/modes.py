"""Benchmark modes of ``python -m mdl_b200 benchmark`` (reference ``src/benchmark.py``:
modes ``:60, 1176-1570``, analytical-FLOP MFU ``:280-355``, GPU-utilisation sampler
``:395-444``, step-time percentiles and the utilisation gate ``:671-848, 1666-1697``).

* ``compute``: training steps on device-resident synthetic batches (no input work);
* ``end-to-end``: the configured input pipeline (Parquet, or synthetic host batches)
  through ``Trainer.step_from_host`` (pinned H2D copy in, loss copy out, every step);
* ``data``: the input pipeline and the H2D copy only (no model work);
* ``embedding``: the embedding lookup, its backward and the sparse optimizer only.

Every step is timed with CUDA events on the launching stream (max over ranks); the
report gives samples/s, mean / p50 / p95 step times, the MFU of the dense GEMM work
(``6 x GEMM weights x rows`` FLOPs per step against the measured bf16 peak when
``MEASURED_PEAKS.json`` is present, else 2.25 PFLOP/s nominal) and the mean GPU
utilisation sampled through NVML during the timed steps.
"""

from __future__ import annotations

import json
import os
import statistics
import threading
import time

import torch
import torch.distributed as dist

MODES = ("compute", "end-to-end", "data", "embedding")


def dense_gemm_flops_per_row(model) -> float:
    """``6 x`` the GEMM weights one row passes through (forward + two backward products).
    Per-token weights ([T, out, in]) count once per row; attention score / value products
    are not included."""

    n = 0
    for name in model.gemm_param_names():
        p = dict(model.named_parameters()).get(name)
        if p is not None:
            n += p.numel()
    return 6.0 * n


def bf16_peak_flops() -> float:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["bf16_tflops"]) * 1e12
    except (OSError, KeyError, ValueError):
        return 2.25e15


class UtilSampler:
    """Mean NVML GPU utilisation (percent) of one device, sampled from a thread."""

    def __init__(self, index: int, period_s: float = 0.05) -> None:
        self.index, self.period = index, period_s
        self.samples: list[float] = []
        self._stop = threading.Event()
        self._t = None

    def start(self) -> "UtilSampler":
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        except Exception:  # noqa: BLE001 - no NVML: no utilisation figure
            return self

        def run():
            while not self._stop.wait(self.period):
                try:
                    self.samples.append(float(pynvml.nvmlDeviceGetUtilizationRates(h).gpu))
                except Exception:  # noqa: BLE001
                    return

        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def stop(self) -> float | None:
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)
        return statistics.fmean(self.samples) if self.samples else None


def run(mode: str, cfg, model, trainer, batches, *, rank: int, world: int, device: torch.device, steps: int,
        warmup: int, min_util: float | None = None) -> dict:
    """Run one benchmark mode; ``batches`` yields host ``PackedBatch``es."""

    if mode not in MODES:
        raise ValueError(f"benchmark mode {mode!r}; choose one of {MODES}")
    cuda = device.type == "cuda"
    pool = [next(batches) for _ in range(3)] if mode == "compute" or mode == "embedding" else None
    dev = [b.to(device) for b in pool] if (pool is not None and cuda) else pool
    anchor = torch.zeros(0, device=device, requires_grad=True)

    def embedding_step(b):
        from ..ops.embedding import fused_lookup

        out = fused_lookup(model.store, model.encoder.plan, b.ids, b.offsets, b.dense, b.rows, anchor)
        out.float().sum().backward()
        model.store.step()

    loss_host = torch.zeros(1, dtype=torch.float32, pin_memory=cuda)

    def one(i):
        if mode == "compute":
            trainer.train_step(dev[i % 3])
        elif mode == "embedding":
            embedding_step(dev[i % 3])
        elif mode == "end-to-end":
            trainer.step_from_host(next(batches), loss_out=loss_host)
        else:  # data
            b = next(batches)
            if cuda:
                b.to(device)

    for i in range(warmup):
        one(i)
    if cuda:
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    util = UtilSampler(device.index or 0).start() if cuda else None
    times = []
    t_wall = time.perf_counter()
    for i in range(steps):
        if cuda:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            one(i)
            e1.record()
            times.append((e0, e1))
        else:
            t0 = time.perf_counter()
            one(i)
            times.append((time.perf_counter() - t0) * 1e3)
    if cuda:
        torch.cuda.synchronize(device)
        ms = [a.elapsed_time(b) for a, b in times]
    else:
        ms = times
    wall_ms = (time.perf_counter() - t_wall) * 1e3
    mean_util = util.stop() if util is not None else None
    # per-step times: the max over ranks of each step
    t = torch.tensor(ms, dtype=torch.float64, device=device if cuda else "cpu")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = sorted(t.tolist())
    total = sum(ms) if mode != "data" else wall_ms
    rows = cfg.training.batch_size * world * steps
    res = {"metric": "train samples/sec" if mode != "data" else "input samples/sec", "mode": mode,
           "value": round(rows / (total / 1e3), 1), "n_gpus": world, "steps": steps,
           "ms_mean": round(total / steps, 4), "ms_p50": round(ms[len(ms) // 2], 4),
           "ms_p95": round(ms[min(len(ms) - 1, int(0.95 * len(ms)))], 4), "model": cfg.model.name,
           "global_batch": cfg.training.batch_size * world}
    if mode in ("compute", "end-to-end"):
        flops = dense_gemm_flops_per_row(model) * cfg.training.batch_size * world
        res["mfu_dense_gemm"] = float(f"{flops / (total / steps / 1e3) / (bf16_peak_flops() * world):.4g}")
    if mean_util is not None:
        res["gpu_util_mean_pct"] = round(mean_util, 1)
        if min_util is not None and mean_util < min_util:
            res["util_gate"] = f"failed: mean GPU utilisation {mean_util:.1f}% < {min_util}%"
    return res
