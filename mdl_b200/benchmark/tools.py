"""Offline benchmark tools: batch-size tuning and benchmark-report summaries.

Counterparts of the reference's ``scripts/tune_batch_size.py`` and
``scripts/summarize_benchmarks.py`` (redesigned):

* ``tune_batch_size``: for each candidate batch size, build the model afresh, run the
  ``compute`` benchmark mode (device-resident synthetic batches, CUDA-event timing) and
  record samples/s, step times and the peak device memory; a CUDA out-of-memory error
  marks the size and ends the sweep upwards (larger sizes only need more memory). The
  recommendation is the fastest size whose peak stays under ``memory_fraction`` of the
  device.
* ``summarize_benchmarks``: JSON lines of ``bench.py`` / ``benchmark`` runs grouped by
  (implementation, model, metric); per group the value at each GPU count and the
  weak-scaling efficiency ``value(N) / (N * value(1))``, as a markdown table.
"""

from __future__ import annotations

import gc
import json
from typing import Callable, Iterable

import torch


def tune_batch_size(build: Callable[[int], tuple], batch_sizes: Iterable[int], *, steps: int = 10, warmup: int = 3,
                    device: torch.device, memory_fraction: float = 0.9) -> dict:
    """``build(batch) -> (cfg, model, trainer, batches)``; returns the per-size results and
    the recommended size."""

    from .modes import run as run_mode

    results = []
    cap = torch.cuda.get_device_properties(device).total_memory if device.type == "cuda" else None
    for b in sorted(int(x) for x in batch_sizes):
        entry = {"batch_size": b}
        try:
            if device.type == "cuda":
                torch.cuda.empty_cache()
                torch.cuda.reset_peak_memory_stats(device)
            cfg, model, trainer, batches = build(b)
            res = run_mode("compute", cfg, model, trainer, batches, rank=0, world=1, device=device, steps=steps,
                           warmup=warmup)
            entry.update(samples_per_s=res["value"], ms_mean=res["ms_mean"], ms_p95=res["ms_p95"])
            if device.type == "cuda":
                entry["peak_bytes"] = int(torch.cuda.max_memory_allocated(device))
                entry["peak_fraction"] = round(entry["peak_bytes"] / cap, 4)
        except torch.cuda.OutOfMemoryError:
            entry["oom"] = True
            results.append(entry)
            break
        finally:
            model = trainer = batches = None  # noqa: F841 - release before the next size
            gc.collect()
        results.append(entry)
    ok = [r for r in results if "samples_per_s" in r and r.get("peak_fraction", 0.0) <= memory_fraction]
    best = max(ok, key=lambda r: r["samples_per_s"]) if ok else None
    return {"results": results, "recommended_batch_size": None if best is None else best["batch_size"]}


def load_reports(paths: Iterable[str]) -> list[dict]:
    """Every JSON object line of the given files (other lines are skipped)."""

    rows = []
    for p in paths:
        with open(p, encoding="utf-8") as fh:
            for line in fh:
                line = line.strip()
                if not line.startswith("{"):
                    continue
                try:
                    obj = json.loads(line)
                except json.JSONDecodeError:
                    continue
                if isinstance(obj, dict) and "value" in obj and ("n_gpus" in obj or "steps" in obj):
                    rows.append(obj)
    return rows


def summarize_benchmarks(rows: list[dict]) -> dict:
    groups: dict[tuple, dict[int, list[float]]] = {}
    for r in rows:
        model = (r.get("config") or {}).get("model") if isinstance(r.get("config"), dict) else r.get("model")
        key = (r.get("impl", "mdl_b200"), str(model), r.get("metric", ""))
        groups.setdefault(key, {}).setdefault(int(r.get("n_gpus", 1)), []).append(float(r["value"]))
    out = []
    for (impl, model, metric), by_n in sorted(groups.items()):
        base = sum(by_n[1]) / len(by_n[1]) if 1 in by_n else None
        for n in sorted(by_n):
            v = sum(by_n[n]) / len(by_n[n])
            eff = None if base is None or base <= 0 else v / (n * base)
            out.append({"impl": impl, "model": model, "metric": metric, "n_gpus": n, "value": round(v, 1),
                        "runs": len(by_n[n]), "weak_scaling_efficiency": None if eff is None else round(eff, 4)})
    return {"rows": out}


def markdown(summary: dict) -> str:
    lines = ["| impl | model | metric | GPUs | value | runs | weak-scaling efficiency |", "|---|---|---|---|---|---|---|"]
    for r in summary["rows"]:
        eff = "" if r["weak_scaling_efficiency"] is None else f"{r['weak_scaling_efficiency']:.3f}"
        lines.append(f"| {r['impl']} | {r['model']} | {r['metric']} | {r['n_gpus']} | {r['value']} | {r['runs']} | "
                     f"{eff} |")
    return "\n".join(lines)
