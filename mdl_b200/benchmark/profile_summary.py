"""``torch.profiler`` summary of training steps: device time by kernel class.

Counterpart of the reference's profiler pass (``src/benchmark.py:851-901``), which lists
attention kernels and communication operators and sums their device time and the
profiler's FLOP estimate. Here every GPU kernel of the profiled steps is put in one
class by its name -- communication (NCCL and this framework's NVLink exchange kernels),
attention, GEMM, embedding, optimizer, normalization, other -- and the report gives
each class's device time per step and share, the top kernels, the framework's named
ranges (``utils/trace.py``) with their CPU time, and the analytical dense-GEMM FLOPs
per step (the profiler's own FLOP counter sees only ATen ops, not these kernels).
"""

from __future__ import annotations

from typing import Callable

import torch

KERNEL_CLASSES: tuple[tuple[str, tuple[str, ...]], ...] = (
    ("communication", ("nccl", "dense_sync", "emb_route", "emb_owner", "barrier_kernel", "multimem",
                       "all_reduce", "allreduce", "all_to_all", "alltoall", "c10d", "reduce_scatter",
                       "all_gather", "allgather")),
    ("attention", ("fmha", "sqa_", "attention", "flash", "scaled_dot_product", "softmax")),
    ("gemm", ("gemm", "cutlass", "cublas", "xmma", "nvjet", "matmul")),
    ("embedding", ("emb_", "embedding")),
    ("optimizer", ("optim", "adagrad", "rmsprop", "adam")),
    ("normalization", ("ln_", "layernorm", "layer_norm", "rmsnorm", "rms_norm")),
)


def classify(name: str) -> str:
    n = name.lower()
    for cls, tokens in KERNEL_CLASSES:
        if any(t in n for t in tokens):
            return cls
    return "other"


def _device_us(evt) -> float:
    for attr in ("self_device_time_total", "self_cuda_time_total", "device_time_total", "cuda_time_total"):
        v = getattr(evt, attr, None)
        if v:
            return float(v)
    return 0.0


def profile_steps(step: Callable[[], None], steps: int, *, device: torch.device,
                  gemm_flops_per_step: float | None = None, top: int = 12) -> dict:
    """Run ``step`` ``steps`` times under ``torch.profiler`` and summarise."""

    if steps <= 0:
        return {"error": "profiling disabled (steps=0)"}
    acts = [torch.profiler.ProfilerActivity.CPU]
    if device.type == "cuda":
        acts.append(torch.profiler.ProfilerActivity.CUDA)
    try:
        with torch.profiler.profile(activities=acts, acc_events=True) as prof:
            for _ in range(steps):
                step()
                prof.step()
            if device.type == "cuda":
                torch.cuda.synchronize(device)
        events = prof.key_averages()
    except Exception as error:  # noqa: BLE001 - profiler support varies by build
        return {"error": f"{type(error).__name__}: {error}"}
    kernels: dict[str, float] = {}
    ranges: dict[str, float] = {}
    for evt in events:
        key = str(evt.key)
        if key.startswith("mdl."):
            ranges[key] = ranges.get(key, 0.0) + float(getattr(evt, "cpu_time_total", 0.0))
            continue
        us = _device_us(evt)
        is_kernel = getattr(evt, "device_type", None) == torch.autograd.DeviceType.CUDA
        if us > 0 and is_kernel:
            kernels[key] = kernels.get(key, 0.0) + us
    total = sum(kernels.values())
    by_class: dict[str, float] = {}
    for k, us in kernels.items():
        c = classify(k)
        by_class[c] = by_class.get(c, 0.0) + us
    out = {
        "steps": steps,
        "device_ms_per_step": round(total / steps / 1e3, 4),
        "by_class_ms_per_step": {c: round(us / steps / 1e3, 4) for c, us in sorted(by_class.items(),
                                                                                  key=lambda kv: -kv[1])},
        "by_class_share": {c: round(us / total, 4) for c, us in by_class.items()} if total else {},
        "top_kernels": [{"name": k[:120], "class": classify(k), "ms_per_step": round(us / steps / 1e3, 4)}
                        for k, us in sorted(kernels.items(), key=lambda kv: -kv[1])[:top]],
        "ranges_cpu_ms_per_step": {k: round(v / steps / 1e3, 4) for k, v in sorted(ranges.items())},
        "communication_kernels": sorted(k[:120] for k in kernels if classify(k) == "communication"),
        "attention_kernels": sorted(k[:120] for k in kernels if classify(k) == "attention"),
    }
    if gemm_flops_per_step is not None:
        out["gemm_flops_per_step"] = float(f"{gemm_flops_per_step:.4g}")
        gemm_ms = by_class.get("gemm", 0.0) / steps / 1e3
        if gemm_ms > 0:
            out["gemm_tflops_achieved"] = round(gemm_flops_per_step / (gemm_ms * 1e-3) / 1e12, 1)
    return out
