"""Stage costs of the input pipeline: where the host time of a batch goes.

Counterpart of the reference's research scripts ``scripts/research_adapter_stage_costs.py``
(scan / adapter / tensorize / pin split of the data producer) and the input-pipeline half
of ``scripts/profile_gpu_utilization_factors.py``. Per raw row group of the inputs it times,
with ``time.perf_counter`` on one thread:

* ``read``: the Parquet row group with the columns the pipeline needs;
* ``expand`` (agg inputs): the legacy whole-table expansion (``AggIndex.flat_table``), or
  for ``agg_direct_mode: direct`` the request-group index and per-pack gathers;
* ``tensorize``: ``Tensorizer`` into a ``PackedBatch``;
* ``pin``: the copy into pinned host buffers (CUDA only);
* ``h2d``: the host-to-device copy, synchronised (CUDA only).

Reports per stage the seconds, the share of the total and the candidate rows per second
the stage alone would sustain, and the pipeline's rows per second; the slowest stage is
named ``bottleneck``.
"""

from __future__ import annotations

import time
from typing import Sequence

import numpy as np
import torch


def stage_costs(config, paths: Sequence[str], batch_plan, seq_names, *, max_tables: int = 8, warmup: int = 1,
                batch_size: int | None = None, device: torch.device | None = None, split: str = "train") -> dict:
    import pyarrow as pa
    import pyarrow.parquet as pq

    from ..data.parquet import RowGroupRef, Tensorizer, plan_row_groups

    sp = getattr(config.data, split) or config.data.train
    tz = Tensorizer(config, batch_plan, split=split, seq_names=seq_names)
    plan = None
    mode = "flat"
    if sp.format in ("adapter_parquet", "agg_parquet"):
        from ..data.agg import AggPlan

        plan = AggPlan.from_config(config, split)
        mode = "direct" if sp.reader.agg_direct_mode in ("direct", "direct_arrow") else "legacy"
    cols = plan.raw_columns() if plan is not None else tz.columns()
    refs: list[RowGroupRef] = plan_row_groups(list(paths), 0, 1, "row_group")[:max_tables + warmup]
    if not refs:
        raise ValueError("no row groups in the inputs")
    bs = int(batch_size or config.training.batch_size)
    cuda = device is not None and device.type == "cuda"
    t = {k: 0.0 for k in ("read", "expand", "tensorize", "pin", "h2d")}
    rows_total = 0
    batches = 0
    for i, ref in enumerate(refs):
        timed = i >= warmup
        mark = time.perf_counter()
        f = pq.ParquetFile(ref.path)
        present = [c for c in cols if c in f.schema_arrow.names]
        table = f.read(columns=present) if ref.index < 0 else f.read_row_group(ref.index, columns=present)
        now = time.perf_counter()
        read_s, mark = now - mark, now
        parts = []   # (candidate table, requests or None) per batch
        if mode == "legacy":
            from ..data.agg import AggIndex

            flat = AggIndex(table, plan).flat_table()
            parts = [(flat.slice(k, bs), None) for k in range(0, flat.num_rows, bs)]
        elif mode == "direct":
            from ..data.agg_direct import _Sources, iter_groups, pack_tables, packs

            sources = _Sources()
            for _k, pack in packs(iter_groups([table], plan, tz, sources), bs):
                cand, req, ri = pack_tables(pack, sources)
                parts.append((cand, (req, ri)))
        else:
            parts = [(table.slice(k, bs), None) for k in range(0, table.num_rows, bs)]
        now = time.perf_counter()
        expand_s, mark = now - mark, now
        packed = [tz(cand, requests=req) for cand, req in parts]
        now = time.perf_counter()
        tens_s, mark = now - mark, now
        pin_s = h2d_s = 0.0
        if cuda:
            pinned = [b.pin_memory() if hasattr(b, "pin_memory") else b for b in packed]
            now = time.perf_counter()
            pin_s, mark = now - mark, now
            for b in pinned:
                b.to(device, non_blocking=True)
            torch.cuda.synchronize(device)
            now = time.perf_counter()
            h2d_s, mark = now - mark, now
        if timed:
            t["read"] += read_s
            t["expand"] += expand_s
            t["tensorize"] += tens_s
            t["pin"] += pin_s
            t["h2d"] += h2d_s
            rows_total += sum(b.rows for b in packed)
            batches += len(packed)
    if not rows_total:
        raise ValueError("no timed rows: raise max_tables or lower warmup")
    total = sum(t.values())
    stages = {k: {"seconds": round(v, 6), "share": round(v / total, 4) if total else 0.0,
                  "rows_per_s": round(rows_total / v, 1) if v > 0 else None}
              for k, v in t.items() if v > 0 or k in ("read", "tensorize")}
    worst = max(stages, key=lambda k: stages[k]["seconds"])
    return {"mode": mode, "tables": len(refs) - warmup, "batches": batches, "rows": rows_total,
            "batch_size": bs, "seconds": round(total, 6), "rows_per_s": round(rows_total / total, 1),
            "stages": stages, "bottleneck": worst}
