"""Per-phase device times of the training step (CUDA events, max over ranks).

    python -m mdl_b200.benchmark.phases [--config N] [--scale S]
    python -m torch.distributed.run --nproc-per-node W --master-addr 127.0.0.1 -m mdl_b200.benchmark.phases

Phases, each timed over 5 repetitions between barriers: the full step, forward +
backward, the dense update, the sparse update, and the embedding lookup forward
alone; then the device time of each phase inside full steps (events between the
forward, backward, dense update and sparse update). Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from ..config import app_config_from_mapping
from ..data.baseline_configs import baseline_config, scaled_config
from ..data.synthetic import BatchPool, SyntheticGenerator
from ..models.factory import build_model
from ..ops.embedding import fused_lookup
from ..train.trainer import Trainer


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--batch", type=int, default=2048)
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    mapping, spec = (scaled_config(args.config, args.scale, batch=args.batch) if args.scale != 1.0
                     else baseline_config(args.config, batch=args.batch))
    cfg = app_config_from_mapping(mapping)
    pg = dist.group.WORLD if world > 1 else None
    model = build_model(cfg, device=dev, rank=rank, world=world, process_group=pg, base_seed=1)
    tr = Trainer(cfg, model, device=dev, rank=rank, world=world, process_group=pg)
    gen = SyntheticGenerator(model.encoder.batch_plan, spec, rank=rank)
    batches = [b.to(dev) for b in BatchPool(gen, args.batch, 3).batches]
    for i in range(4):
        tr.train_step(batches[i % 3])
    torch.cuda.synchronize()
    res: dict[str, float] = {}

    def timed(name, fn, n=5):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        v = torch.tensor([e0.elapsed_time(e1) / n], device=dev)
        if world > 1:
            dist.all_reduce(v, op=dist.ReduceOp.MAX)
        res[name] = round(float(v), 4)

    timed("step_ms", lambda i: tr.train_step(batches[i % 3]))
    # the same steps with events between their phases (device time inside the step)
    tr.enable_phase_events(True)
    for i in range(5):
        tr.train_step(batches[i % 3])
    for name, ms in tr.phase_ms().items():
        v = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(v, op=dist.ReduceOp.MAX)
        res[f"in_step_{name}_ms"] = round(float(v), 4)
    tr.enable_phase_events(False)
    timed("forward_backward_ms", lambda i: tr.forward_backward(batches[i % 3]))
    timed("dense_update_ms", lambda i: tr.dense.step(lr=0.0))
    timed("sparse_update_ms", lambda i: tr.store.step(lr=0.0))
    anchor = torch.zeros(0, device=dev, requires_grad=True)
    timed("lookup_forward_ms", lambda i: fused_lookup(model.store, model.encoder.plan, batches[i % 3].ids,
                                                      batches[i % 3].offsets, batches[i % 3].dense,
                                                      batches[i % 3].rows, anchor))
    if rank == 0:
        print(json.dumps({"world": world, "config": args.config, **res}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
