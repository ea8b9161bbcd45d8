"""One training step of a benchmark workload, for kernel launch lists and
captures of single kernels.

    python -m mdl_b200.benchmark.step [--config N] [--scale S] [--batch B] [--steps K]

Builds the workload (``--scale`` < 1 shrinks the embedding vocabularies, e.g.
for a profiler capture that must stay small), runs warm-up steps, prints the
device time per step (CUDA events), then runs ``--steps`` steps between
``cudaProfilerStart`` / ``cudaProfilerStop`` (capture with the profiler's
"profile from start: off" setting).
"""

from __future__ import annotations

import argparse

import torch

from ..config import app_config_from_mapping
from ..data.baseline_configs import baseline_config, scaled_config
from ..data.synthetic import BatchPool, SyntheticGenerator
from ..models.factory import build_model
from ..train.trainer import Trainer


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--batch", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=2)
    args = ap.parse_args(argv)
    mapping, spec = (scaled_config(args.config, args.scale, batch=args.batch) if args.scale != 1.0
                     else baseline_config(args.config, batch=args.batch))
    cfg = app_config_from_mapping(mapping)
    dev = torch.device("cuda", 0)
    model = build_model(cfg, device=dev, base_seed=1)
    tr = Trainer(cfg, model, device=dev)
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    batches = [b.to(dev) for b in BatchPool(gen, args.batch, 3).batches]
    for i in range(4):
        tr.train_step(batches[i % 3])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(5):
        tr.train_step(batches[i % 3])
    e1.record()
    torch.cuda.synchronize()
    print(f"device time per step {e0.elapsed_time(e1) / 5:.3f} ms", flush=True)
    torch.cuda.cudart().cudaProfilerStart()
    for i in range(args.steps):
        tr.train_step(batches[i % 3])
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
