"""Device times of the multi-rank embedding kernels on ONE GPU (emulated ranks).

    python -m mdl_b200.benchmark.multirank_emulated [--world 2] [--scale 0.05] [--batch 2048]

Lays ``world`` ranks of the workload-2 embedding store out on one GPU
(``parallel/emulate.py``), and times every phase of the owner-push lookup
(``emb_route``, ``emb_owner_fwd``, ``acc_to_bf16``) and of the owner-pull gradient
(``emb_owner_bwd``) for each rank's batch, plus the fused dense reduce-scatter /
optimizer / all-gather (``dense_sync``) over a ``--dense-params`` flat buffer. Peer
traffic is local HBM traffic here, so the times isolate the kernels' own work (the
NVLink share is measured by the multi-GPU phase tool); the small case is what a
single-GPU ncu capture of these kernels runs. Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json

import torch


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--scale", type=float, default=0.05, help="table rows relative to workload 2")
    ap.add_argument("--batch", type=int, default=2048)
    ap.add_argument("--fields", type=int, default=300)
    ap.add_argument("--dense-params", type=int, default=168_000_000)
    ap.add_argument("--iters", type=int, default=5)
    args = ap.parse_args(argv)

    from torch import nn

    from ..config import app_config_from_mapping
    from ..data.baseline_configs import scaled_config
    from ..data.synthetic import SyntheticGenerator
    from ..models.features import FeatureEncoder
    from ..ops.dense import DenseParams
    from ..ops.embedding import (_exchange, owner_collect, owner_pull_grad, owner_push, owner_route,
                                 owner_stage_grad)
    from ..parallel.emulate import EmulatedPeers

    dev = torch.device("cuda", 0)
    W, B = args.world, args.batch
    mapping, spec = scaled_config(2, args.scale, num_fields=args.fields, batch=B)
    cfg = app_config_from_mapping(mapping)
    peers = EmulatedPeers(W, dev, exchange_ids=B * args.fields * 6, exchange_rows=B)
    encs = [FeatureEncoder(cfg, device=dev, rank=r, world=W, slice_tokens=16, base_seed=1, peers=peers)
            for r in range(W)]
    plan = encs[0].plan
    batches = [SyntheticGenerator(encs[0].batch_plan, spec, rank=r).batch(B).to(dev) for r in range(W)]
    for e, b in zip(encs, batches):
        _exchange(e.store, e.plan, b.ids, B)
    grads = [torch.randn(B, plan.out_ld, device=dev).bfloat16() for _ in range(W)]

    def timed(fn) -> float:
        fn()
        torch.cuda.synchronize()
        s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        t.record()
        torch.cuda.synchronize()
        return s.elapsed_time(t) / args.iters

    res = {"world": W, "batch": B, "fields": args.fields, "scale": args.scale}
    res["route_ms"] = timed(lambda: [owner_route(e.store, e.plan, b.ids, b.offsets, b.dense, B)
                                     for e, b in zip(encs, batches)]) / W
    res["owner_fwd_ms"] = timed(lambda: [owner_push(e.store, e.plan, b.ids, b.offsets, B)
                                         for e, b in zip(encs, batches)]) / W
    res["collect_ms"] = timed(lambda: [owner_collect(e.store, e.plan, b.ids, B) for e, b in zip(encs, batches)]) / W
    res["stage_grad_ms"] = timed(lambda: [owner_stage_grad(e.store, e.plan, b.ids, g, B)
                                          for e, b, g in zip(encs, batches, grads)]) / W
    res["owner_bwd_ms"] = timed(lambda: [owner_pull_grad(e.store, e.plan, b.ids, b.offsets, B)
                                         for e, b in zip(encs, batches)]) / W
    n = args.dense_params // W
    dps = [DenseParams([("w", nn.Parameter(torch.zeros(n * W // 1, device="cpu")))], device=dev,
                       bf16_names={"w"}, world=W, rank=r, optimizer="rmsprop", lr=1e-4, comm="fused", peers=peers)
           for r in range(W)]
    res["dense_sync_ms"] = timed(lambda: [dp.update_buckets(1e-4) for dp in dps]) / W
    res["dense_params"] = dps[0].total
    from ..ops._ext import check_error_word

    check_error_word(dev)
    print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in res.items()}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
