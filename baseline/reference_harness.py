"""Reference arm of ``bench.py``: the unmodified reference trained on the same workload.

The reference (``wcrmu/MDL``) is installed, unmodified, under ``baseline/_ref`` (package
``src``). Everything on the timed path is the reference's own code: its config loader
(``src.config.load_app_config``), model factory run on the destination device
(``src.train._build_model_on_device`` -> ``src.model.build_model``), parameter
classification and DDP preparation (``_classify_model_parameters``,
``_prepare_forward_model``, incl. its CUDA-graph backbone prewarm), optimizers
(``_build_dense_optimizer`` RMSprop, ``src.optim.ShardedRowWiseAdagrad``), autocast
context and loss (``_autocast_context``, ``_loss_terms_from_batch``), and its batch
container / H2D helpers (``src.dataloader.FeatureBatch``, ``pin_feature_batch``,
``move_feature_batch``). The step body mirrors the reference hot loop
(``src/train.py:6996-7190``): zero_grad -> autocast forward + loss -> backward ->
optimizer steps.

The workload is a BASELINE config built by ``mdl_b200.data.baseline_configs`` with the
adjustments the reference needs: bag pooling ``mean`` (it has no ``sum``; same cost), its
production ``runtime.cuda_graph_backbone: true`` (RankMixer), and for OneTrans (config 4)
its only pyramid schedule, ``linear`` with ``final_s_tokens: 32`` (queried S tokens per
layer 448, 352, 256, 192, 128, 32 against 512, 256, 256, 128, 128, 64 for halving -- 5%
more query work; run our arm with ``--pyramid linear`` for the like-for-like pair).
Synthetic batches come from the same generator as our arm and are converted to the
reference's ``FeatureBatch`` (sequences as ``{"fields": {name: [B, L]}, "lengths": [B]}``
payloads with the valid events first, as its dataloader delivers them).
"""

from __future__ import annotations

import copy
import os
import sys
import tempfile

import torch
import torch.distributed as dist
import yaml

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def _import_reference():
    if not os.path.isdir(os.path.join(REF, "src")):
        raise RuntimeError("reference not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import src.config as rconfig  # noqa: F401
    import src.dataloader as rdata  # noqa: F401
    import src.train as rtrain  # noqa: F401
    from src import optim as roptim  # noqa: F401

    return rconfig, rdata, rtrain, roptim


def reference_mapping(mapping: dict, cuda_graphs: bool) -> dict:
    """Adapt a benchmark mapping to what the reference supports (see module docstring)."""

    m = copy.deepcopy(mapping)
    for f in m.get("features", []):
        if f.get("pooling") == "sum":
            f["pooling"] = "mean"
    model = m.get("model", {})
    if model.pop("pyramid_schedule", "linear") != "linear":
        model["final_s_tokens"] = 32
    model.pop("pyramid_halve_every", None)
    # the reference has one token per scene (workload 3 asks for 4; recorded in the result)
    model.pop("tokens_per_scenario", None)
    model.pop("sequence_head", None)
    m.setdefault("vocab_strategy", {"defaults": {}, "features": {}})
    m["runtime"]["cuda_graph_backbone"] = bool(cuda_graphs)
    m["runtime"]["distributed"] = "none"
    m["runtime"].pop("kernel_backend", None)
    m["training"].pop("comm", None)
    return m


def to_feature_batch(rdata, packed, plan, device=None, sequences=None):
    """Our PackedBatch -> the reference's FeatureBatch (features dict keyed by name).

    ``sequences``: ``{name: [field names]}`` of the raw sequences in the batch; ours are
    right-aligned (padding first), the reference's payloads carry the valid events first.
    """

    rows = packed.rows
    ids = packed.ids
    off = packed.offsets
    features = {}
    for fi, f in enumerate(plan.features):
        if f.table is None:
            features[f.name] = packed.dense[:, f.dense_col:f.dense_col + f.width]
            continue
        beg = int(off[fi * rows])
        end = int(off[(fi + 1) * rows])
        flat = ids[beg:end]
        if f.pooling == 0:
            features[f.name] = flat.clone()
        else:
            lengths = (off[fi * rows + 1:(fi + 1) * rows + 1] - off[fi * rows:(fi + 1) * rows]).clone()
            features[f.name] = {"values": flat.clone(), "lengths": lengths}
    for name, field_names in (sequences or {}).items():
        seq = packed.sequences[name]
        lengths = seq["lengths"].long()
        L = seq["ids"].shape[1] // rows
        ids = seq["ids"].view(len(field_names), rows, L)
        # left-align: event e of the valid suffix moves to position e
        pos = (torch.arange(L).view(1, L) + (L - lengths).view(rows, 1)).clamp(max=L - 1)
        keep = torch.arange(L).view(1, L) < lengths.view(rows, 1)
        fields = {fn: torch.where(keep, ids[k].gather(1, pos), torch.zeros_like(ids[k])) for k, fn in
                  enumerate(field_names)}
        features[name] = {"fields": fields, "lengths": lengths.clone()}
    batch = rdata.FeatureBatch(features=features, labels=packed.labels.clone(), label_mask=None,
                               scenario_id=packed.scenario_id.clone().long(), group_id=[])
    if device is not None:
        batch = rdata.move_feature_batch(batch, device)
    return batch


class ReferenceTrainer:
    """Builds the reference model + optimizers and runs its training step."""

    def __init__(self, mapping: dict, *, device: torch.device, rank: int, world: int, local: int,
                 cuda_graphs: bool = True) -> None:
        rconfig, rdata, rtrain, roptim = _import_reference()
        self.rdata, self.rtrain = rdata, rtrain
        ref_map = reference_mapping(mapping, cuda_graphs and device.type == "cuda")
        if device.type != "cuda":  # CPU runs (tests): fp32 and the reference's SDPA attention
            ref_map["runtime"].update({"device": "cpu", "precision": "fp32", "attention_backend": "sdpa"})
        with tempfile.NamedTemporaryFile("w", suffix=".yaml", delete=False) as fh:
            yaml.safe_dump(ref_map, fh)
            path = fh.name
        self.config = rconfig.load_app_config(path)
        os.unlink(path)
        self.device = device
        self.context = rtrain.DistributedContext(enabled=world > 1, rank=rank, local_rank=local, world_size=world,
                                                 device=device)
        base = rtrain._build_model_on_device(self.config, {}, device)
        groups = rtrain._classify_model_parameters(base)
        ignored = (*groups.sparse_sync, *groups.sharded_ddp_ignore)
        self.model = rtrain._prepare_forward_model(self.config, base, self.context, ignored)
        self.base = base
        t = self.config.training
        self.optimizers = []
        dense = list(groups.dense_optimizer)
        if dense:
            self.optimizers.append(rtrain._build_dense_optimizer(dense, self.config, device))
        sharded = list(groups.sharded_optimizer)
        if sharded:
            lr = t.lr_sparse or t.lr_dense
            self.optimizers.append(roptim.ShardedRowWiseAdagrad(
                sharded, lr=lr, lr_decay=t.adagrad_lr_decay, weight_decay=t.adagrad_weight_decay,
                initial_accumulator_value=t.adagrad_initial_accumulator_value, eps=t.adagrad_eps))
        replicated = list(groups.embedding_optimizer)
        # tables the reference replicates on every rank (src/train.py:6582-6630): its
        # rank-0 broadcast at start and its touched-row gradient synchronizer per step
        rtrain._synchronize_sparse_parameter_replicas(self.context, groups.sparse_sync)
        self.sparse_sync = rtrain._ReplicatedSparseGradientSynchronizer(self.context, groups.sparse_sync)
        if replicated:
            self.optimizers.append(torch.optim.Adagrad(
                replicated, lr=t.lr_sparse or t.lr_dense, lr_decay=t.adagrad_lr_decay,
                weight_decay=t.adagrad_weight_decay,
                initial_accumulator_value=t.adagrad_initial_accumulator_value, eps=t.adagrad_eps))

    def step(self, batch) -> torch.Tensor:
        rt = self.rtrain
        for opt in self.optimizers:
            opt.zero_grad(set_to_none=True)
        with rt._autocast_context(self.config, self.device):
            output = self.model(batch.features, batch.scenario_id)
            loss, _num, _den = rt._loss_terms_from_batch(
                output, batch, moe_loss_weight=self.config.model.sparse_moe_loss_weight,
                loss_reduction=self.config.training.loss_reduction, task_loss_weights=None, rank_active=True,
                active_rank_count=self.context.world_size)
        loss.backward()
        self.sparse_sync.synchronize(rank_active=True)
        for opt in self.optimizers:
            opt.step()
        return loss.detach()


def synthetic_plan(mapping: dict, spec):
    """A lookup plan of the workload's feature order, only to drive the shared
    synthetic generator (no tables are built on this path)."""

    from mdl_b200.ops.embedding import LookupFeature, LookupPlan, POOL_MEAN, POOL_NONE, POOL_SUM

    feats, col = [], 0
    for f in mapping["features"]:
        if f["kind"] == "dense":
            feats.append(LookupFeature(f["name"], None, width=f["dimension"], out_col=col, dense_col=0))
            col += f["dimension"]
        else:
            pool = {"none": POOL_NONE, "mean": POOL_MEAN, "sum": POOL_SUM}[f.get("pooling", "none")]
            feats.append(LookupFeature(f["name"], f["name"], pooling=pool, width=f["embedding_dim"], out_col=col))
            col += f["embedding_dim"]
    return LookupPlan(feats, out_width=col, dense_width=spec.dense_width)


def reference_batches(trainer: "ReferenceTrainer", mapping: dict, spec, batch: int, count: int, rank: int = 0,
                      device=None):
    """``count`` seeded synthetic batches of the workload as the reference's FeatureBatch."""

    from mdl_b200.data.synthetic import SyntheticGenerator

    plan = synthetic_plan(mapping, spec)
    gen = SyntheticGenerator(plan, spec, rank=rank)
    seqs = {s["name"]: [fl["name"] for fl in s["fields"]] for s in mapping.get("sequences", [])}
    return [to_feature_batch(trainer.rdata, gen.batch(batch), plan, device, seqs) for _ in range(count)]


def run(args, rank: int, world: int, local: int) -> dict:
    from mdl_b200.data.baseline_configs import baseline_config
    from mdl_b200.data.synthetic import BatchPool, SyntheticGenerator
    from mdl_b200.utils.clocks import ClockSampler

    device = torch.device("cuda", local)
    mapping, spec = baseline_config(args.config, batch=args.batch, **({"mdl": True} if args.mdl else {}))
    torch.manual_seed(1234)
    trainer = ReferenceTrainer(mapping, device=device, rank=rank, world=world, local=local,
                               cuda_graphs=not getattr(args, "ref_no_graphs", False))
    plan = synthetic_plan(mapping, spec)
    gen = SyntheticGenerator(plan, spec, rank=rank)
    pool = BatchPool(gen, args.batch, count=args.pool, pin=False)
    rd = trainer.rdata
    seqs = {s["name"]: [fl["name"] for fl in s["fields"]] for s in mapping.get("sequences", [])}
    dev_batches = [to_feature_batch(rd, b, plan, device, seqs) for b in pool.batches]
    host_batches = [rd.pin_feature_batch(to_feature_batch(rd, b, plan, None, seqs)) for b in pool.batches]
    torch.cuda.synchronize(device)

    for i in range(args.warmup):
        trainer.step(dev_batches[i % len(dev_batches)])
    torch.cuda.synchronize(device)

    props = torch.cuda.get_device_properties(device)
    sampler = ClockSampler(f"GPU-{props.uuid}" if getattr(props, "uuid", None) else local).start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        trainer.step(dev_batches[i % len(dev_batches)])
    end.record()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = _max(start.elapsed_time(end), world)

    loss_host = torch.zeros(args.steps, dtype=torch.float32, pin_memory=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(args.steps):
        batch = rd.move_feature_batch(host_batches[i % len(host_batches)], device, non_blocking=True)
        loss = trainer.step(batch)
        loss_host[i:i + 1].copy_(loss.reshape(1).float(), non_blocking=True)
    e2.record()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    ms_e2e = _max(s2.elapsed_time(e2), world)
    rows_total = args.batch * world * args.steps
    h2d = pool.batches[0].nbytes()
    return {
        "impl": "reference",
        "metric": "train samples/sec",
        "value": round(rows_total / (ms / 1000.0), 1),
        "unit": "samples/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (same generator and seeds as the ours arm); random-init weights",
        "config": {
            "model": f"{trainer.config.model.name} (BASELINE config {args.config}) on the unmodified reference; bag "
                     "pooling mean (no sum in the reference); cuda_graph_backbone="
                     + str(bool(trainer.config.runtime.cuda_graph_backbone))
                     + (f"; pyramid linear, final_s_tokens={trainer.config.model.final_s_tokens}"
                        if trainer.config.model.name == "onetrans" else "")
                     + ("; 1 scenario token per scene (the reference has no tokens_per_scenario; ours uses "
                        f"{mapping['model'].get('tokens_per_scenario', 1)})"
                        if trainer.config.model.name == "mdl_rankmixer" else ""),
            "global_batch": args.batch * world,
            "seq_len": (mapping.get("sequences") or [{}])[0].get("max_length"),
            "parallelism": f"ddp{world}+sharded-embeddings{world}",
            "l2": "inputs larger than L2 (same batches as the ours arm)",
        },
        "clocks": clocks,
        "e2e": {"value": round(rows_total / (ms_e2e / 1000.0), 1), "unit": "samples/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4},
        "gpu_launches": 0,
        "final_loss": float(loss_host[-1]),
    }


def _max(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def auc_parity_worker(rank: int, world: int, init_file: str, out_path: str, steps: int = 200,
                      batch: int = 256) -> None:
    """One gloo rank of the AUC parity run (BASELINE workload 1 on CPU).

    Every rank builds this framework's workload-1 model at ``world`` ranks and the
    reference's, both from identical starting weights (the dense weights and full
    embedding tables of a one-rank model built from the same seeds, each rank keeping
    the rows it owns), trains both for ``steps`` steps on its slice of the same union
    batches, scores its slice of the held-out batches, and rank 0 writes both AUCs
    and the losses to ``out_path`` (JSON)."""

    import json

    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import baseline_config
    from mdl_b200.data.synthetic import SyntheticGenerator
    from mdl_b200.metrics.auc import binary_auc
    from mdl_b200.models.factory import build_model
    from mdl_b200.train.trainer import Trainer

    torch.set_num_threads(max(1, (os.cpu_count() or 2) // max(1, world)))
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        mapping, spec = baseline_config(1)
        mapping["training"]["dense_optimizer"] = "rmsprop"  # the reference's only dense optimizer
        cfg = app_config_from_mapping(mapping)
        torch.manual_seed(0)
        full = build_model(cfg, device="cpu", base_seed=0)  # one-rank model: the starting weights
        init_dense = full.reference_state_dict()
        tables = {t.name: full.store.weight(t.name).clone() for t in full.store.layouts}
        torch.manual_seed(0)
        ours = build_model(cfg, device="cpu", rank=rank, world=world, process_group=dist.group.WORLD, base_seed=0)
        ours.load_reference_state_dict(init_dense)
        with torch.no_grad():
            for t in ours.store.layouts:
                gids = t.spec.global_ids(t.num_embeddings, rank)
                ours.store.weight(t.name).copy_(tables[t.name][gids])
        trainer = Trainer(cfg, ours, device=torch.device("cpu"), rank=rank, world=world, process_group=dist.group.WORLD)
        ref = ReferenceTrainer(mapping, device=torch.device("cpu"), rank=rank, world=world, local=rank,
                               cuda_graphs=False)
        ref.base.load_state_dict(init_dense, strict=False)
        with torch.no_grad():
            for name, emb in ref.base.encoder_bank.embeddings.items():
                spec_r = emb.shard_spec
                g = torch.arange(tables[name].shape[0])
                own = g[spec_r.owner(g) == rank]
                emb.weight[spec_r.local_row_ids(own)] = tables[name][own].to(emb.weight.dtype)
        plan = full.encoder.batch_plan
        nf = plan.num_src
        gen = SyntheticGenerator(plan, spec)
        lo, hi = rank * batch, (rank + 1) * batch
        losses_o, losses_r = [], []
        for _ in range(steps):
            union = gen.batch(batch * world)
            mine = union.slice_rows(lo, hi, nf)
            losses_o.append(float(trainer.train_step(mine).loss))
            losses_r.append(float(ref.step(to_feature_batch(ref.rdata, mine, plan))))
        ref.model.eval()
        so, sr, ys = [], [], []
        with torch.no_grad():
            for _ in range(8):
                union = gen.batch(batch * world)
                mine = union.slice_rows(lo, hi, nf)
                so.append(trainer.predict_logits(mine)[:, 0].float())
                fb = to_feature_batch(ref.rdata, mine, plan)
                sr.append(ref.model(fb.features, fb.scenario_id)["logits"][:, 0].float())
                ys.append(mine.labels[:, 0].float())
        local = torch.stack([torch.cat(so), torch.cat(sr), torch.cat(ys)])
        gathered = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(gathered, local)
        if rank == 0:
            allv = torch.cat(gathered, dim=1)
            result = {"auc_ours": binary_auc(allv[0], allv[2]), "auc_reference": binary_auc(allv[1], allv[2]),
                      "first_loss": [losses_o[0], losses_r[0]], "last_loss": [losses_o[-1], losses_r[-1]],
                      "world": world, "steps": steps}
            with open(out_path, "w") as fh:
                json.dump(result, fh)
        dist.barrier()
    finally:
        dist.destroy_process_group()
