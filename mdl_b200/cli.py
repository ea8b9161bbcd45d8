"""Command line: ``python -m mdl_b200 <command> --config CONFIG.yaml ...``.

Commands (reference CLI ``src/main.py:1232-1430``): ``validate-config``,
``plan-shards``, ``profile``, ``fit-vocab``, ``check-checkpoint-store``,
``train``, ``benchmark``, ``evaluate``, ``predict``, plus
``make-synthetic-parquet`` (mock input files of a benchmark workload).

``--set section.key=value`` overrides any config value (YAML-parsed value).
With ``--nproc-per-node N`` (N > 1) ``train`` / ``benchmark`` / ``evaluate``
re-launch themselves under ``torch.distributed.run`` (one process per GPU,
rendezvous on 127.0.0.1). Training data comes from ``data.train.inputs``
(flat Parquet) or, with ``--synthetic`` or no inputs, from the seeded synthetic
generator in the shapes of the config.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import yaml


# ------------------------------------------------------------------ config
def _set_path(mapping: dict, dotted: str, value) -> None:
    keys = dotted.split(".")
    cur = mapping
    for k in keys[:-1]:
        cur = cur.setdefault(k, {})
    cur[keys[-1]] = value


def load_cli_config(args):
    from .config import app_config_from_mapping, load_config_mapping
    from .data.baseline_configs import baseline_config

    if getattr(args, "benchmark_config", None):
        mapping, _ = baseline_config(int(args.benchmark_config))
    else:
        mapping = load_config_mapping(args.config)
    for item in getattr(args, "set", None) or []:
        key, _, raw = item.partition("=")
        _set_path(mapping, key.strip(), yaml.safe_load(raw))
    return app_config_from_mapping(mapping)


def _add_config(p, required=True):
    g = p.add_mutually_exclusive_group(required=required)
    g.add_argument("--config", help="YAML config")
    g.add_argument("--benchmark-config", type=int, help="one of the benchmark workloads (1-5)")
    p.add_argument("--set", action="append", default=[], metavar="KEY=VALUE", help="config override")


# ------------------------------------------------------------------ runtime
def _launched_world() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def _relaunch(args, argv) -> int | None:
    n = getattr(args, "nproc_per_node", None) or 1
    if n <= 1 or "LOCAL_RANK" in os.environ:
        return None
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={args.master_port}", "-m", "mdl_b200", *argv]
    return subprocess.call(cmd)


def _setup_runtime(config):
    import torch

    from .parallel.runtime import set_local_cpu_affinity, setup_distributed

    rank, world, local = _launched_world()
    use_cuda = torch.cuda.is_available() and config.runtime.device != "cpu"
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    if local_world > 1:
        set_local_cpu_affinity(local, local_world)
    global _RUNTIME
    _RUNTIME = setup_distributed(device, timeout_s=600.0, local_world=local_world)
    return rank, world, device


_RUNTIME = None


def _resolve_scenarios(cfg, rank, world):
    from .data.scenarios import resolve_auto_scenarios_distributed

    return resolve_auto_scenarios_distributed(cfg, rank, world)


def load_external_adapter(dotted: str | None):
    """``package.module:function`` or ``package.module.function`` (reference
    ``_load_external_train_adapter`` ``src/train.py:1500-1520``)."""

    import importlib

    if not dotted:
        raise ValueError("external parameter-server training needs training.sparse_parameter_server_adapter")
    module, sep, attr = dotted.partition(":")
    if not sep:
        module, _, attr = dotted.rpartition(".")
    if not module or not attr:
        raise ValueError("sparse_parameter_server_adapter must be 'package.module:function' or 'package.module.function'")
    fn = getattr(importlib.import_module(module), attr)
    if not callable(fn):
        raise TypeError(f"{dotted} is not callable")
    return fn


def _build(config, rank, world, device, seed=1234):
    import torch
    import torch.distributed as dist

    from .models.factory import build_model
    from .train.trainer import Trainer

    torch.manual_seed(seed)
    pg = dist.group.WORLD if world > 1 else None
    vocab_sizes = None
    model = build_model(config, device=device, rank=rank, world=world, process_group=pg, vocab_sizes=vocab_sizes,
                        base_seed=seed)
    trainer = Trainer(config, model, device=device, rank=rank, world=world, process_group=pg)
    return model, trainer


def _batches(config, model, rank, world, *, split="train", synthetic=False, batch=None, loop=True):
    from .data.parquet import ParquetBatchIterator, Tensorizer, discover_parquet_inputs
    from .data.remote_io import RemoteIoPolicy
    from .data.synthetic import SyntheticGenerator, synthetic_spec_from_config

    rows = batch or config.training.batch_size
    sp = getattr(config.data, split) or config.data.train
    if not synthetic and sp.inputs:
        paths = discover_parquet_inputs(sp.inputs)
        r = sp.reader
        if r.host_prepare_prefetch > 0:
            # tensorisation in a spawned child, batches handed over in shared memory
            from .config.schema import thaw
            from .data.prepare_process import ProcessBatchIterator, parquet_batches

            args = (thaw(config), model.encoder.batch_plan, paths, rows, rank, world, split,
                    loop and split == "train", r.shuffle_buffer_rows, r.shuffle_seed, list(model.encoder.seq_plans))
            return ProcessBatchIterator(parquet_batches, args, depth=r.host_prepare_prefetch, pin=r.pin_memory,
                                        startup_timeout_s=r.host_prepare_startup_timeout_sec,
                                        idle_timeout_s=r.host_prepare_idle_timeout_sec)
        tz = Tensorizer(config, model.encoder.batch_plan, split=split, seq_names=list(model.encoder.seq_plans))
        adapter = None
        if sp.format in ("adapter_parquet", "agg_parquet"):
            from .data.agg import AggAdapter, AggPlan

            adapter = AggAdapter(AggPlan.from_config(config, split))
        return ParquetBatchIterator(paths, tz, rows, rank=rank, adapter=adapter,
                                    world=world, shard_unit=r.shard_unit, shuffle_rows=r.shuffle_buffer_rows,
                                    seed=r.shuffle_seed, prefetch=r.prefetch_batches, loop=loop and split == "train",
                                    pin=r.pin_memory, io_policy=RemoteIoPolicy.from_reader(r),
                                    length_buckets=[(b.max_length, b.batch_size) for b in r.length_buckets],
                                    length_bucket_metric=r.length_bucket_metric, overlap=r.overlap_host_prepare,
                                    agg_direct_mode=r.agg_direct_mode)
    seqs = [s for s in config.sequences if s.name in getattr(model.encoder, "seq_plans", {})]
    gen = SyntheticGenerator(model.encoder.batch_plan,
                             synthetic_spec_from_config(config, model.encoder.batch_plan, sequences=seqs), rank=rank)

    def forever():
        while True:
            yield gen.batch(rows)

    return forever()


# ------------------------------------------------------------------ commands
def cmd_validate(args) -> int:
    from .ops.preflight import attention_preflight

    cfg = load_cli_config(args)
    res = cfg.resolved.tokenization
    print(json.dumps({"valid": True, "model": cfg.model.name, "features": len(cfg.features),
                      "attention": attention_preflight(cfg)["paths"],
                      "feature_token_inputs": len(res.feature_token_inputs),
                      "feature_tokens": res.feature_token_count, "scenario_tokens": len(res.scenario_token_specs),
                      "task_tokens": len(res.task_token_specs), "tasks": list(cfg.task_names)}))
    return 0


def cmd_plan_shards(args) -> int:
    from .models.features import FeatureEncoder
    import torch

    cfg = load_cli_config(args)
    enc = FeatureEncoder.__new__(FeatureEncoder)  # plan only: no tables are allocated
    from .parallel.sharding import EmbeddingTableSpec, plan_embedding_shards
    from .models.features import categorical_size, table_name_of

    by_name = {f.name: f for f in cfg.features}
    tables = {}
    for f in cfg.features:
        if f.kind != "categorical":
            continue
        t = table_name_of(cfg, f.name)
        owner = by_name.get(t, f)
        tables[t] = (categorical_size(owner), int(owner.embedding_dim or cfg.model.embedding_dim))
    specs = [EmbeddingTableSpec(n, r, d) for n, (r, d) in sorted(tables.items())]
    plan = plan_embedding_shards(specs, world_size=args.world, strategy=cfg.training.embedding_sharding.strategy,
                                 table_wise_max_rows=cfg.training.embedding_sharding.table_wise_max_rows)
    load = [0] * args.world
    for s in specs:
        sp = plan.tables[s.name]
        for r in range(args.world):
            load[r] += sp.local_rows(s.num_embeddings, r) * s.embedding_dim * 4
    print(json.dumps({"world": args.world, "fingerprint": plan.fingerprint,
                      "row_wise": sum(1 for s in plan.tables.values() if s.strategy == "row_wise"),
                      "table_wise": sum(1 for s in plan.tables.values() if s.strategy == "table_wise"),
                      "bytes_per_rank": load}))
    del enc, torch
    return 0


def cmd_profile(args) -> int:
    import numpy as np

    cfg = load_cli_config(args)
    rank, world, device = 0, 1, "cpu"
    from .models.factory import build_model

    model = build_model(cfg, device="cpu", base_seed=0)
    it = _batches(cfg, model, rank, world, split=args.split, synthetic=args.synthetic, loop=False)
    stats = {"batches": 0, "rows": 0, "ids": 0}
    for i, b in enumerate(it):
        if i >= args.max_batches:
            break
        stats["batches"] += 1
        stats["rows"] += b.rows
        stats["ids"] += int(b.ids.numel())
        if b.labels is not None:
            stats.setdefault("label_sum", np.zeros(b.labels.shape[1]))
            stats["label_sum"] += b.labels.sum(0).numpy()
    if "label_sum" in stats:
        stats["label_rate"] = (stats.pop("label_sum") / max(1, stats["rows"])).tolist()
    _close(it)
    stats["ids_per_row"] = stats["ids"] / max(1, stats["rows"])
    print(json.dumps(stats))
    return 0


def cmd_fit_vocab(args) -> int:
    from .data.parquet import discover_parquet_inputs, fit_vocabs

    cfg = load_cli_config(args)
    out = fit_vocabs(cfg, discover_parquet_inputs(args.inputs or cfg.data.train.inputs), args.out)
    print(json.dumps(out))
    return 0


def cmd_audit_cardinality(args) -> int:
    from .data.audit import audit_cardinality
    from .data.parquet import discover_parquet_inputs

    cfg = load_cli_config(args)
    sp = getattr(cfg.data, args.split) or cfg.data.train
    out = audit_cardinality(cfg, discover_parquet_inputs(args.inputs or sp.inputs), max_rows=args.max_rows)
    print(json.dumps(out))
    return 0 if out["passed"] or not args.strict else 3


def cmd_profile_data(args) -> int:
    from .data.parquet import discover_parquet_inputs
    from .data.profile import profile_parquet

    cfg = load_cli_config(args)
    sp = getattr(cfg.data, args.split) or cfg.data.train
    out = profile_parquet(cfg, discover_parquet_inputs(args.inputs or sp.inputs), max_rows=args.max_rows)
    text = json.dumps(out, indent=1)
    if args.out:
        with open(args.out, "w", encoding="utf-8") as fh:
            fh.write(text)
    print(json.dumps({"rows": out["rows"], "features": len(out["features"]), "out": args.out}))
    return 0


def cmd_recommend(args) -> int:
    from .data.profile import recommend_encodings, recommend_shapes

    def load(path):
        with open(path, encoding="utf-8") as fh:
            return json.load(fh)

    if args.command == "recommend-shapes":
        out = recommend_shapes(load(args.small), load(args.large), horizon_rows=args.horizon_rows, load=args.load,
                               min_dim=args.min_dim, max_dim=args.max_dim)
    else:
        out = recommend_encodings(load(args.profile), bits=args.bits)
    print(json.dumps(out))
    return 0


def cmd_tune_batch_size(args) -> int:
    import dataclasses

    import torch

    from .benchmark.tools import tune_batch_size

    cfg0 = load_cli_config(args)
    rank, world, device = _setup_runtime(cfg0)
    if world != 1:
        raise SystemExit("tune-batch-size runs on one device")

    def build(b):
        cfg = dataclasses.replace(cfg0, training=dataclasses.replace(cfg0.training, batch_size=b))
        model, trainer = _build(cfg, 0, 1, device)
        return cfg, model, trainer, iter(_batches(cfg, model, 0, 1, synthetic=True))

    out = tune_batch_size(build, args.batch_sizes, steps=args.steps, warmup=args.warmup, device=device,
                          memory_fraction=args.memory_fraction)
    print(json.dumps(out))
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    return 0


def cmd_summarize_benchmarks(args) -> int:
    from .benchmark.tools import load_reports, markdown, summarize_benchmarks

    summary = summarize_benchmarks(load_reports(args.files))
    print(markdown(summary) if args.markdown else json.dumps(summary))
    return 0


def cmd_check_store(args) -> int:
    from .checkpoint import latest_committed_checkpoint, open_checkpoint_store

    store = open_checkpoint_store(args.checkpoint_dir)
    payload = os.urandom(args.probe_mib * 2 ** 20)
    t0 = time.time()
    store.write_bytes(payload, "_probe")
    ok = store.read_bytes("_probe") == payload
    store.remove_tree("_probe")
    latest = latest_committed_checkpoint(store)
    print(json.dumps({"store": store.root_uri, "round_trip_ok": ok, "seconds": round(time.time() - t0, 3),
                      "resume_from": None if latest is None else latest.directory}))
    return 0 if ok else 1


def cmd_train(args, argv) -> int:
    rc = _relaunch(args, argv)
    if rc is not None:
        return rc
    import torch

    from .checkpoint import load_training_checkpoint, make_uploader, open_checkpoint_store, save_training_checkpoint
    from .train.watchdog import StepWatchdog, abort_on_cuda_oom

    cfg = load_cli_config(args)
    if cfg.training.sparse_update_mode == "external_parameter_server":
        # the whole run is delegated to the configured adapter (reference src/train.py:6539-6542)
        result = load_external_adapter(cfg.training.sparse_parameter_server_adapter)(config=cfg,
                                                                                      max_steps=args.max_steps)
        print(json.dumps({"done": True, "external": True, "result": repr(result)}), flush=True)
        return 0
    from .ops.preflight import attention_preflight

    attention_preflight(cfg)  # before the runtime and any data scan
    rank, world, device = _setup_runtime(cfg)
    cfg = _resolve_scenarios(cfg, rank, world)
    attention_preflight(cfg, device)
    model, trainer = _build(cfg, rank, world, device)
    if world > 1:
        from .parallel.runtime import validate_shard_metadata

        validate_shard_metadata(model.store)
    ck = cfg.training.checkpoint
    ck_dir = args.checkpoint_dir or (os.path.join(ck.dir, ck.run_name) if ck.dir and ck.run_name else ck.dir)
    run = open_checkpoint_store(ck_dir) if ck_dir else None
    save_every = args.save_every or ck.every_steps
    keep_last = ck.keep_last if args.keep_last is None else args.keep_last
    uploader = None
    start = 0
    if run is not None:
        state = load_training_checkpoint(cfg, trainer, run, args.resume or ck.resume or "auto")
        if state is not None:
            start = state.step
        uploader = make_uploader(cfg, trainer, run, keep_last=keep_last,
                                 local_ranks=int(os.environ.get("LOCAL_WORLD_SIZE", "1")))

    def save(step_no):
        save_training_checkpoint(cfg, trainer, run, step_no, keep_last=keep_last, uploader=uploader,
                                 chunk_bytes=ck.shard_chunk_bytes)
    source = _batches(cfg, model, rank, world, synthetic=args.synthetic)
    batches = iter(source)
    from .train.fixed_eval import FixedTestEval

    fixed = FixedTestEval(cfg, trainer, rank=rank, world=world)
    dog = StepWatchdog(cfg.training.step_watchdog_sec if args.watchdog_sec is None else args.watchdog_sec).start()
    t0 = time.time()
    last = None
    step = start
    # several ranks on finite data: every step votes on the batch supply (train / replay / retry / stop)
    from .train.supply import BATCH_NOT_READY, BudgetedIterator, start_supply_count, supply_verdict, zero_weight

    voting = world > 1 and not args.synthetic
    if voting:
        batches = BudgetedIterator(batches)
    control = _RUNTIME.control_group if _RUNTIME is not None else None
    last_batch = None
    from .train.train_log import TrainLog, environment, environment_line

    tlog = TrainLog(cfg.task_names, world=world, micro_batches=cfg.training.gradient_accumulation_steps,
                    checkpoint_every=save_every if run is not None else 0)
    if rank == 0:
        print(environment_line(environment(cfg, world=world, device=device)), flush=True)
    try:
        while step < args.max_steps:
            t_wait = time.perf_counter()
            starved = False
            if voting:
                try:
                    batch = batches.next_within(args.batch_budget_sec)
                    exhausted = False
                except StopIteration:
                    batch, exhausted = BATCH_NOT_READY, True
                has = batch is not BATCH_NOT_READY
                active, done = start_supply_count(has, exhausted, world, control).wait()
                verdict = supply_verdict(has, active, done, world)
                if verdict == "stop":
                    break
                if verdict == "retry":
                    dog.beat("batch_retry", step)
                    continue
                if verdict == "replay":
                    if last_batch is None:
                        raise RuntimeError(f"rank {rank} has no training data while its peers train")
                    batch = zero_weight(last_batch)
                    starved = True
                last_batch = batch
            else:
                batch = next(batches)
            wait_s = time.perf_counter() - t_wait
            if device.type == "cuda":
                batch = batch.to(device, non_blocking=True)
            res = abort_on_cuda_oom(trainer.train_step, batch)
            step = trainer.step_index
            schedule = getattr(batches, "schedule_next", None)
            if schedule is not None:  # same-thread prepare while the device runs the step
                schedule()
            dog.beat("step", step)
            if rank == 0:
                tlog.step(res, batch, wait_s, starved)
            if step % args.log_every == 0 and rank == 0:
                last = float(res.loss)
                for line in tlog.lines(step, last):
                    print(line, flush=True)
                print(json.dumps({"step": step, "loss": last, "elapsed_s": round(time.time() - t0, 2)}), flush=True)
            if fixed.due(step):
                dog.beat("fixed_test_eval", step)
                ev = fixed.run(model)
                if rank == 0:
                    print(json.dumps({"step": step, "fixed_test_eval": ev}), flush=True)
            if run is not None and save_every and step % save_every == 0:
                dog.beat("checkpoint", step)
                save(step)
    finally:
        dog.stop()
        if voting:
            batches.close()
        _close(source)
    if run is not None:
        if ck.save_on_exit and (not save_every or step % save_every != 0):
            save(step)
        if uploader is not None:
            uploader.close()  # publishes (and on rank 0 commits) every staged step first
            for failed, why in uploader.failed_steps:
                print(json.dumps({"rank": rank, "checkpoint_failed": failed, "error": why}), flush=True)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    if rank == 0:
        print(json.dumps({"done": True, "steps": step, "seconds": round(time.time() - t0, 2)}), flush=True)
    return 0


def cmd_benchmark(args, argv) -> int:
    rc = _relaunch(args, argv)
    if rc is not None:
        return rc
    cfg = load_cli_config(args)
    rank, world, device = _setup_runtime(cfg)
    cfg = _resolve_scenarios(cfg, rank, world)
    model, trainer = _build(cfg, rank, world, device)
    from .benchmark.modes import run as run_mode

    synthetic = args.mode in ("compute", "embedding")
    it = _batches(cfg, model, rank, world, synthetic=synthetic)
    batches = iter(it)
    res = run_mode(args.mode, cfg, model, trainer, batches, rank=rank, world=world, device=device,
                   steps=args.steps, warmup=args.warmup, min_util=args.min_util)
    if args.profile_steps > 0 or args.comm_stats:
        extra = next(batches)
        dev_batch = extra.to(device) if device.type == "cuda" else extra
        if args.comm_stats:
            from .ops.embedding_stats import communication_stats

            stats = communication_stats(model.store, model.encoder.plan, dev_batch.ids, dev_batch.offsets,
                                        dev_batch.rows, collective=world > 1, group=model.store.process_group)
            res["embedding_comm"] = {k: v.as_dict() for k, v in sorted(stats.items())}
            res["embedding_comm_bytes_per_step"] = sum(v.total_communication_bytes for v in stats.values())
        if args.profile_steps > 0:
            from .benchmark.modes import dense_gemm_flops_per_row
            from .benchmark.profile_summary import profile_steps

            flops = dense_gemm_flops_per_row(model) * cfg.training.batch_size
            res["profile"] = profile_steps(lambda: trainer.train_step(dev_batch), args.profile_steps,
                                           device=device, gemm_flops_per_step=flops)
    _close(it)
    if rank == 0:
        print(json.dumps(res), flush=True)
    return 3 if "util_gate" in res else 0


def _close(it) -> None:
    close = getattr(it, "close", None)
    if close is not None:
        close()


def _eval_setup(args, argv):
    from .checkpoint import load_model_checkpoint, open_checkpoint_store
    from .checkpoint.training import MODEL_SUBDIR, resolve_resume_checkpoint

    cfg = load_cli_config(args)
    rank, world, device = _setup_runtime(cfg)
    cfg = _resolve_scenarios(cfg, rank, world)
    model, trainer = _build(cfg, rank, world, device)
    if args.checkpoint:
        store = open_checkpoint_store(args.checkpoint)
        if store.exists("manifest.json"):
            load_model_checkpoint(cfg, trainer, store)
        else:
            ck = resolve_resume_checkpoint(store, "latest")
            if ck is None:
                raise FileNotFoundError(f"no committed checkpoint under {args.checkpoint}")
            load_model_checkpoint(cfg, trainer, store.child(ck.directory, MODEL_SUBDIR))
    split = "test" if cfg.data.test is not None and cfg.data.test.inputs else "train"
    it = _batches(cfg, model, rank, world, split=split, synthetic=args.synthetic, loop=False)

    def limited():
        try:
            for i, b in enumerate(it):
                if i >= args.max_batches:
                    return
                yield b
        finally:
            _close(it)

    return cfg, rank, trainer, limited()


def cmd_evaluate(args, argv) -> int:
    rc = _relaunch(args, argv)
    if rc is not None:
        return rc
    from .train.evaluate import evaluate

    cfg, rank, trainer, batches = _eval_setup(args, argv)
    res = evaluate(trainer, batches, bins=args.auc_bins, group_metric=args.group_metric)
    if rank == 0:
        print(json.dumps(res, default=str), flush=True)
    return 0


def cmd_predict(args, argv) -> int:
    from .train.evaluate import predict

    cfg, rank, trainer, batches = _eval_setup(args, argv)
    probs = predict(trainer, batches, args.output if rank == 0 else None)
    if rank == 0:
        print(json.dumps({"rows": int(probs.shape[0]), "output": args.output}), flush=True)
    return 0


def cmd_make_synthetic(args) -> int:
    from .config import app_config_from_mapping
    from .data.baseline_configs import baseline_config, scaled_config
    from .data.parquet import write_synthetic_parquet
    from .data.synthetic import SyntheticGenerator
    from .models.factory import build_model

    mapping, spec = (scaled_config(args.benchmark, args.scale) if args.scale != 1.0
                     else baseline_config(args.benchmark))
    mapping["runtime"]["device"] = "cpu"
    cfg = app_config_from_mapping(mapping)
    model = build_model(cfg, device="cpu", base_seed=0)
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    os.makedirs(args.out, exist_ok=True)
    for i in range(args.files):
        write_synthetic_parquet(os.path.join(args.out, f"part-{i:05d}.parquet"), gen.batch(args.rows),
                                model.encoder.batch_plan, cfg)
    print(json.dumps({"files": args.files, "rows_per_file": args.rows, "out": args.out}))
    return 0


def cmd_build_config(args) -> int:
    """Config YAMLs of the model families from a field contract (``data/config_builder.py``)."""

    import yaml

    from .config.loader import app_config_from_mapping
    from .config.validate import validate_app_config
    from .data.config_builder import FAMILIES, FieldContract, build_config, memory_summary, render, size_features
    from .data.profile import profile_columns

    with open(args.contract, encoding="utf-8") as fh:
        contract = FieldContract.from_mapping(yaml.safe_load(fh) or {})

    def load(path):
        if not path:
            return None
        with open(path, encoding="utf-8") as fh:
            return json.load(fh)

    profile, shapes = load(args.profile), load(args.shapes)
    if args.profile_inputs:
        from .data.parquet import discover_parquet_inputs

        cols = list(dict.fromkeys([*contract.context_features, *contract.item_features,
                                   *(c for u in contract.ups.values() for c in u["fields"])]))
        cols = [c for c in cols if c not in contract.dense_features]
        profile = profile_columns(discover_parquet_inputs(args.profile_inputs), {c: c for c in cols},
                                  max_rows=args.max_rows)
    if profile is None and shapes is None and not args.estimate_from_names:
        print(json.dumps({"error": "no sizing source: give --profile, --shapes or --profile-inputs, or "
                                   "--estimate-from-names"}), file=sys.stderr)
        return 2
    sizes = size_features(contract, profile=profile, shapes=shapes, load=args.load, growth=args.growth,
                          max_dim=args.max_dim)
    families = list(FAMILIES) if args.family == "all" else [args.family]
    os.makedirs(args.out_dir, exist_ok=True)
    written = []
    for fam in families:
        variants = [False] + ([True] if args.fine and fam.startswith("mdl_") else [])
        for fine in variants:
            m = build_config(contract, fam, sizes=sizes, fine=fine, batch_size=args.batch_size,
                             token_dim=args.token_dim, layers=args.layers, inputs=args.inputs)
            validate_app_config(app_config_from_mapping(m))
            summary = memory_summary(m, world_size=args.world_size, budget_gb=args.budget_gb)
            path = os.path.join(args.out_dir, f"{fam}{'_fine' if fine else ''}.yaml")
            with open(path, "w", encoding="utf-8") as fh:
                fh.write(render(m, summary, sizes))
            written.append({"path": path, **summary})
    print(json.dumps({"configs": written}))
    return 0


def cmd_data_stages(args) -> int:
    """Host-side stage costs of the input pipeline (``benchmark/data_stages.py``)."""

    import torch

    from .benchmark.data_stages import stage_costs
    from .data.parquet import discover_parquet_inputs

    cfg = load_cli_config(args)
    device = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    model, _trainer = _build(cfg, 0, 1, torch.device("cpu"))
    sp = getattr(cfg.data, args.split) or cfg.data.train
    paths = discover_parquet_inputs(args.inputs or sp.inputs)
    res = stage_costs(cfg, paths, model.encoder.batch_plan, list(getattr(model.encoder, "seq_plans", {})),
                      max_tables=args.max_tables, warmup=args.warmup, batch_size=args.batch_size, device=device,
                      split=args.split)
    print(json.dumps(res), flush=True)
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m mdl_b200", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="command", required=True)
    p = sub.add_parser("validate-config")
    _add_config(p)
    p = sub.add_parser("plan-shards")
    _add_config(p)
    p.add_argument("--world", type=int, default=8)
    p = sub.add_parser("profile")
    _add_config(p)
    p.add_argument("--split", choices=["train", "test"], default="train")
    p.add_argument("--max-batches", type=int, default=10)
    p.add_argument("--synthetic", action="store_true")
    p = sub.add_parser("fit-vocab")
    _add_config(p)
    p.add_argument("--inputs", nargs="*")
    p.add_argument("--out", required=True)
    p = sub.add_parser("audit-cardinality")
    _add_config(p)
    p.add_argument("--split", choices=["train", "test"], default="train")
    p.add_argument("--inputs", nargs="*")
    p.add_argument("--max-rows", type=int, default=100_000)
    p.add_argument("--strict", action="store_true", help="exit 3 when a single-value feature holds lists")
    p = sub.add_parser("check-checkpoint-store")
    p.add_argument("--checkpoint-dir", required=True)
    p.add_argument("--probe-mib", type=int, default=8)
    p = sub.add_parser("profile-data", help="categorical profile of Parquet inputs (distinct values, collisions)")
    _add_config(p)
    p.add_argument("--split", choices=["train", "test"], default="train")
    p.add_argument("--inputs", nargs="*")
    p.add_argument("--max-rows", type=int, default=1_000_000)
    p.add_argument("--out")
    p = sub.add_parser("recommend-shapes", help="embedding table sizes / widths from two nested-prefix profiles")
    p.add_argument("--small", required=True)
    p.add_argument("--large", required=True)
    p.add_argument("--horizon-rows", type=int, required=True)
    p.add_argument("--load", type=float, default=0.5)
    p.add_argument("--min-dim", type=int, default=8)
    p.add_argument("--max-dim", type=int, default=128)
    p = sub.add_parser("recommend-encodings", help="per-feature categorical encoding from a profile")
    p.add_argument("--profile", required=True)
    p.add_argument("--bits", type=int, default=20)
    p = sub.add_parser("build-config", help="model config YAMLs from a field contract and a data profile")
    p.add_argument("--contract", required=True, help="field contract YAML (see mdl_b200/data/config_builder.py)")
    p.add_argument("--family", choices=["rankmixer", "mdl_rankmixer", "onetrans", "mdl_onetrans", "all"],
                   default="all")
    p.add_argument("--fine", action="store_true", help="also write the fine-scene siblings of the MDL families")
    p.add_argument("--profile", help="profile-data style JSON report of the raw files")
    p.add_argument("--shapes", help="recommend-shapes JSON")
    p.add_argument("--profile-inputs", nargs="*", help="profile the contract's columns in these Parquet files")
    p.add_argument("--max-rows", type=int, default=1_000_000)
    p.add_argument("--estimate-from-names", action="store_true",
                   help="size tables from column names where no profile covers them (marked in the output)")
    p.add_argument("--load", type=float, default=0.5)
    p.add_argument("--growth", type=float, default=4.0, help="distinct-value growth assumed beyond the profile")
    p.add_argument("--max-dim", type=int, default=64)
    p.add_argument("--batch-size", type=int, default=2048)
    p.add_argument("--token-dim", type=int, default=None)
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--inputs", nargs="*", help="data.train.inputs of the written configs")
    p.add_argument("--world-size", type=int, default=8)
    p.add_argument("--budget-gb", type=float, default=None, help="per-GPU embedding memory budget (GiB)")
    p.add_argument("--out-dir", required=True)
    p = sub.add_parser("data-stages", help="input pipeline stage costs: read, expand, tensorize, pin, H2D")
    _add_config(p)
    p.add_argument("--split", choices=["train", "test"], default="train")
    p.add_argument("--inputs", nargs="*")
    p.add_argument("--max-tables", type=int, default=8)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--batch-size", type=int, default=None)
    p = sub.add_parser("tune-batch-size", help="compute-mode throughput and peak memory per batch size")
    _add_config(p)
    p.add_argument("--batch-sizes", type=int, nargs="+", required=True)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--memory-fraction", type=float, default=0.9)
    p = sub.add_parser("summarize-benchmarks", help="group benchmark JSON lines; weak-scaling efficiency")
    p.add_argument("files", nargs="+")
    p.add_argument("--markdown", action="store_true")
    for name in ("train", "benchmark", "evaluate", "predict"):
        p = sub.add_parser(name)
        _add_config(p)
        p.add_argument("--nproc-per-node", type=int, default=1)
        p.add_argument("--master-port", type=int, default=29533)
        p.add_argument("--synthetic", action="store_true")
        if name == "train":
            p.add_argument("--max-steps", type=int, default=100)
            p.add_argument("--checkpoint-dir")
            p.add_argument("--resume", default=None)
            p.add_argument("--save-every", type=int, default=0)
            p.add_argument("--keep-last", type=int, default=None)
            p.add_argument("--log-every", type=int, default=10)
            p.add_argument("--watchdog-sec", type=float, default=None)
            p.add_argument("--batch-budget-sec", type=float, default=30.0,
                           help="several ranks: seconds to wait for a batch before voting 'not ready'")
        if name == "benchmark":
            p.add_argument("--steps", type=int, default=20)
            p.add_argument("--warmup", type=int, default=5)
            p.add_argument("--mode", choices=["compute", "end-to-end", "data", "embedding"], default="compute",
                           help="compute: device-resident synthetic batches; end-to-end: the input pipeline + "
                                "H2D + training; data: the input pipeline only; embedding: lookup + sparse update")
            p.add_argument("--min-util", type=float, default=None,
                           help="utilisation gate: report a failure (exit 3) below this mean GPU utilisation")
            p.add_argument("--profile-steps", type=int, default=0,
                           help="after the timed steps, profile this many compute steps (device time by kernel "
                                "class, top kernels, named ranges)")
            p.add_argument("--comm-stats", action="store_true",
                           help="add the embedding lookup's per-table communication statistics of one batch")
        if name in ("evaluate", "predict"):
            p.add_argument("--checkpoint")
            p.add_argument("--max-batches", type=int, default=10)
        if name == "evaluate":
            p.add_argument("--group-metric", choices=["qauc", "uauc"], default=None,
                           help="mean per-group AUC over the split's group_id column (one process)")
            p.add_argument("--auc-bins", type=int, default=4096)
        if name == "predict":
            p.add_argument("--output", required=True)
    p = sub.add_parser("make-synthetic-parquet")
    p.add_argument("--benchmark", type=int, default=1)
    p.add_argument("--scale", type=float, default=1.0)
    p.add_argument("--files", type=int, default=2)
    p.add_argument("--rows", type=int, default=1024)
    p.add_argument("--out", required=True)
    return ap


def main(argv=None) -> int:
    from .data.remote_io import RemoteIoStallError

    try:
        return _dispatch(argv)
    except RemoteIoStallError as error:  # a launcher may restart the job on this code
        print(json.dumps({"error": "remote_io_stall", "detail": str(error)}), file=sys.stderr, flush=True)
        return error.exit_code


def _dispatch(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    args = build_parser().parse_args(argv)
    cmd = args.command
    if cmd == "validate-config":
        return cmd_validate(args)
    if cmd == "plan-shards":
        return cmd_plan_shards(args)
    if cmd == "profile":
        return cmd_profile(args)
    if cmd == "fit-vocab":
        return cmd_fit_vocab(args)
    if cmd == "check-checkpoint-store":
        return cmd_check_store(args)
    if cmd == "audit-cardinality":
        return cmd_audit_cardinality(args)
    if cmd == "profile-data":
        return cmd_profile_data(args)
    if cmd in ("recommend-shapes", "recommend-encodings"):
        return cmd_recommend(args)
    if cmd == "data-stages":
        return cmd_data_stages(args)
    if cmd == "build-config":
        return cmd_build_config(args)
    if cmd == "tune-batch-size":
        return cmd_tune_batch_size(args)
    if cmd == "summarize-benchmarks":
        return cmd_summarize_benchmarks(args)
    if cmd == "train":
        return cmd_train(args, argv)
    if cmd == "benchmark":
        return cmd_benchmark(args, argv)
    if cmd == "evaluate":
        return cmd_evaluate(args, argv)
    if cmd == "predict":
        return cmd_predict(args, argv)
    if cmd == "make-synthetic-parquet":
        return cmd_make_synthetic(args)
    raise SystemExit(f"unknown command {cmd}")
