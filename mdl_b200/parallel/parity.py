"""Distributed parity check: W sharded ranks == one rank on the union batch.

The reference's distributed tests assert that the sharded lookup plus sharded
row-wise Adagrad equals a single full-table run on the union of the rank batches
(``tests/test_sharded_embedding.py:49-132``). This module runs the same check for
this framework's whole training step (embeddings, dense model, loss reduction,
gradient exchange and both optimizers) on any backend:

* ``gloo`` on CPU ranks (the PyTorch definitions of every op), and
* ``nccl`` on GPU ranks (the sm_100a kernels, including the NVLink fused paths:
  peer-memory lookup, gradient push to owners, fused dense reduce + optimizer).

Every rank builds the same model with the same seeds, loads identical full
embedding tables into its own shards, trains on its slice of one union batch and
returns gradients and updated weights reassembled to full size; rank 0 also trains
a one-rank model on the whole union batch and compares.
"""

from __future__ import annotations

import datetime
import json
import os
from hashlib import sha256

import torch
import torch.distributed as dist

from ..config import app_config_from_mapping


def tiny_mapping(num_fields: int = 10, batch: int = 64, token_dim: int = 128, tokens: int = 4,
                 optimizer: str = "adam", distribution: str = "sharded",
                 sparse_optimizer: str = "rowwise_adagrad") -> tuple[dict, object]:
    """A small RankMixer workload with row-wise and table-wise tables and multi-hot bags."""

    from ..data.baseline_configs import scaled_config

    m, spec = scaled_config(2, 0.0002, num_fields=num_fields, batch=batch)
    # mix of big (row-wise sharded) and small (table-wise) tables
    for i, f in enumerate(m["features"]):
        if f["kind"] == "categorical":
            rows = 40 + 97 * i if i % 2 else 70000 + 13 * i
            f["encoding"]["max_id"] = rows
            spec.fields[f["name"]].vocab = rows
            f["embedding_dim"] = 32 if i % 3 else 16
    m["model"].update({"token_dim": token_dim, "hidden_dim": 2 * token_dim, "task_head_hidden_dim": 64,
                       "num_heads": 4})
    m["tokenization"]["num_feature_tokens"] = tokens
    m["training"].update({"dense_optimizer": optimizer, "lr_dense": 1e-3, "lr_sparse": 0.05, "lr_warmup_steps": 0,
                          "adagrad_initial_accumulator_value": 0.1, "embedding_distribution": distribution,
                          "sparse_optimizer": sparse_optimizer, "adagrad_lr_decay": 0.01})
    return m, spec


def full_table(name: str, rows: int, dim: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(int.from_bytes(sha256(name.encode()).digest()[:4], "little"))
    t = torch.randn(rows, dim, generator=g) * 0.05
    t[0].zero_()
    return t


@torch.no_grad()
def load_full_tables(store) -> None:
    for t in store.layouts:
        full = full_table(t.name, t.num_embeddings, t.dim)
        ids = t.spec.global_ids(t.num_embeddings, store.rank)
        if ids.numel():
            store.weight(t.name).copy_(full[ids].to(store.slab.device))


@torch.no_grad()
def gather_tables(store, which: str = "weight") -> dict[str, torch.Tensor]:
    """Reassemble full tables (``weight`` or ``grad``) from every rank's shard."""

    out = {}
    for t in store.layouts:
        local = (store.weight(t.name) if which == "weight" else store.grad_view(t.name)).float().cpu()
        ids = t.spec.global_ids(t.num_embeddings, store.rank)
        if store.world > 1 and dist.is_initialized():
            parts = [None] * store.world
            dist.all_gather_object(parts, (ids, local))
        else:
            parts = [(ids, local)]
        full = torch.zeros(t.num_embeddings, t.dim)
        for pid, pval in parts:
            if pid.numel():
                full[pid] = pval
        out[t.name] = full
    return out


def _setup(rank: int, world: int, backend: str, init_file: str, device_type: str):
    if device_type == "cuda":
        torch.cuda.set_device(rank)
    dist.init_process_group(backend, init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))


def run_parity(rank: int, world: int, backend: str, device_type: str, init_file: str, out_path: str,
               optimizer: str = "adam", distribution: str = "sharded", sparse_optimizer: str = "rowwise_adagrad",
               ) -> None:
    _setup(rank, world, backend, init_file, device_type)
    try:
        _run_parity_body(rank, world, device_type, out_path, optimizer, distribution, sparse_optimizer)
    except BaseException:
        # A failed rank exits at once: tearing down a process group whose peers may
        # be blocked in a collective can itself block.
        import traceback

        traceback.print_exc()
        os._exit(1)
    dist.destroy_process_group()


def _run_parity_body(rank: int, world: int, device_type: str, out_path: str, optimizer: str, distribution: str,
                     sparse_optimizer: str) -> None:
    from ..data.synthetic import SyntheticGenerator
    from ..models.factory import build_model
    from ..train.trainer import Trainer

    if True:
        device = torch.device(device_type, rank) if device_type == "cuda" else torch.device("cpu")
        mapping, spec = tiny_mapping(optimizer=optimizer, distribution=distribution,
                                     sparse_optimizer=sparse_optimizer)
        cfg = app_config_from_mapping(mapping)
        B = cfg.training.batch_size
        torch.manual_seed(0)
        model = build_model(cfg, device=device, rank=rank, world=world, process_group=dist.group.WORLD, base_seed=0)
        load_full_tables(model.store)
        model.store.sync_peers()
        trainer = Trainer(cfg, model, device=device, rank=rank, world=world, process_group=dist.group.WORLD)
        F = len(model.encoder.batch_plan.features)
        union = SyntheticGenerator(model.encoder.batch_plan, spec, rank=0).batch(B * world)
        local = union.slice_rows(rank * B, (rank + 1) * B, F)
        batch = local.to(device) if device.type == "cuda" else local
        out = trainer.forward_backward(batch)
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        loss = out["loss"].detach().float().reshape(1).clone()
        dist.all_reduce(loss)  # sum of the per-rank W-scaled losses = W * union loss
        grads_dense = trainer.dense.grad.detach().clone()
        dist.all_reduce(grads_dense)
        grads_dense /= world
        grad_tables = gather_tables(model.store, "grad")
        if model.store.replicas > 1:  # every replica holds its own W-scaled contribution: sum them
            for g in grad_tables.values():
                on_dev = g.to(device)  # NCCL reduces device tensors only
                dist.all_reduce(on_dev)
                g.copy_(on_dev.cpu())
        trainer.optimizer_step()
        if device.type == "cuda":
            torch.cuda.synchronize(device)
            from ..ops._ext import check_error_word

            check_error_word(device)
        master = trainer.dense.gather_master().detach().float().cpu().clone()
        tables = gather_tables(model.store, "weight")
        if rank == 0:
            torch.manual_seed(0)
            ref_model = build_model(cfg, device=device, rank=0, world=1, process_group=None, base_seed=0)
            load_full_tables(ref_model.store)
            ref = Trainer(cfg, ref_model, device=device, rank=0, world=1, process_group=None)
            ubatch = union.to(device) if device.type == "cuda" else union
            rout = ref.forward_backward(ubatch)
            ref_grads = ref.dense.grad.detach().float().cpu().clone()
            ref_grad_tables = gather_tables(ref_model.store, "grad")
            ref.optimizer_step()
            ref_master = ref.dense.gather_master().detach().float().cpu().clone()
            ref_tables = gather_tables(ref_model.store, "weight")

            def rel(a, b):
                n = min(a.numel(), b.numel())
                a, b = a.flatten()[:n], b.flatten()[:n]
                return float((a - b).abs().max() / (b.abs().max() + 1e-12))

            def by_name(dense, flat):
                # flat layouts differ with the world size (bucket padding): compare parameter by parameter
                return torch.cat([flat[dense.offsets[n]:dense.offsets[n] + dense.params[n].numel()]
                                  for n in sorted(dense.offsets)])

            grads_dense = by_name(trainer.dense, grads_dense.float().cpu())
            ref_grads = by_name(ref.dense, ref_grads)
            master, ref_master = by_name(trainer.dense, master), by_name(ref.dense, ref_master)

            result = {
                "loss": float(loss) / world, "ref_loss": float(rout["loss"].detach()),
                "dense_grad_rel": rel(grads_dense.float().cpu(), ref_grads),
                # owners hold the sum over ranks of W-scaled contributions: divide by W
                "table_grad_rel": max(rel(grad_tables[n] / world, ref_grad_tables[n]) for n in ref_grad_tables),
                "dense_param_max_abs": float((master - ref_master).abs().max()),
                "table_max_abs": max(float((tables[n] - ref_tables[n]).abs().max()) for n in ref_tables),
                "lr_dense": cfg.training.lr_dense, "lr_sparse": cfg.training.lr_sparse,
            }
            with open(out_path, "w") as fh:
                json.dump(result, fh)
        dist.barrier()
