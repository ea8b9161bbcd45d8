"""Checkpoints on CPU: save/load round trip, resharding across world sizes (gloo
ranks), commit protocol, retention, and resume reproducing an uninterrupted run."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mdl_b200.checkpoint import (load_model_checkpoint, load_training_checkpoint, open_checkpoint_store,
                                 prune_run_directory, save_model_checkpoint, save_training_checkpoint)
from mdl_b200.checkpoint.training import list_committed_checkpoints, step_directory_name
from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import baseline_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.train.trainer import Trainer


def _cfg():
    m, spec = baseline_config(1)
    m["training"]["embedding_sharding"] = {"strategy": "row_wise"}
    return app_config_from_mapping(m), spec


def _trainer(cfg, rank=0, world=1, group=None, seed=0):
    torch.manual_seed(seed)
    model = build_model(cfg, device="cpu", rank=rank, world=world, process_group=group, base_seed=seed)
    return model, Trainer(cfg, model, device=torch.device("cpu"), rank=rank, world=world, process_group=group)


def _full_tables(tr):
    """Global table contents (weight, acc) rebuilt from one rank's shard (W=1 only)."""

    st = tr.store
    return {t.name: (st.weight(t.name).clone(), st.accumulator(t.name).clone()) for t in st.layouts}


def test_round_trip_same_world(tmp_path):
    cfg, spec = _cfg()
    model, tr = _trainer(cfg)
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    for _ in range(3):
        tr.train_step(gen.batch(64))
    store = open_checkpoint_store(tmp_path / "ck")
    save_model_checkpoint(cfg, tr, store)
    assert (tmp_path / "ck" / "manifest.json").exists()
    assert (tmp_path / "ck" / "shard-0000-rank-00000-of-00001.pt").exists()
    model2, tr2 = _trainer(cfg, seed=123)
    load_model_checkpoint(cfg, tr2, store)
    for n, p in tr.dense.params.items():
        torch.testing.assert_close(tr2.dense.params[n].detach(), p.detach(), rtol=0, atol=0)
    a, b = _full_tables(tr), _full_tables(tr2)
    for n in a:
        torch.testing.assert_close(b[n][0], a[n][0], rtol=0, atol=0)
        torch.testing.assert_close(b[n][1], a[n][1], rtol=0, atol=0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _save_two_ranks(rank, world, port, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, spec = _cfg()
        model, tr = _trainer(cfg, rank, world, dist.group.WORLD)
        gen = SyntheticGenerator(model.encoder.batch_plan, spec, rank=rank)
        for _ in range(2):
            tr.train_step(gen.batch(64))
        save_model_checkpoint(cfg, tr, open_checkpoint_store(path))
        # global tables for the check: every rank's rows scattered into full tables
        out = {}
        for t in tr.store.layouts:
            w = torch.zeros(t.num_embeddings, t.dim)
            a = torch.zeros(t.num_embeddings)
            if t.local_rows:
                if t.spec.strategy == "table_wise":
                    ids = torch.arange(t.local_rows)
                else:
                    ids = (rank - t.spec.cyclic_offset) % world + torch.arange(t.local_rows) * world
                w[ids] = tr.store.weight(t.name)
                a[ids] = tr.store.accumulator(t.name)
            dist.all_reduce(w)
            dist.all_reduce(a)
            out[t.name] = (w, a)
        dense = {n: v.clone() for n, v in tr.dense.state_dict()["params"].items()}
        if rank == 0:
            torch.save({"tables": out, "dense": dense}, os.path.join(path, "expected.pt"))
    finally:
        dist.destroy_process_group()


def test_reshard_two_ranks_to_one(tmp_path):
    path = str(tmp_path / "ck2")
    os.makedirs(path)
    mp.spawn(_save_two_ranks, args=(2, _free_port(), path), nprocs=2, join=True)
    expected = torch.load(os.path.join(path, "expected.pt"))
    cfg, _ = _cfg()
    _, tr = _trainer(cfg, seed=7)
    load_model_checkpoint(cfg, tr, open_checkpoint_store(path))
    for name, (w, a) in expected["tables"].items():
        torch.testing.assert_close(tr.store.weight(name), w, rtol=0, atol=0)
        torch.testing.assert_close(tr.store.accumulator(name), a, rtol=0, atol=0)
    for n, v in expected["dense"].items():
        torch.testing.assert_close(tr.dense.params[n].detach(), v, rtol=0, atol=0)


def test_resume_matches_uninterrupted_run(tmp_path):
    cfg, spec = _cfg()
    batches_model, _ = _trainer(cfg)
    gen = SyntheticGenerator(batches_model.encoder.batch_plan, spec)
    batches = [gen.batch(64) for _ in range(6)]
    _, straight = _trainer(cfg)
    for b in batches:
        straight.train_step(b)
    run = open_checkpoint_store(tmp_path / "run")
    _, first = _trainer(cfg)
    for b in batches[:3]:
        first.train_step(b)
    save_training_checkpoint(cfg, first, run, step=3)
    _, resumed = _trainer(cfg, seed=99)
    state = load_training_checkpoint(cfg, resumed, run, "auto")
    assert state is not None and state.step == 3
    for b in batches[3:]:
        resumed.train_step(b)
    for n, p in straight.dense.params.items():
        torch.testing.assert_close(resumed.dense.params[n].detach(), p.detach(), rtol=1e-6, atol=1e-7)
    a, b = _full_tables(straight), _full_tables(resumed)
    for n in a:
        torch.testing.assert_close(b[n][0], a[n][0], rtol=1e-6, atol=1e-7)


def test_commit_protocol_and_retention(tmp_path):
    cfg, spec = _cfg()
    _, tr = _trainer(cfg)
    run = open_checkpoint_store(tmp_path / "run")
    for step in (1, 2, 3):
        save_training_checkpoint(cfg, tr, run, step=step)
    # an interrupted save: directory without the commit marker
    run.makedirs(step_directory_name(4))
    assert [c.step for c in list_committed_checkpoints(run)] == [1, 2, 3]
    assert run.read_json("_latest.json")["step"] == 3
    assert load_training_checkpoint(cfg, tr, run, "none") is None
    with pytest.raises(FileNotFoundError):
        load_training_checkpoint(cfg, tr, run, 4)
    removed = prune_run_directory(run, keep_last=2)
    assert removed == [step_directory_name(1)]
    assert [c.step for c in list_committed_checkpoints(run)] == [2, 3]


def test_load_rejects_checkpoint_that_misses_a_table(tmp_path):
    # a model table absent from the checkpoint must not keep its random init silently
    import json

    cfg, spec = _cfg()
    model, tr = _trainer(cfg)
    store = open_checkpoint_store(tmp_path / "ck")
    save_model_checkpoint(cfg, tr, store)
    manifest = json.loads((tmp_path / "ck" / "manifest.json").read_text())
    dropped = manifest["chunks"][0]["tables"][0]
    for fname in manifest["chunks"][0]["rank_files"]:
        payload = torch.load(tmp_path / "ck" / fname, weights_only=False)
        payload["tables"].pop(dropped)
        torch.save(payload, tmp_path / "ck" / fname)
    manifest["chunks"][0]["tables"].remove(dropped)
    (tmp_path / "ck" / "manifest.json").write_text(json.dumps(manifest))
    _model2, tr2 = _trainer(cfg, seed=7)
    with pytest.raises(ValueError, match="did not cover all local rows"):
        load_model_checkpoint(cfg, tr2, store)


def test_load_rejects_padding_idx_mismatch(tmp_path):
    cfg, spec = _cfg()
    model, tr = _trainer(cfg)
    store = open_checkpoint_store(tmp_path / "ck")
    save_model_checkpoint(cfg, tr, store)
    fname = tmp_path / "ck" / "shard-0000-rank-00000-of-00001.pt"
    payload = torch.load(fname, weights_only=False)
    first = next(iter(payload["tables"]))
    payload["tables"][first]["padding_idx"] = 3
    torch.save(payload, fname)
    _model2, tr2 = _trainer(cfg, seed=7)
    with pytest.raises(ValueError, match="padding_idx"):
        load_model_checkpoint(cfg, tr2, store)
