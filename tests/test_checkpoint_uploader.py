"""Asynchronous checkpoint publication (stage locally, upload and commit from a thread)
and the staging-space preflight, on CPU: resume from an asynchronously published step,
no commit while a rank's READY marker is missing, commit on two gloo ranks, refusal of
a staging filesystem that is too small."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mdl_b200.checkpoint import (CheckpointStagingSpaceError, CheckpointUploader, check_staging_space,
                                 estimate_staging_bytes, load_training_checkpoint, make_uploader,
                                 open_checkpoint_store, save_training_checkpoint)
from mdl_b200.checkpoint.training import (COMMIT_MARKER, _commit_step, list_committed_checkpoints,
                                          rank_ready_marker, step_directory_name)
from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import baseline_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.train.trainer import Trainer


def _cfg(**ck):
    m, spec = baseline_config(1)
    m["training"]["embedding_sharding"] = {"strategy": "row_wise"}
    m["training"]["checkpoint"] = {"keep_last": 2, **ck}
    return app_config_from_mapping(m), spec


def _trainer(cfg, rank=0, world=1, group=None, seed=0):
    torch.manual_seed(seed)
    model = build_model(cfg, device="cpu", rank=rank, world=world, process_group=group, base_seed=seed)
    return model, Trainer(cfg, model, device=torch.device("cpu"), rank=rank, world=world, process_group=group)


def test_async_saves_publish_commit_and_resume(tmp_path):
    cfg, spec = _cfg(staging_dir=str(tmp_path / "stage"))
    model, tr = _trainer(cfg)
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    batches = [gen.batch(64) for _ in range(5)]
    run = open_checkpoint_store(tmp_path / "run")
    up = make_uploader(cfg, tr, run)
    assert isinstance(up, CheckpointUploader) and up.asynchronous
    for i, b in enumerate(batches[:3]):
        tr.train_step(b)
        save_training_checkpoint(cfg, tr, run, step=i + 1, uploader=up, keep_last=2)
    assert up.flush(timeout=60)
    assert up.failed_steps == [] and up.published_steps == [1, 2, 3]
    # retention ran on the upload thread; staged copies are gone
    assert [c.step for c in list_committed_checkpoints(run)] == [2, 3]
    assert not any(p.is_file() for p in up.staging_root.rglob("*"))
    assert up.uploaded_bytes > 0
    up.close()
    assert not up.staging_root.exists()
    # the published step resumes like a synchronous one
    for b in batches[3:]:
        tr.train_step(b)
    _, resumed = _trainer(cfg, seed=5)
    state = load_training_checkpoint(cfg, resumed, run, "auto")
    assert state is not None and state.step == 3
    for b in batches[3:]:
        resumed.train_step(b)
    for n, p in tr.dense.params.items():
        torch.testing.assert_close(resumed.dense.params[n].detach(), p.detach(), rtol=1e-6, atol=1e-7)


def test_step_without_every_ready_marker_is_not_committed(tmp_path):
    cfg, spec = _cfg()
    model, tr = _trainer(cfg)
    run = open_checkpoint_store(tmp_path / "run")
    # rank 0 of a two-rank run whose peer never publishes: the wait runs out, no commit
    up = CheckpointUploader(run, rank=0, world=2, staging_dir=str(tmp_path / "stage"), ready_timeout_sec=0.3,
                            poll_sec=0.05, asynchronous=False, commit_fn=_commit_step)
    tr.world = 2  # only the manifest's world size and the marker count read it
    try:
        save_training_checkpoint(cfg, tr, run, step=7, uploader=up)
    finally:
        tr.world = 1
    name = step_directory_name(7)
    assert run.exists(name, rank_ready_marker(0)) and not run.exists(name, COMMIT_MARKER)
    assert [s for s, _ in up.failed_steps] == [7] and "not READY" in up.failed_steps[0][1]
    assert list_committed_checkpoints(run) == []
    # once the peer's marker lands, the next save of the step commits
    run.write_bytes(b"", name, rank_ready_marker(1))
    tr.world = 2
    try:
        save_training_checkpoint(cfg, tr, run, step=7, uploader=up)
    finally:
        tr.world = 1
    assert up.published_steps == [7] and run.exists(name, COMMIT_MARKER)
    up.close()


def test_staging_preflight_refuses_small_filesystem(tmp_path):
    cfg, _ = _cfg()
    _, tr = _trainer(cfg)
    est = estimate_staging_bytes(tr, cfg.training.checkpoint.shard_chunk_bytes)
    dense = sum(p.numel() for p in tr.dense.params.values()) * 4
    tables = sum(tr.store.weight(t.name).numel() * 4 + tr.store.accumulator(t.name).numel() * 4
                 for t in tr.store.layouts)
    states = 2 if tr.dense.optimizer == "adam" else 1
    assert est.total_bytes == tables + dense + dense * (1 + states)  # dense.pt, then params + optimizer state
    with pytest.raises(CheckpointStagingSpaceError, match="too little room"):
        check_staging_space(tmp_path, est, local_ranks=8, free=est.total_bytes * 4)
    summary = check_staging_space(tmp_path, est, local_ranks=2, free=est.total_bytes * 4)
    assert "local_ranks=2" in summary
    # synchronous saves need no uploader
    cfg_sync, _ = _cfg(async_upload=False)
    assert make_uploader(cfg_sync, tr, open_checkpoint_store(tmp_path / "r")) is None


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_async(rank, world, port, root):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, spec = _cfg(staging_dir=os.path.join(root, "stage"), ready_timeout_sec=60.0)
        model, tr = _trainer(cfg, rank, world, dist.group.WORLD)
        gen = SyntheticGenerator(model.encoder.batch_plan, spec, rank=rank)
        run = open_checkpoint_store(os.path.join(root, "run"))
        up = make_uploader(cfg, tr, run, local_ranks=world)
        for step in (1, 2):
            tr.train_step(gen.batch(64))
            save_training_checkpoint(cfg, tr, run, step=step, uploader=up, keep_last=2)
        up.close()
        assert up.failed_steps == [], up.failed_steps
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_async_commit_two_gloo_ranks(tmp_path):
    mp.spawn(_two_rank_async, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    run = open_checkpoint_store(tmp_path / "run")
    assert [c.step for c in list_committed_checkpoints(run)] == [1, 2]
    name = step_directory_name(2)
    for r in range(2):
        assert run.exists(name, rank_ready_marker(r))
        assert run.exists(name, "model", f"shard-0000-rank-{r:05d}-of-00002.pt")
    cfg, _ = _cfg()
    _, tr = _trainer(cfg, seed=3)
    assert load_training_checkpoint(cfg, tr, run, "auto").step == 2
