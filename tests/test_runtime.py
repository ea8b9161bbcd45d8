"""Distributed runtime helpers: backend choice, NCCL environment policy, CPU shares,
shard-metadata agreement (gloo ranks), gradient auditor, host memory tools and the
external parameter-server hook."""

import json
import os
import time

import pytest
import torch
import torch.multiprocessing as mp

from mdl_b200.parallel import runtime
from mdl_b200.utils import hostmem


def test_backend_and_nccl_env(monkeypatch):
    monkeypatch.delenv("MDL_DIST_BACKEND", raising=False)
    assert runtime.resolve_backend(torch.device("cpu")) == "gloo"
    assert runtime.resolve_backend(torch.device("cuda", 0)) == "nccl"
    monkeypatch.setenv("MDL_DIST_BACKEND", "gloo")
    assert runtime.resolve_backend(torch.device("cuda", 0)) == "gloo"
    env = {"TORCH_NCCL_ASYNC_ERROR_HANDLING": "0"}
    applied = runtime.configure_nccl_env(8, env=env, p2p_ok=False)
    assert env["TORCH_NCCL_ASYNC_ERROR_HANDLING"] == "0"      # the user's choice stays
    assert applied == {"NCCL_P2P_DISABLE": "1"}
    env = {}
    runtime.configure_nccl_env(8, env=env, p2p_ok=True)
    assert env == {"TORCH_NCCL_ASYNC_ERROR_HANDLING": "1"}


def test_cpu_shares_cover_all_cores_once():
    cpus = list(range(26))
    shares = [runtime.set_local_cpu_affinity(r, 4, cpus, apply=False) for r in range(4)]
    assert sorted(c for s in shares for c in s) == cpus
    assert [len(s) for s in shares] == [6, 6, 6, 8]


def _meta_rank(rank, world, init_file, out_dir, mismatch):
    import torch.distributed as dist

    from mdl_b200.ops.embedding import EmbeddingStore
    from mdl_b200.parallel.sharding import EmbeddingTableSpec, plan_embedding_shards

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    rows = 100 + (7 if (mismatch and rank == 1) else 0)
    plan = plan_embedding_shards([EmbeddingTableSpec("t", rows, 8, 4)], world_size=world, strategy="row_wise",
                                 table_wise_max_rows=0)
    store = EmbeddingStore([("t", rows, 8)], plan, rank=rank, world=world, device="cpu", process_group=None)
    try:
        runtime.validate_shard_metadata(store)
        ok = True
    except RuntimeError:
        ok = False
    with open(os.path.join(out_dir, f"r{rank}.json"), "w") as fh:
        json.dump({"ok": ok}, fh)
    dist.destroy_process_group()


@pytest.mark.parametrize("mismatch", [False, True])
def test_shard_metadata_agreement(tmp_path, mismatch):
    ctx = mp.start_processes(_meta_rank, args=(2, str(tmp_path / "pg"), str(tmp_path), mismatch), nprocs=2,
                             join=False, start_method="spawn")
    deadline = time.monotonic() + 120
    while not ctx.join(timeout=2):
        assert time.monotonic() < deadline, "ranks did not finish"
    res = [json.load(open(tmp_path / f"r{r}.json"))["ok"] for r in range(2)]
    assert res == [not mismatch] * 2


def test_gradient_auditor_flags_unused_parameters():
    class FakeDense:
        names = ["a", "b"]
        offsets = {"a": 0, "b": 4}
        params = {"a": torch.zeros(4), "b": torch.zeros(4)}
        grad = torch.zeros(8)

    d = FakeDense()
    aud = runtime.GradientAuditor(d, steps=2)
    d.grad[:4] = 1.0
    aud.observe()
    aud.observe()
    rep = aud.report()
    assert rep["never_updated"] == ["b"] and rep["static_graph_safe"]


def test_host_memory_tools():
    assert hostmem.process_resident_bytes() > 0
    assert isinstance(hostmem.trim_process_heap(), bool)
    assert hostmem.arrow_pool_bytes() >= 0


def test_external_parameter_server_hook(capsys):
    from mdl_b200.cli import load_external_adapter, main

    assert load_external_adapter("builtins:dict")(config=1, max_steps=2) == {"config": 1, "max_steps": 2}
    with pytest.raises(ValueError):
        load_external_adapter("nodots")
    rc = main(["train", "--benchmark-config", "1", "--max-steps", "3",
               "--set", "training.sparse_update_mode=external_parameter_server",
               "--set", "training.sparse_parameter_server_adapter=builtins.dict"])
    assert rc == 0
    assert '"external": true' in capsys.readouterr().out


def test_benchmark_matrix_summary_and_commands():
    from mdl_b200.benchmark.matrix import bench_command, summarize

    rows = [{"matrix_config": 2, "matrix_gpus": 1, "impl": "ours", "value": 100.0},
            {"matrix_config": 2, "matrix_gpus": 2, "impl": "ours", "value": 180.0},
            {"matrix_config": 2, "matrix_gpus": 1, "impl": "reference", "value": 10.0},
            {"matrix_config": 2, "matrix_gpus": 2, "impl": "ours", "error": "exit 1"}]
    text = summarize(rows)
    assert "| 2 | ours | 2 | 180 | 90 | 0.900 | - |" in text
    assert "| 2 | ours | 1 | 100 | 100 | 1.000 | 10.00 |" in text
    cmd = bench_command(4, 4, "ours", 10, 3, 29999)
    assert "--nproc-per-node=4" in cmd and "--master-addr=127.0.0.1" in cmd and cmd[-1] == "ours"


def test_supply_iterator_and_verdicts():
    import threading

    from mdl_b200.train.supply import BATCH_NOT_READY, BudgetedIterator, supply_verdict

    gate = threading.Event()

    def slow():
        yield 1
        gate.wait(5)
        yield 2

    it = BudgetedIterator(slow())
    assert it.next_within(2.0) == 1
    assert it.next_within(0.05) is BATCH_NOT_READY
    gate.set()
    assert it.next_within(2.0) == 2
    with pytest.raises(StopIteration):
        it.next_within(2.0)
    with pytest.raises(StopIteration):
        it.next_within(2.0)
    assert supply_verdict(True, 1, 1, 2) == "train"
    assert supply_verdict(False, 1, 1, 2) == "replay"
    assert supply_verdict(False, 0, 1, 2) == "retry"
    assert supply_verdict(False, 0, 2, 2) == "stop"


def _vote_rank(rank, world, init_file, out_dir):
    import torch.distributed as dist

    from mdl_b200.train.supply import start_supply_count

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    got = start_supply_count(rank == 0, rank == 1, world).wait()
    with open(os.path.join(out_dir, f"v{rank}.json"), "w") as fh:
        json.dump(list(got), fh)
    dist.destroy_process_group()


def test_supply_vote_over_gloo(tmp_path):
    ctx = mp.start_processes(_vote_rank, args=(2, str(tmp_path / "pg"), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 120
    while not ctx.join(timeout=2):
        assert time.monotonic() < deadline
    assert [json.load(open(tmp_path / f"v{r}.json")) for r in range(2)] == [[1, 1], [1, 1]]


def test_attention_preflight():
    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import scaled_config
    from mdl_b200.ops.preflight import attention_preflight

    m, _ = scaled_config(4, 1e-3, num_fields=8, batch=8)
    assert "flash" in attention_preflight(app_config_from_mapping(m))["paths"]["mixed_causal"]
    m["model"]["num_heads"] = 4           # d=256 / 4 heads = head_dim 64: the CUDA-core kernels
    assert "CUDA-core" in attention_preflight(app_config_from_mapping(m))["paths"]["mixed_causal"]
    m["model"]["num_heads"] = 2           # head_dim 128: no native kernel
    with pytest.raises(ValueError, match="head_dim"):
        attention_preflight(app_config_from_mapping(m))
    m["runtime"] = {**m.get("runtime", {}), "kernel_backend": "torch"}
    assert "PyTorch" in attention_preflight(app_config_from_mapping(m))["paths"]["mixed_causal"]
    m, _ = scaled_config(5, 1e-3, num_fields=8, batch=8, seq_len=64, min_len=8, query_tokens=16)
    paths = attention_preflight(app_config_from_mapping(m))["paths"]
    assert "longer:behavior" in paths and "mixformer_cross" in paths
