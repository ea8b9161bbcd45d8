"""CLI commands on CPU, evaluation metrics against scikit-learn, and the step
watchdog / out-of-memory abort (host-side failures only)."""

import json
import subprocess
import sys
import time

import numpy as np
import pytest
import torch

from mdl_b200.metrics.auc import StreamingHistogramAUC, TaskMonitor, binary_auc, group_auc
from mdl_b200.train.watchdog import StepWatchdog, abort_on_cuda_oom


def _run(*args, cwd=None):
    out = subprocess.run([sys.executable, "-m", "mdl_b200", *args], capture_output=True, text=True, timeout=600,
                         cwd=cwd)
    assert out.returncode == 0, out.stderr[-2000:]
    return [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]


def test_auc_matches_sklearn():
    from sklearn.metrics import roc_auc_score

    rng = np.random.default_rng(0)
    y = (rng.random(5000) < 0.2).astype(np.float64)
    s = rng.normal(size=5000) + y
    s[:100] = np.round(s[:100])  # ties
    ref = roc_auc_score(y, s)
    assert abs(binary_auc(torch.tensor(s), torch.tensor(y)) - ref) < 1e-12
    h = StreamingHistogramAUC(4096)
    h.update(torch.tensor(s), torch.tensor(y))
    assert abs(h.compute() - ref) < 2e-3
    groups = rng.integers(0, 10, size=5000)
    want = np.mean([roc_auc_score(y[groups == g], s[groups == g]) for g in range(10)])
    assert abs(group_auc(torch.tensor(s), torch.tensor(y), groups.tolist()) - want) < 1e-12
    assert binary_auc(torch.ones(3), torch.ones(3)) is None


def test_task_monitor_flags_collapse():
    m = TaskMonitor(["a"])
    m.update(torch.full((100, 1), 5.0), torch.zeros(100, 1))
    s = m.summary()["a"]
    assert s["count"] == 100 and "mean probability above 0.9" in s["warnings"]


def test_watchdog_fires_without_beats_and_not_with_them():
    fired = []
    dog = StepWatchdog(0.3, on_expire=fired.append, poll_sec=0.05).start()
    for _ in range(8):
        time.sleep(0.1)
        dog.beat("step")
    assert not fired
    time.sleep(0.6)
    assert fired and "no training progress" in fired[0]
    dog.stop()


def test_oom_abort_exits_with_70():
    codes = []

    def boom():
        raise torch.cuda.OutOfMemoryError("CUDA out of memory. Tried to allocate 1 GiB")

    abort_on_cuda_oom(boom, exit_fn=codes.append)
    assert codes == [70]
    with pytest.raises(ValueError):
        abort_on_cuda_oom(lambda: (_ for _ in ()).throw(ValueError("other")), exit_fn=codes.append)


def test_cli_train_checkpoint_evaluate_predict(tmp_path):
    data = tmp_path / "data"
    _run("make-synthetic-parquet", "--benchmark", "1", "--files", "2", "--rows", "512", "--out", str(data))
    over = ["--benchmark-config", "1", "--set", f"data.train.inputs=[{str(data)}]", "--set", "training.batch_size=128"]
    prof = _run("profile", *over, "--max-batches", "4")[-1]
    assert prof["rows"] == 512 and prof["batches"] == 4
    run = tmp_path / "run"
    logs = _run("train", *over, "--max-steps", "6", "--checkpoint-dir", str(run), "--save-every", "3",
                "--log-every", "2")
    assert logs[-1]["done"] and logs[-1]["steps"] == 6
    assert (run / "step-000000006" / "_COMMIT").exists() and (run / "step-000000003" / "_COMMIT").exists()
    # resume continues from the last committed step
    logs = _run("train", *over, "--max-steps", "8", "--checkpoint-dir", str(run), "--log-every", "1")
    assert [l["step"] for l in logs if "step" in l and "loss" in l][0] == 7
    ev = _run("evaluate", *over, "--checkpoint", str(run), "--max-batches", "4")[-1]
    auc = ev["tasks"]["click"]["auc"]
    assert ev["batches"] == 4 and auc is not None and 0.0 <= auc <= 1.0
    out = tmp_path / "pred.parquet"
    pr = _run("predict", *over, "--checkpoint", str(run), "--max-batches", "2", "--output", str(out))[-1]
    import pyarrow.parquet as pq

    t = pq.read_table(str(out))
    assert pr["rows"] == 256 and t.num_rows == 256 and "pred_click" in t.column_names
    st = _run("check-checkpoint-store", "--checkpoint-dir", str(run))[-1]
    assert st["round_trip_ok"] and st["resume_from"] == "step-000000008"


def test_cli_fixed_test_eval_during_training(tmp_path):
    data = tmp_path / "data"
    _run("make-synthetic-parquet", "--benchmark", "1", "--files", "2", "--rows", "384", "--out", str(data))
    over = ["--benchmark-config", "1", "--set", f"data.train.inputs=[{str(data)}]",
            "--set", f"data.test.inputs=[{str(data)}]", "--set", "training.batch_size=128",
            "--set", "training.fixed_test_eval.enabled=true", "--set", "training.fixed_test_eval.every_steps=2",
            "--set", "training.fixed_test_eval.files_per_rank=1"]
    logs = _run("train", *over, "--max-steps", "4", "--log-every", "10")
    evals = [l for l in logs if "fixed_test_eval" in l]
    assert [l["step"] for l in evals] == [2, 4]
    ev = evals[-1]["fixed_test_eval"]
    assert ev["batches"] == 3 and 0.0 <= ev["tasks"]["click"]["auc"] <= 1.0


def test_cli_two_ranks_from_parquet_with_checkpoint(tmp_path):
    """Two gloo ranks through the CLI relaunch: runtime set-up, shard-metadata agreement,
    the batch supply vote on Parquet input, a sharded checkpoint, then a resume."""

    data = tmp_path / "data"
    _run("make-synthetic-parquet", "--benchmark", "1", "--files", "2", "--rows", "512", "--out", str(data))
    over = ["--benchmark-config", "1", "--set", f"data.train.inputs=[{str(data)}]", "--set", "training.batch_size=128",
            "--set", "runtime.device=cpu", "--nproc-per-node", "2", "--master-port", "29563"]
    run = tmp_path / "run"
    logs = _run("train", *over, "--max-steps", "4", "--log-every", "2", "--checkpoint-dir", str(run),
                "--save-every", "4")
    assert logs[-1]["done"] and logs[-1]["steps"] == 4
    assert (run / "step-000000004" / "_COMMIT").exists()
    logs = _run("train", *over, "--max-steps", "6", "--log-every", "1", "--checkpoint-dir", str(run))
    assert [l["step"] for l in logs if "loss" in l][0] == 5


def test_cli_replicated_tables_checkpoint_reshards(tmp_path):
    """Replicated tables with full Adagrad on two gloo ranks: rank 0 writes one copy of
    each table; the checkpoint resumes on two ranks and loads into a sharded layout."""

    data = tmp_path / "data"
    _run("make-synthetic-parquet", "--benchmark", "1", "--files", "2", "--rows", "512", "--out", str(data))
    base = ["--benchmark-config", "1", "--set", f"data.train.inputs=[{str(data)}]", "--set", "training.batch_size=128",
            "--set", "runtime.device=cpu", "--set", "training.sparse_optimizer=adagrad"]
    rep = base + ["--set", "training.embedding_distribution=replicated"]
    run = tmp_path / "run"
    logs = _run("train", *rep, "--nproc-per-node", "2", "--master-port", "29565", "--max-steps", "3",
                "--checkpoint-dir", str(run), "--log-every", "1")
    assert logs[-1]["done"]
    manifest = json.loads((run / "step-000000003" / "model" / "manifest.json").read_text())
    assert manifest["embedding_world_size"] == 1
    assert all(len(c["rank_files"]) == 1 for c in manifest["chunks"])
    logs = _run("train", *rep, "--nproc-per-node", "2", "--master-port", "29567", "--max-steps", "4",
                "--checkpoint-dir", str(run), "--log-every", "1")
    assert [l["step"] for l in logs if "loss" in l][0] == 4
    shard = base + ["--set", "training.embedding_distribution=sharded"]
    logs = _run("train", *shard, "--nproc-per-node", "2", "--master-port", "29569", "--max-steps", "5",
                "--checkpoint-dir", str(run), "--log-every", "1")
    assert [l["step"] for l in logs if "loss" in l][0] == 5


def test_cli_benchmark_modes(tmp_path):
    """``benchmark --mode compute | embedding | data | end-to-end`` on CPU: every mode
    reports throughput and step-time percentiles; compute / end-to-end add the dense
    GEMM MFU; end-to-end and data read the Parquet inputs."""

    data = tmp_path / "data"
    _run("make-synthetic-parquet", "--benchmark", "1", "--files", "1", "--rows", "512", "--out", str(data))
    over = ["--benchmark-config", "1", "--set", f"data.train.inputs=[{str(data)}]", "--set", "training.batch_size=64"]
    for mode in ("compute", "embedding", "data", "end-to-end"):
        res = _run("benchmark", *over, "--mode", mode, "--steps", "4", "--warmup", "1")[-1]
        assert res["mode"] == mode and res["value"] > 0 and res["ms_p95"] >= res["ms_p50"] > 0, res
        if mode in ("compute", "end-to-end"):
            assert 0 < res["mfu_dense_gemm"] < 1, res
    # profiler pass and lookup statistics after the timed steps
    res = _run("benchmark", *over, "--mode", "compute", "--steps", "2", "--warmup", "1", "--profile-steps", "2",
               "--comm-stats")[-1]
    prof = res["profile"]
    assert {"mdl.forward", "mdl.backward", "mdl.dense_update", "mdl.sparse_update"} <= set(
        prof["ranges_cpu_ms_per_step"]), prof
    comm = res["embedding_comm"]
    assert comm and all(v["raw_ids"] >= v["active_ids"] >= 0 for v in comm.values())
    assert res["embedding_comm_bytes_per_step"] == 0  # one rank: nothing crosses NVLink
