"""Remote-IO policy: timeouts, retries with backoff, skip budget, stagger, per-file locks,
and the Parquet reader under the policy."""

import time

import pytest

from mdl_b200.data.remote_io import (PerFileLock, RemoteIoPolicy, RemoteIoStallError, call_with_timeout,
                                     retry_with_backoff)


def test_timeout_and_retry():
    with pytest.raises(TimeoutError):
        call_with_timeout(lambda: time.sleep(2), 0.1)
    assert call_with_timeout(lambda: 5, 1.0) == 5
    calls, sleeps = [], []

    def flaky():
        calls.append(1)
        if len(calls) < 3:
            raise OSError("transient")
        return "ok"

    assert retry_with_backoff(flaky, 3, 0.5, sleep=sleeps.append) == "ok"
    assert sleeps == [0.5, 1.0]
    with pytest.raises(RemoteIoStallError) as info:
        retry_with_backoff(lambda: (_ for _ in ()).throw(OSError("down")), 1, 0.0, sleep=lambda s: None)
    assert info.value.exit_code == 70


def test_policy_skips_and_staggers(tmp_path):
    pol = RemoteIoPolicy(retries=0, retry_base_s=0.0, skip_failures=True, lock_dir=str(tmp_path))
    assert pol.run(lambda: (_ for _ in ()).throw(OSError("gone")), "read x") is None and pol.skipped == 1
    pol.file_lock = True
    assert pol.run(lambda: 3, "open y", opening=True, path="hdfs://y") == 3
    slept = []
    RemoteIoPolicy(stagger_s=0.25).stagger(3, sleep=slept.append)
    assert slept == [0.75]
    with PerFileLock("a/b", str(tmp_path)):
        pass


def test_parquet_reader_skips_unreadable_units(tmp_path):
    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import baseline_config
    from mdl_b200.data.parquet import ParquetBatchIterator, Tensorizer
    from mdl_b200.models.factory import build_model

    m, _ = baseline_config(1)
    m["runtime"]["device"] = "cpu"
    cfg = app_config_from_mapping(m)
    model = build_model(cfg, device="cpu", base_seed=0)
    from mdl_b200.cli import main

    assert main(["make-synthetic-parquet", "--benchmark", "1", "--files", "2", "--rows", "256",
                 "--out", str(tmp_path / "d")]) == 0
    good = sorted(str(p) for p in (tmp_path / "d").glob("*.parquet"))
    it = ParquetBatchIterator(good, Tensorizer(cfg, model.encoder.batch_plan), 128,
                              io_policy=RemoteIoPolicy(retries=1, retry_base_s=0.0, skip_failures=True))
    # one planned unit's file disappears before it is read: it is retried, then skipped
    lost = it.refs[1]
    it.refs[1] = type(lost)(str(tmp_path / "missing.parquet"), lost.index, lost.rows)
    kept_rows = sum(r.rows for i, r in enumerate(it.refs) if i != 1)
    batches = list(it)
    assert it.io.skipped == 1
    assert len(batches) == kept_rows // 128
