"""W sharded ranks == one rank on the union batch (gloo on CPU here; NCCL + NVLink kernels on GPUs).

Mirrors the reference's distributed parity tests (``tests/test_sharded_embedding.py``):
spawned ranks, each training on its slice of one union batch, must reproduce the
gradients and updates of a single rank training on the whole batch.
"""

import json
import os
import time

import pytest
import torch
import torch.multiprocessing as mp

from mdl_b200.parallel.parity import run_parity


def _run(tmp_path, world, backend, device_type, optimizer="adam", distribution="sharded",
         sparse_optimizer="rowwise_adagrad"):
    init_file = str(tmp_path / "pg_init")
    out = str(tmp_path / "parity.json")
    ctx = mp.start_processes(run_parity, args=(world, backend, device_type, init_file, out, optimizer, distribution,
                                               sparse_optimizer),
                             nprocs=world, join=False, start_method="spawn")
    deadline = time.monotonic() + 300
    while not ctx.join(timeout=5):
        if time.monotonic() > deadline:
            for proc in ctx.processes:
                if proc.is_alive():
                    proc.kill()
            pytest.fail("parity ranks did not finish within 300 s")
    with open(out) as fh:
        return json.load(fh)


@pytest.mark.parametrize("optimizer,distribution,sparse", [("adam", "sharded", "rowwise_adagrad"),
                                                           ("rmsprop", "sharded", "rowwise_adagrad"),
                                                           ("adam", "sharded", "adagrad"),
                                                           ("adam", "replicated", "adagrad")])
def test_gloo_two_ranks_match_union_batch(tmp_path, optimizer, distribution, sparse):
    r = _run(tmp_path, 2, "gloo", "cpu", optimizer, distribution, sparse)
    assert abs(r["loss"] - r["ref_loss"]) < 1e-5 * max(1.0, abs(r["ref_loss"]))
    assert r["dense_grad_rel"] < 1e-4, r
    assert r["table_grad_rel"] < 1e-4, r
    assert r["table_max_abs"] < 1e-5, r
    assert r["dense_param_max_abs"] < 2e-5, r


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("distribution", [("sharded", "rowwise_adagrad"), ("replicated", "adagrad")])
def test_nccl_nvlink_two_gpus_match_union_batch(tmp_path, distribution):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    r = _run(tmp_path, 2, "nccl", "cuda", "adam", *distribution)
    assert abs(r["loss"] - r["ref_loss"]) < 2e-2 * max(1.0, abs(r["ref_loss"])), r
    assert r["dense_grad_rel"] < 5e-2, r
    assert r["table_grad_rel"] < 5e-2, r
    # one optimizer step moves each weight by at most ~lr; a sign disagreement on a
    # near-zero gradient can at most double that
    assert r["dense_param_max_abs"] < 2.5 * r["lr_dense"], r
    assert r["table_max_abs"] < 2.5 * r["lr_sparse"], r
