"""Sparse optimizers of the embedding store against ``torch.optim.Adagrad`` (full, with
``lr_decay``) and the row-wise rule; the CUDA kernels against the CPU definition."""

import pytest
import torch

from mdl_b200.ops.embedding import EmbeddingStore, _push_grads_cpu
from mdl_b200.parallel.sharding import EmbeddingTableSpec, plan_embedding_shards


def _store(device, optimizer, lr_decay=0.0):
    tables = [("a", 50, 16), ("b", 30, 8)]
    plan = plan_embedding_shards([EmbeddingTableSpec(n, r, d, 4) for n, r, d in tables], world_size=1,
                                 strategy="row_wise", table_wise_max_rows=0,
                                 optimizer_state_layout="full" if optimizer == "full" else "rowwise")
    return EmbeddingStore(tables, plan, rank=0, world=1, device=device, init_std=0.1, lr=0.3, eps=1e-10,
                          initial_accumulator_value=0.1, base_seed=3, optimizer=optimizer, lr_decay=lr_decay)


def _grads(step):
    g = torch.Generator().manual_seed(step)
    ids = torch.randint(1, 50, (20,), generator=g)
    return ids, torch.randn(20, 16, generator=g)


def test_full_adagrad_matches_torch():
    store = _store("cpu", "full", lr_decay=0.05)
    w0 = store.weight("a").clone()
    ref = torch.nn.Parameter(w0.clone())
    opt = torch.optim.Adagrad([ref], lr=0.3, lr_decay=0.05, initial_accumulator_value=0.1, eps=1e-10)
    for step in range(3):
        ids, g = _grads(step)
        _push_grads_cpu(store, "a", ids, g)
        store.step()
        ref.grad = torch.zeros_like(ref).index_add_(0, ids, g).to_sparse()
        opt.step()
    torch.testing.assert_close(store.weight("a"), ref.detach(), atol=1e-6, rtol=1e-5)
    assert store.accumulator("a").shape == (50, 16)


def test_rowwise_adagrad_rule():
    store = _store("cpu", "rowwise")
    w0 = store.weight("a").clone()
    ids, g = _grads(0)
    _push_grads_cpu(store, "a", ids, g)
    store.step()
    dense = torch.zeros(50, 16).index_add_(0, ids, g)
    rows = ids.unique()
    acc = 0.1 + dense[rows].square().mean(1)
    expect = w0[rows] - 0.3 * dense[rows] / (acc.sqrt() + 1e-10).unsqueeze(1)
    torch.testing.assert_close(store.weight("a")[rows], expect)


@pytest.mark.gpu
@pytest.mark.parametrize("optimizer", ["full", "rowwise"])
def test_adagrad_kernels_match_cpu(optimizer):
    cpu, gpu = _store("cpu", optimizer, 0.1), _store("cuda", optimizer, 0.1)
    gpu.slab.copy_(cpu.slab)
    for step in range(2):
        ids, g = _grads(step)
        _push_grads_cpu(cpu, "a", ids, g)
        rows = cpu._cpu_touched.nonzero().flatten()
        gpu.grad.copy_(cpu.grad)
        gpu.flags[rows.cuda()] = 1
        cpu.step()
        gpu.step()
    torch.cuda.synchronize()
    torch.testing.assert_close(gpu.slab.cpu(), cpu.slab, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(gpu.acc.cpu(), cpu.acc, atol=1e-6, rtol=1e-5)
