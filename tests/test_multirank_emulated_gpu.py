"""The multi-rank kernels on ONE GPU: several ranks' buffers laid out on one device
(``EmulatedPeers``), every phase of the protocol issued for each rank in turn on one
stream, results compared with a plain PyTorch fp32 oracle.

Covers the owner-push lookup (``emb_route``, ``emb_owner_fwd``, ``acc_to_bf16``),
the owner-pull gradient (``emb_owner_bwd``) followed by the row-wise Adagrad update
of the owners, and the fused dense reduce-scatter / optimizer / all-gather
(``dense_sync``). Also makes the two bounded device waits run out on purpose (a
peer flag nobody sets, an mbarrier nobody arrives on) and checks that the kernels
return and report the timeout through the error word.
"""

import pytest
import torch

from mdl_b200.ops.embedding import (EmbeddingStore, LookupFeature, LookupPlan, POOL_MEAN, POOL_NONE, POOL_SUM,
                                    _exchange, backward_reference, lookup_reference, owner_collect, owner_pull_grad,
                                    owner_push, owner_route, owner_stage_grad)
from mdl_b200.parallel.emulate import EmulatedPeers
from mdl_b200.parallel.sharding import EmbeddingTableSpec, plan_embedding_shards

pytestmark = pytest.mark.gpu

TABLES = [("big_a", 50_000, 64), ("big_b", 30_000, 32), ("small", 1_000, 16)]


def _plan():
    feats, col = [], 0
    for name, table, pool in (("f_single", "big_a", POOL_NONE), ("f_sum", "big_b", POOL_SUM),
                              ("f_mean", "big_a", POOL_MEAN), ("f_small", "small", POOL_NONE)):
        dim = {t: d for t, _n, d in TABLES}[table]
        feats.append(LookupFeature(name, table, pooling=pool, width=dim, out_col=col))
        col += dim
    feats.append(LookupFeature("dense", None, width=8, out_col=col, dense_col=0))
    col += 8
    return LookupPlan(feats, out_width=col, dense_width=8)


def _batch(plan, rows, seed, device):
    g = torch.Generator().manual_seed(seed)
    nums = {t: n for t, n, _d in TABLES}
    ids, lengths = [], []
    for f in plan.features:
        if f.table is None:
            continue
        if f.pooling == POOL_NONE:
            ln = torch.ones(rows, dtype=torch.int64)
        else:
            ln = torch.randint(0, 7, (rows,), generator=g)  # empty bags included
        x = torch.randint(0, nums[f.table], (int(ln.sum()),), generator=g)
        x[torch.rand(x.numel(), generator=g) < 0.05] = 0  # padding ids
        # a few hot ids shared across bags and ranks (owners see several bundles per row)
        hot = torch.rand(x.numel(), generator=g) < 0.2
        x[hot] = torch.randint(1, 50, (int(hot.sum()),), generator=g)
        ids.append(x)
        lengths.append(ln)
    offsets = torch.cat([torch.zeros(1, dtype=torch.int64), torch.cat(lengths).cumsum(0)])
    dense = torch.randn(rows, 8, generator=g)
    return torch.cat(ids).to(device), offsets.to(device), dense.to(device)


def _stores(world, device, peers):
    specs = [EmbeddingTableSpec(n, r, d) for n, r, d in TABLES]
    plan = plan_embedding_shards(specs, world_size=world, strategy="auto", table_wise_max_rows=5_000,
                                 optimizer_state_layout="row_wise")
    return [EmbeddingStore(TABLES, plan, rank=r, world=world, device=device, base_seed=11, lr=0.1, peers=peers)
            for r in range(world)]


def _oracle_store(stores):
    """One CPU rank holding every table in full, with the sharded ranks' weights."""

    plan1 = plan_embedding_shards([EmbeddingTableSpec(n, r, d) for n, r, d in TABLES], world_size=1,
                                  optimizer_state_layout="row_wise")
    ref = EmbeddingStore(TABLES, plan1, rank=0, world=1, device="cpu", base_seed=0, lr=0.1)
    for name, num, _dim in TABLES:
        for st in stores:
            t = st.layouts[st.index[name]]
            gids = t.spec.global_ids(num, st.rank)
            ref.weight(name)[gids] = st.weight(name).cpu()
            ref.accumulator(name)[gids] = st.accumulator(name).cpu()
    return ref


@pytest.mark.parametrize("world", [2, 4])
def test_owner_push_lookup_gradient_and_adagrad(world):
    dev = torch.device("cuda", 0)
    rows = 300
    plan = _plan()
    peers = EmulatedPeers(world, dev, exchange_ids=4 * rows * 8, exchange_rows=rows)
    stores = _stores(world, dev, peers)
    oracle = _oracle_store(stores)
    batches = [_batch(plan, rows, 100 + r, dev) for r in range(world)]

    # each rank's lookup staging exists before any rank routes (processes agree on its
    # size with an all-reduce at first use; here the emulator gives the size)
    for st, (ids, _off, _d) in zip(stores, batches):
        _exchange(st, plan, ids, rows)
    # forward: every rank routes, then every owner pushes, then every rank collects
    for st, (ids, off, dense) in zip(stores, batches):
        owner_route(st, plan, ids, off, dense, rows)
    for st, (ids, off, _d) in zip(stores, batches):
        owner_push(st, plan, ids, off, rows)
    outs = [owner_collect(st, plan, b[0], rows) for st, b in zip(stores, batches)]
    torch.cuda.synchronize()
    for out, (ids, off, dense) in zip(outs, batches):
        want = lookup_reference(oracle, plan, ids.cpu(), off.cpu(), dense.cpu(), rows)
        torch.testing.assert_close(out.float().cpu(), want, atol=2e-3, rtol=1e-2)

    # backward: every requester stages d(out), then every owner pulls its bundles' slices
    grads = [torch.randn(rows, plan.out_ld, device=dev).bfloat16() for _ in range(world)]
    for st, (ids, _off, _d), g in zip(stores, batches, grads):
        owner_stage_grad(st, plan, ids, g, rows)
    for st, (ids, off, _d) in zip(stores, batches):
        owner_pull_grad(st, plan, ids, off, rows)
    for (ids, off, _d), g in zip(batches, grads):
        backward_reference(oracle, plan, ids.cpu(), off.cpu(), g.float().cpu(), rows)
    torch.cuda.synchronize()
    for name, num, _dim in TABLES:
        for st in stores:
            t = st.layouts[st.index[name]]
            gids = t.spec.global_ids(num, st.rank)
            torch.testing.assert_close(st.grad_view(name).cpu(), oracle.grad_view(name)[gids], atol=1e-4, rtol=1e-4)

    # row-wise Adagrad on each owner (gradient scaled by 1/W, the reference's owner-side mean)
    lr, eps = 0.1, oracle.eps
    for st in stores:
        st.step(lr=lr)
    torch.cuda.synchronize()
    for name, num, _dim in TABLES:
        g = oracle.grad_view(name) / world
        touched = g.abs().sum(dim=1) > 0
        acc = oracle.accumulator(name) + torch.where(touched, g.square().mean(dim=1), torch.zeros(num))
        w = oracle.weight(name) - torch.where(touched.unsqueeze(1), lr * g / (acc.sqrt() + eps).unsqueeze(1),
                                              torch.zeros_like(g))
        for st in stores:
            t = st.layouts[st.index[name]]
            gids = t.spec.global_ids(num, st.rank)
            torch.testing.assert_close(st.weight(name).cpu(), w[gids], atol=1e-5, rtol=1e-4)
            torch.testing.assert_close(st.accumulator(name).cpu(), acc[gids], atol=1e-6, rtol=1e-4)
            assert float(st.grad_view(name).abs().sum()) == 0.0  # gradients cleared for the next step
    from mdl_b200.ops._ext import check_error_word

    check_error_word(dev)


@pytest.mark.parametrize("world", [2, 4])
def test_fused_dense_reduce_scatter_update_all_gather(world):
    from torch import nn

    from mdl_b200.ops.dense import DenseParams

    dev = torch.device("cuda", 0)
    peers = EmulatedPeers(world, dev)
    torch.manual_seed(3)
    shapes = {"w1": (256, 512), "b1": (512,), "w2": (512, 96), "b2": (96,)}
    init = {n: torch.randn(*s) * 0.05 for n, s in shapes.items()}
    dps = []
    for r in range(world):
        params = [(n, nn.Parameter(init[n].clone())) for n in shapes]
        dps.append(DenseParams(params, device=dev, bf16_names={"w1", "w2"}, world=world, rank=r, optimizer="adam",
                               lr=1e-3, comm="fused", buckets=[["w2", "b2"], ["w1", "b1"]], peers=peers))
    grads = [torch.randn(dps[0].total, device=dev) for _ in range(world)]
    for dp, g in zip(dps, grads):
        dp.grad.copy_(g)
    for dp in dps:
        dp.update_buckets(lr=1e-3)
    torch.cuda.synchronize()

    # oracle: mean gradient, one Adam step (bias-corrected), fp32
    b1, b2 = dps[0].betas
    g = torch.stack(grads).mean(0)
    m = (1 - b1) * g
    v = (1 - b2) * g * g
    master0 = torch.zeros_like(g)
    for n in shapes:
        o = dps[0].offsets[n]
        master0[o:o + init[n].numel()] = init[n].flatten().to(dev)
    want = master0 - 1e-3 / (1 - b1) * m / (v.sqrt() / (1 - b2) ** 0.5 + dps[0].eps)
    valid = torch.zeros_like(g, dtype=torch.bool)
    for n in shapes:
        o = dps[0].offsets[n]
        valid[o:o + init[n].numel()] = True
    for dp in dps:
        # every rank's bf16 shadow holds the whole updated model
        torch.testing.assert_close(dp.shadow.float()[valid], want[valid].bfloat16().float(), atol=1e-6, rtol=1e-2)
        # the fp32 master of the owned slice of every bucket is updated exactly
        for begin, end, _fp32_from in dp.buckets:
            chunk = (end - begin) // world
            lo, hi = begin + chunk * dp.rank, begin + chunk * (dp.rank + 1)
            sel = valid[lo:hi]
            torch.testing.assert_close(dp.master[lo:hi][sel], want[lo:hi][sel], atol=1e-6, rtol=1e-5)


def test_peer_barrier_wait_runs_out_and_reports():
    """A device barrier whose peer never arrives: the bounded wait gives up after the
    configured limit, the kernel returns and the error word says PEER_TIMEOUT."""

    from mdl_b200.ops._ext import error_word, ext

    dev = torch.device("cuda", 0)
    C = ext()
    err = error_word(dev)
    torch.cuda.synchronize()
    err.zero_()
    signals = torch.zeros(2, 64, dtype=torch.int32, device=dev)  # rank 1's slot stays 0: nobody arrives
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    C.set_barrier_limit(0.005)
    try:
        C.barrier([signals[0].data_ptr(), signals[1].data_ptr()], counter, 0, err)
        torch.cuda.synchronize()
    finally:
        C.set_barrier_limit(10.0)
    value = int(err.item())
    err.zero_()
    assert value & 2, f"error word 0x{value:x} lacks PEER_TIMEOUT"
    # rank 0 did signal itself and its peer
    assert int(signals[0, 0]) == 1 and int(signals[1, 0]) == 1
    # the context is still usable
    assert float(torch.ones(4, device=dev).sum()) == 4.0


def test_mbarrier_wait_runs_out_and_reports():
    from mdl_b200.ops._ext import ext

    dev = torch.device("cuda", 0)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    returned = torch.zeros(1, dtype=torch.int32, device=dev)
    ext().mbar_timeout_selftest(err, returned)
    torch.cuda.synchronize()
    assert int(err.item()) & 1, "MBAR_TIMEOUT not recorded"
    assert int(returned.item()) == 1
    assert float(torch.ones(4, device=dev).sum()) == 4.0
