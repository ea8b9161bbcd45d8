"""Pinned host buffer pool: slot reuse, growth, shrink against the recent high-water mark,
copies fenced by an event, and packed batches drawing from the pool (CPU; pinning itself
needs CUDA and is skipped here, the bookkeeping is the same)."""

import gc

import torch

from mdl_b200.data.pinned import PinnedPool


class _Ev:
    def __init__(self):
        self.done = False

    def query(self):
        return self.done


def test_reuse_grow_and_shrink():
    pool = PinnedPool(max_free=2, recent_window=8, shrink_factor=2.0)
    (a, b), lease = pool.checkout([(torch.int64, 100), (torch.float32, 50)])
    assert a.numel() == 100 and b.dtype == torch.float32
    lease.release()
    (a2, _), lease2 = pool.checkout([(torch.int64, 90), (torch.float32, 40)])
    assert pool.reuses == 1 and a2.data_ptr() == a.data_ptr()      # same slab lent again
    lease2.release()
    (a3, _), lease3 = pool.checkout([(torch.int64, 1000), (torch.float32, 40)])
    assert pool.grows == 1 and a3.numel() == 1000
    lease3.release()
    # a run of small requests: the big slab exceeds 2x the recent high-water mark and is dropped
    for _ in range(10):
        _, l = pool.checkout([(torch.int64, 10), (torch.float32, 10)])
        l.release()
    assert pool.shrinks >= 1
    assert pool.stats()["free_slots"] <= 2


def test_fenced_slot_waits_for_its_copy():
    pool = PinnedPool()
    (a, _), lease = pool.checkout([(torch.int64, 64), (torch.float32, 8)])
    ev = _Ev()
    lease.fence(ev)
    lease.release()
    (b, _), l2 = pool.checkout([(torch.int64, 64), (torch.float32, 8)])
    assert b.data_ptr() != a.data_ptr() and pool.stats()["pending_slots"] == 1   # copy still running
    l2.release()
    ev.done = True
    (c, _), l3 = pool.checkout([(torch.int64, 64), (torch.float32, 8)])
    assert pool.stats()["pending_slots"] == 0
    l3.release()


def test_lease_returns_when_the_batch_is_collected():
    from mdl_b200.data.batch import PackedBatch
    from mdl_b200.data.pinned import default_pool

    pool = default_pool()
    before = pool.checkouts
    ids = torch.arange(10)
    b = PackedBatch.pack(ids, torch.tensor([0, 10]), None, torch.zeros(1, 1), None, torch.zeros(1, dtype=torch.int64),
                         1, pin=True)
    assert pool.checkouts == before + 1 and torch.equal(b.ids, ids)
    free = pool.stats()["free_slots"]
    del b
    gc.collect()
    assert pool.stats()["free_slots"] >= min(free + 1, pool.max_free)
