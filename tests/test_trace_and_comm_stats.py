"""Profiler ranges, the kernel-class profile summary, and the embedding lookup's
communication statistics (CPU)."""

from types import SimpleNamespace

import torch

from mdl_b200.benchmark.profile_summary import classify, profile_steps
from mdl_b200.ops.embedding import LookupFeature, LookupPlan
from mdl_b200.ops.embedding_stats import BUNDLE_BYTES, EmbeddingCommunicationStats, communication_stats
from mdl_b200.parallel.sharding import EmbeddingShardSpec
from mdl_b200.utils.trace import set_tracing, trace_range, tracing


def test_kernel_classes():
    assert classify("void mdl::dense_sync_kernel<...>") == "communication"
    assert classify("ncclDevKernel_AllReduce_Sum_f32_RING_LL") == "communication"
    assert classify("void mdl::gemm_tcgen05_kernel<false, true, 1, true>") == "gemm"
    assert classify("fmha_fwd_kernel") == "attention"
    assert classify("emb_pool_fwd_kernel") == "embedding"
    assert classify("optim_kernel") == "optimizer"
    assert classify("ln_bwd_kernel<4>") == "normalization"
    assert classify("elementwise_kernel") == "other"


def test_ranges_only_while_profiling():
    assert not tracing()
    with trace_range("mdl.test"):  # no profiler: a no-op context
        pass
    seen = []

    def step():
        with trace_range("mdl.outer"):
            with trace_range("mdl.inner"):
                torch.ones(8).sum()
        seen.append(tracing())

    rep = profile_steps(step, 2, device=torch.device("cpu"), gemm_flops_per_step=1e9)
    assert seen == [True, True]
    assert set(rep["ranges_cpu_ms_per_step"]) == {"mdl.outer", "mdl.inner"}
    assert rep["steps"] == 2 and rep["gemm_flops_per_step"] == 1e9
    set_tracing(True)
    try:
        assert tracing()
    finally:
        set_tracing(False)


def _store(world, rank, num=100, dim=8):
    spec = EmbeddingShardSpec("t", "row_wise", world)
    lay = SimpleNamespace(name="t", num_embeddings=num, dim=dim, spec=spec)
    return SimpleNamespace(world=world, rank=rank, layouts=[lay], index={"t": 0})


def test_comm_stats_bundles_and_bytes():
    # two features on one table, 3 bags each; world 2, rank 0 owns even ids
    plan = LookupPlan(features=[LookupFeature("a", "t", width=8), LookupFeature("b", "t", width=8, out_col=8)],
                      out_width=16)
    rows = 3
    bags = [[2, 3, 5], [4], [0, 7],      # feature a: bag0 {2 local, 3 and 5 -> owner 1}, bag1 local, bag2 {pad, 7}
            [9], [], [6, 8]]             # feature b: bag0 {9 remote}, bag1 empty, bag2 local
    ids = torch.tensor([i for b in bags for i in b])
    offsets = torch.tensor([0] + list(torch.cumsum(torch.tensor([len(b) for b in bags]), 0).tolist()))
    st = communication_stats(_store(2, 0), plan, ids, offsets, rows)["t"]
    assert st.raw_ids == 9 and st.active_ids == 8
    assert st.local_unique_ids == 8
    assert st.remote_ids == 4                  # 3, 5, 7, 9
    assert st.remote_bundles == 3              # (a,bag0,1) with 2 ids, (a,bag2,1), (b,bag0,1)
    assert st.forward_sent_bytes == 3 * BUNDLE_BYTES + 4 * 2
    assert st.forward_received_bytes == 3 * 8 * 4
    assert st.backward_sent_bytes == 3 * 8 * 2
    # one rank: nothing crosses
    one = communication_stats(_store(1, 0), plan, ids, offsets, rows)["t"]
    assert one.remote_ids == 0 and one.total_communication_bytes == 0
    total = EmbeddingCommunicationStats("t")
    total.add_(st)
    total.add_(st)
    assert total.total_communication_bytes == 2 * st.total_communication_bytes
