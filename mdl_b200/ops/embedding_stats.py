"""Per-table communication statistics of the multi-rank embedding lookup.

Counterpart of the reference's ``EmbeddingCommunicationStats`` (``src/embeddings.py:198-240``),
which counts the ids and bytes of its id / embedding all-to-alls. The lookup here moves
different objects, so the counters follow its own traffic (``ops/embedding.py``):

* forward, requester side: one 16-byte descriptor per (bag, remote owner) bundle plus the
  4-byte local row of every id of a multi-row bundle go to the owner; the owner adds one
  pooled fp32 vector per bundle into the requester's accumulator over NVLink;
* backward: the owner reads one bf16 d(out) slice per bundle from the requester.

Bytes are counted from this rank's batch (sent = what leaves this rank as requester,
received = what arrives here as requester). ``collective=True`` adds the owner-side
view, ``received_ids``: ids other ranks route to this rank (one all-reduce of a
``[W, tables]`` count matrix). Computed on demand from the batch with tensor ops,
outside the fused lookup kernels, so the hot path carries no counters.
"""

from __future__ import annotations

from dataclasses import dataclass, fields

import torch
import torch.distributed as dist

BUNDLE_BYTES = 16  # four int32 per routed (bag, owner) bundle


@dataclass
class EmbeddingCommunicationStats:
    table_name: str
    raw_ids: int = 0
    active_ids: int = 0
    local_unique_ids: int = 0
    remote_ids: int = 0            # active ids owned by another rank
    remote_bundles: int = 0        # (bag, owner) bundles routed to another rank
    received_ids: int = 0          # ids other ranks route to this rank (collective only)
    forward_sent_bytes: int = 0
    forward_received_bytes: int = 0
    backward_sent_bytes: int = 0
    backward_received_bytes: int = 0

    @property
    def total_communication_bytes(self) -> int:
        return (self.forward_sent_bytes + self.forward_received_bytes + self.backward_sent_bytes
                + self.backward_received_bytes)

    def add_(self, other: "EmbeddingCommunicationStats") -> None:
        if other.table_name != self.table_name:
            raise ValueError("cannot add communication stats of different tables")
        for f in fields(self):
            if f.name != "table_name":
                setattr(self, f.name, getattr(self, f.name) + getattr(other, f.name))

    def as_dict(self) -> dict:
        d = {f.name: getattr(self, f.name) for f in fields(self)}
        d["total_communication_bytes"] = self.total_communication_bytes
        return d


@torch.no_grad()
def communication_stats(store, plan, ids: torch.Tensor, offsets: torch.Tensor, rows: int, *,
                        collective: bool = False, group=None) -> dict[str, EmbeddingCommunicationStats]:
    """Statistics of one lookup of ``plan`` over the CSR batch ``ids`` / ``offsets``
    (``rows`` bags per feature), keyed by table name."""

    from .embedding import _hash_ids

    W, rank = int(store.world), int(store.rank)
    out: dict[str, EmbeddingCommunicationStats] = {}
    uniq: dict[str, list[torch.Tensor]] = {}
    sent_to = torch.zeros(W, max(1, len(store.layouts)), dtype=torch.int64)
    off = offsets.long()
    for i, f in enumerate(plan.features):
        if f.table is None:
            continue
        t = store.layouts[store.index[f.table]]
        src = plan.src_of(i)
        lo, hi = int(off[src * rows]), int(off[(src + 1) * rows])
        block = _hash_ids(ids[lo:hi].long(), f)
        lengths = off[src * rows + 1:(src + 1) * rows + 1] - off[src * rows:(src + 1) * rows]
        bag = torch.repeat_interleave(torch.arange(rows, device=lengths.device), lengths)
        active = (block > 0) & (block < t.num_embeddings)
        s = out.setdefault(f.table, EmbeddingCommunicationStats(f.table))
        s.raw_ids += int(block.numel())
        s.active_ids += int(active.sum())
        a_ids, a_bag = block[active], bag[active]
        uniq.setdefault(f.table, []).append(a_ids)
        owner = t.spec.owner(a_ids)
        remote = owner != rank
        s.remote_ids += int(remote.sum())
        if W > 1 and bool(remote.any()):
            key = a_bag[remote] * W + owner[remote]
            bundle, per_bundle = torch.unique(key, return_counts=True)
            nb = int(bundle.numel())
            multi_ids = int(per_bundle[per_bundle > 1].sum())
            s.remote_bundles += nb
            s.forward_sent_bytes += nb * BUNDLE_BYTES + 4 * multi_ids
            s.forward_received_bytes += nb * t.dim * 4
            s.backward_sent_bytes += nb * t.dim * 2
            counts = torch.bincount(owner[remote].cpu(), minlength=W)
            sent_to[:, store.index[f.table]] += counts
    for name, parts in uniq.items():
        out[name].local_unique_ids = int(torch.unique(torch.cat(parts)).numel()) if parts else 0
    if collective and W > 1:
        dev = ids.device if (ids.is_cuda and dist.get_backend(group) == "nccl") else torch.device("cpu")
        m = sent_to.to(dev)
        dist.all_reduce(m, group=group)
        for name, s in out.items():
            s.received_ids = int(m[rank, store.index[name]])
    return out
