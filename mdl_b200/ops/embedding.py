"""Sharded embedding tables and the fused embedding-bag lookup.

``EmbeddingStore`` keeps the local shard of every table of a model in one fp32
*slab* per rank (plus the fp32 gradient slab, the row-wise Adagrad
accumulator and one touched-row byte flag per local row). With one rank the
lookup is one kernel that gathers, pools and writes the tokenizer input. With
``world > 1`` (CUDA) every random row access stays on the owner's own HBM
(owner-push, ``csrc/embedding.cu``): each rank routes its bags into per-(bag, owner)
bundles in peer-visible staging; after a device barrier every owner gathers and
pools the rows of the bundles routed to it and adds one pooled vector per bundle
into the requester's fp32 accumulator over NVLink; in the backward every owner
reads each bundle's bf16 output-gradient slice from its requester once and adds it
into its own gradient rows, marking them for the row-wise Adagrad update.

``LookupPlan`` describes one batched lookup: which features, their tables,
pooling and where each pooled result lands in the output matrix (including the
per-token slice padding of the RankMixer tokenizer input).

Reference behaviour reproduced here:
* ownership / local rows (``src/embeddings.py:163-353``), per-table seeded
  ``normal(0, init_std)`` init with the padding row zeroed
  (``src/embeddings.py:724-749``);
* padding id 0 contributes nothing and gets no gradient; ``mean`` pooling
  excludes id 0 (``src/model.py:509-678``); ``sum`` pooling is an addition;
* owner-side gradient = sum over requesters divided by W
  (``src/embeddings.py:615-674``), then row-wise Adagrad (``src/optim.py:31-62``).

On CPU (tests, the gloo plumbing config) the same semantics run in PyTorch;
cross-rank rows are exchanged with ``all_gather`` collectives.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from hashlib import sha256
from typing import Sequence

import torch
import torch.distributed as dist

from ..parallel.sharding import EmbeddingShardingPlan, EmbeddingShardSpec
from ..utils.trace import trace_range
from ._ext import error_word, ext

POOL_NONE, POOL_MEAN, POOL_SUM = 0, 1, 2
HASH_NONE, HASH_PREHASHED = 0, 1


@dataclass
class TableLayout:
    name: str
    num_embeddings: int
    dim: int
    spec: EmbeddingShardSpec
    local_rows: int
    base: int = 0       # element offset in the slab
    row_base: int = 0   # offset in the row space


def table_seed(name: str) -> int:
    return int.from_bytes(sha256(name.encode("utf-8")).digest()[:8], "little")


class EmbeddingStore:
    """All local table shards of one rank, plus sparse optimizer state."""

    def __init__(self, tables: Sequence[tuple[str, int, int]], plan: EmbeddingShardingPlan, *, rank: int,
                 world: int, device: torch.device, init_std: float = 0.02, lr: float = 0.01, eps: float = 1e-10,
                 initial_accumulator_value: float = 0.1,
                 process_group=None, base_seed: int | None = None, optimizer: str = "rowwise",
                 lr_decay: float = 0.0, replicas: int = 1, replica_group=None, peers=None) -> None:
        """``world`` / ``rank`` describe the table sharding; ``replicas > 1`` makes every
        rank of ``replica_group`` hold a full copy (``world == 1``) whose touched-row
        gradients are summed across the replicas before each update.
        ``optimizer``: ``rowwise`` (one accumulator per row) or ``full`` (one per element,
        ``torch.optim.Adagrad`` semantics); ``lr_decay`` gives ``lr / (1 + (step - 1) * lr_decay)``.
        ``peers``: an ``EmulatedPeers`` to lay several ranks out on one GPU (tests of the
        multi-rank kernels); by default ranks are processes joined over CUDA IPC."""

        if optimizer not in ("rowwise", "full"):
            raise ValueError(f"sparse optimizer layout {optimizer!r}")
        if replicas > 1 and world != 1:
            raise ValueError("replicated tables are laid out as one shard (world 1)")
        self.rank = rank
        self.world = world
        self.device = torch.device(device)
        self.lr = lr
        self.eps = eps
        self.full = optimizer == "full"
        self.lr_decay = float(lr_decay)
        self.replicas = int(replicas)
        self.replica_group = replica_group
        self.process_group = process_group
        self._peers = peers
        self.layouts: list[TableLayout] = []
        self.index: dict[str, int] = {}
        elem = 0
        rows = 0
        for name, num, dim in tables:
            spec = plan.tables[name]
            local = spec.local_rows(num, rank)
            layout = TableLayout(name, int(num), int(dim), spec, local, base=elem, row_base=rows)
            self.index[name] = len(self.layouts)
            self.layouts.append(layout)
            elem += ((local * dim + 3) // 4) * 4  # keep each table 16-byte aligned
            rows += local
        self.total_elems = max(elem, 4)
        self.total_rows = max(rows, 1)
        # Every rank's layout (local row counts differ per rank): kernels that reach a
        # peer's slab must use the OWNER's table bases.
        self.base_all: list[list[int]] = []
        self.row_base_all: list[list[int]] = []
        for r in range(world):
            e = rw = 0
            bases, rbases = [], []
            for name, num, dim in tables:
                local = plan.tables[name].local_rows(int(num), r)
                bases.append(e)
                rbases.append(rw)
                e += ((local * int(dim) + 3) // 4) * 4
                rw += local
            self.base_all.append(bases)
            self.row_base_all.append(rbases)
        self._peer_handles: list = []
        self._alloc()
        self.reset_parameters(init_std, base_seed)
        self.acc.fill_(initial_accumulator_value)
        self._meta_cache: dict = {}
        self.step_count = 0
        self.sync_peers()

    def sync_peers(self) -> None:
        """Make this rank's table writes visible before any peer reads them (W > 1 on CUDA)."""

        if self._symm is not None:
            torch.cuda.synchronize(self.device)
            self._symm.barrier_host()

    # ------------------------------------------------------------ storage
    def _alloc(self) -> None:
        dev = self.device
        flag_len = (self.total_rows + 511) // 512 * 512  # the Adagrad scan reads 512 flags per warp
        if dev.type == "cuda" and self.world > 1:
            from ..parallel import symm

            spec = {
                "slab": (self.total_elems, torch.float32),
                "grad": (self.total_elems, torch.float32),
                "flags": (flag_len, torch.uint8),
            }
            if self._peers is not None:
                self._symm = self._peers.buffers("store", self.rank, spec)
            else:
                self._symm = symm.SymmetricBuffers(spec, device=dev, process_group=self.process_group)
            self.slab = self._symm.local("slab")
            self.grad = self._symm.local("grad")
            self.flags = self._symm.local("flags")
            self.grad.zero_()
            self.flags.zero_()
            torch.cuda.synchronize(dev)
            self._symm.barrier_host()
        else:
            self._symm = None
            self.slab = torch.empty(self.total_elems, dtype=torch.float32, device=dev)
            self.grad = torch.zeros(self.total_elems, dtype=torch.float32, device=dev)
            self.flags = torch.zeros(flag_len, dtype=torch.uint8, device=dev)
        self.acc = torch.empty(self.total_elems if self.full else self.total_rows, dtype=torch.float32, device=dev)
        # touched-row list rebuilt every step from the flags (CUDA): the update then walks
        # only those rows, each with coalesced 16-byte lanes
        self.touched_list = (torch.empty(max(self.total_rows, 1), dtype=torch.int32, device=dev)
                             if dev.type == "cuda" else None)
        self.touched_count = torch.zeros(1, dtype=torch.int32, device=dev) if dev.type == "cuda" else None
        self._exchanges: dict = {}  # multi-rank lookup staging per plan
        self.max_dim = max((t.dim for t in self.layouts), default=4)
        # CPU path: dense gradient accumulation per table (sparse rows tracked by a mask)
        self._cpu_touched = torch.zeros(self.total_rows, dtype=torch.bool) if dev.type != "cuda" else None

    def weight(self, name: str) -> torch.Tensor:
        """View of the local shard of table ``name`` as ``[local_rows, dim]``."""

        t = self.layouts[self.index[name]]
        return self.slab[t.base:t.base + t.local_rows * t.dim].view(t.local_rows, t.dim)

    def grad_view(self, name: str) -> torch.Tensor:
        t = self.layouts[self.index[name]]
        return self.grad[t.base:t.base + t.local_rows * t.dim].view(t.local_rows, t.dim)

    def accumulator(self, name: str) -> torch.Tensor:
        """``[local_rows]`` (row-wise) or ``[local_rows, dim]`` (full) Adagrad sums."""

        t = self.layouts[self.index[name]]
        if self.full:
            return self.acc[t.base:t.base + t.local_rows * t.dim].view(t.local_rows, t.dim)
        return self.acc[t.row_base:t.row_base + t.local_rows]

    @torch.no_grad()
    def reset_parameters(self, init_std: float, base_seed: int | None = None) -> None:
        """Per-table seeded normal init, padding row (id 0) zeroed on its owner."""

        seed0 = torch.initial_seed() if base_seed is None else int(base_seed)
        for t in self.layouts:
            if t.local_rows == 0:
                continue
            w = self.weight(t.name)
            seed = (seed0 + table_seed(t.name) + self.rank * 104729) % (2 ** 63 - 1)
            gen = torch.Generator(device=w.device)
            gen.manual_seed(seed)
            w.normal_(0.0, init_std, generator=gen)
            if t.spec.owner_of(0) == self.rank:
                w[0 if t.spec.strategy == "table_wise" else 0 // self.world].zero_()

    # ------------------------------------------------------------ metadata
    def table_meta(self) -> dict[str, torch.Tensor]:
        key = "tables"
        meta = self._meta_cache.get(key)
        if meta is None:
            L = self.layouts
            dev = self.device
            meta = {
                "t_base": torch.tensor([t.base for t in L] or [0], dtype=torch.int64, device=dev),
                "t_row_base": torch.tensor([t.row_base for t in L] or [0], dtype=torch.int64, device=dev),
                "t_dim": torch.tensor([t.dim for t in L] or [4], dtype=torch.int32, device=dev),
                "t_mode": torch.tensor([0 if t.spec.strategy == "row_wise" else 1 for t in L] or [0],
                                       dtype=torch.int32, device=dev),
                "t_cyc": torch.tensor([t.spec.cyclic_offset for t in L] or [0], dtype=torch.int32, device=dev),
                "t_owner": torch.tensor([t.spec.table_owner or 0 for t in L] or [0], dtype=torch.int32, device=dev),
                "t_rows": torch.tensor([t.num_embeddings for t in L] or [1], dtype=torch.int64, device=dev),
                "t_base_all": torch.tensor([b for r in self.base_all for b in r] or [0] * self.world,
                                           dtype=torch.int64, device=dev),
                "t_row_base_all": torch.tensor([b for r in self.row_base_all for b in r] or [0] * self.world,
                                               dtype=torch.int64, device=dev),
            }
            self._meta_cache[key] = meta
        return meta

    def peer_ptrs(self, name: str) -> list[int]:
        if self._symm is not None:
            return self._symm.peer_ptrs(name)
        return [getattr(self, name).data_ptr()]

    # ------------------------------------------------------------ optimizer
    @torch.no_grad()
    def step(self, lr: float | None = None, clip_norm: float | None = None) -> torch.Tensor | None:
        """Adagrad (row-wise or full) on every row touched since the last step.

        Returns the (pre-clip) global sparse gradient norm when ``clip_norm`` is set.
        """

        lr = self.lr if lr is None else lr
        self.step_count += 1
        if self.lr_decay:
            lr = lr / (1.0 + (self.step_count - 1) * self.lr_decay)
        grad_scale = 1.0 / self.world
        if self.replicas > 1:
            self._sync_replicas()
            grad_scale = 1.0 / self.replicas
        if self.device.type != "cuda":
            return self._cpu_step(lr, grad_scale, clip_norm)
        m = self.table_meta()
        if self._symm is not None:
            self._symm.barrier()  # every rank finished pushing gradients
        clip = None
        norm = None
        max_dim = max((t.dim for t in self.layouts), default=4)
        C = ext()
        C.compact_touched(self.flags, self.total_rows, self.touched_list, self.touched_count)
        if clip_norm is not None:
            sq = torch.zeros(1, dtype=torch.float32, device=self.device)
            C.touched_sqnorm(self.grad, self.flags, self.total_rows, m["t_base"], m["t_row_base"], m["t_dim"],
                             grad_scale, sq, self.touched_list, self.touched_count, max_dim)
            if self._symm is not None:
                self._symm.allreduce_small(sq)
            elif self.world > 1:
                dist.all_reduce(sq, group=self.process_group)
            clip = torch.empty(1, dtype=torch.float32, device=self.device)
            ext().clip_factor(sq, float(clip_norm), clip)
            norm = sq.sqrt()
        C.adagrad_apply(self.slab, self.grad, self.acc, self.flags, self.total_rows, m["t_base"], m["t_row_base"],
                        m["t_dim"], float(lr), float(self.eps), grad_scale, clip, error_word(self.device), max_dim,
                        self.touched_list, self.touched_count, self.full)
        if self._symm is not None:
            self._symm.barrier()  # updated rows visible before any peer reads them
        return norm

    def _cpu_step(self, lr: float, grad_scale: float, clip_norm: float | None):
        if self.world > 1 and dist.is_initialized():
            # gradients were accumulated only for owned rows (see _cpu_backward); nothing to exchange
            pass
        touched = self._cpu_touched.nonzero().flatten()
        norm = None
        scale = grad_scale
        if clip_norm is not None:
            sq = torch.zeros(1)
            for t in self.layouts:
                rows = touched[(touched >= t.row_base) & (touched < t.row_base + t.local_rows)] - t.row_base
                if rows.numel():
                    sq += (self.grad_view(t.name)[rows] * grad_scale).square().sum()
            if self.world > 1 and dist.is_initialized():
                dist.all_reduce(sq, group=self.process_group)
            norm = sq.sqrt()
            scale = grad_scale * min(1.0, float(clip_norm) / (float(norm) + 1e-6))
        for t in self.layouts:
            rows = touched[(touched >= t.row_base) & (touched < t.row_base + t.local_rows)] - t.row_base
            if rows.numel() == 0:
                continue
            g = self.grad_view(t.name)[rows] * scale
            acc = self.accumulator(t.name)
            w = self.weight(t.name)
            if self.full:
                acc[rows] += g.square()
                w[rows] -= lr * g / (acc[rows].sqrt() + self.eps)
            else:
                acc[rows] += g.square().mean(dim=1)
                w[rows] -= lr * g / (acc[rows].sqrt() + self.eps).unsqueeze(1)
            self.grad_view(t.name)[rows] = 0.0
        self._cpu_touched.zero_()
        return norm

    # ------------------------------------------------------------ replicas
    def _row_elems(self, rows: torch.Tensor):
        """Element index ``[n, max_dim]`` of each row-space index and its column mask."""

        m = self.table_meta()
        rb = m["t_row_base"].to(rows.device)
        t = torch.searchsorted(rb, rows, right=True) - 1
        dim = m["t_dim"].to(rows.device).long()[t]
        base = m["t_base"].to(rows.device)[t] + (rows - rb[t]) * dim
        col = torch.arange(self.max_dim, device=rows.device)
        mask = col.view(1, -1) < dim.view(-1, 1)
        idx = torch.where(mask, base.view(-1, 1) + col.view(1, -1), torch.zeros_like(base).view(-1, 1))
        return idx, mask

    def _touched_rows(self) -> torch.Tensor:
        if self.device.type == "cuda":
            return self.flags[:self.total_rows].nonzero().flatten()
        return self._cpu_touched.nonzero().flatten()

    def _sync_replicas(self) -> None:
        """Sum the touched-row gradients of every replica into every replica (reference
        ``_ReplicatedSparseGradientSynchronizer`` ``src/train.py:5026-5255``).

        Rows and values are all-gathered (padded to the largest count); every rank then
        reduces the same gathered data in the same order (rows sorted stably, each row's
        contributions added in rank order), so the replicas stay bit-identical."""

        W, group = self.replicas, self.replica_group
        rows = self._touched_rows()
        idx, mask = self._row_elems(rows)
        vals = self.grad[idx] * mask
        dev = rows.device
        n = torch.tensor([rows.numel()], dtype=torch.int64, device=dev)
        counts = [torch.zeros_like(n) for _ in range(W)]
        dist.all_gather(counts, n, group=group)
        cap = max(int(c.item()) for c in counts)
        if cap == 0:
            return
        prow = torch.full((cap,), -1, dtype=torch.int64, device=dev)
        prow[:rows.numel()] = rows
        pval = torch.zeros(cap, self.max_dim, dtype=torch.float32, device=dev)
        pval[:rows.numel()] = vals
        all_rows = [torch.empty_like(prow) for _ in range(W)]
        all_vals = [torch.empty_like(pval) for _ in range(W)]
        dist.all_gather(all_rows, prow, group=group)
        dist.all_gather(all_vals, pval, group=group)
        r = torch.cat(all_rows)
        v = torch.cat(all_vals)
        keep = r >= 0
        r, v = r[keep], v[keep]
        r_sorted, order = torch.sort(r, stable=True)
        v = v[order]
        uniq, cnt = torch.unique_consecutive(r_sorted, return_counts=True)
        starts = torch.cumsum(cnt, 0) - cnt
        total = torch.zeros(uniq.numel(), self.max_dim, dtype=torch.float32, device=dev)
        for k in range(W):
            sel = cnt > k
            total[sel] += v[starts[sel] + k]
        uidx, umask = self._row_elems(uniq)
        self.grad[uidx[umask]] = total[umask]
        if self.device.type == "cuda":
            self.flags[uniq] = 1
        else:
            self._cpu_touched[uniq] = True

    def state_dict(self) -> dict:
        return {
            "tables": {
                t.name: {
                    "weight": self.weight(t.name).detach().cpu().clone(),
                    "sum": self.accumulator(t.name).detach().cpu().clone(),
                    "num_embeddings": t.num_embeddings,
                    "embedding_dim": t.dim,
                    "shard_spec": {"table_name": t.spec.table_name, "strategy": t.spec.strategy,
                                   "world_size": t.spec.world_size, "cyclic_offset": t.spec.cyclic_offset,
                                   "table_owner": t.spec.table_owner},
                }
                for t in self.layouts
            },
            "step": self.step_count,
        }


# ====================================================================== lookup plan
@dataclass
class LookupFeature:
    name: str
    table: str | None          # None -> dense feature
    pooling: int = POOL_NONE
    hash_mode: int = HASH_NONE
    buckets: int = 0
    width: int = 0
    out_col: int = 0
    dense_col: int = 0
    src: int = -1              # feature index in the batch CSR (-1: the feature's own plan index)


@dataclass
class LookupPlan:
    """A batched lookup writing ``[rows, out_ld]`` bf16 (feature columns concatenated).

    ``slice_k``/``slice_stride`` remap logical column ``c`` to
    ``(c // slice_k) * slice_stride + c % slice_k`` so per-token input slices
    of a per-token projection can be padded to a 16-byte multiple (TMA rule).
    """

    features: list[LookupFeature]
    out_width: int               # logical width
    slice_k: int = 0
    slice_stride: int = 0
    dense_width: int = 0
    zero_fill: bool = False      # output has columns no feature writes (must read as zero)
    written_width: int = 0       # logical columns the features write (0: all of out_width)
    _meta: dict = field(default_factory=dict)

    @property
    def out_ld(self) -> int:
        if self.slice_k:
            return (self.out_width + self.slice_k - 1) // self.slice_k * self.slice_stride
        return self.out_width

    def _split(self, f: "LookupFeature") -> int:
        """Columns of ``f`` before its next slice boundary (-1: it crosses more than one)."""

        if not self.slice_k:
            return 1 << 30
        split = self.slice_k - f.out_col % self.slice_k
        return split if f.width <= split + self.slice_k else -1

    def src_of(self, i: int) -> int:
        s = self.features[i].src
        return i if s < 0 else s

    @property
    def num_src(self) -> int:
        """Batch features (CSR blocks) the plan reads."""

        return max((self.src_of(i) for i, f in enumerate(self.features) if f.table is not None), default=-1) + 1

    def zero_unwritten(self, out: torch.Tensor) -> None:
        """Zero the output columns no feature writes (they must read as zero): only the
        per-token slice padding (a few columns per slice, strided) when that is all,
        else the whole matrix (``zero_fill``: reserved summary columns, group padding)."""

        if self.zero_fill:
            out.zero_()
            return
        if not self.slice_k or (self.out_ld == self.out_width and not self.written_width):
            return
        T, K, P = self.out_ld // self.slice_stride, self.slice_k, self.slice_stride
        o3 = out.view(out.shape[0], T, P)
        if P > K:
            o3[:, :, K:].zero_()
        w = self.written_width or self.out_width
        for t in range(w // K, T):  # logical columns past the written ones
            start = max(w - t * K, 0)
            if start < K:
                o3[:, t, start:K].zero_()

    def phys_col(self, c: int) -> int:
        return (c // self.slice_k) * self.slice_stride + c % self.slice_k if self.slice_k else c

    def device_meta(self, store: EmbeddingStore, rows: int) -> tuple[list[torch.Tensor], int]:
        key = (rows, store.device)
        cached = self._meta.get(key)
        if cached is not None:
            return cached
        dev = store.device
        F = len(self.features)
        chunk_prefix = [0]
        bag_prefix = [0]
        lanes_list = []
        for f in self.features:
            lanes = 1
            while lanes * 4 < f.width and lanes < 32:
                lanes *= 2
            if f.width > 4 * lanes * 8:
                raise ValueError(f"feature {f.name}: width {f.width} exceeds the lookup kernel limit")
            lanes_list.append(lanes)
            # one warp per chunk of 32 bags of one feature (csrc/embedding.cu kChunkBags)
            chunk_prefix.append(chunk_prefix[-1] + (rows + 31) // 32)
            bag_prefix.append(bag_prefix[-1] + rows)
        tm = store.table_meta()
        i32 = lambda xs: torch.tensor(xs, dtype=torch.int32, device=dev)
        i64 = lambda xs: torch.tensor(xs, dtype=torch.int64, device=dev)
        meta = [
            i64(chunk_prefix),
            i64(bag_prefix),
            i32([store.index[f.table] if f.table is not None else -1 for f in self.features]),
            i32([f.pooling for f in self.features]),
            i32([f.hash_mode for f in self.features]),
            i64([max(f.buckets, 1) for f in self.features]),
            i32([f.width for f in self.features]),
            i32(lanes_list),
            i64([0] * F),
            i64([self.out_ld] * F),
            i32([f.out_col for f in self.features]),
            i32([self.slice_k] * F),
            i32([self.slice_stride] * F),
            i32([f.dense_col for f in self.features]),
            tm["t_base"], tm["t_row_base"], tm["t_dim"], tm["t_mode"], tm["t_cyc"], tm["t_owner"], tm["t_rows"],
            tm["t_base_all"], tm["t_row_base_all"],
            i64([self.src_of(i) * rows for i in range(F)]),
            i32([self.phys_col(f.out_col) for f in self.features]),
            i32([self._split(f) for f in self.features]),
        ]
        max_vec = max([(f.width + 4 * ln - 1) // (4 * ln) for f, ln in zip(self.features, lanes_list)] or [1])
        result = (meta, chunk_prefix[-1], max_vec)
        self._meta[key] = result
        return result


# ====================================================================== torch reference path
def _hash_ids(ids: torch.Tensor, f: LookupFeature) -> torch.Tensor:
    if f.hash_mode == HASH_PREHASHED:
        return torch.where(ids == 0, torch.zeros_like(ids), (ids & (f.buckets - 1)) + 1)
    return ids


def _gather_rows_cpu(store: EmbeddingStore, table: str, ids: torch.Tensor) -> torch.Tensor:
    """Rows for global ids (any owner); id 0 and out-of-range ids give zeros."""

    t = store.layouts[store.index[table]]
    out = torch.zeros(ids.numel(), t.dim, dtype=torch.float32)
    if store.world == 1 or not dist.is_initialized():
        valid = (ids > 0) & (ids < t.num_embeddings)
        local = t.spec.local_row_ids(ids[valid])
        out[valid] = store.weight(table)[local].float()
        return out
    # gather every rank's request ids, answer the owned ones, sum the answers
    group = store.process_group
    counts = [torch.zeros(1, dtype=torch.int64) for _ in range(store.world)]
    dist.all_gather(counts, torch.tensor([ids.numel()], dtype=torch.int64), group=group)
    cap = int(max(c.item() for c in counts))
    padded = torch.zeros(cap, dtype=torch.int64)
    padded[:ids.numel()] = ids
    all_ids = [torch.zeros(cap, dtype=torch.int64) for _ in range(store.world)]
    dist.all_gather(all_ids, padded, group=group)
    answers = []
    for r in range(store.world):
        req = all_ids[r]
        ans = torch.zeros(cap, t.dim, dtype=torch.float32)
        owner = t.spec.owner(req)
        mine = (owner == store.rank) & (req > 0) & (req < t.num_embeddings)
        if mine.any():
            ans[mine] = store.weight(table)[t.spec.local_row_ids(req[mine])].float()
        answers.append(ans)
    stacked = torch.stack(answers)  # [W, cap, dim]: my answers for every rank
    # reduce-scatter by hand: everyone sums everyone's answers for rank r
    total = stacked.clone()
    dist.all_reduce(total, group=group)
    return total[store.rank, :ids.numel()]


def _push_grads_cpu(store: EmbeddingStore, table: str, ids: torch.Tensor, grads: torch.Tensor) -> None:
    t = store.layouts[store.index[table]]
    valid = (ids > 0) & (ids < t.num_embeddings)
    if store.world == 1 or not dist.is_initialized():
        ids_v = ids[valid]
        local = t.spec.local_row_ids(ids_v)
        store.grad_view(table).index_add_(0, local, grads[valid].float())
        store._cpu_touched[t.row_base + local] = True
        return
    group = store.process_group
    counts = [torch.zeros(1, dtype=torch.int64) for _ in range(store.world)]
    dist.all_gather(counts, torch.tensor([ids.numel()], dtype=torch.int64), group=group)
    cap = int(max(c.item() for c in counts))
    pid = torch.zeros(cap, dtype=torch.int64)
    pid[:ids.numel()] = torch.where(valid, ids, torch.zeros_like(ids))
    pg = torch.zeros(cap, t.dim, dtype=torch.float32)
    pg[:ids.numel()] = grads.float()
    all_ids = [torch.zeros(cap, dtype=torch.int64) for _ in range(store.world)]
    all_g = [torch.zeros(cap, t.dim, dtype=torch.float32) for _ in range(store.world)]
    dist.all_gather(all_ids, pid, group=group)
    dist.all_gather(all_g, pg, group=group)
    for r in range(store.world):
        req = all_ids[r]
        mine = (t.spec.owner(req) == store.rank) & (req > 0)
        if mine.any():
            local = t.spec.local_row_ids(req[mine])
            store.grad_view(table).index_add_(0, local, all_g[r][mine])
            store._cpu_touched[t.row_base + local] = True


def lookup_reference(store: EmbeddingStore, plan: LookupPlan, ids: torch.Tensor, offsets: torch.Tensor,
                     dense: torch.Tensor | None, rows: int, out_dtype=torch.float32) -> torch.Tensor:
    """PyTorch definition of the fused lookup (CPU path and test oracle)."""

    out = torch.zeros(rows, plan.out_ld, dtype=torch.float32, device=ids.device)
    cols = torch.tensor([plan.phys_col(c) for c in range(plan.out_width)], dtype=torch.long)
    logical = torch.zeros(rows, plan.out_width, dtype=torch.float32)
    for fi, f in enumerate(plan.features):
        if f.table is None:
            logical[:, f.out_col:f.out_col + f.width] = dense[:, f.dense_col:f.dense_col + f.width].float().cpu()
            continue
        si = plan.src_of(fi)
        beg = offsets[si * rows:(si + 1) * rows + 1].cpu()
        lengths = beg[1:] - beg[:-1]
        flat = ids[int(beg[0]):int(beg[-1])].cpu()
        flat = _hash_ids(flat, f)
        bag = torch.repeat_interleave(torch.arange(rows), lengths)
        t = store.layouts[store.index[f.table]]
        valid = (flat > 0) & (flat < t.num_embeddings)
        if f.pooling == POOL_NONE:
            # first valid id of each bag
            first = torch.full((rows,), -1, dtype=torch.long)
            idx = torch.arange(flat.numel())
            cand = torch.where(valid, idx, torch.full_like(idx, flat.numel() + 1))
            firsts = torch.full((rows,), flat.numel() + 1, dtype=torch.long).scatter_reduce(0, bag, cand, "amin")
            keep = torch.zeros(flat.numel(), dtype=torch.bool)
            ok = firsts <= flat.numel() - 1
            keep[firsts[ok]] = True
            valid = valid & keep
        rows_v = _gather_rows_cpu(store, f.table, torch.where(valid, flat, torch.zeros_like(flat)))
        pooled = torch.zeros(rows, t.dim).index_add_(0, bag, rows_v * valid.unsqueeze(1).float())
        if f.pooling == POOL_MEAN:
            cnt = torch.zeros(rows).index_add_(0, bag, valid.float()).clamp_min(1.0)
            pooled = pooled / cnt.unsqueeze(1)
        logical[:, f.out_col:f.out_col + t.dim] = pooled
    out[:, cols] = logical.to(out.device)
    return out.to(out_dtype)


def backward_reference(store: EmbeddingStore, plan: LookupPlan, ids: torch.Tensor, offsets: torch.Tensor,
                       grad_out: torch.Tensor, rows: int) -> None:
    cols = torch.tensor([plan.phys_col(c) for c in range(plan.out_width)], dtype=torch.long)
    g_logical = grad_out.float().cpu()[:, cols]
    for fi, f in enumerate(plan.features):
        if f.table is None:
            continue
        si = plan.src_of(fi)
        beg = offsets[si * rows:(si + 1) * rows + 1].cpu()
        lengths = beg[1:] - beg[:-1]
        flat = _hash_ids(ids[int(beg[0]):int(beg[-1])].cpu(), f)
        bag = torch.repeat_interleave(torch.arange(rows), lengths)
        t = store.layouts[store.index[f.table]]
        valid = (flat > 0) & (flat < t.num_embeddings)
        if f.pooling == POOL_NONE:
            idx = torch.arange(flat.numel())
            cand = torch.where(valid, idx, torch.full_like(idx, flat.numel() + 1))
            firsts = torch.full((rows,), flat.numel() + 1, dtype=torch.long).scatter_reduce(0, bag, cand, "amin")
            keep = torch.zeros(flat.numel(), dtype=torch.bool)
            ok = firsts <= flat.numel() - 1
            keep[firsts[ok]] = True
            valid = valid & keep
        g = g_logical[:, f.out_col:f.out_col + t.dim]
        if f.pooling == POOL_MEAN:
            cnt = torch.zeros(rows).index_add_(0, bag, valid.float()).clamp_min(1.0)
            g = g / cnt.unsqueeze(1)
        per_id = g[bag] * valid.unsqueeze(1).float()
        _push_grads_cpu(store, f.table, torch.where(valid, flat, torch.zeros_like(flat)), per_id)


# ====================================================================== autograd op
class _Exchange:
    """Peer-visible staging of one lookup plan's traffic across ranks (CUDA, world > 1).

    Holds this rank's routed bundles (per owner: at most one per bag and
    feature), the owner-local row lists of multi-row bundles, their counts, the
    fp32 accumulator owners add pooled rows into, and the bf16 output gradient
    owners read back. Sizes are agreed on once (collectively) from the first
    batch; row lists hold twice the largest id count of any rank.
    """

    def __init__(self, store: "EmbeddingStore", plan: "LookupPlan", rows: int, n_ids: int) -> None:
        from ..parallel.symm import SymmetricBuffers

        dev = store.device
        peers = store._peers
        if peers is not None:  # emulated ranks: sizes given up front
            t = torch.tensor([max(n_ids, peers.exchange_ids), max(rows, peers.exchange_rows)], dtype=torch.int64)
        else:
            t = torch.tensor([n_ids, rows], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=store.process_group)
        if max((lay.local_rows for lay in store.layouts), default=0) >= 2 ** 31:
            raise ValueError("owner-push lookup keeps 32-bit local row indices")
        if len(plan.features) >= 2 ** 16:
            raise ValueError("owner-push lookup packs the feature index in 16 bits")
        W = store.world
        self.rows_cap = int(t[1])
        self.cap_bundles = max(1, len(plan.features) * self.rows_cap)
        self.cap_rows = 2 * int(t[0]) + 4096
        self.n_out = (self.rows_cap * plan.out_ld + 7) // 8 * 8
        spec = {"bundles": (W * self.cap_bundles * 4, torch.int32), "rows": (W * self.cap_rows, torch.int32),
                "counts": (16, torch.int32), "acc": (self.n_out, torch.float32),
                "grad": (self.n_out, torch.bfloat16)}
        if peers is not None:
            self.symm = peers.buffers(("exchange", len(store._exchanges)), store.rank, spec)
        else:
            self.symm = SymmetricBuffers(spec, device=dev, process_group=store.process_group)
        self.counts = self.symm.local("counts")
        self.acc = self.symm.local("acc")
        self.grad = self.symm.local("grad")

    def ptrs(self) -> tuple[list[int], list[int], list[int], int, int]:
        s = self.symm
        return s.peer_ptrs("bundles"), s.peer_ptrs("rows"), s.peer_ptrs("counts"), self.cap_bundles, self.cap_rows


class _FusedLookup(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, store, plan, ids, offsets, dense, rows):
        ctx.store, ctx.plan, ctx.rows = store, plan, rows
        ctx.save_for_backward(ids, offsets)
        if plan.num_src * rows + 1 > offsets.numel():
            raise ValueError(f"lookup plan reads {plan.num_src} batch features; offsets hold {offsets.numel()}")
        if ids.is_cuda and store.world > 1:
            return _owner_forward(store, plan, ids, offsets, dense, rows)
        if ids.is_cuda:
            meta, chunks, max_vec = plan.device_meta(store, rows)
            out = torch.empty(rows, plan.out_ld, dtype=torch.bfloat16, device=ids.device)
            plan.zero_unwritten(out)
            with trace_range("mdl.embedding.lookup"):
                ext().emb_forward(meta, store.peer_ptrs("slab"), store.rank, ids, offsets, dense,
                                  plan.dense_width, out, chunks, error_word(ids.device), max_vec)
            return out
        return lookup_reference(store, plan, ids, offsets, dense, rows, out_dtype=torch.float32)

    @staticmethod
    def backward(ctx, grad_out):
        ids, offsets = ctx.saved_tensors
        store, plan, rows = ctx.store, ctx.plan, ctx.rows
        if ids.is_cuda and store.world > 1:
            _owner_backward(store, plan, ids, offsets, grad_out, rows)
        elif ids.is_cuda:
            meta, chunks, max_vec = plan.device_meta(store, rows)
            g = grad_out if grad_out.dtype == torch.bfloat16 else grad_out.to(torch.bfloat16)
            ext().emb_backward(meta, store.peer_ptrs("slab"), store.peer_ptrs("grad"), store.peer_ptrs("flags"),
                               store.rank, ids, offsets, g.contiguous(), chunks, error_word(ids.device), max_vec)
        else:
            backward_reference(store, plan, ids, offsets, grad_out, rows)
        return (None,) * 7


def _exchange(store: EmbeddingStore, plan: LookupPlan, ids: torch.Tensor, rows: int) -> _Exchange:
    ex = store._exchanges.get(id(plan))
    if ex is None:
        ex = _Exchange(store, plan, rows, ids.numel())
        store._exchanges[id(plan)] = ex
    if rows > ex.rows_cap or ids.numel() > ex.cap_rows:
        raise RuntimeError(f"batch of {rows} rows / {ids.numel()} ids exceeds the lookup exchange sized for "
                           f"{ex.rows_cap} rows / {ex.cap_rows} ids")
    return ex


def owner_route(store, plan, ids, offsets, dense, rows) -> _Exchange:
    """Owner-push lookup, phase 1 (this rank as requester): zero this rank's
    accumulator and route its bags into per-(bag, owner) bundles in each owner's
    staging (dense columns are written into the accumulator directly)."""

    C = ext()
    ex = _exchange(store, plan, ids, rows)
    meta, chunks, max_vec = plan.device_meta(store, rows)
    ex.counts.zero_()
    ex.acc[:rows * plan.out_ld].zero_()
    bundles, row_lists, counts, capb, capr = ex.ptrs()
    C.emb_route(meta, store.peer_ptrs("slab"), store.rank, ids, offsets, bundles, row_lists, counts, capb, capr,
                ex.acc, dense, plan.dense_width, chunks, error_word(ids.device), max_vec)
    return ex


def owner_push(store, plan, ids, offsets, rows) -> None:
    """Phase 2 (this rank as owner; every rank has routed): gather and pool the rows
    of every bundle routed to this rank from local HBM and add each pooled vector
    into its requester's accumulator over NVLink."""

    ex = _exchange(store, plan, ids, rows)
    meta, _chunks, _max_vec = plan.device_meta(store, rows)
    bundles, row_lists, counts, capb, capr = ex.ptrs()
    ext().emb_owner_forward(meta, store.peer_ptrs("slab"), store.rank, ids, offsets, bundles, row_lists, counts, capb,
                            capr, ex.symm.peer_ptrs("acc"), store.max_dim, error_word(ids.device))


def owner_collect(store, plan, ids, rows) -> torch.Tensor:
    """Phase 3 (every owner has pushed): the accumulator as the bf16 lookup output."""

    ex = _exchange(store, plan, ids, rows)
    out = torch.empty(rows, plan.out_ld, dtype=torch.bfloat16, device=ids.device)
    ext().emb_acc_to_bf16(ex.acc, out)
    return out


def owner_stage_grad(store, plan, ids, grad_out, rows) -> None:
    """Backward, phase 1 (this rank as requester): stage d(out) in peer-visible memory."""

    ex = _exchange(store, plan, ids, rows)
    g = grad_out if grad_out.dtype == torch.bfloat16 else grad_out.to(torch.bfloat16)
    ex.grad[:g.numel()].copy_(g.reshape(-1))


def owner_pull_grad(store, plan, ids, offsets, rows) -> None:
    """Backward, phase 2 (this rank as owner; every requester has staged): read each
    bundle's d(out) slice from its requester once and add it into every local row of
    the bundle, marking the rows touched for the sparse optimizer."""

    ex = _exchange(store, plan, ids, rows)
    meta, _chunks, _max_vec = plan.device_meta(store, rows)
    bundles, row_lists, counts, capb, capr = ex.ptrs()
    ext().emb_owner_backward(meta, store.peer_ptrs("slab"), store.peer_ptrs("grad"), store.peer_ptrs("flags"),
                             store.rank, ids, offsets, bundles, row_lists, counts, capb, capr,
                             ex.symm.peer_ptrs("grad"), store.max_dim, error_word(ids.device))


def _owner_forward(store, plan, ids, offsets, dense, rows):
    """Multi-rank lookup: route (bag, owner) bundles, owners push pooled vectors back."""

    with trace_range("mdl.embedding.route"):
        ex = owner_route(store, plan, ids, offsets, dense, rows)
        ex.symm.barrier()  # every rank's bundles routed, every accumulator zeroed
    with trace_range("mdl.embedding.owner_push"):
        owner_push(store, plan, ids, offsets, rows)
        ex.symm.barrier()  # every owner's vectors have landed
    with trace_range("mdl.embedding.collect"):
        return owner_collect(store, plan, ids, rows)


def _owner_backward(store, plan, ids, offsets, grad_out, rows):
    """Multi-rank gradient: owners pull each requester's d(out) slices into their own grad rows."""

    with trace_range("mdl.embedding.stage_grad"):
        owner_stage_grad(store, plan, ids, grad_out, rows)
        ex = _exchange(store, plan, ids, rows)
        ex.symm.barrier()  # every requester's gradient staged
    with trace_range("mdl.embedding.owner_pull_grad"):
        owner_pull_grad(store, plan, ids, offsets, rows)
        ex.symm.barrier()  # bundles / staged gradients may be overwritten after this point


def fused_lookup(store: EmbeddingStore, plan: LookupPlan, ids: torch.Tensor, offsets: torch.Tensor,
                 dense: torch.Tensor | None, rows: int, anchor: torch.Tensor) -> torch.Tensor:
    """Pooled lookup of all plan features -> ``[rows, plan.out_ld]`` (bf16 on CUDA, fp32 on CPU).

    ``anchor`` is any tensor with ``requires_grad=True``; it only makes autograd
    call the backward, which pushes gradients into the store's gradient slab.
    """

    return _FusedLookup.apply(anchor, store, plan, ids, offsets, dense, rows)
