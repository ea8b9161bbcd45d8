"""Packed model-ready batches.

A ``PackedBatch`` holds every input of one step in a handful of tensors:

* ``ids``: int64 ``[n_ids]``, all categorical ids of all scalar features,
  feature-major (feature 0's bags, then feature 1's ...);
* ``offsets``: int64 ``[F * rows + 1]``, CSR bag boundaries into ``ids``
  (dense features have empty bags);
* ``dense``: fp32 ``[rows, dense_width]``;
* ``labels`` / ``label_mask``: fp32 ``[rows, tasks]``; ``scenario_id``: int64 ``[rows]``;
* ``sequences``: optional dict of per-sequence tensors (ids ``[rows, L, fields]``,
  lengths ``[rows]``) for sequence models.

All int64 leaves are views into one flat buffer and all fp32 leaves into
another, so moving a batch to the GPU is two copies from pinned memory
(reference: coalesced H2D ``src/dataloader.py:11586-11790``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class PackedBatch:
    ids: torch.Tensor
    offsets: torch.Tensor
    dense: torch.Tensor | None
    labels: torch.Tensor | None
    label_mask: torch.Tensor | None
    scenario_id: torch.Tensor
    rows: int
    sequences: dict[str, Any] = field(default_factory=dict)
    group_key: torch.Tensor | None = None   # int64 per row: the split's group_id (QAUC / UAUC), hashed
    _flat: tuple = field(default=(), repr=False)

    @property
    def device(self) -> torch.device:
        return self.ids.device

    def nbytes(self) -> int:
        if self._flat:
            return sum(t.numel() * t.element_size() for t in self._flat)
        return sum(t.numel() * t.element_size() for t in self._leaves() if t is not None)

    def _leaves(self) -> list:
        out = [self.ids, self.offsets, self.dense, self.labels, self.label_mask, self.scenario_id, self.group_key]
        for v in self.sequences.values():
            out.extend(v.values() if isinstance(v, dict) else [v])
        return out

    @staticmethod
    def pack(ids, offsets, dense, labels, label_mask, scenario_id, rows, sequences=None, pin: bool = False,
             group_key=None):
        """Build a batch whose leaves are views of one int64 and one fp32 flat buffer."""

        sequences = sequences or {}
        i64_parts = [("ids", ids), ("offsets", offsets), ("scenario_id", scenario_id), ("group_key", group_key)]
        f32_parts = [("dense", dense), ("labels", labels), ("label_mask", label_mask)]
        for name, seq in sequences.items():
            for k, v in seq.items():
                (i64_parts if v.dtype == torch.int64 else f32_parts).append((f"seq:{name}:{k}", v))
        lease = None
        bufs = {}
        if pin:  # both flat buffers from one slot of the pinned pool (returned with the batch)
            from .pinned import default_pool

            specs = [(dt, max(1, sum(p.numel() for _, p in parts if p is not None)))
                     for dt, parts in ((torch.int64, i64_parts), (torch.float32, f32_parts))]
            views, lease = default_pool().checkout(specs)
            bufs = {torch.int64: views[0], torch.float32: views[1]}

        def flat(parts, dtype):
            total = sum(p.numel() for _, p in parts if p is not None)
            buf = bufs[dtype] if pin else torch.empty(max(total, 1), dtype=dtype)
            views = {}
            off = 0
            for name, p in parts:
                if p is None:
                    views[name] = None
                    continue
                n = p.numel()
                buf[off:off + n].copy_(p.reshape(-1).to(dtype))
                views[name] = (off, tuple(p.shape))
                off += n
            return buf, views
        b64, v64 = flat(i64_parts, torch.int64)
        b32, v32 = flat(f32_parts, torch.float32)
        batch = PackedBatch._from_flat(b64, v64, b32, v32, rows)
        batch._lease = lease
        return batch

    @staticmethod
    def _from_flat(b64, v64, b32, v32, rows):
        def view(buf, spec):
            if spec is None:
                return None
            off, shape = spec
            n = 1
            for s in shape:
                n *= s
            return buf[off:off + n].view(shape)
        seqs: dict[str, dict] = {}
        for views, buf in ((v64, b64), (v32, b32)):
            for name, spec in views.items():
                if name.startswith("seq:"):
                    _, sname, key = name.split(":", 2)
                    seqs.setdefault(sname, {})[key] = view(buf, spec)
        batch = PackedBatch(ids=view(b64, v64["ids"]), offsets=view(b64, v64["offsets"]), dense=view(b32, v32["dense"]),
                            labels=view(b32, v32["labels"]), label_mask=view(b32, v32["label_mask"]),
                            scenario_id=view(b64, v64["scenario_id"]), rows=rows, sequences=seqs,
                            group_key=view(b64, v64.get("group_key")))
        batch._flat = (b64, b32)
        batch._views = (v64, v32)
        return batch

    def to(self, device, non_blocking: bool = True) -> "PackedBatch":
        """Two copies (int64 + fp32 flat buffers) instead of one per leaf."""

        if not self._flat:
            return self.pack(self.ids, self.offsets, self.dense, self.labels, self.label_mask, self.scenario_id,
                             self.rows, self.sequences, group_key=self.group_key).to(device, non_blocking)
        b64, b32 = self._flat
        d64 = b64.to(device, non_blocking=non_blocking)
        d32 = b32.to(device, non_blocking=non_blocking)
        lease = getattr(self, "_lease", None)
        if lease is not None and torch.device(device).type == "cuda":
            ev = torch.cuda.Event()
            ev.record()
            lease.fence(ev)  # the pinned slot is reusable once the copies have run
        v64, v32 = self._views
        return PackedBatch._from_flat(d64, v64, d32, v32, self.rows)

    def copy_into(self, dst: "PackedBatch", non_blocking: bool = True) -> "PackedBatch":
        """Copy this (host) batch into a same-layout device batch in place (static buffers for CUDA graphs)."""

        dst._flat[0].copy_(self._flat[0], non_blocking=non_blocking)
        dst._flat[1].copy_(self._flat[1], non_blocking=non_blocking)
        return dst

    def slice_rows(self, start: int, stop: int, num_features: int) -> "PackedBatch":
        """Rows ``[start, stop)`` as a new packed batch (host tensors; ids re-based per feature)."""

        rows = self.rows
        n = stop - start
        off = self.offsets.cpu()
        ids = self.ids.cpu()
        id_parts, len_parts = [], []
        for f in range(num_features):
            seg = off[f * rows + start:f * rows + stop + 1]
            id_parts.append(ids[int(seg[0]):int(seg[-1])])
            len_parts.append(seg[1:] - seg[:-1])
        offsets = torch.zeros(num_features * n + 1, dtype=torch.int64)
        if len_parts:
            offsets[1:] = torch.cumsum(torch.cat(len_parts), 0)
        cut = lambda t: None if t is None else t.cpu()[start:stop].clone()
        seqs = {name: {k: v.cpu()[start:stop].clone() for k, v in seq.items()} for name, seq in self.sequences.items()}
        return PackedBatch.pack(torch.cat(id_parts) if id_parts else torch.zeros(0, dtype=torch.int64), offsets,
                                cut(self.dense), cut(self.labels), cut(self.label_mask), cut(self.scenario_id), n,
                                seqs, group_key=cut(self.group_key))

    def pin_memory(self) -> "PackedBatch":
        if self._flat and self._flat[0].is_pinned():
            return self
        b = self if self._flat else self.pack(self.ids, self.offsets, self.dense, self.labels, self.label_mask,
                                              self.scenario_id, self.rows, self.sequences, group_key=self.group_key)
        b64, b32 = b._flat
        return PackedBatch._from_flat(b64.pin_memory(), b._views[0], b32.pin_memory(), b._views[1], b.rows)
