"""Several ranks of the NVLink symmetric-memory runtime inside one process, on one GPU.

``EmulatedPeers(world, device)`` stands in for the set of processes that
``SymmetricBuffers`` connects: every emulated rank allocates its named buffers on
the same device and each rank's pointer list names all ranks' buffers, exactly as
the IPC-mapped lists do across processes. The multi-rank kernels (owner-push
lookup, owner-pull gradient, fused dense reduce-scatter / optimizer / all-gather)
therefore run unchanged; what differs is that the caller issues each phase of the
protocol for every rank in turn on one stream, where separate processes would meet
at a device barrier. Barriers are no-ops here: stream order already separates the
phases, and a spin-wait between launches on one GPU is never used (two waiting
kernels on one device are not guaranteed to run at the same time).

This is how the multi-rank kernels are tested on a single GPU; a real multi-GPU
run uses ``SymmetricBuffers`` over CUDA IPC.
"""

from __future__ import annotations

import torch


class EmulatedBuffers:
    """One emulated rank's view of a named buffer set (the ``SymmetricBuffers`` API)."""

    def __init__(self, peers: "EmulatedPeers", key, rank: int) -> None:
        self._peers = peers
        self._key = key
        self.rank = rank
        self.world = peers.world
        self.device = peers.device

    def local(self, name: str) -> torch.Tensor:
        return self._peers._sets[self._key][self.rank][name]

    def peer_ptrs(self, name: str) -> list[int]:
        ranks = self._peers._sets[self._key]
        missing = [r for r in range(self.world) if r not in ranks]
        if missing:
            raise RuntimeError(f"emulated buffers {self._key!r}: ranks {missing} have not allocated yet")
        return [ranks[r][name].data_ptr() for r in range(self.world)]

    def barrier(self) -> None:  # phases are separated by stream order
        pass

    def barrier_host(self) -> None:
        pass

    def allreduce_small(self, values: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError("emulated peers issue ranks one after another; a cross-rank "
                                  "reduction inside one rank's call cannot complete")

    def close(self) -> None:
        pass


class EmulatedPeers:
    def __init__(self, world: int, device: torch.device, *, exchange_ids: int = 0, exchange_rows: int = 0) -> None:
        """``exchange_ids`` / ``exchange_rows``: the per-rank id and row counts the lookup
        staging is sized for (processes agree on them with an all-reduce at first use)."""

        self.world = int(world)
        self.device = torch.device(device)
        self.exchange_ids = int(exchange_ids)
        self.exchange_rows = int(exchange_rows)
        self._sets: dict = {}

    def buffers(self, key, rank: int, spec: dict[str, tuple[int, torch.dtype]]) -> EmulatedBuffers:
        ranks = self._sets.setdefault(key, {})
        if rank in ranks:
            raise RuntimeError(f"emulated buffers {key!r} of rank {rank} allocated twice")
        # 256-byte aligned like the IPC allocations (every tensor starts its own allocation)
        ranks[rank] = {name: torch.zeros(max(int(n), 1), dtype=dt, device=self.device) for name, (n, dt) in spec.items()}
        return EmulatedBuffers(self, key, rank)
