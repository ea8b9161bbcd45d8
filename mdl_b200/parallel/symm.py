"""Symmetric device buffers over CUDA IPC (one process per GPU, one node).

Every rank ``cudaMalloc``'s the same set of named buffers, exports CUDA IPC
handles, exchanges them once with ``torch.distributed.all_gather_object`` and
opens each peer's handle. Kernels then receive the list of per-rank pointers
and address peer HBM directly over NVLink (loads, stores, reductions). The
same object owns a per-rank signal array for the device-side barrier
(``csrc/comm.cu``), so a barrier is a stream-ordered kernel with a bounded wait,
not a host synchronisation.

This replaces the reference's NCCL-only communication layer for the hot paths
(``src/embeddings.py:386-435`` all_to_all, the DDP reducer); NCCL stays for cold
paths (metadata, evaluation histograms).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import error_word, ext

_DTYPE_SIZE = {torch.float32: 4, torch.int32: 4, torch.int64: 8, torch.bfloat16: 2, torch.float16: 2,
               torch.uint8: 1}


class SymmetricBuffers:
    """Named buffers allocated on every rank and mapped by every peer."""

    def __init__(self, spec: dict[str, tuple[int, torch.dtype]], *, device: torch.device, process_group=None) -> None:
        self.device = torch.device(device)
        self.dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.group = process_group
        self.rank = dist.get_rank(process_group)
        self.world = dist.get_world_size(process_group)
        spec = dict(spec)
        spec["__signals"] = (64, torch.int32)
        spec["__scratch"] = (256, torch.float32)
        self.spec = spec
        C = ext()
        self._local_ptrs: dict[str, int] = {}
        handles: dict[str, bytes] = {}
        for name, (numel, dtype) in spec.items():
            nbytes = max(16, int(numel) * _DTYPE_SIZE[dtype])
            nbytes = (nbytes + 255) // 256 * 256
            ptr, handle = C.ipc_alloc(nbytes, self.dev_index)
            self._local_ptrs[name] = ptr
            handles[name] = handle
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, handles, group=process_group)
        self._peer_ptrs: dict[str, list[int]] = {name: [0] * self.world for name in spec}
        self._opened: list[int] = []
        for r in range(self.world):
            for name in spec:
                if r == self.rank:
                    self._peer_ptrs[name][r] = self._local_ptrs[name]
                else:
                    p = C.ipc_open(gathered[r][name], self.dev_index)
                    self._peer_ptrs[name][r] = p
                    self._opened.append(p)
        self._tensors = {name: C.tensor_from_ptr(self._local_ptrs[name], int(numel), dtype, self.dev_index)
                         for name, (numel, dtype) in spec.items()}
        self._tensors["__signals"].zero_()
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        self.barrier_host()

    def local(self, name: str) -> torch.Tensor:
        return self._tensors[name]

    def peer_ptrs(self, name: str) -> list[int]:
        return self._peer_ptrs[name]

    def barrier(self) -> None:
        """Stream-ordered device barrier across all ranks (bounded wait)."""

        ext().barrier(self._peer_ptrs["__signals"], self.counter, self.rank, error_word(self.device))

    def barrier_host(self) -> None:
        dist.barrier(group=self.group)

    def allreduce_small(self, values: torch.Tensor) -> torch.Tensor:
        """Sum a small fp32 vector (<= 256 values) across ranks in place."""

        n = values.numel()
        scratch = self._tensors["__scratch"]
        scratch[:n].copy_(values.flatten())
        self.barrier()
        ext().small_allreduce(self._peer_ptrs["__scratch"], values, n)
        self.barrier()
        return values

    def close(self) -> None:
        C = ext()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            C.ipc_close(p, self.dev_index)
        self._opened = []
        for p in self._local_ptrs.values():
            C.ipc_free(p, self.dev_index)
        self._local_ptrs = {}


class MulticastBuffers:
    """Named buffers of identical size on every rank, in PyTorch symmetric memory,
    with both per-rank pointers (peer loads / stores) and NVSwitch multicast
    addresses (``multimem`` loads with in-switch reduction, multicast stores).

    ``torch.distributed._symmetric_memory`` does the plumbing (physical allocation,
    handle exchange, multicast object); the kernels that use the addresses are this
    library's. Construction raises when the GPUs or the driver offer no multicast,
    and callers fall back to ``SymmetricBuffers``.
    """

    def __init__(self, spec: dict[str, tuple[int, torch.dtype]], *, device: torch.device, process_group=None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.device = torch.device(device)
        self.dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.group = process_group if process_group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if not self.available(self.dev_index):
            raise RuntimeError("no NVSwitch multicast support on this device")
        spec = dict(spec)
        spec["__signals"] = (64, torch.int32)
        spec["__scratch"] = (256, torch.float32)
        self._tensors: dict[str, torch.Tensor] = {}
        self._peer_ptrs: dict[str, list[int]] = {}
        self._mc: dict[str, int] = {}
        self._handles = []
        for name, (numel, dtype) in spec.items():
            n = max(int(numel), 256 // _DTYPE_SIZE[dtype])
            t = symm_mem.empty(n, dtype=dtype, device=self.device)
            h = symm_mem.rendezvous(t, self.group)
            base = list(h.buffer_ptrs)
            off = t.data_ptr() - base[self.rank]
            if off < 0:
                raise RuntimeError(f"symmetric buffer {name}: tensor below its block")
            self._tensors[name] = t
            self._peer_ptrs[name] = [b + off for b in base]
            mc = int(h.multicast_ptr)
            if mc == 0:
                raise RuntimeError(f"symmetric buffer {name}: no multicast address")
            self._mc[name] = mc + off
            self._handles.append(h)
        self._tensors["__signals"].zero_()
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    @staticmethod
    def available(dev_index: int) -> bool:
        try:
            from torch._C._distributed_c10d import _SymmetricMemory

            return bool(_SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, dev_index))
        except Exception:  # noqa: BLE001 - old torch / no symmetric memory: no multicast
            return False

    def local(self, name: str) -> torch.Tensor:
        return self._tensors[name]

    def peer_ptrs(self, name: str) -> list[int]:
        return self._peer_ptrs[name]

    def multicast_ptr(self, name: str) -> int:
        return self._mc[name]

    def barrier(self) -> None:
        ext().barrier(self._peer_ptrs["__signals"], self.counter, self.rank, error_word(self.device))

    def barrier_host(self) -> None:
        dist.barrier(group=self.group)

    def allreduce_small(self, values: torch.Tensor) -> torch.Tensor:
        n = values.numel()
        self._tensors["__scratch"][:n].copy_(values.flatten())
        self.barrier()
        ext().small_allreduce(self._peer_ptrs["__scratch"], values, n)
        self.barrier()
        return values

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        self._handles = []
        self._tensors = {}
