"""Process-group runtime: backend choice, NCCL environment, control group, checks.

Reference counterparts: ``_resolve_process_group_backend`` / ``_setup_distributed`` /
``_cleanup_distributed`` (``src/train.py:1177-1267``), ``_configure_nccl_runtime_env``
(``:719-795``), ``_validate_sharded_embedding_metadata`` (``:4905-4939``),
``_DDPGraphAuditor`` (``:573-630``) and ``_apply_local_rank_cpu_affinity``
(``:815-850``).

* Backend: NCCL on CUDA ranks; gloo when there is no GPU or when
  ``MDL_DIST_BACKEND=gloo`` forces it. A second, gloo *control group* carries
  host-side votes and object gathers so they never queue behind NCCL kernels.
* NCCL environment (set only where the user has not): asynchronous error
  handling on; when two local GPUs cannot reach each other's memory, NCCL's P2P
  transport is disabled. Buffer sizes and channel counts are left to NCCL: on an
  NVSwitch system every peer has full bandwidth and the communication-bound
  paths of this framework run in its own NVLink kernels, not in NCCL.
* ``validate_shard_metadata``: every rank must agree on each table's shape and
  sharding; one all-gather of the descriptors over the control group.
* ``GradientAuditor``: which dense parameters received no gradient in the first
  steps (parameters that never train, or a graph that changes per step).
* ``set_local_cpu_affinity``: the host cores split evenly between local ranks.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def resolve_backend(device: torch.device) -> str:
    forced = os.environ.get("MDL_DIST_BACKEND", "").strip().lower()
    if forced:
        if forced not in ("nccl", "gloo"):
            raise ValueError(f"MDL_DIST_BACKEND must be nccl or gloo, got {forced!r}")
        return forced
    return "nccl" if device.type == "cuda" else "gloo"


def local_p2p_accessible(n: int | None = None) -> bool:
    """True when every pair of the first ``n`` visible GPUs can address each other's memory."""

    if not torch.cuda.is_available():
        return False
    n = torch.cuda.device_count() if n is None else min(n, torch.cuda.device_count())
    return all(torch.cuda.can_device_access_peer(a, b) for a in range(n) for b in range(n) if a != b)


def configure_nccl_env(local_world: int, env: dict | None = None, p2p_ok: bool | None = None) -> dict:
    """Fill the NCCL variables this runtime relies on (without overriding the user's);
    returns the variables it set."""

    env = os.environ if env is None else env
    applied = {}

    def put(key, value):
        if key not in env:
            env[key] = value
            applied[key] = value

    put("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    if local_world > 1:
        ok = local_p2p_accessible(local_world) if p2p_ok is None else p2p_ok
        if not ok:
            put("NCCL_P2P_DISABLE", "1")
    return applied


class Runtime:
    """Rank coordinates, the main process group and the gloo control group."""

    def __init__(self, rank: int, world: int, local_rank: int, device: torch.device, backend: str,
                 control_group=None) -> None:
        self.rank, self.world, self.local_rank = rank, world, local_rank
        self.device, self.backend = device, backend
        self.control_group = control_group

    @property
    def distributed(self) -> bool:
        return self.world > 1 and dist.is_initialized()


def setup_distributed(device: torch.device, *, timeout_s: float = 600.0, local_world: int | None = None) -> Runtime:
    """Initialise the process group from the launcher's environment (``RANK`` / ``WORLD_SIZE``
    / ``LOCAL_RANK``; rendezvous on ``MASTER_ADDR``, default 127.0.0.1)."""

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    backend = resolve_backend(device)
    if world == 1:
        return Runtime(rank, world, local, device, backend)
    if backend == "nccl":
        configure_nccl_env(local_world or int(os.environ.get("LOCAL_WORLD_SIZE", str(world))))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    timeout = datetime.timedelta(seconds=timeout_s)
    if not dist.is_initialized():
        kw = {"device_id": device} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=timeout, **kw)
    control = dist.new_group(backend="gloo", timeout=timeout) if backend == "nccl" else dist.group.WORLD
    return Runtime(rank, world, local, device, backend, control)


def cleanup_distributed(join_timeout_s: float = 30.0) -> bool:
    """Destroy the process group from a helper thread; False when it did not finish in
    time (a peer died mid-collective), in which case the caller should exit hard."""

    if not dist.is_initialized():
        return True
    import threading

    done = threading.Event()

    def run():
        try:
            dist.destroy_process_group()
        finally:
            done.set()

    threading.Thread(target=run, daemon=True).start()
    return done.wait(join_timeout_s)


def shard_descriptors(store) -> list[tuple]:
    return [(t.name, t.num_embeddings, t.dim, t.spec.strategy, t.spec.world_size, t.spec.cyclic_offset,
             t.spec.table_owner) for t in store.layouts]


def validate_shard_metadata(store, group=None, world: int | None = None) -> None:
    """Raise when the ranks disagree on any table's shape or sharding."""

    world = world or (dist.get_world_size(group) if dist.is_initialized() else 1)
    if world <= 1:
        return
    mine = shard_descriptors(store)
    every = [None] * world
    dist.all_gather_object(every, mine, group=group)
    for r, desc in enumerate(every):
        if desc != every[0]:
            diff = sorted(set(map(str, desc)) ^ set(map(str, every[0])))[:4]
            raise RuntimeError(f"embedding shard metadata differs between rank 0 and rank {r}: {diff}")


class GradientAuditor:
    """Counts, over the first ``steps`` backward passes, how often each dense parameter's
    gradient was non-zero (read from the flat gradient buffer before the update)."""

    def __init__(self, dense, steps: int = 3) -> None:
        self.dense, self.steps = dense, steps
        self.seen = 0
        self.hits = {n: 0 for n in dense.names}

    def observe(self) -> None:
        if self.seen >= self.steps:
            return
        g = self.dense.grad
        for n in self.dense.names:
            o = self.dense.offsets[n]
            if bool(g[o:o + self.dense.params[n].numel()].any()):
                self.hits[n] += 1
        self.seen += 1

    def report(self) -> dict:
        never = sorted(n for n, h in self.hits.items() if h == 0)
        sometimes = sorted(n for n, h in self.hits.items() if 0 < h < self.seen)
        return {"steps": self.seen, "never_updated": never, "intermittent": sometimes,
                "static_graph_safe": not sometimes}


def set_local_cpu_affinity(local_rank: int, local_world: int, cpus: list[int] | None = None,
                           apply: bool = True) -> list[int]:
    """This local rank's contiguous share of the allowed cores (the last rank also takes
    the remainder); pins the process (its data threads included) to it when ``apply``."""

    cpus = sorted(os.sched_getaffinity(0)) if cpus is None else sorted(cpus)
    if local_world <= 1 or len(cpus) < local_world:
        return cpus
    per = len(cpus) // local_world
    end = len(cpus) if local_rank == local_world - 1 else (local_rank + 1) * per
    share = cpus[local_rank * per:end]
    if apply:
        os.sched_setaffinity(0, share)
    return share
