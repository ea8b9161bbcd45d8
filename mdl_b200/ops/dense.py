"""Flat storage for the dense (data-parallel) parameters of a model.

Every dense ``nn.Parameter`` is re-homed into one flat fp32 *master* buffer;
its gradient lives in one flat fp32 *grad* buffer and, on CUDA, its bf16
*shadow* (the operand the tcgen05 GEMMs read) in one flat bf16 buffer. The
fused kernels write parameter gradients straight into the grad buffer, and one
optimizer kernel (Adam or RMSprop, with the clip factor applied on the fly)
updates master + state + shadow in a single pass. With ``world > 1`` the grad,
master and shadow buffers are symmetric (IPC-mapped by every peer) and the
update is the fused NVLink reduce-scatter / optimizer / all-gather kernel
(``csrc/comm.cu``), bucket by bucket.

Layout: parameters are grouped into *buckets* in the order their gradients
become final in the backward (a model lists them: heads, last block, ...,
first block, tokenizer; everything else forms a last bucket). Within a bucket
the parameters whose consumers read the bf16 shadow (GEMM weights) come first
and the ones read as fp32 (norm scales, biases, head vectors) after the
bucket's ``fp32_from``; every parameter starts on a 32-element boundary and
every bucket on a multiple of 32 x world.

Overlap: between ``begin_step`` and ``step`` the model calls
``bucket_ready(k)`` as soon as bucket k's gradients are final (a ``GradReady``
node in the autograd graph); the bucket's update (with one rank: the
optimizer, fused with zeroing the gradient; with several: barrier + fused
reduce-scatter / optimizer / all-gather) is then issued on a side stream, so it
runs under the rest of the backward.

Reference counterpart: DDP (``src/train.py:5276-5328``) + RMSprop
(``src/train.py:4826-4893``) + dense clipping (``src/train.py:5745-5775``).
"""

from __future__ import annotations

import math
import os
from typing import Iterable

import torch
import torch.distributed as dist
from torch import nn

from ._ext import ext

ALIGN = 32


def _round(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


class DenseParams:
    def __init__(self, named_params: Iterable[tuple[str, nn.Parameter]], *, device: torch.device,
                 bf16_names: set[str] | None = None, world: int = 1, rank: int = 0, process_group=None,
                 optimizer: str = "adam", lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, rmsprop_alpha: float = 0.99, comm: str = "fused",
                 buckets: list[list[str]] | None = None, overlap: bool = False, peers=None) -> None:
        """``peers``: an ``EmulatedPeers`` to lay several ranks out on one GPU (tests of
        the fused multi-rank update); by default ranks are processes joined over CUDA IPC."""

        self.device = torch.device(device)
        self._peers = peers
        self.world, self.rank, self.group = world, rank, process_group
        self.optimizer, self.lr, self.betas, self.eps = optimizer, lr, betas, eps
        self.weight_decay, self.rmsprop_alpha = weight_decay, rmsprop_alpha
        self.comm = comm
        named = list(named_params)
        bf16_names = set(bf16_names or ()) | {n for n, p in named if getattr(p, "_mdl_gemm", False)}
        by_name = {n: p for n, p in named}
        groups: list[list[str]] = []
        seen: set[str] = set()
        for names in buckets or []:
            grp = [n for n in names if n in by_name and n not in seen]
            seen.update(grp)
            if grp:
                groups.append(grp)
        rest = [n for n, _ in named if n not in seen]
        if rest:
            groups.append(rest)
        self.names: list[str] = []
        self.params: dict[str, nn.Parameter] = {}
        self.offsets: dict[str, int] = {}
        self.buckets: list[tuple[int, int, int]] = []  # (begin, end, fp32_from)
        self.bucket_of: dict[str, int] = {}
        off = 0
        for k, grp in enumerate(groups):
            begin = off
            ordered = [n for n in grp if n in bf16_names] + [n for n in grp if n not in bf16_names]
            fp32_from = None
            for n in ordered:
                if n not in bf16_names and fp32_from is None:
                    fp32_from = off
                self.names.append(n)
                self.params[n] = by_name[n]
                self.offsets[n] = off
                self.bucket_of[n] = k
                off += _round(by_name[n].numel())
            off = _round(max(off, begin + ALIGN), ALIGN * max(1, world))
            self.buckets.append((begin, off, off if fp32_from is None else fp32_from))
        self.total = max(off, ALIGN * max(1, world))
        # single-range view used by callers of the whole buffer
        self.fp32_from = self.buckets[0][2] if len(self.buckets) == 1 else 0
        self._alloc()
        with torch.no_grad():
            for name in self.names:
                p = self.params[name]
                o = self.offsets[name]
                self.master[o:o + p.numel()].copy_(p.detach().flatten().to(self.device, torch.float32))
                p.data = self.master[o:o + p.numel()].view_as(p)
                # autograd accumulates plain-PyTorch gradients straight into the flat buffer;
                # fused nodes write the same memory through _mdl_grad
                p.grad = self.grad[o:o + p.numel()].view_as(p)
                p._mdl_grad = self.grad[o:o + p.numel()].view_as(p)
                if self.shadow is not None:
                    p._mdl_shadow = self.shadow[o:o + p.numel()].view_as(p)
        if self.shadow is not None:
            self.refresh_shadow()
        self.step_count = 0
        # Measured on B200 (RankMixer workload, 1 and 2 GPUs): a side-stream update competes with the
        # backward's kernels for SMs and memory bandwidth and the step gets slower (1 GPU 4.62 -> 5.53
        # ms, 2 GPUs 5.08 -> 5.64 ms), so it is opt-in (MDL_B200_DENSE_OVERLAP=1 or overlap=True).
        env = os.environ.get("MDL_B200_DENSE_OVERLAP")
        on = overlap if env is None else env != "0"
        # per-bucket updates average gradients only through the peer buffers; the NCCL path
        # reduces the whole gradient once, in ``step``
        self.overlap = on and self.device.type == "cuda" and (self.world == 1 or self._symm is not None)
        self._active = False
        self._launched: list[bool] = [False] * len(self.buckets)
        self._side = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None

    def _use_multicast(self) -> bool:
        """NVSwitch multicast for the fused update, when every rank has it (collective)."""

        # Measured on B200 (RankMixer workload, step ms, peer loads vs multicast): 2 GPUs 4.87 vs
        # 5.39, 4 GPUs 5.68 vs 5.61, 8 GPUs 6.31 vs 5.98 (dense update 1.57 vs 1.24). Multicast
        # is the default from 4 ranks on; MDL_B200_NVLS=1 / 0 forces it on / off.
        env = os.environ.get("MDL_B200_NVLS")
        if (env != "1") if env is not None else self.world < 4:
            return False
        from ..parallel.symm import MulticastBuffers

        ok = torch.tensor([1 if MulticastBuffers.available(self.device.index if self.device.index is not None else torch.cuda.current_device()) else 0], dtype=torch.int32,
                          device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        return bool(int(ok.item()))

    def _alloc(self) -> None:
        dev = self.device
        n = self.total
        self._symm = None
        self._mc: list[int] = []  # multicast addresses of grad / master / shadow (NVLS path)
        if dev.type == "cuda" and self.world > 1 and self.comm == "fused":
            from ..parallel.symm import SymmetricBuffers

            spec = {"master": (n, torch.float32), "grad": (n, torch.float32), "shadow": (n, torch.bfloat16)}
            if self._peers is not None:
                self._symm = self._peers.buffers("dense", self.rank, spec)
            elif self._use_multicast():
                from ..parallel.symm import MulticastBuffers

                self._symm = MulticastBuffers(spec, device=dev, process_group=self.group)
                self._mc = [self._symm.multicast_ptr(k) for k in ("grad", "master", "shadow")]
            else:
                self._symm = SymmetricBuffers(spec, device=dev, process_group=self.group)
            self.master = self._symm.local("master")
            self.grad = self._symm.local("grad")
            self.shadow = self._symm.local("shadow")
            self.master.zero_()
        else:
            self.master = torch.zeros(n, dtype=torch.float32, device=dev)
            self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
            self.shadow = torch.zeros(n, dtype=torch.bfloat16, device=dev) if dev.type == "cuda" else None
        self.grad.zero_()
        self.state1 = torch.zeros(n, dtype=torch.float32, device=dev)
        self.state2 = torch.zeros(n, dtype=torch.float32, device=dev) if self.optimizer == "adam" else None
        self._sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self._clip = torch.ones(1, dtype=torch.float32, device=dev)

    def refresh_shadow(self) -> None:
        if self.shadow is not None:
            ext().cast_bf16(self.master, self.shadow)

    def zero_grad(self) -> None:
        self.grad.zero_()

    def broadcast_from_rank0(self) -> None:
        """Make every rank start from rank 0's dense weights (DDP init semantics)."""

        if self.world > 1 and dist.is_initialized():
            dist.broadcast(self.master, src=0, group=self.group)
            self.refresh_shadow()

    # ------------------------------------------------------------------ step
    def _hyper(self, lr: float) -> dict:
        b1, b2 = self.betas
        t = self.step_count
        return dict(lr=lr, b1=b1, b2=b2, bc1=1.0 - b1 ** t, bc2=1.0 - b2 ** t, opt=0 if self.optimizer == "adam" else 1)

    def begin_step(self, lr: float | None = None, clip_norm: float | None = None) -> bool:
        """Open an optimizer step whose bucket updates may start during the backward.

        Returns whether overlapping is on (CUDA and no global clipping: the clip factor
        needs every gradient before any update)."""

        self._active = False
        if not self.overlap or clip_norm is not None:
            return False
        self.step_count += 1
        self._h = self._hyper(self.lr if lr is None else lr)
        self._launched = [False] * len(self.buckets)
        self._active = True
        return True

    def bucket_ready(self, k: int) -> None:
        """Bucket k's gradients are final: issue its update on the side stream."""

        if not self._active or self._launched[k]:
            return
        self._launched[k] = True
        cur = torch.cuda.current_stream(self.device)
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            self._update_bucket(k, self._h, max_blocks=self._side_blocks())

    def _side_blocks(self) -> int:
        # a few SMs' worth of 256-thread blocks: enough in flight for NVLink, little HBM pressure
        env = os.environ.get("MDL_B200_SIDE_BLOCKS")
        return int(env) if env else 0

    def _update_bucket(self, k: int, h: dict, max_blocks: int = 0) -> None:
        C = ext()
        begin, end, fp32_from = self.buckets[k]
        scale = 1.0 / self.world
        if self._symm is not None:
            sym = self._symm
            sym.barrier()  # every rank's gradients of this bucket are final
            C.dense_sync(sym.peer_ptrs("grad"), sym.peer_ptrs("master"), sym.peer_ptrs("shadow"), self.state1,
                         self.state2, begin, end, fp32_from, self.rank, h["opt"], h["lr"], h["b1"], h["b2"], self.eps,
                         self.weight_decay, h["bc1"], h["bc2"], self.rmsprop_alpha, scale, None, None, 0, max_blocks,
                         self._mc)
            return
        sl = slice(begin, end)
        shadow = None if self.shadow is None else self.shadow[sl]
        if h["opt"] == 0:
            C.adam(self.master[sl], self.grad[sl], self.state1[sl], self.state2[sl], shadow, h["lr"], h["b1"],
                   h["b2"], self.eps, self.weight_decay, h["bc1"], h["bc2"], scale, None, True, max_blocks)
        else:
            C.rmsprop(self.master[sl], self.grad[sl], self.state1[sl], shadow, h["lr"], self.rmsprop_alpha, self.eps,
                      self.weight_decay, scale, None, True, max_blocks)

    @torch.no_grad()
    def update_buckets(self, lr: float | None = None) -> None:
        """One optimizer step of this rank's buckets without the closing barrier and
        gradient reset of ``step``: with emulated peers the caller issues every rank's
        update, then resets the gradients, in stream order."""

        self.step_count += 1
        h = self._hyper(self.lr if lr is None else lr)
        for k in range(len(self.buckets)):
            self._update_bucket(k, h)

    @torch.no_grad()
    def step(self, lr: float | None = None, clip_norm: float | None = None) -> torch.Tensor | None:
        """Average gradients over ranks and apply the optimizer. Returns the grad norm if clipping.

        After ``begin_step`` this only issues the buckets the backward did not report
        and joins the side stream."""

        if self._active:
            self._active = False
            cur = torch.cuda.current_stream(self.device)
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                for k, done in enumerate(self._launched):
                    if not done:
                        self._update_bucket(k, self._h, max_blocks=0)
                if self._symm is not None:
                    self._symm.barrier()  # no rank reads this rank's gradients any more
                    self.grad.zero_()
            cur.wait_stream(self._side)
            return None
        lr = self.lr if lr is None else lr
        self.step_count += 1
        h = self._hyper(lr)
        if self.device.type != "cuda":
            return self._cpu_step(lr, clip_norm, h["bc1"], h["bc2"])
        C = ext()
        scale = 1.0 / self.world
        norm = None
        if self._symm is not None:
            sym = self._symm
            sym.barrier()
            clip = None
            if clip_norm is not None:
                self._sq.zero_()
                for begin, end, fp32_from in self.buckets:
                    C.dense_sync(sym.peer_ptrs("grad"), sym.peer_ptrs("master"), sym.peer_ptrs("shadow"), self.state1,
                                 self.state2, begin, end, fp32_from, self.rank, h["opt"], lr, h["b1"], h["b2"],
                                 self.eps, self.weight_decay, h["bc1"], h["bc2"], self.rmsprop_alpha, scale, None,
                                 self._sq, 1, 0, self._mc)
                sym.allreduce_small(self._sq)
                C.clip_factor(self._sq, float(clip_norm), self._clip)
                norm = self._sq.sqrt()
                clip = self._clip
            for begin, end, fp32_from in self.buckets:
                C.dense_sync(sym.peer_ptrs("grad"), sym.peer_ptrs("master"), sym.peer_ptrs("shadow"), self.state1,
                             self.state2, begin, end, fp32_from, self.rank, h["opt"], lr, h["b1"], h["b2"], self.eps,
                             self.weight_decay, h["bc1"], h["bc2"], self.rmsprop_alpha, scale, clip, None,
                             2 if clip_norm is not None else 0, 0, self._mc)
            sym.barrier()
            self.grad.zero_()
            return norm
        if self.world > 1 and dist.is_initialized():
            dist.all_reduce(self.grad, group=self.group)  # NCCL baseline path
        clip = None
        if clip_norm is not None:
            self._sq.zero_()
            C.sqnorm(self.grad, scale, self._sq)
            C.clip_factor(self._sq, float(clip_norm), self._clip)
            clip = self._clip
            norm = self._sq.sqrt()
        if h["opt"] == 0:
            C.adam(self.master, self.grad, self.state1, self.state2, self.shadow, lr, h["b1"], h["b2"], self.eps,
                   self.weight_decay, h["bc1"], h["bc2"], scale, clip, True, 0)
        else:
            C.rmsprop(self.master, self.grad, self.state1, self.shadow, lr, self.rmsprop_alpha, self.eps,
                      self.weight_decay, scale, clip, True, 0)
        return norm

    def _cpu_step(self, lr, clip_norm, bc1, bc2):
        g = self.grad
        if self.world > 1 and dist.is_initialized():
            dist.all_reduce(g, group=self.group)
        g = g / self.world
        norm = None
        if clip_norm is not None:
            norm = g.norm()
            g = g * min(1.0, float(clip_norm) / (float(norm) + 1e-6))
        if self.weight_decay:
            g = g + self.weight_decay * self.master
        if self.optimizer == "adam":
            b1, b2 = self.betas
            self.state1.mul_(b1).add_(g, alpha=1 - b1)
            self.state2.mul_(b2).addcmul_(g, g, value=1 - b2)
            denom = (self.state2.sqrt() / math.sqrt(bc2)).add_(self.eps)
            self.master.addcdiv_(self.state1, denom, value=-lr / bc1)
        else:
            a = self.rmsprop_alpha
            self.state1.mul_(a).addcmul_(g, g, value=1 - a)
            self.master.addcdiv_(g, self.state1.sqrt().add_(self.eps), value=-lr)
        self.grad.zero_()
        return norm

    @torch.no_grad()
    def gather(self, buf: torch.Tensor) -> torch.Tensor:
        """``buf`` (master or optimizer state) complete on every rank.

        With the fused NVLink update rank r keeps the authoritative values of its
        slice ``[begin + r * c, begin + (r + 1) * c)`` of every bucket only (peers
        receive the bf16 shadow, plus fp32 for the non-GEMM parameters); this
        all-gathers the owned slices bucket by bucket.
        """

        if self._symm is None or self.world == 1:
            return buf
        full = torch.empty_like(buf)
        for begin, end, _ in self.buckets:
            c = (end - begin) // self.world
            mine = buf[begin + self.rank * c:begin + (self.rank + 1) * c].contiguous()
            dist.all_gather_into_tensor(full[begin:end], mine, group=self.group)
        return full

    def gather_master(self) -> torch.Tensor:
        """The full fp32 master vector on every rank (see ``gather``)."""

        return self.gather(self.master)

    def state_dict(self) -> dict:
        """Parameters by name and optimizer state by name (collective when the update is sharded)."""

        master = self.gather(self.master).detach().cpu()
        s1 = self.gather(self.state1).detach().cpu()
        s2 = None if self.state2 is None else self.gather(self.state2).detach().cpu()

        def by_name(buf):
            return {n: buf[self.offsets[n]:self.offsets[n] + p.numel()].view_as(p).clone()
                    for n, p in self.params.items()}

        return {"params": by_name(master), "state1": by_name(s1), "state2": None if s2 is None else by_name(s2),
                "step": self.step_count, "optimizer": self.optimizer}

    def load_state_dict(self, state: dict) -> None:
        with torch.no_grad():
            for n, v in state["params"].items():
                if n in self.params:
                    o = self.offsets[n]
                    self.master[o:o + v.numel()].copy_(v.flatten().to(self.master.device))
            for key, buf in (("state1", self.state1), ("state2", self.state2)):
                saved = state.get(key)
                if buf is None or not isinstance(saved, dict):
                    continue
                for n, v in saved.items():
                    if n in self.params:
                        o = self.offsets[n]
                        buf[o:o + v.numel()].copy_(v.flatten().to(buf.device))
            if "step" in state:
                self.step_count = int(state["step"])
        self.refresh_shadow()


class GradReadyFn(torch.autograd.Function):
    """Identity whose backward tells ``DenseParams`` that bucket ``k`` is final.

    Placed on the input of a module: autograd reaches this node's backward only
    after the module's backward (which wrote its parameter gradients) has run.
    """

    @staticmethod
    def forward(ctx, x, dense, k):
        ctx.dense, ctx.k = dense, k
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        ctx.dense.bucket_ready(ctx.k)
        return g, None, None


def grad_ready(x: torch.Tensor, dense: "DenseParams | None", k: int) -> torch.Tensor:
    if dense is None or not x.requires_grad:
        return x
    return GradReadyFn.apply(x, dense, k)
