"""Training step engine shared by ``train``, ``benchmark`` and ``bench.py``.

One ``Trainer`` owns a model, its flat dense parameters (``DenseParams``) and
its embedding store, and runs the reference's optimizer-step semantics
(``train_mdl`` ``src/train.py:6529-7431``, hot loop :6832-7360):

* loss reduction ``sum`` / ``mean_per_task`` / ``mean_per_request_per_task``
  with per-task weights, scaled so that the rank-averaged gradient equals the
  global objective (``_loss_terms_from_batch`` ``src/train.py:5890-6031``);
* LR schedule: linear warmup then constant or cosine (``src/train.py:5495-5512``);
* dense optimizer (RMSprop or Adam) after the gradient average, optional
  global clip (``src/train.py:5745-5826``);
* row-wise Adagrad on the touched embedding rows with the owner-side ``1/W``
  gradient scale and optional global sparse clip;
* gradient accumulation over ``gradient_accumulation_steps`` micro-batches.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..config.schema import AppConfig
from ..ops.dense import DenseParams
from ..utils.trace import trace_range


def lr_multiplier(config: AppConfig, step: int, decay_steps: int | None = None) -> float:
    t = config.training
    warm = t.lr_warmup_steps if t.warmup_steps is None else t.warmup_steps
    if warm > 0 and step <= warm:
        return float(step) / float(warm)
    if t.lr_schedule == "constant":
        return 1.0
    decay = decay_steps if decay_steps is not None else t.lr_decay_steps
    if decay is None:
        raise RuntimeError("cosine lr_schedule requires lr_decay_steps")
    if decay <= warm:
        return min(1.0, float(step) / float(max(warm, 1)))
    progress = min(max(float(step - warm) / float(decay - warm), 0.0), 1.0)
    return t.lr_min_ratio + (1.0 - t.lr_min_ratio) * 0.5 * (1.0 + math.cos(math.pi * progress))


@dataclass
class StepResult:
    loss: torch.Tensor
    logits: torch.Tensor | None = None
    dense_grad_norm: torch.Tensor | None = None
    sparse_grad_norm: torch.Tensor | None = None
    extras: dict = field(default_factory=dict)


class Trainer:
    def __init__(self, config: AppConfig, model, *, device: torch.device, rank: int = 0, world: int = 1,
                 process_group=None) -> None:
        self.config = config
        self.model = model
        self.device = torch.device(device)
        self.rank, self.world, self.group = rank, world, process_group
        t = config.training
        buckets = model.dense_buckets() if hasattr(model, "dense_buckets") else None
        self.dense = DenseParams(
            model.named_parameters(), device=self.device, bf16_names=model.gemm_param_names(), world=world,
            rank=rank, process_group=process_group, optimizer=t.dense_optimizer, lr=t.lr_dense,
            betas=(t.adam_beta1, t.adam_beta2), eps=t.adam_eps if t.dense_optimizer == "adam" else 1e-8,
            weight_decay=t.weight_decay, rmsprop_alpha=t.rmsprop_alpha, comm=t.comm, buckets=buckets)
        self.dense.broadcast_from_rank0()
        # the model reports finished gradient buckets during the backward (overlapped updates)
        model.dense_hooks = self.dense
        self.store = model.store
        names = list(config.task_names)
        self.task_weights = torch.tensor([float(t.task_loss_weights.get(n, 1.0)) for n in names],
                                         dtype=torch.float32, device=self.device)
        self.step_index = 0
        self.micro_index = 0
        from ..ops.moe import moe_modules

        self.moe = moe_modules(model)

    def task_scale(self, batch) -> torch.Tensor:
        """Per-task multiplier of the summed BCE terms (see module docstring)."""

        red = self.config.training.loss_reduction
        W = float(self.world)
        if red == "sum":
            return self.task_weights * W
        if batch.label_mask is None:
            counts = torch.full_like(self.task_weights, float(batch.rows))
            global_counts = counts * W  # equal local batch on every rank
        else:
            counts = batch.label_mask.float().sum(dim=0).to(self.device)
            global_counts = counts.clone()
            if self.world > 1 and dist.is_initialized():
                dist.all_reduce(global_counts, group=self.group)
        scale = torch.where(global_counts > 0, W / global_counts.clamp_min(1.0), torch.zeros_like(global_counts))
        return scale * self.task_weights

    def enable_phase_events(self, on: bool = True) -> None:
        """Record CUDA events between the phases of every step (forward, backward,
        dense update, sparse update); ``phase_ms()`` then gives their device times."""

        self._phase_marks: list | None = [] if on else None

    def _mark(self, name: str) -> None:
        marks = getattr(self, "_phase_marks", None)
        if marks is not None and self.device.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

    def phase_ms(self) -> dict[str, float]:
        """Mean device time of each phase over the recorded steps (synchronizes)."""

        marks = getattr(self, "_phase_marks", None) or []
        torch.cuda.synchronize(self.device)
        sums: dict[str, float] = {}
        counts: dict[str, int] = {}
        for (_n0, e0), (n1, e1) in zip(marks, marks[1:]):
            if n1 == "start":
                continue
            sums[n1] = sums.get(n1, 0.0) + e0.elapsed_time(e1)
            counts[n1] = counts.get(n1, 0) + 1
        self._phase_marks = []
        return {k: sums[k] / counts[k] for k in sums}

    def request_weights(self, batch):
        """``mean_per_request_per_task`` (reference ``_loss_terms_from_batch``
        ``src/train.py:5921-5957``): each request's candidates share one mean per task.

        Returns ``(batch with per-row weights, task_scale)``: the label mask becomes
        ``mask / count(request, task)`` for rows of requests with a labelled candidate,
        and the per-task scale is ``W / global number of such requests`` -- the same
        loss as averaging per request, then over requests, then summing over tasks."""

        import dataclasses

        rows = batch.rows
        ri = None
        for seq in (batch.sequences or {}).values():
            cand = seq.get("row_indices") if isinstance(seq, dict) else None
            if cand is not None and cand.numel() == rows:
                if ri is not None and not torch.equal(ri, cand.to(ri.device)):
                    raise ValueError("request-level loss requires one consistent row_indices mapping")
                ri = cand
        if ri is None:
            raise ValueError("mean_per_request_per_task requires request-deduplicated features with "
                             "candidate-to-request row_indices")
        dev = self.device
        ri = ri.to(dev).long()
        ntask = len(self.config.task_names)
        mask = (batch.label_mask.to(dev).float() if batch.label_mask is not None
                else torch.ones(rows, ntask, device=dev))
        _req, inv = torch.unique(ri, sorted=True, return_inverse=True)
        counts = torch.zeros(_req.numel(), ntask, device=dev).index_add_(0, inv, mask)
        per_row = mask / counts[inv].clamp_min(1.0)
        valid = (counts > 0).float().sum(dim=0)
        if self.world > 1 and dist.is_initialized():
            dist.all_reduce(valid, group=self.group)
        W = float(self.world)
        scale = torch.where(valid > 0, W / valid.clamp_min(1.0), torch.zeros_like(valid)) * self.task_weights
        return dataclasses.replace(batch, label_mask=per_row), scale

    def forward_backward(self, batch) -> dict:
        self._mark("start")
        with trace_range("mdl.forward"):
            if self.config.training.loss_reduction == "mean_per_request_per_task":
                batch, scale = self.request_weights(batch)
            else:
                scale = self.task_scale(batch)
            out = self.model(batch, task_scale=scale)
        self._mark("forward")
        with trace_range("mdl.backward"):
            out["loss"].backward()
        self._mark("backward")
        return out

    def _lrs(self, step: int) -> tuple[float, float]:
        t = self.config.training
        mult = lr_multiplier(self.config, step)
        lr_sparse = t.lr_sparse if t.lr_sparse is not None else t.lr_dense
        return t.lr_dense * mult, lr_sparse * mult

    def optimizer_step(self) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        self.step_index += 1
        t = self.config.training
        lr_dense, lr_sparse = self._lrs(self.step_index)
        if self.moe:
            from ..ops.moe import step_moe_controllers

            step_moe_controllers(self.moe, self.world, self.group)
        with trace_range("mdl.dense_update"):
            dn = self.dense.step(lr=lr_dense, clip_norm=t.dense_clip_norm)
        self._mark("dense_update")
        with trace_range("mdl.sparse_update"):
            sn = self.store.step(lr=lr_sparse, clip_norm=t.sparse_clip_norm)
        self._mark("sparse_update")
        return dn, sn

    def train_step(self, batch) -> StepResult:
        """One micro-batch; runs the optimizers every ``gradient_accumulation_steps`` micro-batches.

        On the last micro-batch of a step the dense update is opened before the
        backward, so buckets whose gradients are final update while the rest of
        the backward runs."""

        t = self.config.training
        final = (self.micro_index + 1) % t.gradient_accumulation_steps == 0
        if final:
            self.dense.begin_step(lr=self._lrs(self.step_index + 1)[0], clip_norm=t.dense_clip_norm)
        out = self.forward_backward(batch)
        self.micro_index += 1
        dn = sn = None
        if final:
            dn, sn = self.optimizer_step()
        return StepResult(loss=out["loss"].detach(), logits=out.get("logits"), dense_grad_norm=dn,
                          sparse_grad_norm=sn)

    def step_from_host(self, host_batch, loss_out: torch.Tensor | None = None) -> StepResult:
        """Public end-to-end step: copy a (pinned) host batch to the device, train, and copy
        the loss back into ``loss_out`` (a pinned host scalar) without a host sync."""

        if self.device.type == "cuda":
            batch = host_batch.to(self.device, non_blocking=True)
        else:
            batch = host_batch
        result = self.train_step(batch)
        if loss_out is not None:
            loss_out.copy_(result.loss.reshape(loss_out.shape), non_blocking=True)
        return result

    def train_from_host(self, host_batches, loss_out: torch.Tensor | None = None) -> int:
        """Public end-to-end loop: train one step per (pinned) host batch, copying batch
        k+1 to the device on a side stream while step k runs, and the loss of step i into
        ``loss_out[i]`` (pinned host) without a host sync. Returns the number of steps."""

        n = 0
        if self.device.type != "cuda":
            for b in host_batches:
                res = self.train_step(b)
                if loss_out is not None:
                    loss_out[n:n + 1].copy_(res.loss.reshape(1))
                n += 1
            return n
        from ..data.parquet import DevicePrefetcher

        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)  # one per trainer (allocator pools)
        for dev in DevicePrefetcher(host_batches, self.device, self._copy_stream):
            res = self.train_step(dev)
            if loss_out is not None:
                loss_out[n:n + 1].copy_(res.loss.reshape(1), non_blocking=True)
            n += 1
        return n

    @torch.no_grad()
    def predict_logits(self, batch) -> torch.Tensor:
        out = self.model(batch, task_scale=self.task_scale(batch))
        return out["logits"].detach()
