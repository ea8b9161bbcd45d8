"""Task heads with the fused last layer + BCE loss.

``TaskHeads`` holds one two-layer tower per task (reference ``TaskHead``
``src/model.py:869-882``: ``Linear(D, Hh) -> act -> Dropout -> Linear(Hh, 1)``),
stacked over tasks so that all towers run as one grouped GEMM. Input is one
``D``-vector per (sample, task): ``x [B, ntask, D]`` (MDL task tokens) or a
shared vector broadcast to every task.

CUDA: grouped GEMM with a GELU/ReLU epilogue, then one kernel for the last
layer, the masked BCE loss and its gradient (``head_bce``); the backward is two
grouped GEMMs plus a column sum. CPU: the same math in PyTorch.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..ops._ext import ext
from ..ops.gemm import ACT_GELU, ACT_RELU, bgemm
from ..ops.layers import _grad, _kaiming_uniform_, _shadow, gemm_param


class TaskHeadsBCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, labels, mask, task_scale, relu):
        B, nt, D = x.shape
        Hh = w2.shape[1]
        dev = x.device
        x = x.contiguous()
        pre = torch.empty(B, nt * Hh, dtype=torch.bfloat16, device=dev)
        act = torch.empty_like(pre)
        if relu:
            bgemm(x, _shadow(w1), act, M=B, N=Hh, K=D, G=nt, lda=nt * D, gsA=D, ldb=D, gsB=Hh * D, ldc=nt * Hh,
                  gsC=Hh, bias=b1, gs_bias=Hh, act=ACT_RELU)
            pre = act
        else:
            bgemm(x, _shadow(w1), pre, M=B, N=Hh, K=D, G=nt, lda=nt * D, gsA=D, ldb=D, gsB=Hh * D, ldc=nt * Hh,
                  gsC=Hh, out2=act, bias=b1, gs_bias=Hh, act=ACT_GELU)
        logits = torch.empty(B, nt, dtype=torch.float32, device=dev)
        loss = torch.zeros(1, dtype=torch.float32, device=dev)
        ext().head_bce(act, pre, w2, b2, labels, mask, task_scale, logits, loss, None, None, None, B, nt, Hh,
                       bool(relu))
        ctx.save_for_backward(x, pre, act, labels, mask if mask is not None else labels.new_empty(0), task_scale)
        ctx.meta = (w1, b1, w2, b2, relu, mask is not None)
        ctx.mark_non_differentiable(logits)
        return loss.reshape(()), logits

    @staticmethod
    def backward(ctx, dloss, _dlogits):
        x, pre, act, labels, mask, task_scale = ctx.saved_tensors
        w1, b1, w2, b2, relu, has_mask = ctx.meta
        B, nt, D = x.shape
        Hh = w2.shape[1]
        scale = task_scale * dloss.reshape(1).to(torch.float32)
        dpre = torch.empty_like(act)
        C = ext()
        C.head_bce(act, pre, w2, b2, labels, mask if has_mask else None, scale, None, None, dpre, _grad(w2), _grad(b2),
                   B, nt, Hh, bool(relu))
        C.colsum(dpre, _grad(b1).reshape(-1), 1, B, nt * Hh, nt * Hh, 0, 1.0)
        # dW1[t] += dpre_t^T @ x_t
        bgemm(dpre, x, _grad(w1), M=Hh, N=D, K=B, G=nt, lda=nt * Hh, gsA=Hh, a_mn=True, ldb=nt * D, gsB=D,
              b_mn=True, ldc=D, gsC=Hh * D, accumulate=True)
        dx = torch.empty(B, nt, D, dtype=torch.bfloat16, device=x.device)
        bgemm(dpre, _shadow(w1), dx, M=B, N=D, K=Hh, G=nt, lda=nt * Hh, gsA=Hh, ldb=D, gsB=Hh * D, b_mn=True,
              ldc=nt * D, gsC=D)
        return dx, None, None, None, None, None, None, None, None


class SharedInputHeadsBCEFn(torch.autograd.Function):
    """Every task reads the same ``x [B, D]`` (row stride ``x.stride(0)``): the
    first layers of all towers are one GEMM against the stacked ``w1``."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, labels, mask, task_scale, relu):
        B, D = x.shape
        nt, Hh = w2.shape
        dev = x.device
        lda = x.stride(0)
        pre = torch.empty(B, nt * Hh, dtype=torch.bfloat16, device=dev)
        act = torch.empty_like(pre)
        w1s = _shadow(w1).reshape(nt * Hh, D)
        if relu:
            bgemm(x, w1s, act, M=B, N=nt * Hh, K=D, lda=lda, ldb=D, ldc=nt * Hh, bias=b1.reshape(-1), act=ACT_RELU)
            pre = act
        else:
            bgemm(x, w1s, pre, M=B, N=nt * Hh, K=D, lda=lda, ldb=D, ldc=nt * Hh, out2=act, bias=b1.reshape(-1),
                  act=ACT_GELU)
        logits = torch.empty(B, nt, dtype=torch.float32, device=dev)
        loss = torch.zeros(1, dtype=torch.float32, device=dev)
        ext().head_bce(act, pre, w2, b2, labels, mask, task_scale, logits, loss, None, None, None, B, nt, Hh,
                       bool(relu))
        ctx.save_for_backward(x, pre, act, labels, mask if mask is not None else labels.new_empty(0), task_scale)
        ctx.meta = (w1, b1, w2, b2, relu, mask is not None)
        ctx.mark_non_differentiable(logits)
        return loss.reshape(()), logits

    @staticmethod
    def backward(ctx, dloss, _dlogits):
        x, pre, act, labels, mask, task_scale = ctx.saved_tensors
        w1, b1, w2, b2, relu, has_mask = ctx.meta
        B, D = x.shape
        nt, Hh = w2.shape
        scale = task_scale * dloss.reshape(1).to(torch.float32)
        dpre = torch.empty_like(act)
        C = ext()
        C.head_bce(act, pre, w2, b2, labels, mask if has_mask else None, scale, None, None, dpre, _grad(w2), _grad(b2),
                   B, nt, Hh, bool(relu))
        C.colsum(dpre, _grad(b1).reshape(-1), 1, B, nt * Hh, nt * Hh, 0, 1.0)
        bgemm(dpre, x, _grad(w1).reshape(nt * Hh, D), M=nt * Hh, N=D, K=B, lda=nt * Hh, a_mn=True, ldb=x.stride(0),
              b_mn=True, ldc=D, accumulate=True)
        dx = torch.empty(B, D, dtype=torch.bfloat16, device=x.device)
        bgemm(dpre, _shadow(w1).reshape(nt * Hh, D), dx, M=B, N=D, K=nt * Hh, lda=nt * Hh, ldb=D, b_mn=True, ldc=D)
        return dx, None, None, None, None, None, None, None, None


class TaskHeads(nn.Module):
    def __init__(self, num_tasks: int, input_dim: int, hidden_dim: int, activation: str = "gelu", device=None):
        super().__init__()
        nt, D, Hh = num_tasks, input_dim, hidden_dim
        self.num_tasks, self.input_dim, self.hidden_dim = nt, D, Hh
        self.relu = activation == "relu"
        self.w1 = gemm_param(torch.empty(nt, Hh, D, device=device))
        self.b1 = nn.Parameter(torch.empty(nt, Hh, device=device))
        self.w2 = nn.Parameter(torch.empty(nt, Hh, device=device))
        self.b2 = nn.Parameter(torch.empty(nt, device=device))
        for t in range(nt):
            _kaiming_uniform_(self.w1.data[t], D)
            _kaiming_uniform_(self.b1.data[t], D)
            _kaiming_uniform_(self.w2.data[t], Hh)
            _kaiming_uniform_(self.b2.data[t:t + 1], Hh)

    def forward(self, x: torch.Tensor, labels: torch.Tensor | None, mask: torch.Tensor | None,
                task_scale: torch.Tensor) -> dict[str, torch.Tensor]:
        """``x [B, ntask, D]`` -> ``{"logits": [B, ntask], "loss": scalar}`` (loss only with labels)."""

        if (x.is_cuda and labels is not None and hasattr(self.w1, "_mdl_shadow") and self.input_dim % 8 == 0
                and self.hidden_dim % 8 == 0):
            loss, logits = TaskHeadsBCEFn.apply(x.to(torch.bfloat16), self.w1, self.b1, self.w2, self.b2,
                                                labels.float(), None if mask is None else mask.float(),
                                                task_scale.float(), self.relu)
            return {"loss": loss, "logits": logits}
        act = F.relu if self.relu else F.gelu
        hid = act(torch.einsum("btd,thd->bth", x.float(), self.w1) + self.b1.unsqueeze(0))
        logits = (hid * self.w2.unsqueeze(0)).sum(-1) + self.b2.unsqueeze(0)
        out = {"logits": logits}
        if labels is not None:
            bce = F.binary_cross_entropy_with_logits(logits, labels.float(), reduction="none")
            if mask is not None:
                bce = bce * mask.float()
            out["loss"] = (bce * task_scale.unsqueeze(0).to(bce.dtype)).sum()
        return out

    def forward_shared(self, x: torch.Tensor, labels: torch.Tensor | None, mask: torch.Tensor | None,
                       task_scale: torch.Tensor) -> dict[str, torch.Tensor]:
        """``x [B, D]`` read by every task (reference default readout: the flattened
        NS tokens feed each ``TaskHead``, ``src/model.py:7970-8022``)."""

        if (x.is_cuda and labels is not None and hasattr(self.w1, "_mdl_shadow") and self.input_dim % 8 == 0
                and self.hidden_dim % 8 == 0 and x.stride(1) == 1 and x.stride(0) % 8 == 0):
            loss, logits = SharedInputHeadsBCEFn.apply(x.to(torch.bfloat16), self.w1, self.b1, self.w2, self.b2,
                                                       labels.float(), None if mask is None else mask.float(),
                                                       task_scale.float(), self.relu)
            return {"loss": loss, "logits": logits}
        return self.forward(x.unsqueeze(1).expand(-1, self.num_tasks, -1), labels, mask, task_scale)

    def reference_state_dict(self, prefix: str = "logit_layers") -> dict[str, torch.Tensor]:
        sd = {}
        for t in range(self.num_tasks):
            p = f"{prefix}.{t}.network."
            sd[p + "0.weight"] = self.w1.detach()[t].clone()
            sd[p + "0.bias"] = self.b1.detach()[t].clone()
            sd[p + "3.weight"] = self.w2.detach()[t].view(1, -1).clone()
            sd[p + "3.bias"] = self.b2.detach()[t:t + 1].clone()
        return sd


class TaskQueryReadout(nn.Module):
    """Equal-readout control (``model.readout: task_query``; reference
    ``TaskQueryReadout`` ``src/model.py:900-946``): one learned query per task reads the
    final feature tokens with domain-aware attention, then a per-token FFN with a
    residual, giving one ``token_dim`` state per task for the task heads."""

    def __init__(self, num_tasks: int, token_dim: int, num_heads: int, num_feature_tokens: int, hidden_dim: int,
                 activation: str, init_std: float, device=None) -> None:
        super().__init__()
        from ..ops.layers import DomainAwareAttention, PerTokenFFN

        self.queries = nn.Parameter(torch.empty(num_tasks, token_dim, device=device).normal_(0.0, init_std))
        self.attention = DomainAwareAttention(token_dim, num_heads, num_tasks, num_feature_tokens, hidden_dim,
                                              activation, device=device)
        self.ffn = PerTokenFFN(num_tasks, token_dim, hidden_dim, activation, device=device)

    def forward(self, feature_tokens: torch.Tensor) -> torch.Tensor:
        B = feature_tokens.shape[0]
        dt = torch.bfloat16 if feature_tokens.is_cuda else feature_tokens.dtype
        q = self.queries.to(dt).unsqueeze(0).expand(B, -1, -1)
        states = q + self.attention(q, feature_tokens).to(dt)
        return states + self.ffn(states).to(dt)
