"""RankMixer ranker: per-token tokenizer -> L x (token mixing + per-token FFN) -> task heads.

Reference: ``RankMixerModel`` (``src/model.py:6691-6911``), ``RankMixerBlock``
(:6654-6665), ``RankMixerSliceTokenizer`` (:4318-4432), ``TaskHead`` (:869-882),
token mixing (``src/modules/attention.py:345-363``) and ``StackedPerTokenFFN``
(``src/modules/mlp.py:135-207``).

Two execution paths with one set of parameters:

* CUDA: the fused lookup kernel writes the tokenizer input (per-token slices,
  padded to a 16-byte multiple) straight from the embedding tables; then
  ``PerTokenLinearFn``, one ``RankMixerBlockFn`` per layer and ``HeadsBCEFn``
  run the sm_100a kernels (``ops/fused.py``).
* CPU: the same math in plain PyTorch fp32 (``forward_reference``), used for
  the gloo plumbing runs and as the oracle of the GPU tests.

Parameter layout deviations from the reference (converted by
``reference_state_dict`` / ``load_reference_state_dict``): the tokenizer weight
is stored ``[T, D, Kpad]`` (K padded with zero columns) and the task towers are
stacked over tasks (``heads.w1 [ntask, Hh, D]`` ...) so that all tasks run as
one GEMM.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..config.schema import AppConfig
from .features import FeatureEncoder


def _kaiming_uniform_(t: torch.Tensor, fan_in: int) -> None:
    bound = 1.0 / math.sqrt(fan_in)  # kaiming_uniform(a=sqrt(5)) bound = sqrt(6 / ((1 + 5) * fan_in))
    nn.init.uniform_(t, -bound, bound)


def token_mix(x: torch.Tensor) -> torch.Tensor:
    """RankMixer token mixing: ``[B,T,T,D/T] -> permute(0,2,1,3)``."""

    B, T, D = x.shape
    return x.view(B, T, T, D // T).permute(0, 2, 1, 3).reshape(B, T, D)


class RankMixerModel(nn.Module):
    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1,
                 process_group=None, vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None) -> None:
        super().__init__()
        self.config = config
        mc = config.model
        res = config.resolved.tokenization
        self.T = int(res.feature_token_count)
        self.D = int(mc.token_dim)
        self.H = int(mc.hidden_dim)
        self.L = int(mc.num_layers)
        self.tasks = list(config.task_names)
        self.ntask = len(self.tasks)
        self.Hh = int(mc.task_head_hidden_dim or mc.hidden_dim)
        self.head_relu = mc.task_head_activation == "relu"
        self.ffn_relu = mc.ffn_activation == "relu"
        self.moe = mc.rankmixer_ffn_type == "sparse_moe"
        if self.D % self.T:
            raise ValueError("rankmixer requires token_dim divisible by the feature token count")
        groupwise = config.tokenization.feature_tokenizer == "groupwise"
        token_groups = [list(g.inputs) for g in res.feature_token_groups] if groupwise else None
        if groupwise and len(token_groups) != self.T:
            raise ValueError(f"groupwise tokenizer: {len(token_groups)} groups for {self.T} tokens")
        self.encoder = FeatureEncoder(config, device=device, rank=rank, world=world, process_group=process_group,
                                      vocab_sizes=vocab_sizes, slice_tokens=0 if groupwise else self.T,
                                      base_seed=base_seed, token_groups=token_groups)
        from .sequence_encoders import SequenceSummaries

        # sequences summarised into feature-token inputs (mean_pool / attention_pool / longer / stca)
        self.summaries = SequenceSummaries(config, self.encoder, self.encoder.summary_names, device=device)
        if groupwise:
            self.K = self.Kpad = self.encoder.group_k_pad
            fan_in = self.encoder.group_widths
        else:
            self.K = self.encoder.slice_k
            self.Kpad = self.encoder.slice_stride
            fan_in = [self.K] * self.T
        T, D, H, K, Kp = self.T, self.D, self.H, self.K, self.Kpad
        dev = torch.device(device)
        self.tok_weight = nn.Parameter(torch.zeros(T, D, Kp, device=dev))
        self.tok_bias = nn.Parameter(torch.empty(T, D, device=dev))
        for t in range(T):  # each token's fan-in is its own input width; padded columns stay zero
            _kaiming_uniform_(self.tok_weight.data[t, :, :fan_in[t]], fan_in[t])
            _kaiming_uniform_(self.tok_bias.data[t], fan_in[t])
        self.blocks = nn.ModuleList()
        for _ in range(self.L):
            blk = nn.Module()
            blk.ln1_weight = nn.Parameter(torch.ones(D, device=dev))
            blk.ln1_bias = nn.Parameter(torch.zeros(D, device=dev))
            if self.moe:
                from ..ops.moe import build_rankmixer_moe

                blk.ffn = build_rankmixer_moe(config, T, device=dev)
            else:
                blk.w_in = nn.Parameter(torch.empty(T, H, D, device=dev))
                blk.b_in = nn.Parameter(torch.empty(T, H, device=dev))
                blk.w_out = nn.Parameter(torch.empty(T, D, H, device=dev))
                blk.b_out = nn.Parameter(torch.empty(T, D, device=dev))
                for t in range(T):
                    _kaiming_uniform_(blk.w_in.data[t], D)
                    _kaiming_uniform_(blk.b_in.data[t], D)
                    _kaiming_uniform_(blk.w_out.data[t], H)
                    _kaiming_uniform_(blk.b_out.data[t], H)
            blk.ln2_weight = nn.Parameter(torch.ones(D, device=dev))
            blk.ln2_bias = nn.Parameter(torch.zeros(D, device=dev))
            self.blocks.append(blk)
        Hh, nt = self.Hh, self.ntask
        self.head_w1 = nn.Parameter(torch.empty(nt, Hh, D, device=dev))
        self.head_b1 = nn.Parameter(torch.empty(nt, Hh, device=dev))
        self.head_w2 = nn.Parameter(torch.empty(nt, Hh, device=dev))
        self.head_b2 = nn.Parameter(torch.empty(nt, device=dev))
        for t in range(nt):
            _kaiming_uniform_(self.head_w1.data[t], D)
            _kaiming_uniform_(self.head_b1.data[t], D)
            _kaiming_uniform_(self.head_w2.data[t], Hh)
            _kaiming_uniform_(self.head_b2.data[t:t + 1], Hh)
        self.ln_eps = 1e-5

    # ------------------------------------------------------------------ params
    def gemm_param_names(self) -> set[str]:
        """Parameters consumed as bf16 GEMM operands (get a bf16 shadow)."""

        names = {"tok_weight", "head_w1"}
        for i in range(self.L):
            if not self.moe:
                names |= {f"blocks.{i}.w_in", f"blocks.{i}.w_out"}
        names |= {n for n, p in self.blocks.named_parameters(prefix="blocks") if getattr(p, "_mdl_gemm", False)}
        names |= {n for n, p in self.summaries.named_parameters(prefix="summaries") if getattr(p, "_mdl_gemm", False)}
        return names

    def dense_buckets(self) -> list[list[str]]:
        """Parameter groups in the order their gradients become final in the backward."""

        heads = ["head_w1", "head_b1", "head_w2", "head_b2"]
        blocks = [[n for n, _ in self.blocks[i].named_parameters(prefix=f"blocks.{i}")]
                  for i in reversed(range(self.L))]
        return [heads, *blocks,
                ["tok_weight", "tok_bias", *[n for n, _ in self.summaries.named_parameters(prefix="summaries")]]]

    @property
    def store(self):
        return self.encoder.store

    # ------------------------------------------------------------------ forward
    def forward(self, batch, task_scale: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        """Training forward. ``batch`` is a ``PackedBatch``; returns ``loss`` and ``logits``."""

        anchor = torch.zeros(0, device=batch.ids.device, requires_grad=True)
        from ..ops.embedding import fused_lookup

        x0 = fused_lookup(self.store, self.encoder.plan, batch.ids, batch.offsets, batch.dense, batch.rows, anchor)
        native = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
        if self.summaries.names:
            from .sequence_encoders import add_summaries

            x0 = add_summaries(x0, self.summaries(self.encoder, batch, anchor, native),
                               self.encoder.summary_cols["plan"])
        if native:
            out = self._forward_cuda(x0, batch, task_scale)
        else:
            out = self.forward_reference(x0, batch, task_scale)
        if self.moe:
            from ..ops.moe import add_moe_loss

            add_moe_loss(out, self, float(self.config.model.sparse_moe_loss_weight))
        return out

    def _forward_cuda(self, x0, batch, task_scale):
        from ..ops.fused import HeadsBCEFn, PerTokenLinearFn, RankMixerBlockFn

        if self.ffn_relu:
            raise NotImplementedError("fused RankMixer block implements the gelu FFN (reference default)")
        from ..ops.dense import grad_ready

        hooks = getattr(self, "dense_hooks", None)  # bucket k final -> its update starts (see dense_buckets)
        x0 = grad_ready(x0, hooks, self.L + 1)
        x = PerTokenLinearFn.apply(x0, self.tok_weight, self.tok_bias, self.T, self.K, self.Kpad)
        for i, blk in enumerate(self.blocks):
            x = grad_ready(x, hooks, self.L - i)
            if self.moe:
                from ..ops.fused import MixLayerNormFn
                from ..ops.layers import LayerNormFn

                m = MixLayerNormFn.apply(x, blk.ln1_weight, blk.ln1_bias, self.ln_eps)
                x = LayerNormFn.apply(blk.ffn(m) + m, blk.ln2_weight, blk.ln2_bias, self.ln_eps)
                continue
            x = RankMixerBlockFn.apply(x, blk.ln1_weight, blk.ln1_bias, blk.w_in, blk.b_in, blk.w_out, blk.b_out,
                                       blk.ln2_weight, blk.ln2_bias, self.ln_eps)
        x = grad_ready(x, hooks, 0)
        if task_scale is None:
            task_scale = torch.full((self.ntask,), 1.0 / max(1, batch.rows), device=x.device)
        loss, logits = HeadsBCEFn.apply(x, self.head_w1, self.head_b1, self.head_w2, self.head_b2, batch.labels,
                                        batch.label_mask, task_scale, self.head_relu)
        return {"loss": loss, "logits": logits}

    def forward_reference(self, x0, batch, task_scale=None):
        """Plain PyTorch fp32 definition (CPU path and test oracle)."""

        B = batch.rows
        T, K, Kp, D = self.T, self.K, self.Kpad, self.D
        xin = x0.float().view(B, T, Kp)[:, :, :K]
        w = self.tok_weight[:, :, :K]
        x = torch.einsum("btk,tdk->btd", xin, w) + self.tok_bias.unsqueeze(0)
        act_fn = F.relu if self.ffn_relu else F.gelu
        for blk in self.blocks:
            m = F.layer_norm(token_mix(x) + x, (D,), blk.ln1_weight, blk.ln1_bias, self.ln_eps)
            if self.moe:
                f = blk.ffn(m).float()
            else:
                h = act_fn(torch.einsum("btd,thd->bth", m, blk.w_in) + blk.b_in.unsqueeze(0))
                f = torch.einsum("bth,tdh->btd", h, blk.w_out) + blk.b_out.unsqueeze(0)
            x = F.layer_norm(f + m, (D,), blk.ln2_weight, blk.ln2_bias, self.ln_eps)
        pooled = x.mean(dim=1)
        head_act = F.relu if self.head_relu else F.gelu
        hid = head_act(torch.einsum("bd,thd->bth", pooled, self.head_w1) + self.head_b1.unsqueeze(0))
        logits = (hid * self.head_w2.unsqueeze(0)).sum(-1) + self.head_b2.unsqueeze(0)
        out = {"logits": logits}
        if batch.labels is not None:
            if task_scale is None:
                task_scale = torch.full((self.ntask,), 1.0 / max(1, B), device=logits.device)
            bce = F.binary_cross_entropy_with_logits(logits, batch.labels.float(), reduction="none")
            if batch.label_mask is not None:
                bce = bce * batch.label_mask.float()
            out["loss"] = (bce * task_scale.unsqueeze(0).to(bce.dtype)).sum()
        return out

    # ------------------------------------------------------------------ reference layout
    def reference_state_dict(self) -> dict[str, torch.Tensor]:
        """Dense weights under the reference's parameter names and shapes."""

        sd: dict[str, torch.Tensor] = {}
        K = self.K
        sd["feature_projector.projection.weight"] = self.tok_weight.detach()[:, :, :K].clone()
        sd["feature_projector.projection.bias"] = self.tok_bias.detach().clone()
        for i, blk in enumerate(self.blocks):
            p = f"blocks.{i}."
            sd[p + "feature_norm.weight"] = blk.ln1_weight.detach().clone()
            sd[p + "feature_norm.bias"] = blk.ln1_bias.detach().clone()
            if self.moe:
                sd.update(blk.ffn.reference_state_dict(p + "feature_ffn."))
            else:
                sd[p + "feature_ffn.input_weight"] = blk.w_in.detach().clone()
                sd[p + "feature_ffn.input_bias"] = blk.b_in.detach().clone()
                sd[p + "feature_ffn.output_weight"] = blk.w_out.detach().clone()
                sd[p + "feature_ffn.output_bias"] = blk.b_out.detach().clone()
            sd[p + "feature_ffn_norm.weight"] = blk.ln2_weight.detach().clone()
            sd[p + "feature_ffn_norm.bias"] = blk.ln2_bias.detach().clone()
        for t in range(self.ntask):
            p = f"logit_layers.{t}.network."
            sd[p + "0.weight"] = self.head_w1.detach()[t].clone()
            sd[p + "0.bias"] = self.head_b1.detach()[t].clone()
            sd[p + "3.weight"] = self.head_w2.detach()[t].view(1, -1).clone()
            sd[p + "3.bias"] = self.head_b2.detach()[t:t + 1].clone()
        return sd

    @torch.no_grad()
    def load_reference_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        if self.moe:
            raise NotImplementedError("loading reference weights covers the dense per-token FFN")
        K = self.K
        self.tok_weight[:, :, :K].copy_(sd["feature_projector.projection.weight"])
        self.tok_weight[:, :, K:].zero_()
        self.tok_bias.copy_(sd["feature_projector.projection.bias"])
        for i, blk in enumerate(self.blocks):
            p = f"blocks.{i}."
            blk.ln1_weight.copy_(sd[p + "feature_norm.weight"])
            blk.ln1_bias.copy_(sd[p + "feature_norm.bias"])
            blk.w_in.copy_(sd[p + "feature_ffn.input_weight"])
            blk.b_in.copy_(sd[p + "feature_ffn.input_bias"])
            blk.w_out.copy_(sd[p + "feature_ffn.output_weight"])
            blk.b_out.copy_(sd[p + "feature_ffn.output_bias"])
            blk.ln2_weight.copy_(sd[p + "feature_ffn_norm.weight"])
            blk.ln2_bias.copy_(sd[p + "feature_ffn_norm.bias"])
        for t in range(self.ntask):
            p = f"logit_layers.{t}.network."
            self.head_w1[t].copy_(sd[p + "0.weight"])
            self.head_b1[t].copy_(sd[p + "0.bias"])
            self.head_w2[t].copy_(sd[p + "3.weight"].view(-1))
            self.head_b2[t:t + 1].copy_(sd[p + "3.bias"])
