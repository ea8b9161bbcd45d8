"""MDL multi-domain ranker on a OneTrans backbone (``model.name: mdl_onetrans``).

Reference: ``MDLOneTransModel`` (``src/model.py:8205-8435``) and ``MDLDomainBlock``
(``:8025-8202``).

The OneTrans backbone (tokenizer, mixed causal layers, pyramid) runs
unchanged; after backbone layer ``i`` the domain block ``i`` updates the
scenario and task tokens:

* by default each domain set reads the layer's NS tokens (fixed count ``N``)
  with domain-aware attention (per-token FFN projections), or the RankMixer
  interaction ablation -- the same reader as ``mdl_rankmixer``;
* from ``model.first_domain_sequence_layer`` on, each set instead reads the
  whole retained token sequence ``[Q_S; NS]`` (padded S tokens masked) with
  shared-projection attention (``SequenceDomainAttention``), so one pool
  holds sequence and NS evidence alike;
* task tokens add the pooled active scene (DomainFused); both sets pass their
  per-token FFN with a residual.

The scene feature bias conditions the NS tokens before the first layer; the
readout is ``_mdl_logits`` over the final NS tokens and the domain tokens,
read by one task head per task.

CUDA: the backbone is the OneTrans CUDA path (tcgen05 GEMMs writing the token
buffer, tcgen05 flash attention); every per-token FFN and projector is a
grouped tcgen05 GEMM pair reading the NS rows of the token buffer in place,
and attention over the NS tokens is the few-query kernel. CPU: the fp32
PyTorch definitions of both.
"""

from __future__ import annotations

import torch
from torch import nn

from ..config.schema import AppConfig
from .mdl import MDLDomainMixin, scenario_mask_from_ids
from .onetrans import OneTransAssembleFn, OneTransLayerFn, OneTransModel, OneTransTokenizeFn


class MDLOneTransModel(MDLDomainMixin, OneTransModel):
    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1, process_group=None,
                 vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None) -> None:
        nn.Module.__init__(self)
        dom_inputs = self._domain_specs(config)
        OneTransModel.__init__(self, config, device=device, rank=rank, world=world, process_group=process_group,
                               vocab_sizes=vocab_sizes, base_seed=base_seed, domain_tokens=dom_inputs or None,
                               task_heads=False)
        dev = torch.device(device)
        D, H, N = self.token_dim, self.hidden_dim, self.num_ns
        self.D = D
        self._init_domain_inputs(config, dev, D, H)
        first_seq = config.model.first_domain_sequence_layer
        blocks = []
        for i in range(len(self.layers)):
            blk = nn.Module()
            self._add_domain_modules(blk, dev, N, D, H, sequence=first_seq is not None and i >= int(first_seq))
            blocks.append(blk)
        self.blocks = nn.ModuleList(blocks)
        self._init_domain_outputs(config, dev, D, H)

    # ------------------------------------------------------------------ params
    def dense_buckets(self) -> list[list[str]]:
        """Heads, then (backbone layer i, domain block i) from the last layer down, then
        the tokenizer, projectors and the rest."""

        names = [n for n, _ in self.named_parameters()]
        heads = [n for n in names if n.startswith("heads.")]
        layers = [[n for n in names if n.startswith((f"layers.{i}.", f"blocks.{i}."))]
                  for i in reversed(range(len(self.layers)))]
        rest = [n for n in names if not n.startswith(("heads.", "layers.", "blocks."))]
        return [heads, *layers, rest]

    # ------------------------------------------------------------------ forward
    def forward(self, batch, task_scale: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        from ..ops.dense import grad_ready

        B = batch.rows
        anchor = torch.zeros(0, device=batch.ids.device, requires_grad=True)
        seq_in, ns_in, kstart = self._inputs(batch, anchor)
        cuda = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
        hooks = getattr(self, "dense_hooks", None) if cuda else None
        nl = len(self.layers)
        L = self.L
        if cuda:
            seq_in = grad_ready(seq_in, hooks, nl + 1)
            if self.ns_mode != "auto_split":
                ns_in = self.ns_tokens(ns_in).to(torch.bfloat16)
            if self.head_dim != 32:
                raise NotImplementedError(f"OneTrans head_dim {self.head_dim}: the tcgen05 attention kernels take "
                                          "head_dim 32 (set runtime.kernel_backend: torch for this model)")
            if self.multi:
                X = OneTransAssembleFn.apply(seq_in.to(torch.bfloat16), ns_in, kstart, self, L)
            else:
                X = OneTransTokenizeFn.apply(seq_in, ns_in, kstart, self, L)
            ks = kstart
        else:
            X = self.tokenize_reference(seq_in, ns_in, kstart, B)
            ks = kstart.to(X.device).long()
        dt = X.dtype
        mask = scenario_mask_from_ids(batch.scenario_id, self.S).to(X.device)
        s_prompt, t_prompt = self._domain_prompts(batch, B, anchor, cuda, dt)
        s, t = self._initial_states(s_prompt, t_prompt, B, dt)
        if self.scene_feature_bias is not None:
            ns = self._apply_scene_bias(X[:, L:, :], s_prompt, mask).to(dt)
            X = torch.cat([X[:, :L, :], ns], dim=1)
        w_fused = self._scene_weights(mask, include_global=self.use_global) if s is not None else None
        s_in = L
        for i, (layer, blk) in enumerate(zip(self.layers, self.blocks)):
            q = self.query_counts[i]
            if cuda:
                X = grad_ready(X, hooks, nl - i)  # layer i's and block i's gradients are final once d(X_in) is
                X = OneTransLayerFn.apply(X, ks, layer, s_in, q, self.attn_heads, self.eps)
            else:
                X = layer.forward_reference(X, ks, s_in, q, self.attn_heads, self.eps)
            ks = (ks - (s_in - q)).clamp(min=0)
            s_in = q
            seq_reader = blk.scenario_sequence_attention or blk.task_sequence_attention
            memory = (X, ks) if seq_reader is not None else None
            s, t = self._domain_step(blk, X[:, s_in:, :], s, t, s_prompt, t_prompt, w_fused, memory)
        pred = self._readout(X[:, s_in:, :], s, t, mask)
        if task_scale is None:
            task_scale = torch.full((self.ntask,), 1.0 / max(1, B), device=X.device)
        pred = grad_ready(pred, hooks, 0)
        return self.heads(pred, batch.labels, batch.label_mask, task_scale)
