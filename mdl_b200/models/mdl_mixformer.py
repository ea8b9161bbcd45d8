"""MDL multi-domain ranker on a MixFormer backbone (``model.name: mdl_mixformer``).

Reference: ``MDLMixFormerModel`` (``src/model.py:8698-8950``), ``MDLMixFormerBlock``
(``:8622-8695``), ``ScenarioConditionedQueryRouter`` (``:8581-8619``).

Per block: the MixFormer Query Mixer updates the feature heads; with
``model.mdl_mixformer_query_conditioning`` (and scenario tokens) the pooled
active-scene state is routed into the queries (``ScenarioQueryRouter``); the
heads read the behaviour sequence (cross attention) and pass Output Fusion;
then the scenario and task tokens read the ``N`` feature heads exactly as the
MDL domain block of ``mdl_rankmixer`` does. The scene feature bias conditions
the initial heads; the readout is ``_mdl_logits`` over the final heads and
domain tokens, one task head per task.

CUDA: the MixFormer CUDA path (RMSNorm kernels, grouped tcgen05 SwiGLU
GEMMs) plus the MDL domain machinery (grouped tcgen05 per-token FFNs,
few-query attention kernel).
"""

from __future__ import annotations

import torch
from torch import nn

from ..config.schema import AppConfig
from .mdl import MDLDomainMixin, scenario_mask_from_ids
from .mixformer import MixFormerModel, ScenarioQueryRouter


class MDLMixFormerModel(MDLDomainMixin, MixFormerModel):
    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1, process_group=None,
                 vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None) -> None:
        nn.Module.__init__(self)
        dom_inputs = self._domain_specs(config)
        MixFormerModel.__init__(self, config, device=device, rank=rank, world=world, process_group=process_group,
                                vocab_sizes=vocab_sizes, base_seed=base_seed, domain_tokens=dom_inputs or None,
                                task_heads=False)
        dev = torch.device(device)
        D, H, N = self.D, int(config.model.hidden_dim), self.N
        self._init_domain_inputs(config, dev, D, H)
        route = bool(config.model.mdl_mixformer_query_conditioning) and self.use_scen
        blocks = []
        for _ in self.mixer.blocks:
            blk = nn.Module()
            self._add_domain_modules(blk, dev, N, D, H)
            blk.query_router = ScenarioQueryRouter(N, D, device=dev) if route else None
            blocks.append(blk)
        self.blocks = nn.ModuleList(blocks)
        self._init_domain_outputs(config, dev, D, H)

    def dense_buckets(self) -> list[list[str]]:
        names = [n for n, _ in self.named_parameters()]
        heads = [n for n in names if n.startswith("heads.")]
        return [heads, [n for n in names if not n.startswith("heads.")]]

    def forward(self, batch, task_scale: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        native = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
        anchor = torch.zeros(0, device=batch.ids.device, requires_grad=True)
        B = batch.rows
        feat_in, tokens, valid = self._inputs(batch, anchor, native)
        x, seq = self.mixer.inputs(feat_in, tokens, native)
        dt = x.dtype
        mask = scenario_mask_from_ids(batch.scenario_id, self.S).to(x.device)
        s_prompt, t_prompt = self._domain_prompts(batch, B, anchor, native, dt)
        s, t = self._initial_states(s_prompt, t_prompt, B, dt)
        if self.scene_feature_bias is not None:
            x = self._apply_scene_bias(x, s_prompt, mask).to(dt)
        w_fused = self._scene_weights(mask, include_global=self.use_global) if s is not None else None
        for mf, blk in zip(self.mixer.blocks, self.blocks):
            q = mf.query_mix(x, native)
            if blk.query_router is not None:
                q = blk.query_router(q, self._pool(s, w_fused), native)
            x = mf.output_fusion(mf.cross_attention(q, seq, valid, native), native)
            s, t = self._domain_step(blk, x, s, t, s_prompt, t_prompt, w_fused)
        pred = self._readout(x, s, t, mask)
        if task_scale is None:
            task_scale = torch.full((self.ntask,), 1.0 / max(1, B), device=x.device)
        return self.heads(pred, batch.labels, batch.label_mask, task_scale)
