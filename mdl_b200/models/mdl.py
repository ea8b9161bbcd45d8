"""MDL multi-domain ranker on a RankMixer backbone (``model.name: mdl_rankmixer``).

Reference: ``MDLRankMixerModel`` (``src/model.py:7543-7967``), ``MDLRankMixerBlock``
(:7418-7465), domain interaction (:6953-7228), readout (:7238-7416),
``DomainTokenProjector`` (:4469-4498), ``SceneFeatureBias`` (:4501-4547),
``ScenarioTower`` (:6914-6950), ``DomainAwareAttention`` /
``RankMixerDomainInteraction`` / ``masked_scenario_pool`` / ``DomainFusedModule``
(``src/modules/attention.py:366-512, 719-789``).

Per sample the model carries three token sets through ``L`` blocks:

* feature tokens ``[B, T, D]``: the RankMixer tokenizer and blocks (token
  mixing + LayerNorm + per-token FFN, with the second residual + LayerNorm for
  ``mdl_feature_interaction: residual_ffn``);
* scenario tokens ``[B, Ns, D]``: ``tokens_per_scenario`` tokens per scene plus
  an optional global token, built by per-token MLPs (``Linear -> act ->
  Linear -> ReLU``) from their configured inputs;
* task tokens ``[B, ntask, D]``, built the same way.

In every block each domain token set reads the feature tokens with
domain-aware attention (per-token FFN projections of queries, keys and values;
``few_query_attention``), task tokens add the masked mean of the active
scene's tokens (DomainFused), and both sets pass a per-token FFN with a
residual. The task heads read one task token each.

Execution on CUDA: the embedding lookup writes the tokenizer input and the
domain-token inputs (two lookups over one batch), every per-token MLP/FFN is a
grouped tcgen05 GEMM pair, attention is the few-query kernel, the RankMixer
block is the fused block, heads + BCE are one grouped GEMM and one kernel. On
CPU the same modules run their PyTorch definitions.

``tokens_per_scenario`` (default 1, the reference layout) generalises the
scenario tokens: scene ``s`` owns tokens ``[s * k, (s + 1) * k)`` and every
pooling over "the active scene" averages its ``k`` tokens.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..config.schema import AppConfig
from ..ops.layers import DomainAwareAttention, Linear, PerTokenFFN, gemm_param, layer_norm
from .features import FeatureEncoder
from .heads import TaskHeads
from .rankmixer import token_mix


def _kaiming_uniform_(t: torch.Tensor, fan_in: int) -> None:
    bound = 1.0 / math.sqrt(max(1, fan_in))
    nn.init.uniform_(t, -bound, bound)


def scenario_mask_from_ids(scenario_id: torch.Tensor, num_scenarios: int) -> torch.Tensor:
    """``[B]`` integer ids -> one-hot ``[B, S]`` float; a ``[B, S]`` mask passes through
    (reference ``_scenario_mask_from_ids`` ``src/model.py:414-480``, without the
    per-step validation sync)."""

    if scenario_id.dim() == 2:
        if scenario_id.size(1) != num_scenarios:
            raise ValueError(f"scenario mask width must be {num_scenarios}, got {scenario_id.size(1)}")
        return scenario_id.float()
    if scenario_id.dim() != 1:
        raise ValueError("scenario_id must have shape [batch] or [batch, num_scenarios]")
    return F.one_hot(scenario_id.long().clamp(0, num_scenarios - 1), num_scenarios).float()


class RankMixerDomainInteraction(nn.Module):
    """Ablation of domain-aware attention: RankMixer mixing over ``[feature; domain]``
    tokens, zero-padded to a width divisible by the token count, residual +
    LayerNorm, domain outputs cropped back (``src/modules/attention.py:366-422``)."""

    def __init__(self, token_dim: int, num_domain_tokens: int, num_feature_tokens: int, device=None) -> None:
        super().__init__()
        self.token_dim = token_dim
        self.num_feature_tokens = num_feature_tokens
        self.num_tokens = num_feature_tokens + num_domain_tokens
        self.mixing_dim = math.ceil(token_dim / self.num_tokens) * self.num_tokens
        self.norm = nn.LayerNorm(self.mixing_dim, device=device)

    def forward(self, domain_tokens: torch.Tensor, feature_tokens: torch.Tensor) -> torch.Tensor:
        tokens = torch.cat([feature_tokens, domain_tokens.to(feature_tokens.dtype)], dim=1)
        if self.mixing_dim != self.token_dim:
            tokens = F.pad(tokens, (0, self.mixing_dim - self.token_dim))
        mixed = token_mix(tokens) + tokens
        out = F.layer_norm(mixed.float(), (self.mixing_dim,), self.norm.weight, self.norm.bias, self.norm.eps)
        return out.to(tokens.dtype)[:, self.num_feature_tokens:, :self.token_dim]


class SequenceDomainAttention(nn.Module):
    """Domain tokens read a masked token sequence (reference
    ``VariableLengthDomainAttention`` ``src/modules/attention.py:568-716``).

    ``LayerNorm`` on the queries and on the memory, shared ``Linear`` Q/K/V
    projections (valid for any sequence length, which the OneTrans pyramid
    changes per layer), attention over the memory tokens ``j >= kstart[b]``
    (prefix padding), ``Linear`` output projection. The OneTrans memory always
    holds the NS tokens, so every sample has a visible key.

    CUDA: LayerNorm kernels and tcgen05 GEMMs for the norms and projections;
    the few-query score/softmax/value products are batched matmuls.
    """

    def __init__(self, token_dim: int, num_heads: int, device=None) -> None:
        super().__init__()
        if token_dim % num_heads:
            raise ValueError("token_dim must be divisible by num_heads")
        D = token_dim
        self.num_heads = num_heads
        self.query_norm = nn.LayerNorm(D, device=device)
        self.memory_norm = nn.LayerNorm(D, device=device)
        self.query_projection = Linear(D, D, device=device)
        self.key_projection = Linear(D, D, device=device)
        self.value_projection = Linear(D, D, device=device)
        self.output_projection = Linear(D, D, device=device)

    def forward(self, domain_tokens: torch.Tensor, memory: torch.Tensor, kstart: torch.Tensor) -> torch.Tensor:
        B, Nq, D = domain_tokens.shape
        Lk = memory.shape[1]
        h = self.num_heads
        hd = D // h
        native = memory.is_cuda and hasattr(self.key_projection.weight, "_mdl_shadow")
        qn = layer_norm(domain_tokens, self.query_norm.weight, self.query_norm.bias, 1e-5, native)
        mn = layer_norm(memory, self.memory_norm.weight, self.memory_norm.bias, 1e-5, native)
        q = self.query_projection(qn.reshape(B * Nq, D)).view(B, Nq, h, hd).transpose(1, 2)
        mflat = mn.reshape(B * Lk, D)
        k = self.key_projection(mflat).view(B, Lk, h, hd).transpose(1, 2)
        v = self.value_projection(mflat).view(B, Lk, h, hd).transpose(1, 2)
        s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * (1.0 / math.sqrt(hd))   # [B, h, Nq, Lk]
        keep = torch.arange(Lk, device=memory.device).view(1, 1, 1, Lk) >= kstart.to(memory.device).view(B, 1, 1, 1)
        p = torch.softmax(s.masked_fill(~keep, float("-inf")), dim=-1)
        o = torch.matmul(p.to(v.dtype), v).transpose(1, 2).reshape(B * Nq, D)
        return self.output_projection(o.contiguous()).view(B, Nq, D)


class MDLDomainMixin:
    """MDL domain tokens over a backbone's feature tokens.

    Shared by the RankMixer (``mdl_rankmixer``) and OneTrans (``mdl_onetrans``)
    backbones: the scenario / task projectors and readout seeds, one domain
    block per backbone layer (reference ``MDLDomainBlock`` ``src/model.py:8025-8202``
    and the domain half of ``MDLRankMixerBlock`` ``:7418-7465``), the scene
    feature bias, the scenario tower ablation and the readout
    (``_mdl_logits`` ``:7375-7415``).
    """

    def _domain_specs(self, config: AppConfig) -> list[list[str]]:
        """Reads the domain options; returns the inputs of each domain token (scenario
        tokens first) for the feature encoder."""

        mc = config.model
        res = config.resolved.tokenization
        self.tasks = list(config.task_names)
        self.ntask = len(self.tasks)
        self.S = len(config.scenarios.names)
        self.tps = max(1, int(mc.tokens_per_scenario))
        self.heads_n = int(mc.num_heads)
        self.act = mc.ffn_activation
        self.use_scen = bool(mc.use_scenario_tokens)
        self.use_task = bool(mc.use_task_tokens)
        self.use_global = bool(mc.use_global_scenario_token) and self.use_scen
        self.split = mc.mdl_token_state == "split"
        if self.split and not (self.use_scen or self.use_task):
            raise ValueError("model.mdl_token_state=split requires task or scenario tokens")
        if int(mc.token_dim) % self.heads_n:
            raise ValueError("token_dim must be divisible by num_heads")
        scen_specs = [s for s in res.scenario_token_specs
                      if self.use_scen and (s.kind != "global" or self.use_global)]
        task_specs = list(res.task_token_specs) if self.use_task else []
        self.Ns, self.Nt = len(scen_specs), len(task_specs)
        dom_inputs = [s.resolved_inputs() for s in scen_specs + task_specs]
        for spec, inputs in zip(scen_specs + task_specs, dom_inputs):
            if not inputs:
                raise ValueError(f"domain token {spec.name!r} has no inputs")
        return dom_inputs

    def _init_domain_inputs(self, config: AppConfig, dev, D: int, H: int) -> None:
        """Domain-token projectors (reference ``DomainTokenProjector``: ``Linear -> act ->
        Linear -> ReLU``) and the split-mode readout seeds."""

        off = getattr(self, "_dom_offset", 0)  # leading per-token inputs that are not domain tokens
        widths = self.encoder.domain_widths[off:]
        Kd = self.encoder.domain_k_pad
        self.Kd = Kd
        self.scenario_projector = None
        self.task_projector = None
        if self.Ns:
            self.scenario_projector = PerTokenFFN(self.Ns, Kd, H, self.act, output_relu=True, device=dev, out_dim=D)
            self.scenario_projector.restrict_inputs(widths[:self.Ns])
        if self.Nt:
            self.task_projector = PerTokenFFN(self.Nt, Kd, H, self.act, output_relu=True, device=dev, out_dim=D)
            self.task_projector.restrict_inputs(widths[self.Ns:])
        std = float(config.model.init_std)
        self.scenario_readout_seed = (nn.Parameter(torch.randn(1, self.Ns, D, device=dev) * std)
                                      if self.split and self.Ns else None)
        self.task_readout_seed = (nn.Parameter(torch.randn(1, self.Nt, D, device=dev) * std)
                                  if self.split and self.Nt else None)

    def _init_domain_outputs(self, config: AppConfig, dev, D: int, H: int) -> None:
        mc = config.model
        self.scene_feature_bias = None
        if mc.scene_feature_bias != "none":
            if not self.use_scen:
                raise ValueError("scene_feature_bias needs scenario tokens")
            out = D if mc.scene_feature_bias == "additive" else 2 * D
            self.scene_feature_bias = Linear(D, out, device=dev)
            nn.init.zeros_(self.scene_feature_bias.weight)
            nn.init.zeros_(self.scene_feature_bias.bias)
        self.scene_bias_mode = mc.scene_feature_bias
        # scenario tower ablation (no scenario tokens): one MLP per scene over the pooled feature state
        self.scenario_tower = (PerTokenFFN(self.S, D, H, self.act, device=dev) if not self.use_scen else None)
        Hh = int(mc.task_head_hidden_dim or mc.hidden_dim)
        self.heads = TaskHeads(self.ntask, D, Hh, mc.task_head_activation, device=dev)

    def _add_domain_modules(self, blk: nn.Module, dev, num_feature_tokens: int, D: int, H: int,
                            sequence: bool = False) -> None:
        """Scenario / task readers and FFNs of one domain block: domain-aware attention
        over ``num_feature_tokens`` fixed tokens (or the RankMixer interaction ablation),
        or, with ``sequence``, attention over the variable-length token sequence."""

        mc = self.config.model
        blk.scenario_attention = blk.scenario_rankmixer = blk.scenario_ffn = None
        blk.task_attention = blk.task_rankmixer = blk.task_ffn = None
        blk.scenario_sequence_attention = blk.task_sequence_attention = None
        T = num_feature_tokens
        if self.split and not sequence and ((self.Ns and not mc.use_scenario_feature_interaction)
                                            or (self.Nt and not mc.use_task_feature_interaction)):
            raise ValueError("model.mdl_token_state=split requires domain-aware attention")
        if self.Ns:
            if sequence:
                blk.scenario_sequence_attention = SequenceDomainAttention(D, self.heads_n, device=dev)
            elif mc.use_scenario_feature_interaction:
                blk.scenario_attention = DomainAwareAttention(D, self.heads_n, self.Ns, T, H, self.act, device=dev)
            else:
                blk.scenario_rankmixer = RankMixerDomainInteraction(D, self.Ns, T, device=dev)
            blk.scenario_ffn = PerTokenFFN(self.Ns, D, H, self.act, device=dev)
        if self.Nt:
            if sequence:
                blk.task_sequence_attention = SequenceDomainAttention(D, self.heads_n, device=dev)
            elif mc.use_task_feature_interaction:
                blk.task_attention = DomainAwareAttention(D, self.heads_n, self.Nt, T, H, self.act, device=dev)
            else:
                blk.task_rankmixer = RankMixerDomainInteraction(D, self.Nt, T, device=dev)
            blk.task_ffn = PerTokenFFN(self.Nt, D, H, self.act, device=dev)

    def _scene_weights(self, mask: torch.Tensor, include_global: bool) -> torch.Tensor:
        """``[B, Ns]`` weights of the masked mean over the active scene's tokens (and the
        global token when ``include_global``); reference ``masked_scenario_pool``."""

        w = mask.repeat_interleave(self.tps, dim=1)
        if self.use_global:
            g = torch.full_like(w[:, :1], 1.0 if include_global else 0.0)
            w = torch.cat([w, g], dim=1)
        return w / w.sum(dim=1, keepdim=True).clamp_min(1.0)

    @staticmethod
    def _pool(tokens: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        return torch.einsum("bn,bnd->bd", weights.to(tokens.dtype), tokens)

    @staticmethod
    def _interact(domain: torch.Tensor, feature: torch.Tensor, attention, rankmixer) -> torch.Tensor:
        if attention is not None:
            return domain + attention(domain, feature).to(domain.dtype)
        return rankmixer(domain, feature)

    def _domain_prompts(self, batch, B: int, anchor: torch.Tensor, cuda: bool, dt: torch.dtype,
                        summaries: dict | None = None):
        """Scenario / task prompts ``[B, Ns, D]`` / ``[B, Nt, D]`` from the domain-token
        lookup (``None`` for a disabled set). Sequence summaries among the domain inputs
        (prior sequences) are added into their columns; they are computed here unless
        the caller passes them."""

        from ..ops.embedding import fused_lookup

        enc = self.encoder
        s_prompt = t_prompt = None
        if self.Ns + self.Nt:
            d0 = fused_lookup(self.store, enc.domain_plan, batch.ids, batch.offsets, batch.dense, B, anchor)
            cols = enc.summary_cols["domain"]
            if cols:
                from .sequence_encoders import add_summaries

                if summaries is None:
                    summaries = self.summaries(enc, batch, anchor, cuda)
                d0 = add_summaries(d0, summaries, cols)
            off = getattr(self, "_dom_offset", 0)
            dom = d0.view(B, -1, self.Kd)[:, off:off + self.Ns + self.Nt]
            if not cuda:
                dom = dom.float()
            if self.Ns:
                s_prompt = self.scenario_projector(dom[:, :self.Ns]).to(dt)
            if self.Nt:
                t_prompt = self.task_projector(dom[:, self.Ns:]).to(dt)
        return s_prompt, t_prompt

    def _initial_states(self, s_prompt, t_prompt, B: int, dt: torch.dtype):
        s = t = None
        if s_prompt is not None:
            s = s_prompt if self.scenario_readout_seed is None else \
                self.scenario_readout_seed.to(dt).expand(B, -1, -1)
        if t_prompt is not None:
            t = t_prompt if self.task_readout_seed is None else self.task_readout_seed.to(dt).expand(B, -1, -1)
        return s, t

    def _apply_scene_bias(self, x: torch.Tensor, s_prompt: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        """Reference ``SceneFeatureBias`` (``src/model.py:4513-4540``): additive or FiLM
        conditioning of the feature tokens on the active scene's prompt tokens."""

        dt = x.dtype
        w = self._scene_weights(mask, include_global=False)
        scene = self._pool(s_prompt, w)
        params = self.scene_feature_bias(scene).to(dt)
        if self.scene_bias_mode == "additive":
            return x + params.unsqueeze(1)
        gamma, beta = params.chunk(2, dim=-1)
        return (1.0 + gamma).unsqueeze(1) * x + beta.unsqueeze(1)

    def _domain_step(self, blk, x, s, t, s_prompt, t_prompt, w_fused, memory=None):
        """One domain block: each domain set reads the feature tokens ``x`` (or the
        sequence ``memory = (tokens, kstart)``), task tokens add the pooled active
        scene (DomainFused), both sets pass their per-token FFN with a residual."""

        def read(state, prompt, attention, rankmixer, seq_attention):
            dt = state.dtype
            query = prompt + state if self.split else state
            if seq_attention is not None:
                return state + seq_attention(query, *memory).to(dt)
            if self.split:
                return state + attention(query, x).to(dt)
            return self._interact(state, x, attention, rankmixer)

        s_hat = None
        if s is not None:
            s_hat = read(s, s_prompt, blk.scenario_attention, blk.scenario_rankmixer,
                         blk.scenario_sequence_attention)
            s = s_hat + blk.scenario_ffn(s_hat).to(s_hat.dtype)
        if t is not None:
            t_hat = read(t, t_prompt, blk.task_attention, blk.task_rankmixer, blk.task_sequence_attention)
            if s_hat is not None:
                t_hat = t_hat + self._pool(s_hat, w_fused).unsqueeze(1)
            t = t_hat + blk.task_ffn(t_hat).to(t_hat.dtype)
        return s, t

    def _readout(self, x: torch.Tensor, s, t, mask: torch.Tensor) -> torch.Tensor:
        """Prediction tokens ``[B, ntask, D]`` of the task heads (reference ``_mdl_logits``)."""

        B = x.shape[0]
        dt = x.dtype
        context = None
        if not self.use_scen:
            pooled = x.mean(dim=1)
            states = self.scenario_tower(pooled.unsqueeze(1).expand(B, self.S, x.shape[-1]).contiguous()).to(dt)
            wm = mask / mask.sum(dim=1, keepdim=True).clamp_min(1.0)
            context = self._pool(states, wm)
        elif not self.use_task:
            context = self._pool(s, self._scene_weights(mask, include_global=self.use_global))
        if self.use_task:
            return t if context is None else t + context.unsqueeze(1)
        v = x.mean(dim=1)
        if context is not None:
            v = v + context
        return v.unsqueeze(1).expand(B, self.ntask, x.shape[-1]).contiguous()


class MDLRankMixerModel(MDLDomainMixin, nn.Module):
    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1,
                 process_group=None, vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None) -> None:
        super().__init__()
        self.config = config
        mc = config.model
        res = config.resolved.tokenization
        dev = torch.device(device)
        self.T = int(res.feature_token_count)
        self.D = int(mc.token_dim)
        self.H = int(mc.hidden_dim)
        self.L = int(mc.num_layers)
        self.ffn_relu = mc.ffn_activation == "relu"
        self.residual_ffn = mc.mdl_feature_interaction == "residual_ffn"
        self.ln_eps = 1e-5
        T, D, H = self.T, self.D, self.H
        if D % T:
            raise ValueError("mdl_rankmixer requires token_dim divisible by the feature token count")
        self.moe = mc.rankmixer_ffn_type == "sparse_moe"
        dom_inputs = self._domain_specs(config)
        groupwise = config.tokenization.feature_tokenizer == "groupwise"
        token_groups = [list(g.inputs) for g in res.feature_token_groups] if groupwise else None
        if groupwise and len(token_groups) != T:
            raise ValueError(f"groupwise tokenizer: {len(token_groups)} groups for {T} tokens")
        self.encoder = FeatureEncoder(config, device=dev, rank=rank, world=world, process_group=process_group,
                                      vocab_sizes=vocab_sizes, slice_tokens=0 if groupwise else T, base_seed=base_seed,
                                      domain_tokens=dom_inputs or None, token_groups=token_groups)
        from .sequence_encoders import SequenceSummaries

        # sequences summarised into feature-token or domain-token inputs
        self.summaries = SequenceSummaries(config, self.encoder, self.encoder.summary_names, device=dev)
        if groupwise:
            self.K = self.Kpad = self.encoder.group_k_pad
            fan_in = self.encoder.group_widths
        else:
            self.K = self.encoder.slice_k
            self.Kpad = self.encoder.slice_stride
            fan_in = [self.K] * T
        # feature tokenizer: T per-token linear maps of the concatenated (or grouped) inputs
        self.tok_weight = gemm_param(torch.zeros(T, D, self.Kpad, device=dev))
        self.tok_bias = nn.Parameter(torch.empty(T, D, device=dev))
        for t in range(T):
            _kaiming_uniform_(self.tok_weight.data[t, :, :fan_in[t]], fan_in[t])
            _kaiming_uniform_(self.tok_bias.data[t], fan_in[t])
        self._init_domain_inputs(config, dev, D, H)
        self.blocks = nn.ModuleList(self._make_block(dev) for _ in range(self.L))
        self._init_domain_outputs(config, dev, D, H)

    def _make_block(self, dev) -> nn.Module:
        T, D, H = self.T, self.D, self.H
        blk = nn.Module()
        blk.ln1_weight = nn.Parameter(torch.ones(D, device=dev))
        blk.ln1_bias = nn.Parameter(torch.zeros(D, device=dev))
        if self.moe:
            from ..ops.moe import build_rankmixer_moe

            blk.ffn = build_rankmixer_moe(self.config, T, device=dev)
        else:
            blk.w_in = gemm_param(torch.empty(T, H, D, device=dev))
            blk.b_in = nn.Parameter(torch.empty(T, H, device=dev))
            blk.w_out = gemm_param(torch.empty(T, D, H, device=dev))
            blk.b_out = nn.Parameter(torch.empty(T, D, device=dev))
            for t in range(T):
                _kaiming_uniform_(blk.w_in.data[t], D)
                _kaiming_uniform_(blk.b_in.data[t], D)
                _kaiming_uniform_(blk.w_out.data[t], H)
                _kaiming_uniform_(blk.b_out.data[t], H)
        if self.residual_ffn:
            blk.ln2_weight = nn.Parameter(torch.ones(D, device=dev))
            blk.ln2_bias = nn.Parameter(torch.zeros(D, device=dev))
        self._add_domain_modules(blk, dev, T, D, H)
        return blk

    # ------------------------------------------------------------------ params
    def gemm_param_names(self) -> set[str]:
        return {n for n, p in self.named_parameters() if getattr(p, "_mdl_gemm", False)}

    def dense_buckets(self) -> list[list[str]]:
        """Parameter groups in the order their gradients become final in the backward
        (heads, last block, ..., first block; the rest finishes last)."""

        names = [n for n, _ in self.named_parameters()]
        groups = [[n for n in names if n.startswith("heads.")]]
        for i in reversed(range(self.L)):
            groups.append([n for n in names if n.startswith(f"blocks.{i}.")])
        return groups

    @property
    def store(self):
        return self.encoder.store

    # ------------------------------------------------------------------ pieces
    def _cuda(self, batch) -> bool:
        return batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"

    def _tokenize(self, x0: torch.Tensor, B: int, cuda: bool) -> torch.Tensor:
        if cuda:
            from ..ops.fused import PerTokenLinearFn

            return PerTokenLinearFn.apply(x0, self.tok_weight, self.tok_bias, self.T, self.K, self.Kpad)
        xin = x0.float().view(B, self.T, self.Kpad)[:, :, :self.K]
        return torch.einsum("btk,tdk->btd", xin, self.tok_weight[:, :, :self.K]) + self.tok_bias.unsqueeze(0)

    def _feature_block(self, blk, x: torch.Tensor, cuda: bool) -> torch.Tensor:
        D = self.D
        if self.moe:
            if cuda:
                from ..ops.fused import MixLayerNormFn
                from ..ops.layers import LayerNormFn

                m = MixLayerNormFn.apply(x, blk.ln1_weight, blk.ln1_bias, self.ln_eps)
                f = blk.ffn(m)
                if not self.residual_ffn:
                    return f
                return LayerNormFn.apply(f + m, blk.ln2_weight, blk.ln2_bias, self.ln_eps)
            xf = x.float()
            m = F.layer_norm(token_mix(xf) + xf, (D,), blk.ln1_weight, blk.ln1_bias, self.ln_eps)
            f = blk.ffn(m).float()
            if not self.residual_ffn:
                return f.to(x.dtype)
            return F.layer_norm(f + m, (D,), blk.ln2_weight, blk.ln2_bias, self.ln_eps).to(x.dtype)
        if cuda and not self.ffn_relu:
            from ..ops.fused import MixLayerNormFn, RankMixerBlockFn
            from ..ops.layers import PerTokenFFNFn

            if self.residual_ffn:
                return RankMixerBlockFn.apply(x, blk.ln1_weight, blk.ln1_bias, blk.w_in, blk.b_in, blk.w_out,
                                              blk.b_out, blk.ln2_weight, blk.ln2_bias, self.ln_eps)
            m = MixLayerNormFn.apply(x, blk.ln1_weight, blk.ln1_bias, self.ln_eps)
            return PerTokenFFNFn.apply(m, blk.w_in, blk.b_in, blk.w_out, blk.b_out, False)
        act_fn = F.relu if self.ffn_relu else F.gelu
        xf = x.float()
        m = F.layer_norm(token_mix(xf) + xf, (D,), blk.ln1_weight, blk.ln1_bias, self.ln_eps)
        h = act_fn(torch.einsum("btd,thd->bth", m, blk.w_in) + blk.b_in.unsqueeze(0))
        f = torch.einsum("bth,tdh->btd", h, blk.w_out) + blk.b_out.unsqueeze(0)
        if not self.residual_ffn:
            return f.to(x.dtype)
        return F.layer_norm(f + m, (D,), blk.ln2_weight, blk.ln2_bias, self.ln_eps).to(x.dtype)

    # ------------------------------------------------------------------ forward
    def forward(self, batch, task_scale: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        from ..ops.dense import grad_ready
        from ..ops.embedding import fused_lookup

        B = batch.rows
        cuda = self._cuda(batch)
        anchor = torch.zeros(0, device=batch.ids.device, requires_grad=True)
        x0 = fused_lookup(self.store, self.encoder.plan, batch.ids, batch.offsets, batch.dense, B, anchor)
        summaries = self.summaries(self.encoder, batch, anchor, cuda) if self.summaries.names else {}
        if summaries and self.encoder.summary_cols["plan"]:
            from .sequence_encoders import add_summaries

            x0 = add_summaries(x0, summaries, self.encoder.summary_cols["plan"])
        x = self._tokenize(x0, B, cuda)
        dt = x.dtype
        mask = scenario_mask_from_ids(batch.scenario_id, self.S).to(x.device)
        s_prompt, t_prompt = self._domain_prompts(batch, B, anchor, cuda, dt, summaries)
        s, t = self._initial_states(s_prompt, t_prompt, B, dt)
        if self.scene_feature_bias is not None:
            x = self._apply_scene_bias(x, s_prompt, mask)
        w_fused = self._scene_weights(mask, include_global=self.use_global) if (s is not None) else None
        hooks = getattr(self, "dense_hooks", None) if cuda else None
        for i, blk in enumerate(self.blocks):
            x = grad_ready(x, hooks, self.L - i)  # block i's gradients are final once d(x_in) is
            x = self._feature_block(blk, x, cuda)
            s, t = self._domain_step(blk, x, s, t, s_prompt, t_prompt, w_fused)
        pred = self._readout(x, s, t, mask)
        if task_scale is None:
            task_scale = torch.full((self.ntask,), 1.0 / max(1, B), device=x.device)
        pred = grad_ready(pred, hooks, 0)
        out = self.heads(pred, batch.labels, batch.label_mask, task_scale)
        if self.moe:
            from ..ops.moe import add_moe_loss

            add_moe_loss(out, self, float(self.config.model.sparse_moe_loss_weight))
        return out
