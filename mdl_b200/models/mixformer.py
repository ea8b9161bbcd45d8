"""MixFormer: feature heads that read one long behaviour sequence through cross attention.

Reference: ``src/modules/mixformer.py`` (``MixFormerRMSNorm`` :28, ``DenseSwiGLUFFN`` :56,
``StackedPerHeadSwiGLUFFN`` :82-115, ``MixFormerHeadMixing`` :118-174,
``MixFormerQueryMixer`` :177, ``MixFormerOutputFusion`` :203,
``MixFormerCrossAttention`` :226-784, ``MixFormerBlock`` :787-845) and
``MixFormerModel`` ``src/model.py:8473-8578``.

Block (``N`` heads of width ``D``, sequence width ``N * D``):

* Query Mixer: ``x + HeadMixing(RMSNorm(x))`` (parameter-free transpose of the
  ``[N, N, D/N]`` chunks), then ``+ SwiGLU_n(RMSNorm(.))`` per head;
* Cross Attention: ``hist = s + SwiGLU(RMSNorm(s))`` viewed ``[L, N, D]``; head
  ``n`` is one full-width query: ``q' = RMSNorm(x_n) W_k[n]``,
  ``w = softmax(q' . hist[:, n] / sqrt(D))`` over valid events,
  ``x_n + (sum_l w_l hist[l, n]) W_v[n]^T`` (the reordered form: no length-sized
  K/V are materialised);
* Output Fusion: ``x + SwiGLU_n(RMSNorm(x))``.

The SwiGLU networks (per head and the sequence one) are grouped tcgen05 GEMMs
(``ops.layers.SwiGLUFn``); RMSNorm runs on the CUDA kernel.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..ops.layers import gemm_param, rms_norm, swiglu


def _kaiming_uniform_a5_(t: torch.Tensor) -> None:
    """``nn.init.kaiming_uniform_(a=sqrt(5))`` on each [out, in] slice (nn.Linear's default)."""

    for i in range(t.shape[0]):
        nn.init.kaiming_uniform_(t[i], a=math.sqrt(5))


class SwiGLUStack(nn.Module):
    """``N`` bias-free SwiGLU FFNs; ``w_ug`` stacks each head's up and gate weights."""

    def __init__(self, num: int, dim: int, hidden: int, device=None) -> None:
        super().__init__()
        self.num, self.dim, self.hidden = num, dim, hidden
        self.w_ug = gemm_param(torch.empty(num, 2 * hidden, dim, device=device))
        self.w_o = gemm_param(torch.empty(num, dim, hidden, device=device))
        _kaiming_uniform_a5_(self.w_ug.data[:, :hidden])
        _kaiming_uniform_a5_(self.w_ug.data[:, hidden:])
        _kaiming_uniform_a5_(self.w_o.data)

    def forward(self, x: torch.Tensor, native: bool) -> torch.Tensor:
        return swiglu(x, self.w_ug, self.w_o, native)


def head_mixing(x: torch.Tensor, user_heads: int | None = None) -> torch.Tensor:
    """``[B, N, D] -> [B, N, N, D/N] -> transpose(1, 2) -> [B, N, D]``.

    With ``user_heads = u`` (UI-MixFormer decoupling, reference
    ``MixFormerHeadMixing`` ``src/modules/mixformer.py:118-174``) the first ``u``
    output heads keep only the chunks that came from the first ``u`` input heads
    (columns ``[0, u * D/N)``); item heads keep everything."""

    B, N, D = x.shape
    y = x.reshape(B, N, N, D // N).transpose(1, 2).reshape(B, N, D)
    if user_heads is None:
        return y
    keep = torch.ones(N, D, dtype=y.dtype, device=y.device)
    keep[:user_heads, user_heads * (D // N):] = 0
    return y * keep


class MixFormerBlock(nn.Module):
    def __init__(self, num_heads: int, dim: int, hidden: int, seq_hidden: int, device=None,
                 user_heads: int | None = None) -> None:
        super().__init__()
        if dim % num_heads:
            raise ValueError("MixFormer head width must be divisible by the head count")
        if user_heads is not None and not 0 < user_heads < num_heads:
            raise ValueError("mixformer_user_head_count must be inside (0, heads)")
        N, D = num_heads, dim
        self.N, self.D = N, D
        self.user_heads = user_heads
        self.qm_norm = nn.Parameter(torch.ones(D, device=device))
        self.qm_ffn_norm = nn.Parameter(torch.ones(D, device=device))
        self.qm_ffn = SwiGLUStack(N, D, hidden, device=device)
        self.seq_norm = nn.Parameter(torch.ones(N * D, device=device))
        self.seq_ffn = SwiGLUStack(1, N * D, seq_hidden, device=device)
        self.key_weight = nn.Parameter(torch.empty(N, D, D, device=device))
        self.value_weight = nn.Parameter(torch.empty(N, D, D, device=device))
        for n in range(N):
            nn.init.xavier_uniform_(self.key_weight.data[n])
            nn.init.xavier_uniform_(self.value_weight.data[n])
        self.q_norm = nn.Parameter(torch.ones(D, device=device))
        self.of_norm = nn.Parameter(torch.ones(D, device=device))
        self.of_ffn = SwiGLUStack(N, D, hidden, device=device)

    def history(self, seq: torch.Tensor, native: bool) -> torch.Tensor:
        """``s + SwiGLU(RMSNorm(s))`` viewed ``[B, L, N, D]``."""

        B, L, W = seq.shape
        flat = seq.reshape(B * L, 1, W)
        h = flat + self.seq_ffn(rms_norm(flat, self.seq_norm, native=native), native)
        return h.view(B, L, self.N, self.D)

    def query_mix(self, x: torch.Tensor, native: bool) -> torch.Tensor:
        """Query Mixer: ``x + HeadMixing(RMSNorm(x))``, then ``+ SwiGLU_n(RMSNorm(.))``."""

        x = x + head_mixing(rms_norm(x, self.qm_norm, native=native), self.user_heads)
        return x + self.qm_ffn(rms_norm(x, self.qm_ffn_norm, native=native), native)

    def output_fusion(self, x: torch.Tensor, native: bool) -> torch.Tensor:
        return x + self.of_ffn(rms_norm(x, self.of_norm, native=native), native)

    def forward(self, x: torch.Tensor, seq: torch.Tensor, valid: torch.Tensor, native: bool) -> torch.Tensor:
        """``x [B, N, D]`` heads, ``seq [B, L, N*D]``, ``valid [B, L]`` -> ``[B, N, D]``."""

        return self.output_fusion(self.cross_attention(self.query_mix(x, native), seq, valid, native), native)

    def cross_attention(self, x: torch.Tensor, seq: torch.Tensor, valid: torch.Tensor, native: bool) -> torch.Tensor:
        """Reordered single-query cross attention of each head over the history."""

        hist = self.history(seq, native)
        B, L = hist.shape[0], hist.shape[1]
        if native:
            # fused kernel: the bf16 history is streamed once, in place (valid events are a suffix)
            from ..ops.attention import single_query_attention

            qn = rms_norm(x, self.q_norm, native=native).float()
            sq = torch.einsum("bno,noi->bni", qn, self.key_weight)
            kstart = (L - valid.sum(dim=1)).to(torch.int32)
            ctx = single_query_attention(sq, hist, kstart, 1.0 / math.sqrt(self.D))
            return x + torch.einsum("bni,noi->bno", ctx, self.value_weight).to(x.dtype)
        # one fp32 copy of the history in head-major order [B, N, L, D] (conversion and
        # transpose in a single pass), read by both batched products
        hf = torch.empty(B, self.N, L, self.D, dtype=torch.float32, device=hist.device)
        hf.copy_(hist.permute(0, 2, 1, 3))
        qn = rms_norm(x, self.q_norm, native=native).float()
        sq = torch.einsum("bno,noi->bni", qn, self.key_weight)                 # q' = q W_k
        scores = torch.matmul(sq.unsqueeze(2), hf.transpose(-1, -2)).squeeze(2) / math.sqrt(self.D)  # [B, N, L]
        mask = valid.bool().unsqueeze(1)
        scores = scores.masked_fill(~mask, float("-inf"))
        w = torch.nan_to_num(torch.softmax(scores, dim=-1)) * mask
        ctx = torch.matmul(w.unsqueeze(2), hf).squeeze(2)                      # [B, N, D]
        return x + torch.einsum("bni,noi->bno", ctx, self.value_weight).to(x.dtype)

    def reference_state_dict(self, prefix: str) -> dict[str, torch.Tensor]:
        H = self.qm_ffn.hidden
        Hs = self.seq_ffn.hidden
        sd = {prefix + "query_mixer.input_norm.weight": self.qm_norm,
              prefix + "query_mixer.ffn_norm.weight": self.qm_ffn_norm,
              prefix + "query_mixer.ffn.up_weight": self.qm_ffn.w_ug[:, :H],
              prefix + "query_mixer.ffn.gate_weight": self.qm_ffn.w_ug[:, H:],
              prefix + "query_mixer.ffn.output_weight": self.qm_ffn.w_o,
              prefix + "cross_attention.sequence_norm.weight": self.seq_norm,
              prefix + "cross_attention.sequence_ffn.up_projection.weight": self.seq_ffn.w_ug[0, :Hs],
              prefix + "cross_attention.sequence_ffn.gate_projection.weight": self.seq_ffn.w_ug[0, Hs:],
              prefix + "cross_attention.sequence_ffn.output_projection.weight": self.seq_ffn.w_o[0],
              prefix + "cross_attention.key_weight": self.key_weight,
              prefix + "cross_attention.value_weight": self.value_weight,
              prefix + "cross_attention.query_norm.weight": self.q_norm,
              prefix + "output_fusion.norm.weight": self.of_norm,
              prefix + "output_fusion.ffn.up_weight": self.of_ffn.w_ug[:, :H],
              prefix + "output_fusion.ffn.gate_weight": self.of_ffn.w_ug[:, H:],
              prefix + "output_fusion.ffn.output_weight": self.of_ffn.w_o}
        return {k: v.detach().clone() for k, v in sd.items()}


class MixFormerHead(nn.Module):
    """Feature heads (an ``auto_split`` MLP of the scalar inputs to ``N x D``) that read
    a token sequence ``[B, L, W]`` (projected to ``N * D``) through MixFormer blocks;
    the heads are flattened for the task heads."""

    def __init__(self, k_in: int, k_log: int, seq_width: int, num_heads: int, dim: int, hidden: int, seq_hidden: int,
                 layers: int, device=None, user_heads: int | None = None) -> None:
        super().__init__()
        from .longer import _MLP  # deferred: longer imports this module

        self.N, self.D = num_heads, dim
        self.feature_mlp = _MLP(k_in, k_log, hidden, num_heads * dim, device=device)
        self.seq_proj = gemm_param(torch.empty(num_heads * dim, seq_width, device=device))
        nn.init.kaiming_uniform_(self.seq_proj.data, a=math.sqrt(5))
        self.blocks = nn.ModuleList(MixFormerBlock(num_heads, dim, hidden, seq_hidden, device=device,
                                                   user_heads=user_heads) for _ in range(layers))
        self.output_dim = num_heads * dim

    def inputs(self, feat_in: torch.Tensor, seq: torch.Tensor, native: bool):
        """Feature heads ``[B, N, D]`` and the projected sequence ``[B, L, N * D]``."""

        B, L, W = seq.shape
        x = self.feature_mlp(feat_in, native).view(B, self.N, self.D)
        if native:
            from ..ops.layers import LinearFn

            s = LinearFn.apply(seq.reshape(B * L, W).to(torch.bfloat16), self.seq_proj, None).view(B, L, -1)
        else:
            s = (seq.float().reshape(B * L, W) @ self.seq_proj.t()).view(B, L, self.N * self.D)
        return x, s

    def forward(self, feat_in: torch.Tensor, seq: torch.Tensor, valid: torch.Tensor, native: bool) -> torch.Tensor:
        x, s = self.inputs(feat_in, seq, native)
        for blk in self.blocks:
            x = blk(x, s, valid, native)
        return x.reshape(x.shape[0], self.N * self.D)


class MixFormerModel(nn.Module):
    """``model.name: mixformer``: ``num_ns_tokens`` (or the feature-token count) feature
    heads of width ``token_dim`` from the scalar inputs (``auto_split`` MLP), one raw
    behaviour sequence whose events (field embeddings through a step MLP) form the
    ``N * token_dim`` sequence, ``num_layers`` MixFormer blocks, flattened heads ->
    task heads (reference ``MixFormerModel`` ``src/model.py:8473-8578``)."""

    def __init__(self, config, *, device: torch.device, rank: int = 0, world: int = 1, process_group=None,
                 vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None,
                 domain_tokens: list[list[str]] | None = None, task_heads: bool = True) -> None:
        super().__init__()
        from .features import FeatureEncoder
        from .heads import TaskHeads
        from .longer import _MLP

        m = config.model
        seq_by_name = {s.name: s for s in config.sequences}
        groups = config.resolved.tokenization.sequence_token_groups
        if groups:
            raw = []
            for g in groups:
                if len(g.inputs) != 1 or g.inputs[0] not in seq_by_name:
                    raise NotImplementedError(f"MixFormer sequence token group {g.name!r}: a group holds one raw "
                                              "sequence")
                raw.append(seq_by_name[g.inputs[0]])
        else:
            raw = [s for s in config.sequences if s.encoder == "raw"]
        if not raw or any(not s.max_length for s in raw):
            raise ValueError("MixFormer needs at least one raw sequence with max_length")
        self.config = config
        self.seq = raw[0]
        self.group_seqs = raw
        self.multi = len(raw) > 1
        by_name = {f.name: f for f in config.features}
        ns_inputs = [n for n in config.resolved.tokenization.feature_token_inputs if n in by_name]
        self.encoder = FeatureEncoder(config, device=device, rank=rank, world=world, process_group=process_group,
                                      vocab_sizes=vocab_sizes, input_names=ns_inputs, slice_tokens=1,
                                      base_seed=base_seed, sequences=raw, domain_tokens=domain_tokens)
        from .sequence_encoders import SequenceSummaries

        # prior sequences of the MDL domain tokens (mean_pool / attention_pool / longer / stca)
        self.summaries = SequenceSummaries(config, self.encoder, self.encoder.summary_names, device=device)
        N = int(m.num_ns_tokens or config.resolved.tokenization.feature_token_count)
        Dh = int(m.token_dim)
        self.N, self.D, self.L = N, Dh, int(self.seq.max_length)
        if self.multi:
            # several behaviour sequences: one bias-free alignment to N * D per group, then
            # SEP tokens (intent_ordered) or type embeddings + time order (timestamp_aware)
            from .sequence_fusion import SequenceGroups

            self.seq_groups = SequenceGroups(config, self.encoder, raw, N * Dh, projection="linear", device=device)
            self.L = self.seq_groups.S
        else:
            plan = self.encoder.seq_plans[self.seq.name]
            self.step = _MLP(plan.out_ld, plan.out_width, int(m.hidden_dim), N * Dh, device=device)
        self.mixer = MixFormerHead(self.encoder.plan.out_ld, self.encoder.plan.out_width, N * Dh, N, Dh,
                                   int(m.hidden_dim), int(m.hidden_dim), max(1, int(m.num_layers)), device=device,
                                   user_heads=m.mixformer_user_head_count)
        self.ntask = len(config.task_names)
        self.task_query = None
        if task_heads:
            head_in = N * Dh
            if m.readout == "task_query":
                from .heads import TaskQueryReadout

                self.task_query = TaskQueryReadout(self.ntask, Dh, int(m.num_heads), N, int(m.hidden_dim),
                                                   m.ffn_activation, float(m.init_std), device=device)
                head_in = Dh
            self.heads_mod = TaskHeads(self.ntask, head_in, int(m.task_head_hidden_dim or 4 * Dh),
                                       m.task_head_activation, device=device)

    def gemm_param_names(self) -> set[str]:
        return {n for n, p in self.named_parameters() if getattr(p, "_mdl_gemm", False)}

    def dense_buckets(self) -> list[list[str]]:
        names = [n for n, _ in self.named_parameters()]
        return [[n for n in names if n.startswith("heads_mod.")], [n for n in names if not n.startswith("heads_mod.")]]

    @property
    def store(self):
        return self.encoder.store

    def _inputs(self, batch, anchor, native: bool):
        """Scalar inputs ``[B, K]``, event tokens ``[B, L, N * D]`` and their validity ``[B, L]``."""

        from ..ops.embedding import fused_lookup
        from .features import lookup_sequence

        B, L = batch.rows, self.L
        feat_in = fused_lookup(self.store, self.encoder.plan, batch.ids, batch.offsets, batch.dense, B, anchor)
        if self.multi:
            tokens, lengths = self.seq_groups(self.encoder, batch, anchor, native)
            if native:
                tokens = tokens.to(torch.bfloat16)
        else:
            seq_in, lengths = lookup_sequence(self.encoder, batch, self.seq.name, B, L, anchor)
            tokens = self.step(seq_in, native).view(B, L, self.N * self.D)
        e = torch.arange(L, device=tokens.device)
        valid = e.view(1, -1) >= (L - lengths.clamp(0, L)).view(-1, 1)
        return feat_in, tokens, valid

    def forward(self, batch, task_scale: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        native = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
        anchor = torch.zeros(0, device=batch.ids.device, requires_grad=True)
        B = batch.rows
        feat_in, tokens, valid = self._inputs(batch, anchor, native)
        # the head's sequence projection sees the already N*D-wide event tokens
        readout = self.mixer(feat_in, tokens, valid, native)
        if task_scale is None:
            task_scale = torch.full((self.ntask,), 1.0 / max(1, B), device=readout.device)
        if self.task_query is not None:
            states = self.task_query(readout.view(B, self.N, self.D))
            return self.heads_mod(states, batch.labels, batch.label_mask, task_scale)
        return self.heads_mod.forward_shared(readout, batch.labels, batch.label_mask, task_scale)


class ScenarioQueryRouter(nn.Module):
    """Routes the active scene's state into the MixFormer query heads (reference
    ``ScenarioConditionedQueryRouter`` ``src/model.py:8581-8619``):
    ``q + sigmoid(W_g c + b_g)[:, :, None] * (W_d c)[:, None]`` with ``c = RMSNorm(ctx)``;
    ``W_d`` starts at zero (the router starts as the identity) and ``b_g`` at -2."""

    def __init__(self, num_heads: int, dim: int, device=None) -> None:
        super().__init__()
        from ..ops.layers import Linear

        self.context_norm = nn.Parameter(torch.ones(dim, device=device))
        self.head_gate = Linear(dim, num_heads, device=device)
        self.context_delta = Linear(dim, dim, bias=False, device=device)
        nn.init.kaiming_uniform_(self.head_gate.weight, a=math.sqrt(5))
        nn.init.constant_(self.head_gate.bias, -2.0)
        nn.init.zeros_(self.context_delta.weight)

    def forward(self, queries: torch.Tensor, context: torch.Tensor, native: bool) -> torch.Tensor:
        c = rms_norm(context.unsqueeze(1), self.context_norm, native=native).squeeze(1)
        if not native:
            c = c.float()
        gates = torch.sigmoid(self.head_gate(c).float()).unsqueeze(-1)
        delta = self.context_delta(c.contiguous()).float().unsqueeze(1)
        return (queries.float() + gates * delta).to(queries.dtype)


def build_mixformer(config, **kw):
    if config.model.name == "mixformer":
        return MixFormerModel(config, **kw)
    from .mdl_mixformer import MDLMixFormerModel

    return MDLMixFormerModel(config, **kw)
