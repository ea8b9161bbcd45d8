"""Sequence summaries that feed feature tokens (and MDL domain tokens).

A sequence whose ``encoder`` is ``mean_pool``, ``attention_pool``, ``longer`` or
``stca`` is summarised into a fixed-width vector that takes the place of a scalar
input: its columns are reserved in the tokenizer (or domain-token) input matrix
and filled after the embedding lookup. Counterpart of the sequence branch of the
reference ``FeatureEncoderBank`` (``src/model.py:2519-2790`` construction,
``_pool_sequence`` :3451-3588):

* events: the concatenated field values of each event (categorical embeddings,
  then dense fields, looked up once per event by the fused lookup kernel);
* ``mean_pool`` / ``attention_pool``: ``Linear(event width -> pool_dim)`` plus a
  learned position embedding, then the masked mean, or a masked softmax over
  ``tokens . q / sqrt(pool_dim)`` with the query projected from the
  ``target_inputs`` (or a learned query without targets); output width
  ``pool_dim * rankmixer_summary_tokens``;
* ``longer``: the LONGER encoder (projection MLP, global tokens = user globals,
  CLS tokens and candidate globals projected from ``target_inputs``, cross block
  over the most recent ``longer_query_tokens`` events, self blocks); output the
  global tokens (``longer_output: summary``) or every token (``full``);
* ``stca``: the STCA encoder (``models/stca.py``).

Positions: event ``e`` of a left-padded window of ``L`` events with ``n`` valid
events has position ``e - (L - n)`` (0 = oldest kept event); padding rows are
masked. For ``longer`` the position embedding is added to the event columns
before ``time_delta_field`` (the reference keeps the time delta out of it).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

SUMMARY_ENCODERS = ("mean_pool", "attention_pool", "longer", "stca")


def summary_width(seq) -> int:
    """Columns a sequence summary occupies in a token input matrix."""

    if seq.encoder == "stca":
        return int(seq.stca_dim)
    if seq.encoder in ("mean_pool", "attention_pool"):
        return int(seq.pool_dim) * int(seq.rankmixer_summary_tokens)
    if seq.encoder == "longer":
        dim = int(seq.longer_dim) * int(seq.longer_token_merge)
        tokens = int(seq.rankmixer_summary_tokens)
        if seq.longer_output != "summary":
            tokens += int(seq.longer_query_tokens)
        return tokens * dim
    raise ValueError(f"sequence {seq.name!r}: encoder {seq.encoder!r} has no summary")


def valid_mask(lengths: torch.Tensor, L: int) -> torch.Tensor:
    """``[B, L]`` validity of a left-padded window (the last ``lengths[b]`` events)."""

    e = torch.arange(L, device=lengths.device)
    return e.view(1, -1) >= (L - lengths.clamp(0, L)).view(-1, 1)


def positions(lengths: torch.Tensor, L: int) -> torch.Tensor:
    """``[B, L]`` position of every event (0 = oldest valid event; clamped at 0 on padding)."""

    e = torch.arange(L, device=lengths.device)
    return (e.view(1, -1) - (L - lengths.clamp(0, L)).view(-1, 1)).clamp(min=0)


class PoolSequenceEncoder(nn.Module):
    """``mean_pool`` / ``attention_pool`` summary of one sequence."""

    def __init__(self, seq, k_in: int, k_log: int, target_k: int, target_log: int, init_std: float,
                 device=None) -> None:
        super().__init__()
        from ..ops.layers import Linear

        self.mode = seq.encoder
        self.L = int(seq.max_length)
        self.P = int(seq.pool_dim)
        self.S = int(seq.rankmixer_summary_tokens)
        self.step = Linear(k_in, self.P, device=device)
        with torch.no_grad():  # padded input columns contribute nothing
            self.step.weight[:, k_log:].zero_()
        self.pos = nn.Parameter(torch.randn(self.L, self.P, device=device) * init_std)
        self.query = None
        self.query_proj = None
        if self.mode == "attention_pool":
            if target_k:
                self.query_proj = Linear(target_k, self.S * self.P, device=device)
                with torch.no_grad():
                    self.query_proj.weight[:, target_log:].zero_()
            else:
                self.query = nn.Parameter(torch.randn(1, self.S, self.P, device=device) * init_std)

    def forward(self, seq_in: torch.Tensor, lengths: torch.Tensor, target: torch.Tensor | None,
                row_indices: torch.Tensor | None = None) -> torch.Tensor:
        """``seq_in``/``lengths`` per request (``row_indices``: candidate -> request) or per
        candidate; the event projection and the mean pool run once per request."""

        from .features import expand_requests

        R, L, P = lengths.shape[0], self.L, self.P
        tokens = self.step(seq_in).float().view(R, L, P)
        tokens = tokens + self.pos.float()[positions(lengths, L)]
        mask = valid_mask(lengths, L)
        m = mask.unsqueeze(-1).float()
        if self.mode == "mean_pool":
            pooled = (tokens * m).sum(dim=1) / m.sum(dim=1).clamp_min(1.0)
            pooled = expand_requests(pooled, row_indices)
            return pooled.repeat(1, self.S) if self.S > 1 else pooled
        tokens = expand_requests(tokens, row_indices)
        mask = expand_requests(mask, row_indices)
        B = tokens.shape[0]
        if self.query_proj is not None:
            q = self.query_proj(target).float().view(B, self.S, P)
        else:
            q = self.query.float().expand(B, -1, -1)
        scores = torch.einsum("blp,bsp->bsl", tokens, q) / math.sqrt(P)
        scores = scores.masked_fill(~mask.unsqueeze(1), -1.0e9)
        w = torch.softmax(scores, dim=-1) * mask.unsqueeze(1).float()
        w = w / w.sum(dim=-1, keepdim=True).clamp_min(1.0e-9)
        return torch.einsum("bsl,blp->bsp", w, tokens).reshape(B, self.S * P)


class LongerSummaryEncoder(nn.Module):
    """``encoder: longer`` as a feature encoder: LONGER tokens -> summary vector."""

    def __init__(self, config, seq, encoder, target_k: int, target_log: int, user_k: int, user_log: int,
                 device=None) -> None:
        super().__init__()
        from .longer import LongerEncoder, _SlicePlan

        self.summary = seq.longer_output == "summary"
        self.cls = int(seq.longer_cls_tokens)
        self.longer = LongerEncoder(config, seq, encoder, _SlicePlan(target_k, target_log) if target_k else None,
                                    _SlicePlan(user_k, user_log) if user_k else None, device=device,
                                    extra_globals=self.cls, time_delta=_time_delta_cols(seq, encoder))
        D = self.longer.D
        self.cls_tokens = (nn.Parameter(torch.randn(1, self.cls, D, device=device) * float(config.model.init_std))
                           if self.cls else None)
        want = int(seq.rankmixer_summary_tokens)
        if self.longer.G != want:
            raise ValueError(f"LONGER sequence {seq.name!r}: {self.longer.G} global tokens (user "
                             f"{self.longer.Gu} + cls {self.cls} + candidate {self.longer.Gc}) != "
                             f"rankmixer_summary_tokens {want}")

    def forward(self, seq_in, lengths, target, user, native: bool, row_indices=None) -> torch.Tensor:
        from .features import expand_requests
        from .longer import LongerEncoder

        # event tokens once per request, then each candidate takes its request's tokens
        tokens = expand_requests(self.longer.project(seq_in, lengths, native), row_indices)
        lengths = expand_requests(lengths, row_indices)
        X = self.longer(None, lengths, target, user, native, cls_tokens=self.cls_tokens, tokens=tokens,
                        summary_only=self.summary)
        G = self.longer.G
        B = lengths.shape[0]
        if self.summary:
            return X.reshape(B, -1).float()  # the G global tokens
        return LongerEncoder.reference_order(X, G).reshape(B, -1).float()


def _time_delta_cols(seq, encoder) -> tuple[int, int] | None:
    """Logical columns ``[c0, c1)`` of ``time_delta_field`` in the event rows."""

    if not seq.time_delta_field:
        return None
    plan = encoder.seq_plans[seq.name]
    name = f"{seq.name}.{seq.time_delta_field}"
    for lf in plan.features:
        if lf.name == name:
            return (lf.out_col, lf.out_col + lf.width)
    raise ValueError(f"sequence {seq.name!r}: time_delta_field {seq.time_delta_field!r} is not one of its fields")


class SequenceSummaries(nn.Module):
    """Every summary sequence of a model, evaluated once per batch.

    ``forward`` returns ``{sequence name: [B, summary_width] fp32}``; the caller adds
    each summary into the columns the feature encoder reserved for it."""

    def __init__(self, config, encoder, names: list[str], device=None) -> None:
        super().__init__()
        from .longer import _MLP
        from .stca import STCAEncoder

        seq_by_name = {s.name: s for s in config.sequences}
        self.names = [n for n in names if n in seq_by_name]
        self.mods = nn.ModuleDict()
        self.meta: dict[str, tuple] = {}
        kp = encoder.target_k_pad
        for name in self.names:
            seq = seq_by_name[name]
            sp = encoder.seq_plans[name]
            tgt = encoder.target_index.get((name, "target"))
            usr = encoder.target_index.get((name, "user"))
            tlog = encoder.target_widths[tgt] if tgt is not None else 0
            ulog = encoder.target_widths[usr] if usr is not None else 0
            if seq.encoder in ("mean_pool", "attention_pool"):
                if seq.encoder == "attention_pool" and tgt is None and seq.target_inputs:
                    raise ValueError(f"sequence {name!r}: target inputs are not scalar features")
                mod = PoolSequenceEncoder(seq, sp.out_ld, sp.out_width, kp if tgt is not None else 0, tlog,
                                          float(config.model.init_std), device=device)
            elif seq.encoder == "longer":
                mod = LongerSummaryEncoder(config, seq, encoder, kp if tgt is not None else 0, tlog,
                                           kp if usr is not None else 0, ulog, device=device)
            elif seq.encoder == "stca":
                if tgt is None:
                    raise ValueError(f"STCA sequence {name!r} needs target_inputs")
                d = int(seq.stca_dim)
                ratio = int(seq.stca_expansion_ratio)
                mod = nn.Module()
                mod.step = _MLP(sp.out_ld, sp.out_width, d * ratio, d, device=device)
                mod.target = _MLP(kp, kp, d * ratio, d, device=device)
                mod.encoder = STCAEncoder(d, int(seq.stca_num_heads or config.model.num_heads), int(seq.stca_layers),
                                          ratio, device=device)
            else:
                raise ValueError(f"sequence {name!r}: encoder {seq.encoder!r} is not a summary encoder")
            self.mods[name] = mod
            self.meta[name] = (seq.encoder, int(seq.max_length or 0), tgt, usr)

    def forward(self, model_encoder, batch, anchor: torch.Tensor, native: bool) -> dict[str, torch.Tensor]:
        from ..ops.embedding import fused_lookup
        from .features import lookup_sequence

        if not self.names:
            return {}
        B = batch.rows
        enc = model_encoder
        targets = None
        if enc.target_plan is not None:
            targets = fused_lookup(enc.store, enc.target_plan, batch.ids, batch.offsets, batch.dense, B, anchor)
        kp = enc.target_k_pad

        def group(i):
            if i is None:
                return None
            g = targets[:, i * kp:(i + 1) * kp]
            return g if native else g.float()

        out = {}
        for name in self.names:
            kind, L, ti, ui = self.meta[name]
            mod = self.mods[name]
            seq_in, lengths, ri = lookup_sequence(enc, batch, name, B, L, anchor, expand=False)
            if not native:
                seq_in = seq_in.float()
            if kind in ("mean_pool", "attention_pool"):
                out[name] = mod(seq_in, lengths, group(ti), ri)
            elif kind == "longer":
                out[name] = mod(seq_in, lengths, group(ti), group(ui), native, ri)
            else:  # stca: history projection and per-layer transforms once per request
                hist = mod.step(seq_in, native).view(lengths.shape[0], L, -1)
                target = mod.target(group(ti), native)
                out[name] = mod.encoder(hist, valid_mask(lengths, L), target, native, row_indices=ri).float()
        return out


def add_summaries(x: torch.Tensor, summaries: dict[str, torch.Tensor], cols: list) -> torch.Tensor:
    """Add each summary into its reserved (physical) columns of ``x``."""

    for name, idx in cols:
        x = x.index_add(1, idx.to(x.device), summaries[name].to(x.dtype))
    return x
