"""Several raw sequences fused into one token sequence (OneTrans S tokens, MixFormer
behaviour tokens).

Counterpart of the reference ``OneTransTokenizer`` sequence part
(``src/model.py:4571-5296``; ``_sequence_token_part`` :5143-5218) and the
``MixFormerTokenizer`` alignment (:5347-5476):

* every sequence token group (one raw sequence here) has its own projection of
  the event values: the OneTrans projection MLP (``Linear -> GELU -> Linear`` to
  ``token_dim``) or the MixFormer bias-free ``Linear`` to ``N * token_dim``;
* ``intent_ordered``: groups in configured order, a learned SEP token between
  consecutive groups (``model.use_sep_tokens``), then the valid tokens compacted
  in order (padding first: the per-sample ``kstart`` of the attention kernels);
* ``timestamp_aware``: a learned type embedding per group is added to its tokens,
  then every valid event of all groups is ordered oldest to newest by its
  ``timestamp_field`` (ascending) or ``time_delta_field`` (descending age), padding
  first; ``model.global_sequence_max_length`` keeps only that many newest events.

``forward`` returns ``(tokens [B, S, width], valid_count [B])`` with the valid tokens
at the end of the ``S = sum(max_length) + separators`` positions.
"""

from __future__ import annotations

import torch
from torch import nn


class SequenceGroups(nn.Module):
    def __init__(self, config, encoder, sequences: list, width: int, *, projection: str, hidden: int = 0,
                 device=None) -> None:
        super().__init__()
        from ..ops.layers import Linear
        from .longer import _MLP

        m = config.model
        self.names = [s.name for s in sequences]
        self.lengths = [int(s.max_length) for s in sequences]
        for s in sequences:
            if not s.max_length:
                raise ValueError(f"sequence {s.name!r} needs max_length")
        self.fusion = m.sequence_fusion
        if self.fusion not in ("intent_ordered", "timestamp_aware"):
            raise ValueError(f"model.sequence_fusion {self.fusion!r}")
        self.width = int(width)
        self.kind = projection
        self.proj = nn.ModuleList()
        for s in sequences:
            plan = encoder.seq_plans[s.name]
            if projection == "mlp":
                self.proj.append(_MLP(plan.out_ld, plan.out_width, int(hidden), self.width, device=device))
            else:
                lin = Linear(plan.out_ld, self.width, bias=False, device=device)
                with torch.no_grad():
                    lin.weight[:, plan.out_width:].zero_()
                self.proj.append(lin)
        G = len(sequences)
        std = float(m.init_std)
        self.seps = G - 1 if (self.fusion == "intent_ordered" and m.use_sep_tokens) else 0
        self.sep = nn.Parameter(torch.randn(self.seps, self.width, device=device) * std) if self.seps else None
        self.type_emb = (nn.Parameter(torch.randn(G, self.width, device=device) * std)
                         if self.fusion == "timestamp_aware" else None)
        self.S = sum(self.lengths) + self.seps
        # timestamp_aware with model.global_sequence_max_length: only the newest events of
        # all groups together are kept (reference ``_global_timestamp_sequence_token_part``)
        limit = getattr(m, "global_sequence_max_length", None)
        self.keep = int(limit) if (limit and self.fusion == "timestamp_aware" and int(limit) < self.S) else 0
        if self.keep:
            self.S = self.keep
        # temporal keys (timestamp_aware): the dense column of each sequence's time field
        self.time_cols: list[tuple[int, float]] = []
        if self.fusion == "timestamp_aware":
            for s in sequences:
                field, sign = (s.timestamp_field, 1.0) if s.timestamp_field else (s.time_delta_field, -1.0)
                if not field:
                    raise ValueError(f"timestamp_aware fusion: sequence {s.name!r} has neither timestamp_field "
                                     "nor time_delta_field")
                dens = encoder.seq_dense_fields[s.name]
                if field not in dens:
                    raise ValueError(f"sequence {s.name!r}: temporal field {field!r} must be a dense field")
                col = 0
                for fl in s.fields:
                    if fl.kind == "dense":
                        if fl.name == field:
                            break
                        col += int(fl.dimension)
                self.time_cols.append((col, sign))

    def _project(self, g: int, x: torch.Tensor, native: bool) -> torch.Tensor:
        if self.kind == "mlp":
            return self.proj[g](x, native)
        return self.proj[g](x if native else x.float())

    def forward(self, encoder, batch, anchor: torch.Tensor, native: bool):
        from .features import expand_requests, lookup_sequence

        B = batch.rows
        parts, masks, keys = [], [], []
        for g, (name, L) in enumerate(zip(self.names, self.lengths)):
            # events projected once per request, then handed to the request's candidates
            seq_in, lengths, ri = lookup_sequence(encoder, batch, name, B, L, anchor, expand=False)
            tok = self._project(g, seq_in, native).view(lengths.shape[0], L, self.width)
            tok = expand_requests(tok, ri)
            lengths = expand_requests(lengths, ri)
            if not native:
                tok = tok.float()
            if self.type_emb is not None:
                tok = tok + self.type_emb[g].to(tok.dtype)
            e = torch.arange(L, device=tok.device)
            valid = e.view(1, -1) >= (L - lengths.clamp(0, L)).view(-1, 1)
            parts.append(tok)
            masks.append(valid)
            if self.type_emb is not None:
                col, sign = self.time_cols[g]
                seq = batch.sequences[name]
                t = seq["dense"][:, col].float().view(-1, L)
                ri = seq.get("row_indices")
                if ri is not None:
                    t = t.index_select(0, ri.to(t.device))
                keys.append(t.to(tok.device) * sign)
            elif self.sep is not None and g < self.seps:
                parts.append(self.sep[g].to(tok.dtype).view(1, 1, -1).expand(B, 1, -1))
                masks.append(torch.ones(B, 1, dtype=torch.bool, device=tok.device))
        tokens = torch.cat(parts, dim=1)
        mask = torch.cat(masks, dim=1)
        if self.type_emb is not None:
            key = torch.cat(keys, dim=1).masked_fill(~mask, float("-inf"))
            order = torch.argsort(key, dim=1, stable=True)
        else:
            order = torch.argsort(mask.to(torch.int8), dim=1, stable=True)  # padding first, order kept
        if self.keep:
            order = order[:, -self.keep:]  # the newest events (padding sorts first)
        tokens = tokens.gather(1, order.unsqueeze(-1).expand(-1, -1, tokens.shape[-1]))
        kept = mask.gather(1, order)
        tokens = tokens * kept.unsqueeze(-1).to(tokens.dtype)
        return tokens, kept.sum(dim=1)
