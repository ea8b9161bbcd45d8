"""STCA: stacked target-to-history cross attention, a sequence encoder with one query.

Reference: ``src/modules/stca.py`` (``SwiGLUFFN`` :70-95, ``SingleQueryTargetAttention``
:97-610, ``STCAInputLayer`` :613-677, ``STCASequenceEncoder`` :680-975); the
encoder's output token ``z`` is a feature-token input of the ranker
(``FeatureEncoderBank`` ``src/model.py:2678-2700``).

Per layer ``i``: ``X_i = LN_i(SwiGLU_i(X))`` (history transform), attention of the
single query ``q_i`` over ``X_i`` (per head ``h``: ``s = (q W_Q)_h W_K[h]``,
``w = softmax(s . X_i / sqrt(d_h))`` over valid events, ``(sum_l w_l X_i[l]) W_V[h]^T``,
heads concatenated, output projection -- the reordered single-query form, no
length-sized K/V), then ``q_{i+1} = LN_{i+1}(SwiGLU_{i+1}(P_i [o_0 .. o_i, x_t]))``;
``z = SwiGLU_f(P_f [o_0 .. o_{M-1}, x_t])``. ``q_0 = LN_0(SwiGLU_0(x_t))`` for the target
token ``x_t``. Projections are bias-free (the paper's parameterisation).

History transforms are grouped-GEMM SwiGLUs and LayerNorm on the CUDA kernels; the
per-sample attention of the H score vectors over the history is the shared-history kernel of
``csrc/sqa.cu`` (one warp per sample, the bf16 history read once for every head; the
history gradient summed over the heads in the same pass).
"""

from __future__ import annotations

import math

import torch
from torch import nn

from ..ops.attention import shared_query_attention, shared_query_supported
from ..ops.layers import gemm_param, layer_norm, linear_nb, swiglu


def _linear_init(t: torch.Tensor) -> None:
    nn.init.kaiming_uniform_(t, a=math.sqrt(5))


class _SwiGLU(nn.Module):
    def __init__(self, dim: int, hidden: int, device=None) -> None:
        super().__init__()
        self.dim, self.hidden = dim, hidden
        self.w_ug = gemm_param(torch.empty(1, 2 * hidden, dim, device=device))
        self.w_o = gemm_param(torch.empty(1, dim, hidden, device=device))
        _linear_init(self.w_ug.data[0, :hidden])
        _linear_init(self.w_ug.data[0, hidden:])
        _linear_init(self.w_o.data[0])

    def forward(self, x: torch.Tensor, native: bool) -> torch.Tensor:
        shape = x.shape
        y = swiglu(x.reshape(-1, 1, shape[-1]), self.w_ug, self.w_o, native)
        return y.view(shape)


class STCALayer(nn.Module):
    def __init__(self, dim: int, heads: int, ratio: int, device=None) -> None:
        super().__init__()
        self.dim, self.heads, self.hd = dim, heads, dim // heads
        self.ffn = _SwiGLU(dim, ratio * dim, device=device)
        self.ln_w = nn.Parameter(torch.ones(dim, device=device))
        self.ln_b = nn.Parameter(torch.zeros(dim, device=device))
        self.wq = gemm_param(torch.empty(dim, dim, device=device))
        self.wk = nn.Parameter(torch.empty(dim, dim, device=device))
        self.wv = nn.Parameter(torch.empty(dim, dim, device=device))
        self.wo = gemm_param(torch.empty(dim, dim, device=device))
        for w in (self.wq, self.wk, self.wv, self.wo):
            _linear_init(w.data)

    def transform(self, x: torch.Tensor, native: bool) -> torch.Tensor:
        return layer_norm(self.ffn(x, native), self.ln_w, self.ln_b, 1e-5, native)

    def attend(self, q: torch.Tensor, hist: torch.Tensor, valid: torch.Tensor, native: bool) -> torch.Tensor:
        """``q [B, d]`` over ``hist [B, L, d]`` -> ``[B, d]``."""

        B = q.shape[0]
        H, hd, d = self.heads, self.hd, self.dim
        pq = linear_nb(q, self.wq, native).float().view(B, H, hd)
        sv = torch.einsum("bhk,hkd->bhd", pq, self.wk.view(H, hd, d))          # score vector per head
        if native and hist.is_cuda and shared_query_supported(H, d):
            # valid is a suffix mask (left-padded window): its first valid event is L - count
            kstart = (hist.shape[1] - valid.sum(dim=-1)).to(torch.int32)
            ctx = shared_query_attention(sv, hist, kstart, 1.0 / math.sqrt(hd))  # [B, H, d]
        else:
            hf = hist.float()
            scores = torch.einsum("bhd,bld->bhl", sv, hf) / math.sqrt(hd)
            mask = valid.bool().unsqueeze(1)
            w = torch.nan_to_num(torch.softmax(scores.masked_fill(~mask, float("-inf")), dim=-1)) * mask
            ctx = torch.einsum("bhl,bld->bhd", w, hf)                           # [B, H, d]
        vals = torch.einsum("bhd,hkd->bhk", ctx, self.wv.view(H, hd, d)).reshape(B, d)
        return linear_nb(vals, self.wo, native)


class STCAEncoder(nn.Module):
    def __init__(self, dim: int, heads: int, layers: int, ratio: int, device=None) -> None:
        super().__init__()
        if dim % heads:
            raise ValueError("stca_dim must be divisible by the head count")
        self.dim, self.M = dim, layers
        self.layers = nn.ModuleList(STCALayer(dim, heads, ratio, device=device) for _ in range(layers))
        self.fusion = nn.ParameterList(gemm_param(torch.empty(dim, (i + 2) * dim, device=device))
                                       for i in range(layers - 1))
        for w in self.fusion:
            _linear_init(w.data)
        self.final_proj = gemm_param(torch.empty(dim, (layers + 1) * dim, device=device))
        _linear_init(self.final_proj.data)
        self.final_ffn = _SwiGLU(dim, ratio * dim, device=device)

    def transform_histories(self, history: torch.Tensor, native: bool) -> list[torch.Tensor]:
        """Every layer's transformed history ``LN_i(SwiGLU_i(X))``: candidate-independent, so
        computed once per request (reference ``STCASequenceCache`` ``src/modules/stca.py:28-44``)."""

        return [layer.transform(history, native) for layer in self.layers]

    def forward(self, history: torch.Tensor | None, valid: torch.Tensor, target: torch.Tensor, native: bool,
                row_indices: torch.Tensor | None = None,
                transformed: list[torch.Tensor] | None = None) -> torch.Tensor:
        """``history [R, L, d]`` / ``valid [R, L]`` per request (or per row), ``target [B, d]`` per
        candidate row; ``row_indices [B]`` maps candidates to requests (request-level
        batching: the history transforms run once per request). ``transformed`` replaces
        ``history`` with cached ``transform_histories`` output."""

        hs = transformed if transformed is not None else self.transform_histories(history, native)
        if row_indices is not None:
            ri = row_indices.to(valid.device).long()
            valid = valid.index_select(0, ri)
        outs: list[torch.Tensor] = []
        q = self.layers[0].transform(target, native)
        for i, layer in enumerate(self.layers):
            hist = hs[i] if row_indices is None else hs[i].index_select(0, ri.to(hs[i].device))
            outs.append(layer.attend(q, hist, valid, native).to(target.dtype))
            if i + 1 < self.M:
                fused = linear_nb(torch.cat([*outs, target], dim=-1), self.fusion[i], native)
                q = self.layers[i + 1].transform(fused, native)
        final = linear_nb(torch.cat([*outs, target], dim=-1), self.final_proj, native)
        return self.final_ffn(final, native)
