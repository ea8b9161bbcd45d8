"""OneTrans non-sequence (NS) token encoders other than ``auto_split``.

* ``dcnv2`` (reference ``CrossNetV2Layer`` / ``DCNv2NSEncoder``
  ``src/model.py:763-866``): ``z0 = Linear(x)`` (identity when the widths
  match), ``L`` cross layers ``z <- z0 * (W z + b) + z`` (full or low-rank
  ``W = U V^T``), an optional deep MLP on ``z0``, and ``Linear([z; deep])`` to
  ``N * d``;
* ``groupwise`` (``OneTransTokenizer._ns_tokens_groupwise`` ``:5085-5090``):
  one ``Linear -> act -> Linear`` per NS group over the concatenation of the
  group's inputs, i.e. a per-token FFN over per-group input slices.

CUDA: every ``Linear`` is a tcgen05 GEMM (``ops.layers.Linear`` when its
widths are multiples of 8), the groupwise projections are one grouped GEMM
pair (``PerTokenFFN``); the cross-layer products ``z0 * c + z`` are PyTorch
elementwise ops.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..ops.layers import Linear, PerTokenFFN


def _xavier_(t: torch.Tensor) -> None:
    bound = math.sqrt(6.0 / (t.shape[0] + t.shape[1]))
    nn.init.uniform_(t, -bound, bound)


class CrossLayer(nn.Module):
    def __init__(self, dim: int, low_rank: int | None = None, device=None) -> None:
        super().__init__()
        if low_rank is not None and not 0 < low_rank <= dim:
            raise ValueError(f"ns_dcn_low_rank must be in [1, {dim}]")
        self.low_rank = low_rank
        if low_rank is None:
            self.proj = Linear(dim, dim, device=device)
            _xavier_(self.proj.weight.data)
            nn.init.zeros_(self.proj.bias)
        else:
            self.u = nn.Parameter(torch.empty(dim, low_rank, device=device))
            self.v = nn.Parameter(torch.empty(dim, low_rank, device=device))
            self.bias = nn.Parameter(torch.zeros(dim, device=device))
            _xavier_(self.u.data)
            _xavier_(self.v.data)

    def forward(self, z0: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
        if self.low_rank is None:
            c = self.proj(z)
        else:
            dt = torch.bfloat16 if z.is_cuda else z.dtype
            c = F.linear(F.linear(z.to(dt), self.v.t().to(dt)), self.u.to(dt), self.bias.to(dt))
        return z0 * c.to(z0.dtype) + z


class DCNv2Encoder(nn.Module):
    """``[B, k_ld]`` lookup rows (logical width ``k_log``, zero padding after it) ->
    ``[B, out_dim]``."""

    def __init__(self, k_ld: int, k_log: int, out_dim: int, projection_dim: int, cross_layers: int,
                 deep_layers: int, deep_dim: int, activation: str, low_rank: int | None = None, device=None) -> None:
        super().__init__()
        if cross_layers <= 0 or projection_dim <= 0 or deep_layers < 0:
            raise ValueError("dcnv2 needs cross_layers > 0, projection_dim > 0, deep_layers >= 0")
        self.k_log = k_log
        self.act = F.relu if activation == "relu" else F.gelu
        self.input_proj = None
        if k_log != projection_dim:
            self.input_proj = Linear(k_ld, projection_dim, device=device)
            with torch.no_grad():      # fan-in of the logical inputs; padded input columns stay zero
                bound = 1.0 / math.sqrt(k_log)
                self.input_proj.weight.uniform_(-bound, bound)
                self.input_proj.weight[:, k_log:] = 0
                self.input_proj.bias.uniform_(-bound, bound)
        self.cross = nn.ModuleList(CrossLayer(projection_dim, low_rank, device=device) for _ in range(cross_layers))
        self.deep = nn.ModuleList()
        width = projection_dim
        for _ in range(deep_layers):
            self.deep.append(Linear(width, deep_dim, device=device))
            width = deep_dim
        self.output_proj = Linear(projection_dim + (deep_dim if deep_layers else 0), out_dim, device=device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        z0 = self.input_proj(x) if self.input_proj is not None else x[:, :self.k_log]
        if not x.is_cuda:
            z0 = z0.float()
        z = z0
        for layer in self.cross:
            z = layer(z0, z)
        if len(self.deep):
            h = z0
            for lin in self.deep:
                h = self.act(lin(h))
            z = torch.cat([z, h.to(z.dtype)], dim=-1)
        return self.output_proj(z.contiguous())

    def reference_state_dict(self, prefix: str) -> dict[str, torch.Tensor]:
        sd = {}
        if self.input_proj is not None:
            sd[prefix + "input_proj.weight"] = self.input_proj.weight[:, :self.k_log]
            sd[prefix + "input_proj.bias"] = self.input_proj.bias
        for i, layer in enumerate(self.cross):
            if layer.low_rank is None:
                sd[f"{prefix}cross_layers.{i}.weight"] = layer.proj.weight
                sd[f"{prefix}cross_layers.{i}.bias"] = layer.proj.bias
            else:
                sd[f"{prefix}cross_layers.{i}.u"] = layer.u
                sd[f"{prefix}cross_layers.{i}.v"] = layer.v
                sd[f"{prefix}cross_layers.{i}.bias"] = layer.bias
        for i, lin in enumerate(self.deep):
            sd[f"{prefix}deep.{2 * i}.weight"] = lin.weight
            sd[f"{prefix}deep.{2 * i}.bias"] = lin.bias
        sd[prefix + "output_proj.weight"] = self.output_proj.weight
        sd[prefix + "output_proj.bias"] = self.output_proj.bias
        return {k: v.detach().clone() for k, v in sd.items()}


class GroupwiseNS(nn.Module):
    """One projection MLP per NS group; input ``[B, N * kp]`` (group ``n`` at columns
    ``[n * kp, n * kp + widths[n])``), output ``[B, N, d]``."""

    def __init__(self, widths: list[int], kp: int, token_dim: int, hidden_dim: int, activation: str,
                 device=None) -> None:
        super().__init__()
        self.widths, self.kp = list(widths), kp
        self.ffn = PerTokenFFN(len(widths), kp, hidden_dim, activation, device=device, out_dim=token_dim)
        self.ffn.restrict_inputs(self.widths)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B = x.shape[0]
        v = x.view(B, len(self.widths), self.kp)
        return self.ffn(v if x.is_cuda else v.float())

    def reference_state_dict(self, prefix: str) -> dict[str, torch.Tensor]:
        f = self.ffn
        sd = {}
        for n, w in enumerate(self.widths):
            sd[f"{prefix}{n}.0.weight"] = f.input_weight[n, :, :w]
            sd[f"{prefix}{n}.0.bias"] = f.input_bias[n]
            sd[f"{prefix}{n}.2.weight"] = f.output_weight[n]
            sd[f"{prefix}{n}.2.bias"] = f.output_bias[n]
        return {k: v.detach().clone() for k, v in sd.items()}
