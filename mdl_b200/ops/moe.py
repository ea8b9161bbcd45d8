"""Sparse-MoE per-token FFN (ReLU router with an L1 regulariser, DTSI dense router).

Reference: ``SparseMoEPerTokenFFN`` (``src/modules/mlp.py:210-504``), its
controller step ``_step_sparse_moe_controllers`` (``src/train.py:5830-5850``) and
the loss term (``src/train.py:6018-6029``).

Each of the ``T`` tokens owns ``E`` experts ``Linear(D,H) -> act -> Linear(H,D)``,
a sparse router ``relu(x W_s + b_s)`` and (DTSI) a dense router
``softmax(x W_d + b_d)``. Training evaluates every expert and mixes them with
one effective gate per (sample, token, expert):

* DTSI ``dense_router``: the dense gates; ``mean``: the mean of the dense and
  sparse gates; without DTSI: the sparse gates;
* inference: the sparse gates above ``inference_threshold`` (others give
  exactly zero).

The regularisation loss is ``coefficient * mean_t mean_b sum_e relu-gate``; the
coefficient is multiplied by ``multiplier ** sign(active_ratio - target)`` after
each optimizer step (on the device, no host sync).

Layout: the experts of a token are concatenated, ``w_in [T, E*H, D]`` and
``w_out [T, D, E*H]``, so the whole layer is two grouped tcgen05 GEMMs over
the tokens: ``act = gelu(x_t W_in[t]^T)`` (all experts at once, ``N = E*H``)
and ``y_t = (g * act) W_out[t]^T`` (the gate-weighted sum over experts is the
``K = E*H`` reduction). The gate scaling, the gate gradient
``dg = sum_h dh * act + dy . b_out`` and the bias terms are PyTorch
elementwise ops around them.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ._ext import ext
from .gemm import ACT_GELU_GRAD, ACT_RELU, bgemm
from .layers import _grad, _shadow, gemm_param


class MoEExpertsFn(torch.autograd.Function):
    """``y[b,t] = sum_e g[b,t,e] * (act(x[b,t] W_in[t,e]^T + b_in[t,e]) W_out[t,e]^T + b_out[t,e])``."""

    @staticmethod
    def forward(ctx, x, g, w_in, b_in, w_out, b_out, relu):
        B, T, D = x.shape
        E = g.shape[2]
        EH = w_in.shape[1]
        H = EH // E
        dev = x.device
        if not (x.stride(2) == 1 and x.stride(1) == D and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0):
            x = x.contiguous()
        act = torch.empty(T, B, EH, dtype=torch.bfloat16, device=dev)
        if relu:
            gp = None
            bgemm(x, _shadow(w_in), act, M=B, N=EH, K=D, G=T, lda=x.stride(0), gsA=D, ldb=D, gsB=EH * D, ldc=EH,
                  gsC=B * EH, bias=b_in, gs_bias=EH, act=ACT_RELU)
        else:
            gp = torch.empty_like(act)  # gelu'(pre-activation)
            bgemm(x, _shadow(w_in), gp, M=B, N=EH, K=D, G=T, lda=x.stride(0), gsA=D, ldb=D, gsB=EH * D, ldc=EH,
                  gsC=B * EH, out2=act, bias=b_in, gs_bias=EH, act=ACT_GELU_GRAD)
        gt = g.permute(1, 0, 2).to(torch.bfloat16).unsqueeze(-1)          # [T, B, E, 1]
        hg = (act.view(T, B, E, H) * gt).view(T, B, EH)
        y = torch.empty(B, T, D, dtype=torch.bfloat16, device=dev)
        bgemm(hg, _shadow(w_out), y, M=B, N=D, K=EH, G=T, lda=EH, gsA=B * EH, ldb=EH, gsB=D * EH, ldc=T * D, gsC=D)
        y += torch.einsum("bte,ted->btd", g.float(), b_out).to(torch.bfloat16)
        ctx.save_for_backward(x, g, act, gp if gp is not None else act)
        ctx.meta = (w_in, b_in, w_out, b_out, bool(relu))
        return y

    @staticmethod
    def backward(ctx, dy):
        x, g, act, gp = ctx.saved_tensors
        w_in, b_in, w_out, b_out, relu = ctx.meta
        B, T, D = x.shape
        E = g.shape[2]
        EH = w_in.shape[1]
        H = EH // E
        dev = x.device
        dy = dy.contiguous().to(torch.bfloat16)
        gt = g.permute(1, 0, 2).to(torch.bfloat16).unsqueeze(-1)
        dhg = torch.empty(T, B, EH, dtype=torch.bfloat16, device=dev)
        bgemm(dy, _shadow(w_out), dhg, M=B, N=EH, K=D, G=T, lda=T * D, gsA=D, ldb=EH, gsB=D * EH, b_mn=True,
              ldc=EH, gsC=B * EH)
        hg = (act.view(T, B, E, H) * gt).view(T, B, EH)
        bgemm(dy, hg, _grad(w_out), M=D, N=EH, K=B, G=T, lda=T * D, gsA=D, a_mn=True, ldb=EH, gsB=B * EH, b_mn=True,
              ldc=EH, gsC=D * EH, accumulate=True)
        del hg
        _grad(b_out).add_(torch.einsum("bte,btd->ted", g.float(), dy.float()))
        dh4 = dhg.view(T, B, E, H)
        dg = (dh4.float() * act.view(T, B, E, H).float()).sum(-1).permute(1, 0, 2)
        dg = dg + torch.einsum("btd,ted->bte", dy.float(), b_out.float())
        if relu:
            dpre = (dh4 * gt * (act.view(T, B, E, H) > 0)).view(T, B, EH)
        else:
            dpre = (dh4 * gt * gp.view(T, B, E, H)).view(T, B, EH)
        del dhg, dh4
        ext().colsum(dpre, _grad(b_in), T, B, EH, EH, B * EH, 1.0)
        bgemm(dpre, x, _grad(w_in), M=EH, N=D, K=B, G=T, lda=EH, gsA=B * EH, a_mn=True, ldb=x.stride(0), gsB=D,
              b_mn=True, ldc=D, gsC=EH * D, accumulate=True)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(B, T, D, dtype=torch.bfloat16, device=dev)
            bgemm(dpre, _shadow(w_in), dx, M=B, N=D, K=EH, G=T, lda=EH, gsA=B * EH, ldb=D, gsB=EH * D, b_mn=True,
                  ldc=T * D, gsC=D)
        return dx, dg.to(g.dtype), None, None, None, None, None


class SparseMoEPerTokenFFN(nn.Module):
    def __init__(self, num_tokens: int, token_dim: int, hidden_dim: int, num_experts: int = 4,
                 activation: str = "gelu", use_dtsi: bool = True, inference_threshold: float = 0.0,
                 target_active_ratio: float = 0.25, regularization_initial: float = 1e-8,
                 regularization_multiplier: float = 1.2, dtsi_training_output: str | None = None,
                 device=None) -> None:
        super().__init__()
        if use_dtsi and dtsi_training_output not in ("dense_router", "mean"):
            raise ValueError("DTSI needs sparse_moe_dtsi_training_output dense_router or mean")
        if not 0.0 < target_active_ratio <= 1.0:
            raise ValueError("target_active_ratio must be in (0, 1]")
        if regularization_multiplier <= 1.0 or regularization_initial <= 0.0:
            raise ValueError("regularization multiplier must be > 1 and the initial coefficient > 0")
        T, D, H, E = num_tokens, token_dim, hidden_dim, num_experts
        self.num_tokens, self.token_dim, self.hidden_dim, self.num_experts = T, D, H, E
        self.relu = activation == "relu"
        self.use_dtsi = use_dtsi
        self.dtsi_training_output = dtsi_training_output
        self.inference_threshold = float(inference_threshold)
        self.target_active_ratio = float(target_active_ratio)
        self.regularization_multiplier = float(regularization_multiplier)
        self.w_in = gemm_param(torch.empty(T, E * H, D, device=device))
        self.b_in = nn.Parameter(torch.empty(T, E * H, device=device))
        self.w_out = gemm_param(torch.empty(T, D, E * H, device=device))
        self.b_out = nn.Parameter(torch.empty(T, E, D, device=device))
        # nn.Linear default init per expert and router (kaiming_uniform(a=sqrt(5)) == U(+-1/sqrt(fan_in)))
        bi, bo = 1.0 / math.sqrt(D), 1.0 / math.sqrt(H)
        nn.init.uniform_(self.w_in, -bi, bi)
        nn.init.uniform_(self.b_in, -bi, bi)
        nn.init.uniform_(self.w_out, -bo, bo)
        nn.init.uniform_(self.b_out, -bo, bo)
        self.sparse_router_weight = nn.Parameter(torch.empty(T, E, D, device=device).uniform_(-bi, bi))
        self.sparse_router_bias = nn.Parameter(torch.empty(T, E, device=device).uniform_(-bi, bi))
        if use_dtsi:
            self.dense_router_weight = nn.Parameter(torch.empty(T, E, D, device=device).uniform_(-bi, bi))
            self.dense_router_bias = nn.Parameter(torch.empty(T, E, device=device).uniform_(-bi, bi))
        else:
            self.dense_router_weight = self.dense_router_bias = None
        self.register_buffer("regularization_coefficient",
                             torch.tensor(float(regularization_initial), device=device))
        self.last_regularization_loss: torch.Tensor | None = None
        self.last_active_ratio: torch.Tensor | None = None
        self.update_pending = False

    # ------------------------------------------------------------------ gates
    def gates(self, x: torch.Tensor) -> torch.Tensor:
        """Effective expert weights ``[B, T, E]`` (fp32); records the regulariser."""

        xf = x.float()
        sparse = torch.relu(torch.einsum("btd,ted->bte", xf, self.sparse_router_weight)
                            + self.sparse_router_bias.unsqueeze(0))
        # L1 of the sparse gates: mean over tokens of the per-token batch mean of the expert sum
        self.last_regularization_loss = self.regularization_coefficient * sparse.sum(-1).mean()
        self.last_active_ratio = (sparse > 0).float().mean().detach()
        self.update_pending = self.training
        if not self.training:
            return sparse * (sparse > self.inference_threshold)
        if not self.use_dtsi:
            return sparse
        dense = torch.softmax(torch.einsum("btd,ted->bte", xf, self.dense_router_weight)
                              + self.dense_router_bias.unsqueeze(0), dim=-1)
        if self.dtsi_training_output == "dense_router":
            return dense
        return 0.5 * (dense + sparse)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, D = x.shape
        g = self.gates(x)
        if x.is_cuda and hasattr(self.w_in, "_mdl_shadow"):
            return MoEExpertsFn.apply(x.to(torch.bfloat16), g, self.w_in, self.b_in, self.w_out, self.b_out,
                                      self.relu)
        E, H = self.num_experts, self.hidden_dim
        act = F.relu if self.relu else F.gelu
        h = act(torch.einsum("btd,thd->bth", x.float(), self.w_in) + self.b_in.unsqueeze(0))    # [B, T, E*H]
        hg = (h.view(B, T, E, H) * g.unsqueeze(-1)).view(B, T, E * H)
        return torch.einsum("bth,tdh->btd", hg, self.w_out) + torch.einsum("bte,ted->btd", g, self.b_out)

    # ------------------------------------------------------------------ controller
    @torch.no_grad()
    def step_regularization_controller(self, active_ratio: torch.Tensor) -> None:
        if not self.update_pending:
            return
        direction = torch.sign(active_ratio.to(self.regularization_coefficient) - self.target_active_ratio)
        self.regularization_coefficient.mul_(torch.pow(torch.full_like(direction, self.regularization_multiplier),
                                                       direction))
        self.update_pending = False

    def reference_state_dict(self, prefix: str) -> dict[str, torch.Tensor]:
        """Per-expert ``nn.Linear`` / router tensors under the reference's names."""

        T, E, H = self.num_tokens, self.num_experts, self.hidden_dim
        sd = {}
        for t in range(T):
            for e in range(E):
                p = f"{prefix}experts.{t}.{e}."
                sd[p + "0.weight"] = self.w_in[t, e * H:(e + 1) * H]
                sd[p + "0.bias"] = self.b_in[t, e * H:(e + 1) * H]
                sd[p + "3.weight"] = self.w_out[t, :, e * H:(e + 1) * H]
                sd[p + "3.bias"] = self.b_out[t, e]
            sd[f"{prefix}sparse_routers.{t}.weight"] = self.sparse_router_weight[t]
            sd[f"{prefix}sparse_routers.{t}.bias"] = self.sparse_router_bias[t]
            if self.use_dtsi:
                sd[f"{prefix}dense_routers.{t}.weight"] = self.dense_router_weight[t]
                sd[f"{prefix}dense_routers.{t}.bias"] = self.dense_router_bias[t]
        sd[prefix + "regularization_coefficient"] = self.regularization_coefficient
        return {k: v.detach().clone() for k, v in sd.items()}


def moe_modules(model: nn.Module) -> list[SparseMoEPerTokenFFN]:
    return [m for m in model.modules() if isinstance(m, SparseMoEPerTokenFFN)]


def moe_outputs(model: nn.Module) -> dict[str, torch.Tensor]:
    """``moe_regularization_loss`` (sum over layers) and ``moe_active_ratio`` (mean) of the
    last forward (reference ``_sparse_moe_outputs`` ``src/model.py:6638-6651``)."""

    mods = [m for m in moe_modules(model) if m.last_regularization_loss is not None]
    if not mods:
        return {}
    return {"moe_regularization_loss": torch.stack([m.last_regularization_loss for m in mods]).sum(),
            "moe_active_ratio": torch.stack([m.last_active_ratio for m in mods]).mean()}


@torch.no_grad()
def step_moe_controllers(modules: list[SparseMoEPerTokenFFN], world: int = 1, group=None) -> None:
    """After a training step: the active ratio of each MoE layer, averaged over the ranks
    with one all-reduce, moves its regularisation coefficient."""

    mods = [m for m in modules if m.update_pending and m.last_active_ratio is not None]
    if not mods:
        return
    ratios = torch.stack([m.last_active_ratio.float() for m in mods])
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(ratios, group=group)
        ratios /= float(world)
    for m, r in zip(mods, ratios):
        m.step_regularization_controller(r)


def add_moe_loss(out: dict, model: nn.Module, weight: float) -> dict:
    """Adds ``weight * moe_regularization_loss`` to ``out["loss"]`` (reference
    ``_loss_terms_from_batch`` ``src/train.py:6018-6029``) and reports both terms."""

    extra = moe_outputs(model)
    if extra:
        out.update(extra)
        if "loss" in out and weight > 0.0:
            out["loss"] = out["loss"] + weight * extra["moe_regularization_loss"].to(out["loss"].dtype)
    return out


def build_rankmixer_moe(config, num_tokens: int, device=None) -> SparseMoEPerTokenFFN:
    m = config.model
    return SparseMoEPerTokenFFN(num_tokens, int(m.token_dim), int(m.hidden_dim), int(m.sparse_moe_num_experts),
                                m.ffn_activation, bool(m.sparse_moe_use_dtsi), float(m.sparse_moe_inference_threshold),
                                float(m.sparse_moe_target_active_ratio), float(m.sparse_moe_regularization_initial),
                                float(m.sparse_moe_regularization_multiplier), m.sparse_moe_dtsi_training_output,
                                device=device)
