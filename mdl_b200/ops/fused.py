"""Fused autograd nodes of the RankMixer family (CUDA: native kernels only).

Each node runs a whole sub-graph with the sm_100a kernels and writes the
gradients of its dense parameters straight into the flat gradient buffer
(``param._mdl_grad``, see ``ops/dense.py``); GEMM operands are the bf16 shadow
copies (``param._mdl_shadow``). On CPU the modules in ``models/rankmixer.py``
use the plain PyTorch definitions instead (autograd, fp32), which are also the
oracles of the GPU tests.

* ``PerTokenLinearFn``: ``y[b,t] = x[b,t,:K] @ W[t]^T + b[t]`` (reference
  ``PerTokenLinear`` ``src/modules/mlp.py:10-42``) as one grouped GEMM; the
  backward's weight gradient is a second grouped GEMM, the bias gradient a
  column-sum epilogue.
* ``RankMixerBlockFn``: ``m = LN(mix(x) + x)``, ``f = FFN_t(m_t)``,
  ``y = LN(f + m)`` (reference ``RankMixerBlock`` ``src/model.py:6654-6665``,
  ``StackedPerTokenFFN`` ``src/modules/mlp.py:135-207``) in 4 kernels forward
  (mix+LN, GEMM+bias+GELU, GEMM+bias, add+LN) and 7 backward.
* ``HeadsBCEFn``: mean over tokens, the task towers' first layer for all tasks
  as one GEMM with a GELU epilogue, then one kernel for the last layer, the
  masked BCE loss and its gradient (reference ``TaskHead`` ``src/model.py:869-882``,
  ``_loss_terms_from_batch`` ``src/train.py:5890-6031``).
"""

from __future__ import annotations

import torch

from ._ext import ext
from .gemm import ACT_DMUL, ACT_GELU, ACT_GELU_GRAD, ACT_NONE, bgemm


def _shadow(p: torch.Tensor) -> torch.Tensor:
    s = getattr(p, "_mdl_shadow", None)
    if s is None:
        raise RuntimeError("parameter has no bf16 shadow (not registered in DenseParams)")
    return s


def _grad(p: torch.Tensor) -> torch.Tensor:
    g = getattr(p, "_mdl_grad", None)
    if g is None:
        raise RuntimeError("parameter has no flat gradient view (not registered in DenseParams)")
    return g


# ----------------------------------------------------------------------------- per-token linear
class PerTokenLinearFn(torch.autograd.Function):
    """x: [B, T*Kpad] bf16 (token t's slice at columns t*Kpad .. t*Kpad+K); weight [T, N, Kpad]."""

    @staticmethod
    def forward(ctx, x, weight, bias, T, K, Kpad):
        B = x.shape[0]
        N = weight.shape[1]
        w = _shadow(weight)
        out = torch.empty(B, T, N, dtype=torch.bfloat16, device=x.device)
        bgemm(x, w, out, M=B, N=N, K=K, G=T, lda=T * Kpad, gsA=Kpad, ldb=Kpad, gsB=N * Kpad, ldc=T * N, gsC=N,
              bias=bias, gs_bias=N)
        ctx.save_for_backward(x)
        ctx.meta = (weight, bias, T, K, Kpad, N)
        return out

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        weight, bias, T, K, Kpad, N = ctx.meta
        B = x.shape[0]
        dy = dy.contiguous() if dy.stride(-1) != 1 else dy
        ldy = dy.stride(0)
        # dW[t] += dy[:,t,:]^T @ x[:,t,:K]      (M=N, N=K, K=B; both operands MN-major)
        bgemm(dy, x, _grad(weight), M=N, N=K, K=B, G=T, lda=ldy, gsA=N, a_mn=True, ldb=T * Kpad, gsB=Kpad,
              b_mn=True, ldc=Kpad, gsC=N * Kpad, accumulate=True)
        ext().colsum(dy, _grad(bias), T, B, N, ldy, N, 1.0)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.zeros(B, T * Kpad, dtype=torch.bfloat16, device=x.device) if Kpad != K else \
                torch.empty(B, T * Kpad, dtype=torch.bfloat16, device=x.device)
            # dx[:,t,:K] = dy[:,t,:] @ W[t]         (M=B, N=K, K=N; W MN-major)
            bgemm(dy, _shadow(weight), dx, M=B, N=K, K=N, G=T, lda=ldy, gsA=N, ldb=Kpad, gsB=N * Kpad, b_mn=True,
                  ldc=T * Kpad, gsC=Kpad)
        return dx, None, None, None, None, None


# ----------------------------------------------------------------------------- RankMixer block
class RankMixerBlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, g1, b1n, w_in, b_in, w_out, b_out, g2, b2n, eps):
        B, T, D = x.shape
        H = w_in.shape[1]
        dev = x.device
        C = ext()
        x = x.contiguous()
        m = torch.empty_like(x)
        mean1 = torch.empty(B * T, dtype=torch.float32, device=dev)
        rstd1 = torch.empty_like(mean1)
        C.ln_fwd(x, None, g1, b1n, m, mean1, rstd1, B, T, D, True, eps)
        pre = torch.empty(T, B, H, dtype=torch.bfloat16, device=dev)
        act = torch.empty_like(pre)
        bgemm(m, _shadow(w_in), pre, M=B, N=H, K=D, G=T, lda=T * D, gsA=D, ldb=D, gsB=H * D, ldc=H, gsC=B * H,
              out2=act, bias=b_in, gs_bias=H, act=ACT_GELU_GRAD)  # pre <- gelu'(pre-activation)
        f = torch.empty_like(x)
        bgemm(act, _shadow(w_out), f, M=B, N=D, K=H, G=T, lda=H, gsA=B * H, ldb=H, gsB=D * H, ldc=T * D, gsC=D,
              bias=b_out, gs_bias=D)
        y = torch.empty_like(x)
        mean2 = torch.empty_like(mean1)
        rstd2 = torch.empty_like(mean1)
        C.ln_fwd(f, m, g2, b2n, y, mean2, rstd2, B, T, D, False, eps)
        ctx.save_for_backward(x, m, pre, act, f, mean1, rstd1, mean2, rstd2)
        ctx.params = (g1, b1n, w_in, b_in, w_out, b_out, g2, b2n)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, m, pre, act, f, mean1, rstd1, mean2, rstd2 = ctx.saved_tensors
        g1, b1n, w_in, b_in, w_out, b_out, g2, b2n = ctx.params
        B, T, D = x.shape
        H = w_in.shape[1]
        dev = x.device
        C = ext()
        grid = C.ln_bwd_grid(B)
        partials = torch.empty(grid, 2 * D, dtype=torch.float32, device=dev)
        df = torch.empty_like(x)
        dm = torch.empty_like(x)
        if dy.dim() == 3 and dy.stride(1) == 0:
            dyb, dyf = dy[:, 0, :], None  # gradient of a mean over tokens: broadcast, never materialised
            if dyb.stride(-1) != 1:
                dyb = dyb.contiguous()
        else:
            dyb, dyf = None, dy.contiguous()
        C.ln_bwd(dyf, dyb, 1.0, f, m, mean2, rstd2, g2, df, dm, partials, _grad(g2), _grad(b2n), B, T, D, False, grid)
        # d b_out[t] = sum_b df[b, t, :]
        C.colsum(df, _grad(b_out), T, B, D, T * D, D, 1.0)
        # dPre = (df_t @ W_out[t]) * gelu'(pre);  colsum -> d b_in
        dpre = torch.empty_like(pre)
        bgemm(df, _shadow(w_out), dpre, M=B, N=H, K=D, G=T, lda=T * D, gsA=D, ldb=H, gsB=D * H, b_mn=True, ldc=H,
              gsC=B * H, aux=pre, ld_aux=H, gs_aux=B * H, colsum=_grad(b_in), gs_colsum=H, act=ACT_DMUL)
        # dW_out[t] += df_t^T @ act_t
        bgemm(df, act, _grad(w_out), M=D, N=H, K=B, G=T, lda=T * D, gsA=D, a_mn=True, ldb=H, gsB=B * H, b_mn=True,
              ldc=H, gsC=D * H, accumulate=True)
        # dW_in[t] += dPre_t^T @ m_t
        bgemm(dpre, m, _grad(w_in), M=H, N=D, K=B, G=T, lda=H, gsA=B * H, a_mn=True, ldb=T * D, gsB=D, b_mn=True,
              ldc=D, gsC=H * D, accumulate=True)
        # dm += dPre_t @ W_in[t]
        bgemm(dpre, _shadow(w_in), dm, M=B, N=D, K=H, G=T, lda=H, gsA=B * H, ldb=D, gsB=H * D, b_mn=True,
              ldc=T * D, gsC=D, accumulate=True)
        dx = torch.empty_like(x)
        # the first grid * 2D floats of `partials` are reused (no per-token sums here)
        C.ln_bwd(dm, None, 1.0, x, None, mean1, rstd1, g1, dx, None, partials, _grad(g1), _grad(b1n),
                 B, T, D, True, grid)
        return dx, None, None, None, None, None, None, None, None, None


# ----------------------------------------------------------------------------- heads + BCE
class HeadsBCEFn(torch.autograd.Function):
    """Returns (loss scalar fp32, logits [B, ntask] fp32). Only the loss carries a gradient."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, labels, mask, task_scale, relu):
        B, T, D = x.shape
        ntask, Hh = w2.shape
        dev = x.device
        C = ext()
        pooled = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        C.token_mean(x.contiguous(), pooled, B, T, D)
        pre = torch.empty(B, ntask * Hh, dtype=torch.bfloat16, device=dev)
        act = torch.empty_like(pre)
        w1s = _shadow(w1).reshape(ntask * Hh, D)
        from .gemm import ACT_RELU
        if relu:
            bgemm(pooled, w1s, pre, M=B, N=ntask * Hh, K=D, lda=D, ldb=D, ldc=ntask * Hh, bias=b1.reshape(-1))
            act = torch.relu(pre)
        else:
            bgemm(pooled, w1s, pre, M=B, N=ntask * Hh, K=D, lda=D, ldb=D, ldc=ntask * Hh, out2=act,
                  bias=b1.reshape(-1), act=ACT_GELU)
        logits = torch.empty(B, ntask, dtype=torch.float32, device=dev)
        loss = torch.zeros(1, dtype=torch.float32, device=dev)
        C.head_bce(act, pre, w2, b2, labels, mask, task_scale, logits, loss, None, None, None, B, ntask, Hh, bool(relu))
        ctx.save_for_backward(pooled, pre, act, labels, mask if mask is not None else labels.new_empty(0), task_scale)
        ctx.meta = (w1, b1, w2, b2, B, T, D, ntask, Hh, relu, mask is not None)
        ctx.mark_non_differentiable(logits)
        return loss.reshape(()), logits

    @staticmethod
    def backward(ctx, dloss, _dlogits):
        pooled, pre, act, labels, mask, task_scale = ctx.saved_tensors
        w1, b1, w2, b2, B, T, D, ntask, Hh, relu, has_mask = ctx.meta
        C = ext()
        dev = pooled.device
        scale = task_scale * dloss.reshape(1).to(torch.float32)
        dpre = torch.empty_like(pre)
        C.head_bce(act, pre, w2, b2, labels, mask if has_mask else None, scale, None, None, dpre, _grad(w2),
                   _grad(b2), B, ntask, Hh, bool(relu))
        C.colsum(dpre, _grad(b1).reshape(-1), 1, B, ntask * Hh, ntask * Hh, 0, 1.0)
        # dW1 += dpre^T @ pooled
        bgemm(dpre, pooled, _grad(w1).reshape(ntask * Hh, D), M=ntask * Hh, N=D, K=B, lda=ntask * Hh, a_mn=True,
              ldb=D, b_mn=True, ldc=D, accumulate=True)
        # d pooled / T, broadcast over tokens as a stride-0 view
        dpooled = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        bgemm(dpre, _shadow(w1).reshape(ntask * Hh, D), dpooled, M=B, N=D, K=ntask * Hh, lda=ntask * Hh, ldb=D,
              b_mn=True, ldc=D, alpha=1.0 / T)
        dx = dpooled.unsqueeze(1).expand(B, T, D)
        return dx, None, None, None, None, None, None, None, None


# ----------------------------------------------------------------------------- token mixing + LayerNorm
class MixLayerNormFn(torch.autograd.Function):
    """``LayerNorm(token_mix(x) + x)`` over ``[B, T, D]`` as one kernel each way
    (the first half of a RankMixer block, reference ``src/model.py:6663``)."""

    @staticmethod
    def forward(ctx, x, g, b, eps):
        B, T, D = x.shape
        x = x.contiguous()
        m = torch.empty_like(x)
        mean = torch.empty(B * T, dtype=torch.float32, device=x.device)
        rstd = torch.empty_like(mean)
        ext().ln_fwd(x, None, g, b, m, mean, rstd, B, T, D, True, eps)
        ctx.save_for_backward(x, mean, rstd)
        ctx.params = (g, b)
        return m

    @staticmethod
    def backward(ctx, dm):
        x, mean, rstd = ctx.saved_tensors
        g, b = ctx.params
        B, T, D = x.shape
        C = ext()
        grid = C.ln_bwd_grid(B)
        partials = torch.empty(grid, 2 * D, dtype=torch.float32, device=x.device)
        dx = torch.empty_like(x)
        C.ln_bwd(dm.contiguous().to(torch.bfloat16), None, 1.0, x, None, mean, rstd, g, dx, None, partials, _grad(g),
                 _grad(b), B, T, D, True, grid)
        return dx, None, None, None
