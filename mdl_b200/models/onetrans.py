"""OneTrans: one causal transformer over sequence (S) and non-sequence (NS) tokens.

Reference: ``OneTransTokenizer`` ``src/model.py:4571-5296``, ``MixedCausalAttention``
``:5479-5721``, ``MixedFFN`` ``:5724-5818``, ``OneTransBlock`` ``:5821-6071``,
``OneTransBackbone`` ``:6097-6560``, ``OneTransModel`` ``:7970-8022``.

Token sequence of one sample: ``[S_0 .. S_{L-1}, NS_0 .. NS_{N-1}]`` with the
S tokens left-padded (a sample's valid events are its last ``len`` events; the
first valid token index is ``kstart``).

* S tokens: the embeddings of each event's fields (one lookup per field, rows =
  events) through a ``Linear -> GELU -> Linear`` projection;
* NS tokens (``auto_split``): the concatenated scalar inputs through one
  ``Linear -> GELU -> Linear`` to ``N * d``;
* learned absolute positions counted over valid tokens only (``e - kstart``),
  added to valid tokens;
* per layer (pre-RMSNorm): mixed causal attention -- shared Q/K/V weights for
  S tokens, one weight set per NS token, a shared output projection -- over a
  query suffix (the last ``q_l`` S tokens + all NS tokens, the pyramid), then a
  mixed FFN (shared for S, per NS token), both residual;
* readout: the final NS tokens flattened into the task heads.

Layouts. The whole sequence of a sample lives in one ``[B, L + N, d]`` buffer
(S rows then NS rows): shared-weight products run as GEMMs grouped over the
batch with one weight (batch stride 0), per-token products as GEMMs grouped
over the NS tokens, both writing straight into the buffer, and the weight
gradient of a shared weight sums the per-sample row ranges inside one GEMM. The
attention is the tcgen05 flash attention of ``ops/attention.py``.

Pyramid schedules: ``linear`` is the reference's (``_layer_s_count``
``src/model.py:6181-6198``); ``halve`` keeps ``initial >> ((l + 1) // k)`` S
queries at layer ``l`` (halving every ``k`` layers), rounded like ``linear``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..config.schema import AppConfig
from ..ops._ext import error_word, ext
from ..ops.attention import (NATIVE_HEAD_DIMS, attention_bwd, attention_fwd, suffix_attention,
                             suffix_attention_reference)
from ..ops.gemm import ACT_ADD, ACT_DMUL, ACT_GELU_GRAD, bgemm
from ..ops.layers import _grad, _kaiming_uniform_, _shadow, gemm_param
from .features import FeatureEncoder
from .heads import TaskHeads


# ----------------------------------------------------------------------------- schedule
def pyramid_query_counts(config: AppConfig, initial_s: int, num_ns: int) -> list[int]:
    """S tokens queried (and kept) by each layer."""

    m = config.model
    counts, cur = [], initial_s
    for layer in range(m.num_layers):
        if not m.use_pyramid or initial_s == 0:
            counts.append(cur)
            continue
        final = m.final_s_tokens
        if m.pyramid_schedule == "halve":
            target = initial_s >> ((layer + 1) // max(1, m.pyramid_halve_every))
            if final is not None:
                target = max(min(final, initial_s), target)
                if layer == m.num_layers - 1:
                    target = min(final, initial_s)
        else:
            final = min(num_ns, initial_s) if final is None else min(final, initial_s)
            if layer == m.num_layers - 1:
                target = final
            else:
                progress = float(layer + 1) / float(m.num_layers)
                target = round(initial_s - (initial_s - final) * progress)
            if target > m.pyramid_round_to:
                target = max(final, int(round(target / m.pyramid_round_to) * m.pyramid_round_to))
        if m.pyramid_schedule == "halve" and m.pyramid_round_to < target < initial_s:
            target = int(round(target / m.pyramid_round_to) * m.pyramid_round_to)
        cur = max(0, min(cur, target))
        counts.append(cur)
    return counts


def _off(t: torch.Tensor, n: int) -> torch.Tensor:
    """Flat view of a contiguous tensor starting ``n`` elements in (a GEMM operand base)."""

    return t.view(-1)[n:]


# ----------------------------------------------------------------------------- mixed GEMMs
def _mixed_fwd(x, L, s, K, w_s, b_s, w_ns, b_ns, out, Nout, act=0, out2=None, aux=None):
    """``out [B, L, Nout] = x [B, L, K] W^T + b`` with W shared for rows < s and per token above."""

    B = x.shape[0]
    n = L - s
    if s > 0:
        bgemm(x, w_s, out, M=s, N=Nout, K=K, G=B, lda=K, gsA=L * K, ldb=K, gsB=0, ldc=Nout, gsC=L * Nout,
              out2=out2, bias=b_s, gs_bias=0, aux=aux, ld_aux=Nout, gs_aux=L * Nout, act=act)
    if n > 0:
        bgemm(_off(x, s * K), w_ns, _off(out, s * Nout), M=B, N=Nout, K=K, G=n, lda=L * K, gsA=K, ldb=K,
              gsB=Nout * K, ldc=L * Nout, gsC=Nout, out2=None if out2 is None else _off(out2, s * Nout),
              bias=b_ns, gs_bias=Nout, aux=None if aux is None else _off(aux, s * Nout), ld_aux=L * Nout,
              gs_aux=Nout, act=act)


def _mixed_dgrad(dy, L, s, Nout, K, w_s, w_ns, dx, act=0, aux=None, colsum_s=None, colsum_ns=None):
    """``dx [B, L, K] = dy [B, L, Nout] W`` (optionally times ``aux``, with column sums of the result)."""

    B = dy.shape[0]
    n = L - s
    if s > 0:
        bgemm(dy, w_s, dx, M=s, N=K, K=Nout, G=B, lda=Nout, gsA=L * Nout, ldb=K, gsB=0, b_mn=True, ldc=K,
              gsC=L * K, aux=aux, ld_aux=K, gs_aux=L * K, act=act, colsum=colsum_s, gs_colsum=0)
    if n > 0:
        bgemm(_off(dy, s * Nout), w_ns, _off(dx, s * K), M=B, N=K, K=Nout, G=n, lda=L * Nout, gsA=Nout, ldb=K,
              gsB=Nout * K, b_mn=True, ldc=L * K, gsC=K, aux=None if aux is None else _off(aux, s * K),
              ld_aux=L * K, gs_aux=K, act=act, colsum=colsum_ns, gs_colsum=K)


def _mixed_wgrad(dy, x, L, s, Nout, K, gw_s, gw_ns):
    """``gw_s += sum over S rows of dy^T x``; ``gw_ns[t] += dy_t^T x_t`` (fp32 gradients)."""

    B = dy.shape[0]
    n = L - s
    if s > 0:
        bgemm(dy, x, gw_s, M=Nout, N=K, K=s, lda=Nout, a_mn=True, ldb=K, b_mn=True, ldc=K, accumulate=True,
              kg=B, ksA=L * Nout, ksB=L * K)
    if n > 0:
        bgemm(_off(dy, s * Nout), _off(x, s * K), gw_ns, M=Nout, N=K, K=B, G=n, lda=L * Nout, gsA=Nout, a_mn=True,
              ldb=L * K, gsB=K, b_mn=True, ldc=K, gsC=Nout * K, accumulate=True)


def _mixed_bias_grad(dy, L, s, Nout, gb_s, gb_ns):
    B = dy.shape[0]
    n = L - s
    C = ext()
    if s > 0:
        C.colsum(dy, gb_s, B, s, Nout, Nout, L * Nout, 1.0, 0)
    if n > 0:
        C.colsum(_off(dy, s * Nout), gb_ns, n, B, Nout, L * Nout, Nout, 1.0, Nout)


# ----------------------------------------------------------------------------- fused layer
class OneTransLayerFn(torch.autograd.Function):
    """One OneTrans block on the CUDA path: ``X [B, Lk, d] -> Y [B, q + N, d]``."""

    @staticmethod
    def forward(ctx, X, kstart, layer, s_in, q, heads, eps):
        C = ext()
        B, Lk, D = X.shape
        N = Lk - s_in
        Lq = q + N
        Hd = layer.hidden_dim
        dev = X.device
        X = X.contiguous()
        xn = torch.empty_like(X)
        rstd1 = torch.empty(B * Lk, dtype=torch.float32, device=dev)
        C.rms_fwd(X, layer.norm1, xn, rstd1, B * Lk, D, eps)
        qkv = torch.empty(B, Lk, 3 * D, dtype=torch.bfloat16, device=dev)
        _mixed_fwd(xn, Lk, s_in, D, _shadow(layer.wqkv_s), layer.bqkv_s, _shadow(layer.wqkv_ns), layer.bqkv_ns, qkv,
                   3 * D)
        ks = kstart.to(torch.int32).contiguous()
        att = torch.empty(B, Lq, D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(B, heads, Lq, dtype=torch.float32, device=dev)
        attention_fwd(qkv, ks, att, lse, heads, Lq, True)
        h = torch.empty(B, Lq, D, dtype=torch.bfloat16, device=dev)
        # h = X[:, Lk-Lq:] + att W_o^T + b_o
        bgemm(att, _shadow(layer.wo), h, M=Lq, N=D, K=D, G=B, lda=D, gsA=Lq * D, ldb=D, gsB=0, ldc=D, gsC=Lq * D,
              bias=layer.bo, aux=_off(X, (Lk - Lq) * D), ld_aux=D, gs_aux=Lk * D, act=ACT_ADD)
        hn = torch.empty_like(h)
        rstd2 = torch.empty(B * Lq, dtype=torch.float32, device=dev)
        C.rms_fwd(h, layer.norm2, hn, rstd2, B * Lq, D, eps)
        ug = torch.empty(B, Lq, Hd, dtype=torch.bfloat16, device=dev)
        u = torch.empty_like(ug)
        _mixed_fwd(hn, Lq, q, D, _shadow(layer.w1_s), layer.b1_s, _shadow(layer.w1_ns), layer.b1_ns, ug, Hd,
                   act=ACT_GELU_GRAD, out2=u)
        Y = torch.empty(B, Lq, D, dtype=torch.bfloat16, device=dev)
        _mixed_fwd(u, Lq, q, Hd, _shadow(layer.w2_s), layer.b2_s, _shadow(layer.w2_ns), layer.b2_ns, Y, D,
                   act=ACT_ADD, aux=h)
        ctx.save_for_backward(X, xn, rstd1, qkv, ks, att, lse, h, hn, rstd2, ug, u)
        ctx.meta = (layer, s_in, q, heads)
        return Y

    @staticmethod
    def backward(ctx, dY):
        X, xn, rstd1, qkv, ks, att, lse, h, hn, rstd2, ug, u = ctx.saved_tensors
        layer, s_in, q, heads = ctx.meta
        C = ext()
        B, Lk, D = X.shape
        N = Lk - s_in
        Lq = q + N
        Hd = layer.hidden_dim
        dev = X.device
        dY = dY.to(torch.bfloat16).contiguous()
        # ---- FFN
        du = torch.empty(B, Lq, Hd, dtype=torch.bfloat16, device=dev)
        _mixed_dgrad(dY, Lq, q, D, Hd, _shadow(layer.w2_s), _shadow(layer.w2_ns), du, act=ACT_DMUL, aux=ug,
                     colsum_s=_grad(layer.b1_s), colsum_ns=_grad(layer.b1_ns))
        _mixed_wgrad(dY, u, Lq, q, D, Hd, _grad(layer.w2_s), _grad(layer.w2_ns))
        _mixed_bias_grad(dY, Lq, q, D, _grad(layer.b2_s), _grad(layer.b2_ns))
        dhn = torch.empty(B, Lq, D, dtype=torch.bfloat16, device=dev)
        _mixed_dgrad(du, Lq, q, Hd, D, _shadow(layer.w1_s), _shadow(layer.w1_ns), dhn)
        _mixed_wgrad(du, hn, Lq, q, Hd, D, _grad(layer.w1_s), _grad(layer.w1_ns))
        del du
        dh = torch.empty_like(dhn)
        C.rms_bwd(h, layer.norm2, rstd2, dhn, dh, _grad(layer.norm2), B * Lq, D, dres=dY)
        # ---- attention output projection
        datt = torch.empty_like(dh)
        bgemm(dh, _shadow(layer.wo), datt, M=B * Lq, N=D, K=D, lda=D, ldb=D, b_mn=True, ldc=D)
        bgemm(dh, att, _grad(layer.wo), M=D, N=D, K=B * Lq, lda=D, a_mn=True, ldb=D, b_mn=True, ldc=D,
              accumulate=True)
        C.colsum(dh, _grad(layer.bo), 1, B * Lq, D, D, 0, 1.0)
        # ---- attention
        dqkv = torch.empty_like(qkv)
        attention_bwd(qkv, ks, att, lse, datt, dqkv, heads, Lq, True)
        del datt
        # ---- Q/K/V projections
        dxn = torch.empty_like(X)
        _mixed_dgrad(dqkv, Lk, s_in, 3 * D, D, _shadow(layer.wqkv_s), _shadow(layer.wqkv_ns), dxn)
        _mixed_wgrad(dqkv, xn, Lk, s_in, 3 * D, D, _grad(layer.wqkv_s), _grad(layer.wqkv_ns))
        _mixed_bias_grad(dqkv, Lk, s_in, 3 * D, _grad(layer.bqkv_s), _grad(layer.bqkv_ns))
        dX = torch.empty_like(X)
        C.rms_bwd(X, layer.norm1, rstd1, dxn, dX, _grad(layer.norm1), B * Lk, D, dres=dh, res_period=Lk,
                  res_tail=Lq)
        return dX, None, None, None, None, None, None


class OneTransTokenizeFn(torch.autograd.Function):
    """S tokens (event projection MLP) + NS tokens + positions -> ``[B, L + N, d]``.

    ``auto_split`` NS tokens are computed here (MLP GEMMs writing the NS rows);
    for the other NS encoders ``ns_in`` is the finished ``[B, N * d]`` token
    matrix, copied into the NS rows (its gradient is the NS rows of ``dX0``)."""

    @staticmethod
    def forward(ctx, seq_in, ns_in, kstart, model, L):
        C = ext()
        B = ns_in.shape[0]
        D, N, Hd = model.token_dim, model.num_ns, model.hidden_dim
        Ks, Kn = seq_in.shape[1], ns_in.shape[1]
        Lt = L + N
        dev = ns_in.device
        ug = torch.empty(B * L, Hd, dtype=torch.bfloat16, device=dev)
        u = torch.empty_like(ug)
        bgemm(seq_in, _shadow(model.seq_w1), ug, M=B * L, N=Hd, K=Ks, lda=seq_in.stride(0), ldb=Ks, ldc=Hd, out2=u,
              bias=model.seq_b1, act=ACT_GELU_GRAD)
        X0 = torch.empty(B, Lt, D, dtype=torch.bfloat16, device=dev)
        bgemm(u, _shadow(model.seq_w2), X0, M=L, N=D, K=Hd, G=B, lda=Hd, gsA=L * Hd, ldb=Hd, gsB=0, ldc=D,
              gsC=Lt * D, bias=model.seq_b2)
        vg, v = _ns_rows_forward(model, ns_in, X0, L)
        ks = kstart.to(torch.int32).contiguous()
        C.position_add(X0, model.pos, ks, B, Lt, D)
        ctx.save_for_backward(seq_in, ns_in, ks, ug, u, vg, v)
        ctx.meta = (model, L)
        return X0

    @staticmethod
    def backward(ctx, dX0):
        seq_in, ns_in, ks, ug, u, vg, v = ctx.saved_tensors
        model, L = ctx.meta
        C = ext()
        B = ns_in.shape[0]
        D, N, Hd = model.token_dim, model.num_ns, model.hidden_dim
        Ks, Kn = seq_in.shape[1], ns_in.shape[1]
        Lt = L + N
        dev = ns_in.device
        dX0 = dX0.to(torch.bfloat16).contiguous()
        C.position_grad(dX0, _grad(model.pos), ks, B, Lt, D)
        # S: projection MLP over events
        du = torch.empty(B * L, Hd, dtype=torch.bfloat16, device=dev)
        bgemm(dX0, _shadow(model.seq_w2), du, M=L, N=Hd, K=D, G=B, lda=D, gsA=Lt * D, ldb=Hd, gsB=0, b_mn=True,
              ldc=Hd, gsC=L * Hd, aux=ug, ld_aux=Hd, gs_aux=L * Hd, act=ACT_DMUL, colsum=_grad(model.seq_b1),
              gs_colsum=0)
        bgemm(dX0, u, _grad(model.seq_w2), M=D, N=Hd, K=L, lda=D, a_mn=True, ldb=Hd, b_mn=True, ldc=Hd,
              accumulate=True, kg=B, ksA=Lt * D, ksB=L * Hd)
        C.colsum(dX0, _grad(model.seq_b2), B, L, D, D, Lt * D, 1.0, 0)
        bgemm(du, seq_in, _grad(model.seq_w1), M=Hd, N=Ks, K=B * L, lda=Hd, a_mn=True, ldb=seq_in.stride(0),
              b_mn=True, ldc=Ks, accumulate=True)
        dseq = torch.empty(B * L, Ks, dtype=torch.bfloat16, device=dev)
        bgemm(du, _shadow(model.seq_w1), dseq, M=B * L, N=Ks, K=Hd, lda=Hd, ldb=Ks, b_mn=True, ldc=Ks)
        del du
        return dseq, _ns_rows_backward(model, ns_in, dX0, L, vg, v), None, None, None


def _ns_rows_forward(model, ns_in, X0, L):
    """NS rows ``[L, L + N)`` of the token buffer: the ``auto_split`` MLP (GEMMs writing
    the rows in place) or a copy of the finished ``[B, N * d]`` tokens."""

    B = ns_in.shape[0]
    D, N, Hd = model.token_dim, model.num_ns, model.hidden_dim
    Kn, Lt, dev = ns_in.shape[1], L + N, ns_in.device
    if model.ns_mode == "auto_split":
        vg = torch.empty(B, Hd, dtype=torch.bfloat16, device=dev)
        v = torch.empty_like(vg)
        bgemm(ns_in, _shadow(model.ns_w1), vg, M=B, N=Hd, K=Kn, lda=ns_in.stride(0), ldb=Kn, ldc=Hd, out2=v,
              bias=model.ns_b1, act=ACT_GELU_GRAD)
        bgemm(v, _shadow(model.ns_w2), _off(X0, L * D), M=B, N=N * D, K=Hd, lda=Hd, ldb=Hd, ldc=Lt * D,
              bias=model.ns_b2)
        return vg, v
    X0[:, L:, :].copy_(ns_in.view(B, N, D))
    empty = ns_in.new_empty(0)
    return empty, empty


def _ns_rows_backward(model, ns_in, dX0, L, vg, v):
    """Gradient of ``ns_in`` from the NS rows of ``dX0`` (weight gradients accumulated)."""

    B = ns_in.shape[0]
    D, N, Hd = model.token_dim, model.num_ns, model.hidden_dim
    Kn, Lt, dev = ns_in.shape[1], L + N, ns_in.device
    if model.ns_mode != "auto_split":
        return dX0[:, L:, :].reshape(B, N * D)
    C = ext()
    dns_tok = _off(dX0, L * D)
    dv = torch.empty(B, Hd, dtype=torch.bfloat16, device=dev)
    bgemm(dns_tok, _shadow(model.ns_w2), dv, M=B, N=Hd, K=N * D, lda=Lt * D, ldb=Hd, b_mn=True, ldc=Hd, aux=vg,
          ld_aux=Hd, act=ACT_DMUL, colsum=_grad(model.ns_b1))
    bgemm(dns_tok, v, _grad(model.ns_w2), M=N * D, N=Hd, K=B, lda=Lt * D, a_mn=True, ldb=Hd, b_mn=True, ldc=Hd,
          accumulate=True)
    C.colsum(dns_tok, _grad(model.ns_b2), 1, B, N * D, Lt * D, 0, 1.0)
    bgemm(dv, ns_in, _grad(model.ns_w1), M=Hd, N=Kn, K=B, lda=Hd, a_mn=True, ldb=ns_in.stride(0), b_mn=True,
          ldc=Kn, accumulate=True)
    dns = torch.empty(B, Kn, dtype=torch.bfloat16, device=dev)
    bgemm(dv, _shadow(model.ns_w1), dns, M=B, N=Kn, K=Hd, lda=Hd, ldb=Kn, b_mn=True, ldc=Kn)
    return dns


class OneTransAssembleFn(torch.autograd.Function):
    """Finished S tokens (several fused sequence groups) + NS tokens + positions ->
    ``[B, S + N, d]`` (the multi-group counterpart of ``OneTransTokenizeFn``)."""

    @staticmethod
    def forward(ctx, s_tokens, ns_in, kstart, model, S):
        B = ns_in.shape[0]
        D, N = model.token_dim, model.num_ns
        X0 = torch.empty(B, S + N, D, dtype=torch.bfloat16, device=ns_in.device)
        X0[:, :S].copy_(s_tokens)
        vg, v = _ns_rows_forward(model, ns_in, X0, S)
        ks = kstart.to(torch.int32).contiguous()
        ext().position_add(X0, model.pos, ks, B, S + N, D)
        ctx.save_for_backward(ns_in, ks, vg, v)
        ctx.meta = (model, S)
        return X0

    @staticmethod
    def backward(ctx, dX0):
        ns_in, ks, vg, v = ctx.saved_tensors
        model, S = ctx.meta
        B = ns_in.shape[0]
        D, N = model.token_dim, model.num_ns
        dX0 = dX0.to(torch.bfloat16).contiguous()
        ext().position_grad(dX0, _grad(model.pos), ks, B, S + N, D)
        dns = _ns_rows_backward(model, ns_in, dX0, S, vg, v)
        return dX0[:, :S], dns, None, None, None


# ----------------------------------------------------------------------------- modules
def _rms_reference(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _mixed_reference(x, s, w_s, b_s, w_ns, b_ns):
    """fp32: rows < s with the shared weight, rows >= s with their own."""

    ys = x[:, :s] @ w_s.t() + b_s
    if x.shape[1] == s:  # S rows only (the request side of a request cache)
        return ys
    yn = torch.einsum("bnk,nok->bno", x[:, s:], w_ns) + b_ns.unsqueeze(0)
    return torch.cat([ys, yn], dim=1)


class OneTransLayer(nn.Module):
    """Parameters of one block (reference ``OneTransBlock`` ``src/model.py:5821-5840``)."""

    def __init__(self, token_dim: int, hidden_dim: int, num_ns: int, device=None) -> None:
        super().__init__()
        D, H, N = token_dim, hidden_dim, num_ns
        self.token_dim, self.hidden_dim, self.num_ns = D, H, N
        self.norm1 = nn.Parameter(torch.ones(D, device=device))
        self.wqkv_s = gemm_param(torch.empty(3 * D, D, device=device))
        self.bqkv_s = nn.Parameter(torch.empty(3 * D, device=device))
        self.wqkv_ns = gemm_param(torch.empty(N, 3 * D, D, device=device))
        self.bqkv_ns = nn.Parameter(torch.empty(N, 3 * D, device=device))
        self.wo = gemm_param(torch.empty(D, D, device=device))
        self.bo = nn.Parameter(torch.empty(D, device=device))
        self.norm2 = nn.Parameter(torch.ones(D, device=device))
        self.w1_s = gemm_param(torch.empty(H, D, device=device))
        self.b1_s = nn.Parameter(torch.empty(H, device=device))
        self.w1_ns = gemm_param(torch.empty(N, H, D, device=device))
        self.b1_ns = nn.Parameter(torch.empty(N, H, device=device))
        self.w2_s = gemm_param(torch.empty(D, H, device=device))
        self.b2_s = nn.Parameter(torch.empty(D, device=device))
        self.w2_ns = gemm_param(torch.empty(N, D, H, device=device))
        self.b2_ns = nn.Parameter(torch.empty(N, D, device=device))
        # nn.Linear's default init per projection (kaiming-uniform weight, bias U(+-1/sqrt(fan_in)))
        for w, b, fan in ((self.wqkv_s, self.bqkv_s, D), (self.wo, self.bo, D), (self.w1_s, self.b1_s, D),
                          (self.w2_s, self.b2_s, H)):
            _kaiming_uniform_(w.data, fan)
            _kaiming_uniform_(b.data, fan)
        for w, b, fan in ((self.wqkv_ns, self.bqkv_ns, D), (self.w1_ns, self.b1_ns, D), (self.w2_ns, self.b2_ns, H)):
            _kaiming_uniform_(w.data, fan)
            _kaiming_uniform_(b.data, fan)

    def forward_reference(self, X, kstart, s_in, q, heads, eps):
        B, Lk, D = X.shape
        N = Lk - s_in
        Lq = q + N
        xn = _rms_reference(X, self.norm1, eps)
        qkv = _mixed_reference(xn, s_in, self.wqkv_s, self.bqkv_s, self.wqkv_ns, self.bqkv_ns)
        att = suffix_attention_reference(qkv, kstart, heads, Lq)
        h = X[:, Lk - Lq:].float() + att @ self.wo.t() + self.bo
        hn = _rms_reference(h, self.norm2, eps)
        u = F.gelu(_mixed_reference(hn, q, self.w1_s, self.b1_s, self.w1_ns, self.b1_ns))
        return h + _mixed_reference(u, q, self.w2_s, self.b2_s, self.w2_ns, self.b2_ns)

    def reference_state_dict(self, prefix: str) -> dict[str, torch.Tensor]:
        D = self.token_dim
        sd = {prefix + "norm_attention.weight": self.norm1, prefix + "norm_ffn.weight": self.norm2,
              prefix + "attention.output.weight": self.wo, prefix + "attention.output.bias": self.bo,
              prefix + "ffn.s_ffn.0.weight": self.w1_s, prefix + "ffn.s_ffn.0.bias": self.b1_s,
              prefix + "ffn.s_ffn.2.weight": self.w2_s, prefix + "ffn.s_ffn.2.bias": self.b2_s}
        for j, part in enumerate(("query", "key", "value")):
            sd[prefix + f"attention.s_{part}.weight"] = self.wqkv_s[j * D:(j + 1) * D]
            sd[prefix + f"attention.s_{part}.bias"] = self.bqkv_s[j * D:(j + 1) * D]
            for n in range(self.num_ns):
                sd[prefix + f"attention.ns_{part}.{n}.weight"] = self.wqkv_ns[n, j * D:(j + 1) * D]
                sd[prefix + f"attention.ns_{part}.{n}.bias"] = self.bqkv_ns[n, j * D:(j + 1) * D]
        for n in range(self.num_ns):
            sd[prefix + f"ffn.ns_ffn.{n}.0.weight"] = self.w1_ns[n]
            sd[prefix + f"ffn.ns_ffn.{n}.0.bias"] = self.b1_ns[n]
            sd[prefix + f"ffn.ns_ffn.{n}.2.weight"] = self.w2_ns[n]
            sd[prefix + f"ffn.ns_ffn.{n}.2.bias"] = self.b2_ns[n]
        return {k: v.detach().clone() for k, v in sd.items()}


class OneTransModel(nn.Module):
    """OneTrans ranker (``model.name: onetrans``) with ``auto_split`` NS tokens and one
    ``intent_ordered`` sequence group."""

    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1, process_group=None,
                 vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None,
                 domain_tokens: list[list[str]] | None = None, task_heads: bool = True) -> None:
        super().__init__()
        m = config.model
        self.ns_mode = m.ns_tokenizer
        if self.ns_mode not in ("auto_split", "dcnv2", "groupwise"):
            raise NotImplementedError(f"OneTrans ns_tokenizer {m.ns_tokenizer!r}")
        groups = config.resolved.tokenization.sequence_token_groups
        seq_by_name = {s.name: s for s in config.sequences}
        if not groups:
            raise ValueError("OneTrans requires at least one sequence token group")
        group_seqs = []
        for g in groups:
            if len(g.inputs) != 1 or g.inputs[0] not in seq_by_name:
                raise NotImplementedError(f"OneTrans sequence token group {g.name!r}: a group holds one raw sequence")
            group_seqs.append(seq_by_name[g.inputs[0]])
        if m.token_dim % m.num_heads:
            raise ValueError("token_dim must be divisible by num_heads")
        self.head_dim = m.token_dim // m.num_heads
        self.config = config
        self.seq = group_seqs[0]
        self.group_seqs = group_seqs
        self.multi = len(group_seqs) > 1
        if not self.seq.max_length:
            raise ValueError(f"sequence {self.seq.name!r} needs max_length")
        self.L = int(self.seq.max_length)
        ns_inputs = list(config.resolved.tokenization.feature_token_inputs)
        # groupwise NS tokens read per-group input slices: the encoder's per-token input plan
        # (shared with the MDL domain tokens, which follow the NS groups)
        ns_groups = [list(g.inputs) for g in config.resolved.tokenization.ns_token_groups]
        if self.ns_mode == "groupwise":
            if not ns_groups:
                raise ValueError("groupwise OneTrans tokenizer requires tokenization.ns_tokens or scalar features")
            ns_inputs = []
            domain_tokens = ns_groups + list(domain_tokens or [])
        self._dom_offset = len(ns_groups) if self.ns_mode == "groupwise" else 0
        self.encoder = FeatureEncoder(config, device=device, rank=rank, world=world, process_group=process_group,
                                      vocab_sizes=vocab_sizes, input_names=ns_inputs, slice_tokens=1,
                                      base_seed=base_seed, sequences=group_seqs, domain_tokens=domain_tokens or None)
        from .sequence_encoders import SequenceSummaries

        # prior sequences of the MDL domain tokens (mean_pool / attention_pool / longer / stca)
        self.summaries = SequenceSummaries(config, self.encoder, self.encoder.summary_names, device=device)
        D, Hd = int(m.token_dim), int(m.hidden_dim)
        if self.ns_mode == "groupwise":
            N = len(ns_groups)
        else:
            N = int(m.num_ns_tokens or max(1, len(ns_inputs)))
        self.token_dim, self.hidden_dim, self.num_ns, self.attn_heads = D, Hd, N, int(m.num_heads)
        self.eps = 1e-6
        self.Kn, self.Kn_log = self.encoder.plan.out_ld, self.encoder.plan.out_width
        if self.multi:
            # several groups: per-group projection MLPs, SEP tokens / time order, compaction
            from .sequence_fusion import SequenceGroups

            self.seq_groups = SequenceGroups(config, self.encoder, group_seqs, D, projection="mlp", hidden=Hd,
                                             device=device)
            self.L = self.seq_groups.S
        else:
            seq_plan = self.encoder.seq_plans[self.seq.name]
            self.Ks, self.Ks_log = seq_plan.out_ld, seq_plan.out_width
            self.seq_w1 = gemm_param(torch.zeros(Hd, self.Ks, device=device))
            self.seq_b1 = nn.Parameter(torch.empty(Hd, device=device))
            self.seq_w2 = gemm_param(torch.empty(D, Hd, device=device))
            self.seq_b2 = nn.Parameter(torch.empty(D, device=device))
            _kaiming_uniform_(self.seq_w1.data[:, :self.Ks_log], self.Ks_log)  # padded input columns stay zero
            _kaiming_uniform_(self.seq_b1.data, self.Ks_log)
            _kaiming_uniform_(self.seq_w2.data, Hd)
            _kaiming_uniform_(self.seq_b2.data, Hd)
        if self.ns_mode == "auto_split":
            self.ns_w1 = gemm_param(torch.zeros(Hd, self.Kn, device=device))
            self.ns_b1 = nn.Parameter(torch.empty(Hd, device=device))
            self.ns_w2 = gemm_param(torch.empty(N * D, Hd, device=device))
            self.ns_b2 = nn.Parameter(torch.empty(N * D, device=device))
            _kaiming_uniform_(self.ns_w1.data[:, :self.Kn_log], self.Kn_log)
            _kaiming_uniform_(self.ns_b1.data, self.Kn_log)
            _kaiming_uniform_(self.ns_w2.data, Hd)
            _kaiming_uniform_(self.ns_b2.data, Hd)
        elif self.ns_mode == "dcnv2":
            from .ns_encoders import DCNv2Encoder

            proj = int(m.ns_dcn_projection_dim or Hd)
            self.ns_dcn = DCNv2Encoder(self.Kn, self.Kn_log, N * D, proj, int(m.ns_dcn_cross_layers),
                                       int(m.ns_dcn_deep_layers), int(m.ns_dcn_deep_dim or proj), m.ffn_activation,
                                       m.ns_dcn_low_rank, device=device)
        else:
            from .ns_encoders import GroupwiseNS

            self.ns_group = GroupwiseNS(self.encoder.domain_widths[:N], self.encoder.domain_k_pad, D, Hd,
                                        m.ffn_activation, device=device)
        P = max(int(config.resolved.onetrans_max_position_embeddings), self.L + N)
        self.pos = nn.Parameter(torch.empty(P, D, device=device).normal_(0.0, m.init_std))
        self.layers = nn.ModuleList(OneTransLayer(D, Hd, N, device=device) for _ in range(m.num_layers))
        self.query_counts = pyramid_query_counts(config, self.L, N)
        self.ntask = len(config.task_names)
        self.task_query = None
        if task_heads:
            head_in = N * D
            if m.readout == "task_query":
                from .heads import TaskQueryReadout

                self.task_query = TaskQueryReadout(self.ntask, D, int(m.num_heads), N, Hd, m.ffn_activation,
                                                   float(m.init_std), device=device)
                head_in = D
            self.heads_mod = TaskHeads(self.ntask, head_in, int(m.task_head_hidden_dim or Hd),
                                       m.task_head_activation, device=device)

    # ------------------------------------------------------------------ params
    def gemm_param_names(self) -> set[str]:
        return {n for n, p in self.named_parameters() if getattr(p, "_mdl_gemm", False)}

    def dense_buckets(self) -> list[list[str]]:
        names = [n for n, _ in self.named_parameters()]
        heads = [n for n in names if n.startswith("heads_mod.")]
        layers = [[n for n in names if n.startswith(f"layers.{i}.")] for i in reversed(range(len(self.layers)))]
        rest = [n for n in names if not n.startswith(("heads_mod.", "layers."))]
        return [heads, *layers, rest]

    @property
    def store(self):
        return self.encoder.store

    # ------------------------------------------------------------------ inputs
    def _inputs(self, batch, anchor):
        from ..ops.embedding import fused_lookup
        from .features import lookup_sequence

        B, L = batch.rows, self.L
        if self.multi:
            native = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
            seq_in, valid = self.seq_groups(self.encoder, batch, anchor, native)  # finished S tokens
            kstart = (L - valid.to(torch.int64)).to(torch.int32)
        else:
            seq_in, lengths = lookup_sequence(self.encoder, batch, self.seq.name, B, L, anchor)
            kstart = (L - lengths.to(torch.int64).clamp(0, L)).to(torch.int32)
        if self.ns_mode == "groupwise":
            ns_in = fused_lookup(self.store, self.encoder.domain_plan, batch.ids, batch.offsets, batch.dense, B, anchor)
        else:
            ns_in = fused_lookup(self.store, self.encoder.plan, batch.ids, batch.offsets, batch.dense, B, anchor)
        return seq_in, ns_in, kstart

    def ns_tokens(self, ns_in: torch.Tensor) -> torch.Tensor:
        """``[B, N * d]`` NS tokens of the ``dcnv2`` / ``groupwise`` encoders (``auto_split``
        runs inside the tokenizer)."""

        B = ns_in.shape[0]
        if self.ns_mode == "dcnv2":
            return self.ns_dcn(ns_in)
        kp = self.encoder.domain_k_pad
        v = ns_in.as_strided((B, self.num_ns * kp), (ns_in.stride(0), 1))
        return self.ns_group(v).reshape(B, self.num_ns * self.token_dim)

    # ------------------------------------------------------------------ forward
    def forward(self, batch, task_scale: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        anchor = torch.zeros(0, device=batch.ids.device, requires_grad=True)
        seq_in, ns_in, kstart = self._inputs(batch, anchor)
        if task_scale is None:
            task_scale = torch.full((self.ntask,), 1.0 / max(1, batch.rows), device=batch.ids.device)
        if batch.ids.is_cuda and self.config.runtime.kernel_backend == "native":
            return self._forward_cuda(seq_in, ns_in, kstart, batch, task_scale)
        return self.forward_reference(seq_in, ns_in, kstart, batch, task_scale)

    def _forward_cuda(self, seq_in, ns_in, kstart, batch, task_scale):
        from ..ops.dense import grad_ready

        hooks = getattr(self, "dense_hooks", None)
        nl = len(self.layers)
        seq_in = grad_ready(seq_in, hooks, nl + 1)
        if self.ns_mode != "auto_split":
            ns_in = self.ns_tokens(ns_in).to(torch.bfloat16)
        if self.head_dim not in NATIVE_HEAD_DIMS:
            raise NotImplementedError(f"OneTrans head_dim {self.head_dim}: the native attention kernels take "
                                      f"{NATIVE_HEAD_DIMS} (set runtime.kernel_backend: torch for this model)")
        if self.multi:
            X = OneTransAssembleFn.apply(seq_in.to(torch.bfloat16), ns_in, kstart, self, self.L)
        else:
            X = OneTransTokenizeFn.apply(seq_in, ns_in, kstart, self, self.L)
        s_in, ks = self.L, kstart
        for i, layer in enumerate(self.layers):
            X = grad_ready(X, hooks, nl - i)
            q = self.query_counts[i]
            X = OneTransLayerFn.apply(X, ks, layer, s_in, q, self.attn_heads, self.eps)
            ks = (ks - (s_in - q)).clamp(min=0)
            s_in = q
        X = grad_ready(X, hooks, 0)
        return self._task_logits(X[:, s_in:, :], batch, task_scale)

    def _task_logits(self, ns: torch.Tensor, batch, task_scale) -> dict[str, torch.Tensor]:
        """Heads over the flattened final NS tokens, or over the task-query states
        (reference ``_task_readout_logits`` ``src/model.py:960-972``)."""

        if self.task_query is not None:
            return self.heads_mod(self.task_query(ns), batch.labels, batch.label_mask, task_scale)
        B = ns.shape[0]
        return self.heads_mod.forward_shared(ns.reshape(B, -1), batch.labels, batch.label_mask, task_scale)

    def tokenize_reference(self, seq_in, ns_in, kstart, B):
        """fp32 PyTorch tokenizer: ``[B, L + N, d]`` with positions on the valid tokens."""

        L, D, N = self.L, self.token_dim, self.num_ns
        if self.multi:
            s = seq_in.float().view(B, L, D)
        else:
            s = F.gelu(seq_in.float()[:, :self.Ks_log] @ self.seq_w1[:, :self.Ks_log].t() + self.seq_b1)
            s = (s @ self.seq_w2.t() + self.seq_b2).view(B, L, D)
        if self.ns_mode == "auto_split":
            v = F.gelu(ns_in.float()[:, :self.Kn_log] @ self.ns_w1[:, :self.Kn_log].t() + self.ns_b1)
            ns = (v @ self.ns_w2.t() + self.ns_b2).view(B, N, D)
        else:
            ns = self.ns_tokens(ns_in).float().view(B, N, D)
        X = torch.cat([s, ns], dim=1)
        e = torch.arange(L + N, device=X.device)
        ks = kstart.to(X.device).long()
        valid = e.view(1, -1) >= ks.view(-1, 1)
        pid = (e.view(1, -1) - ks.view(-1, 1)).clamp(min=0)
        return X + self.pos[pid] * valid.unsqueeze(-1)

    def forward_reference(self, seq_in, ns_in, kstart, batch, task_scale=None):
        """Plain PyTorch fp32 definition (CPU path and test oracle)."""

        B, L, D, N = batch.rows, self.L, self.token_dim, self.num_ns
        X = self.tokenize_reference(seq_in, ns_in, kstart, B)
        ks = kstart.to(X.device).long()
        s_in = L
        for i, layer in enumerate(self.layers):
            q = self.query_counts[i]
            X = layer.forward_reference(X, ks, s_in, q, self.attn_heads, self.eps)
            ks = (ks - (s_in - q)).clamp(min=0)
            s_in = q
        return self._task_logits(X[:, s_in:, :], batch, task_scale)

    # ------------------------------------------------------------------ request cache
    @torch.no_grad()
    def precompute_request_cache(self, batch) -> dict:
        """Candidate-independent OneTrans state per request (reference
        ``OneTransBackbone.precompute_request_cache`` ``src/model.py:6200-6398``). S tokens
        precede the NS tokens and the attention is causal, so every S token's output is
        independent of the candidate: per layer the cache keeps the K/V of the layer's S
        keys and their padding count; candidates then run only their NS tokens. Rows are the
        requests of the sequence payload (``row_indices``; one per row without it)."""

        from .features import lookup_sequence

        if self.multi:
            raise NotImplementedError("OneTrans request cache: one sequence token group")
        anchor = torch.zeros(0, device=batch.ids.device)
        L, D = self.L, self.token_dim
        seq_in, lengths, _ri = lookup_sequence(self.encoder, batch, self.seq.name, batch.rows, L, anchor,
                                               expand=False)
        R = lengths.numel()
        ks = (L - lengths.to(seq_in.device).long().clamp(0, L))
        x = F.gelu(seq_in.float()[:, :self.Ks_log] @ self.seq_w1[:, :self.Ks_log].t() + self.seq_b1)
        S = (x @ self.seq_w2.t() + self.seq_b2).view(R, L, D)
        e = torch.arange(L, device=S.device)
        valid = e.view(1, -1) >= ks.view(-1, 1)
        S = S + self.pos[(e.view(1, -1) - ks.view(-1, 1)).clamp(min=0)] * valid.unsqueeze(-1)
        layers, s_in, kst = [], L, ks
        for i, layer in enumerate(self.layers):
            q = self.query_counts[i]
            xn = _rms_reference(S, layer.norm1, self.eps)
            kv = xn @ layer.wqkv_s[D:].t() + layer.bqkv_s[D:]                   # [R, s_in, 2D]
            layers.append((kv, kst))
            S = layer.forward_reference(S, kst, s_in, q, self.attn_heads, self.eps)  # S-only: q outputs
            kst = (kst - (s_in - q)).clamp(min=0)
            s_in = q
        return {"layers": layers, "kstart": ks, "lengths": lengths}

    @torch.no_grad()
    def forward_with_cache(self, batch, request_cache: dict) -> torch.Tensor:
        """Logits ``[rows, tasks]`` of candidate rows from a request cache: the NS tokens
        attend to their request's cached S keys (valid from the cached padding count) and
        causally to each other; the per-NS-token projections and FFNs run per candidate."""

        from ..ops.embedding import fused_lookup

        anchor = torch.zeros(0, device=batch.ids.device)
        B, L, D, N, H = batch.rows, self.L, self.token_dim, self.num_ns, self.attn_heads
        plan = self.encoder.domain_plan if self.ns_mode == "groupwise" else self.encoder.plan
        ns_in = fused_lookup(self.store, plan, batch.ids, batch.offsets, batch.dense, B, anchor).float()
        ri = (batch.sequences.get(self.seq.name) or {}).get("row_indices")
        ri = (torch.arange(B, device=ns_in.device) if ri is None else ri.to(ns_in.device).long())
        if self.ns_mode == "auto_split":
            v = F.gelu(ns_in[:, :self.Kn_log] @ self.ns_w1[:, :self.Kn_log].t() + self.ns_b1)
            X = (v @ self.ns_w2.t() + self.ns_b2).view(B, N, D)
        else:
            X = self.ns_tokens(ns_in).float().view(B, N, D)
        ks0 = request_cache["kstart"].index_select(0, ri)
        X = X + self.pos[(L + torch.arange(N, device=X.device).view(1, -1) - ks0.view(-1, 1)).clamp(min=0)]
        hd = D // H
        causal = torch.ones(N, N, dtype=torch.bool, device=X.device).tril()
        for layer, (kv_s, kst) in zip(self.layers, request_cache["layers"]):
            xn = _rms_reference(X, layer.norm1, self.eps)
            qkv = torch.einsum("bnk,nok->bno", xn, layer.wqkv_ns) + layer.bqkv_ns.unsqueeze(0)   # [B, N, 3D]
            kv = torch.cat([kv_s.index_select(0, ri), qkv[..., D:]], dim=1)                    # [B, s + N, 2D]
            s_in = kv_s.shape[1]
            k = kv[..., :D].reshape(B, s_in + N, H, hd).transpose(1, 2)
            v = kv[..., D:].reshape(B, s_in + N, H, hd).transpose(1, 2)
            qh = qkv[..., :D].reshape(B, N, H, hd).transpose(1, 2)
            s_ok = torch.arange(s_in, device=X.device).view(1, 1, s_in) >= kst.index_select(0, ri).view(B, 1, 1)
            allowed = torch.cat([s_ok.expand(B, N, s_in), causal.view(1, N, N).expand(B, N, N)], dim=2)
            sc = (qh @ k.transpose(-1, -2)) / math.sqrt(hd)
            att = torch.softmax(sc.masked_fill(~allowed.unsqueeze(1), float("-inf")), -1) @ v
            h = X + att.transpose(1, 2).reshape(B, N, D) @ layer.wo.t() + layer.bo
            hn = _rms_reference(h, layer.norm2, self.eps)
            u = F.gelu(torch.einsum("bnk,nok->bno", hn, layer.w1_ns) + layer.b1_ns.unsqueeze(0))
            X = h + torch.einsum("bnk,nok->bno", u, layer.w2_ns) + layer.b2_ns.unsqueeze(0)
        scale = torch.ones(self.ntask, device=X.device)
        from types import SimpleNamespace

        return self._task_logits(X, SimpleNamespace(labels=None, label_mask=None), scale)["logits"]

    # ------------------------------------------------------------------ reference layout
    def reference_state_dict(self) -> dict[str, torch.Tensor]:
        """Dense weights under the reference's parameter names (``OneTransModel``)."""

        p = "backbone."
        sd = {p + "tokenizer.sequence_projectors.0.0.weight": self.seq_w1[:, :self.Ks_log],
              p + "tokenizer.sequence_projectors.0.0.bias": self.seq_b1,
              p + "tokenizer.sequence_projectors.0.2.weight": self.seq_w2,
              p + "tokenizer.sequence_projectors.0.2.bias": self.seq_b2,
              p + "unified_position_embeddings.weight": self.pos}
        if self.ns_mode == "auto_split":
            sd.update({p + "tokenizer.auto_ns_projection.0.weight": self.ns_w1[:, :self.Kn_log],
                       p + "tokenizer.auto_ns_projection.0.bias": self.ns_b1,
                       p + "tokenizer.auto_ns_projection.2.weight": self.ns_w2,
                       p + "tokenizer.auto_ns_projection.2.bias": self.ns_b2})
        sd = {k: v.detach().clone() for k, v in sd.items()}
        if self.ns_mode == "dcnv2":
            sd.update(self.ns_dcn.reference_state_dict(p + "tokenizer.dcn_ns_encoder."))
        elif self.ns_mode == "groupwise":
            sd.update(self.ns_group.reference_state_dict(p + "tokenizer.ns_projectors."))
        for i, layer in enumerate(self.layers):
            sd.update(layer.reference_state_dict(f"{p}blocks.{i}."))
        sd.update(self.heads_mod.reference_state_dict())
        if self.task_query is not None:
            sd.update({"task_query_readout." + k: v.detach().clone()
                       for k, v in self.task_query.state_dict().items()})
        return sd


def build_onetrans(config: AppConfig, **kw):
    if config.model.name == "onetrans":
        return OneTransModel(config, **kw)
    from .mdl_onetrans import MDLOneTransModel

    return MDLOneTransModel(config, **kw)
