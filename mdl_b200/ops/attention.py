"""Causal attention of a query suffix over its own token sequence.

``suffix_attention(qkv, kstart, heads, lq)`` is the attention of the OneTrans
mixed causal attention (reference ``MixedCausalAttention.attend_causal_suffix``
``src/model.py:5617-5695``; flash-attn varlen with bottom-right causality over
the packed valid tokens):

* ``qkv [B, Lk, 3*D]``: per token Q | K | V (head ``h`` at columns
  ``h*hd : (h+1)*hd`` of each part);
* the queries are the last ``lq`` tokens; query row ``p`` (token index) sees
  key ``j`` iff ``kstart[b] <= j <= p`` (``j <= p`` only when ``causal``);
* padding is a per-sample prefix (``kstart``), which is how the reference lays
  out valid tokens (valid S tokens at the end of the S block, NS tokens always
  valid), so a query row before ``kstart`` has no visible key and outputs zero;
* ``ktail`` (causal only): the last ``ktail`` tokens see every key and are seen
  by every query -- LONGER's mixed visibility (``mixed_allowed_mask``
  ``src/model.py:1110-1158``: global tokens see everything, recent queries are
  bottom-right causal and see the globals) with the globals placed after the
  sequence instead of before it;
* ``kexcl`` (``<= ktail``): the last ``kexcl`` of those tokens are seen only by
  each other -- LONGER's candidate global tokens, which attend to everything
  while no user global or sequence token attends to them (the reference keeps
  them out of the request-side keys, ``LongerSequenceEncoder.forward``
  ``src/model.py:2036-2296``);
* returns ``[B, lq, D]``.

CUDA: the tcgen05 flash attention in ``csrc/fmha.cu`` (forward saves the
base-2 log-sum-exp; backward writes ``dqkv`` in the input layout). CPU: the
same contract in fp32 PyTorch, also the oracle of the GPU tests.
"""

from __future__ import annotations

import math

import torch

from ._ext import error_word, ext
from ..utils.trace import trace_range

LOG2E = 1.4426950408889634


def suffix_attention_reference(qkv: torch.Tensor, kstart: torch.Tensor, heads: int, lq: int, causal: bool = True,
                               scale: float | None = None, ktail: int = 0, kexcl: int = 0) -> torch.Tensor:
    """fp32 PyTorch definition (differentiable)."""

    B, Lk, W = qkv.shape
    D = W // 3
    hd = D // heads
    scale = scale if scale else 1.0 / math.sqrt(hd)
    x = qkv.float()
    q = x[:, Lk - lq:, :D].reshape(B, lq, heads, hd).transpose(1, 2)
    k = x[:, :, D:2 * D].reshape(B, Lk, heads, hd).transpose(1, 2)
    v = x[:, :, 2 * D:].reshape(B, Lk, heads, hd).transpose(1, 2)
    s = torch.matmul(q, k.transpose(-1, -2)) * scale                   # [B, H, lq, Lk]
    kpos = torch.arange(Lk, device=qkv.device)
    qpos = torch.arange(Lk - lq, Lk, device=qkv.device)
    ks = kstart.to(qkv.device).long().view(B, 1, 1)
    allowed = kpos.view(1, 1, Lk) >= ks
    if causal:
        tail0 = Lk - ktail
        allowed = allowed & ((kpos.view(1, 1, Lk) <= qpos.view(1, lq, 1)) | (kpos.view(1, 1, Lk) >= tail0)
                             | (qpos.view(1, lq, 1) >= tail0))
        excl0 = Lk - kexcl
        allowed = allowed & ((kpos.view(1, 1, Lk) < excl0) | (qpos.view(1, lq, 1) >= excl0))
    allowed = allowed & (qpos.view(1, lq, 1) >= ks)                      # padded queries output zero
    s = s.masked_fill(~allowed.unsqueeze(1), float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.where(allowed.unsqueeze(1), p, torch.zeros_like(p))       # rows without a visible key
    o = torch.matmul(p, v)                                              # [B, H, lq, hd]
    return o.transpose(1, 2).reshape(B, lq, D)


NATIVE_HEAD_DIMS = (8, 16, 32, 64)


def attention_fwd(qkv, ks, out, lse, heads: int, lq: int, causal: bool, ktail: int = 0, kexcl: int = 0) -> None:
    """Native forward of the suffix attention: the tcgen05 flash attention for head width
    32, the CUDA-core kernels (``csrc/attn_simt.cu``) for 8, 16 and 64."""

    hd = qkv.shape[2] // 3 // heads
    if hd == 32:
        ext().fmha_fwd(qkv, ks, out, lse, heads, lq, bool(causal), 0.0, error_word(qkv.device), int(ktail),
                       int(kexcl))
    elif hd in NATIVE_HEAD_DIMS:
        ext().attn_simt_fwd(qkv, ks, out, lse, heads, lq, bool(causal), 0.0, int(ktail), int(kexcl))
    else:
        raise NotImplementedError(f"attention head width {hd}: the native kernels take {NATIVE_HEAD_DIMS}")


def attention_bwd(qkv, ks, out, lse, dout, dqkv, heads: int, lq: int, causal: bool, ktail: int = 0,
                  kexcl: int = 0) -> None:
    hd = qkv.shape[2] // 3 // heads
    dsum = torch.empty(lse.shape, dtype=torch.float32, device=qkv.device)
    if hd == 32:
        dq_acc = torch.empty(out.shape, dtype=torch.float32, device=qkv.device)
        ext().fmha_bwd(qkv, ks, out, lse, dout, dqkv, dq_acc, dsum, heads, lq, bool(causal), 0.0,
                       error_word(qkv.device), int(ktail), int(kexcl))
    elif hd in NATIVE_HEAD_DIMS:
        ext().attn_simt_bwd(qkv, ks, out, lse, dout, dqkv, dsum, heads, lq, bool(causal), 0.0, int(ktail),
                            int(kexcl))
    else:
        raise NotImplementedError(f"attention head width {hd}: the native kernels take {NATIVE_HEAD_DIMS}")


class SuffixAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, kstart, heads, lq, causal, ktail=0, kexcl=0):
        B, Lk, W = qkv.shape
        D = W // 3
        qkv = qkv.contiguous()
        ks = kstart.to(torch.int32).contiguous()
        out = torch.empty(B, lq, D, dtype=torch.bfloat16, device=qkv.device)
        lse = torch.empty(B, heads, lq, dtype=torch.float32, device=qkv.device)
        attention_fwd(qkv, ks, out, lse, heads, lq, causal, ktail, kexcl)
        ctx.save_for_backward(qkv, ks, out, lse)
        ctx.meta = (heads, lq, bool(causal), int(ktail), int(kexcl))
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, ks, out, lse = ctx.saved_tensors
        heads, lq, causal, ktail, kexcl = ctx.meta
        dout = dout.to(torch.bfloat16).contiguous()
        dqkv = torch.empty_like(qkv)
        attention_bwd(qkv, ks, out, lse, dout, dqkv, heads, lq, causal, ktail, kexcl)
        return dqkv, None, None, None, None, None, None


def suffix_attention(qkv: torch.Tensor, kstart: torch.Tensor, heads: int, lq: int, causal: bool = True,
                     ktail: int = 0, kexcl: int = 0) -> torch.Tensor:
    with trace_range("mdl.attention.suffix"):
        if qkv.is_cuda:
            return SuffixAttentionFn.apply(qkv, kstart, heads, lq, causal, ktail, kexcl)
        return suffix_attention_reference(qkv, kstart, heads, lq, causal, ktail=ktail, kexcl=kexcl)


# ----------------------------------------------------------------------------- single-query attention
def single_query_attention_reference(q: torch.Tensor, hist: torch.Tensor, kstart: torch.Tensor,
                                     scale: float) -> torch.Tensor:
    """fp32 definition: per sample and head, ``softmax(scale * q . h_l)`` over the events
    ``l >= kstart[b]`` of ``hist [B, L, N, D]``, weighted sum of ``h_l``; ``q [B, N, D]``;
    a sample without a valid event gives zero."""

    B, L, N, D = hist.shape
    hf = hist.float().permute(0, 2, 1, 3)                                   # [B, N, L, D]
    s = torch.matmul(q.float().unsqueeze(2), hf.transpose(-1, -2)).squeeze(2) * scale   # [B, N, L]
    valid = torch.arange(L, device=hist.device).view(1, 1, L) >= kstart.to(hist.device).long().view(B, 1, 1)
    w = torch.nan_to_num(torch.softmax(s.masked_fill(~valid, float("-inf")), dim=-1)) * valid
    return torch.matmul(w.unsqueeze(2), hf).squeeze(2)


class SingleQueryAttentionFn(torch.autograd.Function):
    """CUDA kernels of ``csrc/sqa.cu``: one warp per (sample, head) streams the bf16 history
    once (online softmax); the backward recomputes the weights from the saved log-sum-exp."""

    @staticmethod
    def forward(ctx, q, hist, kstart, scale):
        q = q.float().contiguous()
        hist = hist.to(torch.bfloat16).contiguous()
        ks = kstart.to(torch.int32).contiguous()
        B, L, N, D = hist.shape
        out = torch.empty(B, N, D, dtype=torch.float32, device=q.device)
        lse = torch.empty(B, N, dtype=torch.float32, device=q.device)
        ext().sqa_fwd(q, hist, ks, out, lse, float(scale))
        ctx.save_for_backward(q, hist, ks, out, lse)
        ctx.scale = float(scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, hist, ks, out, lse = ctx.saved_tensors
        dq = torch.empty_like(q)
        dhist = torch.empty_like(hist)
        ext().sqa_bwd(q, hist, ks, out, lse, dout.float().contiguous(), dq, dhist, ctx.scale)
        return dq, dhist, None, None


def single_query_attention(q: torch.Tensor, hist: torch.Tensor, kstart: torch.Tensor, scale: float) -> torch.Tensor:
    with trace_range("mdl.attention.single_query"):
        if q.is_cuda:
            return SingleQueryAttentionFn.apply(q, hist, kstart, scale)
        return single_query_attention_reference(q, hist, kstart, scale)


def shared_query_attention_reference(q: torch.Tensor, hist: torch.Tensor, kstart: torch.Tensor,
                                     scale: float) -> torch.Tensor:
    """fp32 definition: for sample ``b`` and query ``g`` of ``q [B, G, D]``,
    ``softmax(scale * q_g . h_l)`` over the events ``l >= kstart[b]`` of the shared history
    ``hist [B, L, D]`` (keys = values = the rows), weighted sum of ``h_l``; a sample without a
    valid event gives zero."""

    B, L, D = hist.shape
    hf = hist.float()
    s = torch.matmul(q.float(), hf.transpose(-1, -2)) * scale                       # [B, G, L]
    valid = torch.arange(L, device=hist.device).view(1, 1, L) >= kstart.to(hist.device).long().view(B, 1, 1)
    w = torch.nan_to_num(torch.softmax(s.masked_fill(~valid, float("-inf")), dim=-1)) * valid
    return torch.matmul(w, hf)


class SharedQueryAttentionFn(torch.autograd.Function):
    """CUDA kernels ``sqa_shared_*`` of ``csrc/sqa.cu``: one warp per sample runs all G queries
    over the bf16 history, which is read once for all of them; the backward recomputes the
    weights from the saved log-sum-exp and writes the history gradient summed over the queries."""

    @staticmethod
    def forward(ctx, q, hist, kstart, scale):
        q = q.float().contiguous()
        hist = hist.to(torch.bfloat16).contiguous()
        ks = kstart.to(torch.int32).contiguous()
        B, G, D = q.shape
        out = torch.empty(B, G, D, dtype=torch.float32, device=q.device)
        lse = torch.empty(B, G, dtype=torch.float32, device=q.device)
        ext().sqa_shared_fwd(q, hist, ks, out, lse, float(scale))
        ctx.save_for_backward(q, hist, ks, out, lse)
        ctx.scale = float(scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, hist, ks, out, lse = ctx.saved_tensors
        dq = torch.empty_like(q)
        dhist = torch.empty_like(hist)
        ext().sqa_shared_bwd(q, hist, ks, out, lse, dout.float().contiguous(), dq, dhist, ctx.scale)
        return dq, dhist, None, None


def shared_query_supported(groups: int, width: int) -> bool:
    """Shapes of the native kernels: ``width`` even and at most 256, ``groups`` at most 8,
    and (groups rounded up to 2, 4 or 8) x (ceil(width / 64) rounded up to 1, 2 or 4) <= 16."""

    if groups < 1 or groups > 8 or width < 1 or width > 256 or width % 2:
        return False
    g = 2 if groups <= 2 else (4 if groups <= 4 else 8)
    p = 1 if width <= 64 else (2 if width <= 128 else 4)
    return g * p <= 16


def shared_query_attention(q: torch.Tensor, hist: torch.Tensor, kstart: torch.Tensor, scale: float) -> torch.Tensor:
    """``q [B, G, D]`` over ``hist [B, L, D]`` with prefix padding ``kstart [B]`` -> ``[B, G, D]``
    fp32 (CUDA: the native kernels; CPU: the fp32 definition). CUDA shapes outside
    ``shared_query_supported`` raise."""

    with trace_range("mdl.attention.shared_query"):
        if q.is_cuda:
            if not shared_query_supported(q.shape[1], q.shape[2]):
                raise NotImplementedError(f"shared-history attention: {q.shape[1]} queries of width {q.shape[2]}")
            return SharedQueryAttentionFn.apply(q, hist, kstart, scale)
        return shared_query_attention_reference(q, hist, kstart, scale)
