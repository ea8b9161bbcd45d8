"""LONGER: long-sequence encoder (cross block with recent queries + global tokens, self blocks).

Reference: ``LongerSequenceAttentionBlock`` ``src/model.py:1033-1414``,
``LongerTokenMerger`` ``:1417-1517``, ``LongerSequenceEncoder`` ``:1520-2296``,
``LongerModel`` ``:6563-6612``.

* Sequence tokens: each event's field embeddings (one lookup per field, rows =
  events) through a ``Linear -> GELU -> Linear`` step projector to ``d``
  (``longer_dim``). The token merger groups ``m`` (``longer_token_merge``)
  consecutive events (left-padded to a multiple of ``m``), runs
  ``longer_inner_layers`` blocks at width ``d`` inside each group, zeroes padding
  slots and lays each group's slots side by side: ``ceil(L / m)`` tokens of width
  ``m * d``, the width of every later block, global token and output token.
* Global tokens: candidate globals from the sequence's ``target_inputs`` and user
  globals from ``longer_user_global_inputs``, each group concatenated and
  projected by an MLP to ``count * d``.
* Cross block: queries = the global tokens + the last ``R`` (``longer_query_tokens``)
  sequence tokens, keys = globals + all sequence tokens. User / CLS globals see
  every valid key except the candidate globals; recent queries are bottom-right
  causal and see the user / CLS globals (``mixed_allowed_mask`` ``:1110-1158``);
  candidate globals see every valid key and are seen by no other query, so every
  output but theirs is independent of the candidate (the reference's request-side
  / candidate-side split, ``:1706-1730, 2036-2296``). Self blocks: the same
  visibility over the cross block's ``R + G`` outputs. Every block: pre-LayerNorm
  queries and keys (separate norms), Q and fused K/V projections, attention,
  output projection, residual, pre-LayerNorm GELU FFN, residual.
* Output: the ``G + R`` tokens flattened (``longer_output: full``).

Layout. A sample's tokens are ``[sequence (left-padded); user; CLS; candidate
globals]`` -- the globals after the sequence, so the visibility is the causal
query suffix plus ``ktail = G`` trailing global tokens, of which the last
``kexcl = Gc`` are hidden from the others, in the tcgen05 flash attention
(``ops/attention.py``), and padding stays a per-sample prefix. The query order
inside the model is ``[recent; globals]``; ``reference_order`` maps it to the
reference's ``[globals; recent]``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ..config.schema import AppConfig
from ..ops._ext import error_word, ext
from ..ops.attention import NATIVE_HEAD_DIMS, attention_bwd, attention_fwd, suffix_attention_reference
from ..ops.gemm import ACT_ADD, ACT_DMUL, ACT_GELU_GRAD, bgemm
from ..ops.layers import _grad, _kaiming_uniform_, _shadow, gemm_param
from .features import FeatureEncoder
from .heads import TaskHeads
from .mixformer import MixFormerHead


def _off(t: torch.Tensor, n: int) -> torch.Tensor:
    return t.view(-1)[n:]


def _ln_fwd(x2d, w, b, eps):
    rows, D = x2d.shape
    out = torch.empty_like(x2d)
    mean = torch.empty(rows, dtype=torch.float32, device=x2d.device)
    rstd = torch.empty_like(mean)
    ext().ln_fwd(x2d, None, w, b, out, mean, rstd, rows, 1, D, False, eps)
    return out, mean, rstd


def _ln_bwd(dy2d, x2d, mean, rstd, w, b, res=None):
    """LayerNorm backward; ``res`` (same shape, bf16) is added to the input gradient in the
    same pass (a residual branch's gradient)."""

    rows, D = x2d.shape
    C = ext()
    grid = C.ln_bwd_grid(rows)
    partials = torch.empty(grid, 2 * D, dtype=torch.float32, device=x2d.device)
    dx = torch.empty_like(x2d)
    C.ln_bwd(dy2d.contiguous(), None, 1.0, x2d, None, mean, rstd, w, dx, None, partials, _grad(w), _grad(b), rows, 1,
             D, False, grid, None if res is None else res.contiguous())
    return dx


class LongerBlockFn(torch.autograd.Function):
    """One LONGER attention block on the CUDA path: ``X [B, Lk, d] -> Y [B, Lq, d]``
    (queries are the last ``Lq`` tokens)."""

    @staticmethod
    def forward(ctx, X, kstart, blk, Lq, heads, causal, ktail, kexcl=0):
        B, Lk, D = X.shape
        Hd = blk.hidden_dim
        dev = X.device
        eps = blk.eps
        X = X.contiguous()
        xk, mean_k, rstd_k = _ln_fwd(X.view(B * Lk, D), blk.lnk_w, blk.lnk_b, eps)
        xq_in = X[:, Lk - Lq:].contiguous().view(B * Lq, D)
        xq, mean_q, rstd_q = _ln_fwd(xq_in, blk.lnq_w, blk.lnq_b, eps)
        qkv = torch.empty(B, Lk, 3 * D, dtype=torch.bfloat16, device=dev)
        r0 = max(0, Lk - 128 * ((Lq + 127) // 128))
        if Lk - Lq > r0:  # Q of rows in the first query tile that are not queries must be finite
            qkv[:, r0:Lk - Lq, :D].zero_()
        if Lq == Lk:  # every token is a query: one flat product instead of B tiny ones
            bgemm(xq, _shadow(blk.wq), qkv, M=B * Lk, N=D, K=D, lda=D, ldb=D, ldc=3 * D, bias=blk.bq)
        else:
            bgemm(xq, _shadow(blk.wq), _off(qkv, (Lk - Lq) * 3 * D), M=Lq, N=D, K=D, G=B, lda=D, gsA=Lq * D, ldb=D,
                  gsB=0, ldc=3 * D, gsC=Lk * 3 * D, bias=blk.bq, gs_bias=0)
        bgemm(xk, _shadow(blk.wkv), _off(qkv, D), M=B * Lk, N=2 * D, K=D, lda=D, ldb=D, ldc=3 * D, bias=blk.bkv)
        ks = kstart.to(torch.int32).contiguous()
        att = torch.empty(B, Lq, D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(B, heads, Lq, dtype=torch.float32, device=dev)
        attention_fwd(qkv, ks, att, lse, heads, Lq, bool(causal), int(ktail), int(kexcl))
        h = torch.empty(B, Lq, D, dtype=torch.bfloat16, device=dev)
        if Lq == Lk:
            bgemm(att, _shadow(blk.wo), h, M=B * Lq, N=D, K=D, lda=D, ldb=D, ldc=D, bias=blk.bo, aux=X, ld_aux=D,
                  act=ACT_ADD)
        else:
            bgemm(att, _shadow(blk.wo), h, M=Lq, N=D, K=D, G=B, lda=D, gsA=Lq * D, ldb=D, gsB=0, ldc=D, gsC=Lq * D,
                  bias=blk.bo, aux=_off(X, (Lk - Lq) * D), ld_aux=D, gs_aux=Lk * D, act=ACT_ADD)
        hn, mean_f, rstd_f = _ln_fwd(h.view(B * Lq, D), blk.lnf_w, blk.lnf_b, eps)
        ug = torch.empty(B * Lq, Hd, dtype=torch.bfloat16, device=dev)
        u = torch.empty_like(ug)
        bgemm(hn, _shadow(blk.w1), ug, M=B * Lq, N=Hd, K=D, lda=D, ldb=D, ldc=Hd, out2=u, bias=blk.b1,
              act=ACT_GELU_GRAD)
        Y = torch.empty(B, Lq, D, dtype=torch.bfloat16, device=dev)
        bgemm(u, _shadow(blk.w2), Y, M=B * Lq, N=D, K=Hd, lda=Hd, ldb=Hd, ldc=D, bias=blk.b2, aux=h, ld_aux=D,
              act=ACT_ADD)
        ctx.save_for_backward(X, xk, mean_k, rstd_k, xq_in, xq, mean_q, rstd_q, qkv, ks, att, lse, h, hn, mean_f,
                              rstd_f, ug, u)
        ctx.meta = (blk, Lq, heads, bool(causal), int(ktail), int(kexcl))
        return Y

    @staticmethod
    def backward(ctx, dY):
        (X, xk, mean_k, rstd_k, xq_in, xq, mean_q, rstd_q, qkv, ks, att, lse, h, hn, mean_f, rstd_f, ug,
         u) = ctx.saved_tensors
        blk, Lq, heads, causal, ktail, kexcl = ctx.meta
        B, Lk, D = X.shape
        Hd = blk.hidden_dim
        dev = X.device
        C = ext()
        dY = dY.to(torch.bfloat16).contiguous().view(B * Lq, D)
        # FFN
        du = torch.empty(B * Lq, Hd, dtype=torch.bfloat16, device=dev)
        bgemm(dY, _shadow(blk.w2), du, M=B * Lq, N=Hd, K=D, lda=D, ldb=Hd, b_mn=True, ldc=Hd, aux=ug, ld_aux=Hd,
              act=ACT_DMUL, colsum=_grad(blk.b1))
        bgemm(dY, u, _grad(blk.w2), M=D, N=Hd, K=B * Lq, lda=D, a_mn=True, ldb=Hd, b_mn=True, ldc=Hd, accumulate=True)
        C.colsum(dY, _grad(blk.b2), 1, B * Lq, D, D, 0, 1.0)
        dhn = torch.empty(B * Lq, D, dtype=torch.bfloat16, device=dev)
        bgemm(du, _shadow(blk.w1), dhn, M=B * Lq, N=D, K=Hd, lda=Hd, ldb=D, b_mn=True, ldc=D)
        bgemm(du, hn, _grad(blk.w1), M=Hd, N=D, K=B * Lq, lda=Hd, a_mn=True, ldb=D, b_mn=True, ldc=D, accumulate=True)
        del du
        dh = _ln_bwd(dhn, h.view(B * Lq, D), mean_f, rstd_f, blk.lnf_w, blk.lnf_b, res=dY)
        # output projection
        datt = torch.empty_like(dh)
        bgemm(dh, _shadow(blk.wo), datt, M=B * Lq, N=D, K=D, lda=D, ldb=D, b_mn=True, ldc=D)
        bgemm(dh, att, _grad(blk.wo), M=D, N=D, K=B * Lq, lda=D, a_mn=True, ldb=D, b_mn=True, ldc=D, accumulate=True)
        C.colsum(dh, _grad(blk.bo), 1, B * Lq, D, D, 0, 1.0)
        # attention
        dqkv = torch.empty_like(qkv)
        attention_bwd(qkv, ks, att, lse, datt.view(B, Lq, D), dqkv, heads, Lq, causal, ktail, kexcl)
        del datt
        # Q projection (query rows only)
        dq_rows = _off(dqkv, (Lk - Lq) * 3 * D)
        dxq = torch.empty(B * Lq, D, dtype=torch.bfloat16, device=dev)
        if Lq == Lk:
            bgemm(dq_rows, _shadow(blk.wq), dxq, M=B * Lq, N=D, K=D, lda=3 * D, ldb=D, b_mn=True, ldc=D)
            bgemm(dq_rows, xq, _grad(blk.wq), M=D, N=D, K=B * Lq, lda=3 * D, a_mn=True, ldb=D, b_mn=True, ldc=D,
                  accumulate=True)
            C.colsum(dq_rows, _grad(blk.bq), 1, B * Lq, D, 3 * D, 0, 1.0)
        else:
            bgemm(dq_rows, _shadow(blk.wq), dxq, M=Lq, N=D, K=D, G=B, lda=3 * D, gsA=Lk * 3 * D, ldb=D, gsB=0,
                  b_mn=True, ldc=D, gsC=Lq * D)
            bgemm(dq_rows, xq, _grad(blk.wq), M=D, N=D, K=Lq, lda=3 * D, a_mn=True, ldb=D, b_mn=True, ldc=D,
                  accumulate=True, kg=B, ksA=Lk * 3 * D, ksB=Lq * D)
            C.colsum(dq_rows, _grad(blk.bq), B, Lq, D, 3 * D, Lk * 3 * D, 1.0, 0)
        # K/V projection (all rows)
        dkv = _off(dqkv, D)
        dxk = torch.empty(B * Lk, D, dtype=torch.bfloat16, device=dev)
        bgemm(dkv, _shadow(blk.wkv), dxk, M=B * Lk, N=D, K=2 * D, lda=3 * D, ldb=D, b_mn=True, ldc=D)
        bgemm(dkv, xk, _grad(blk.wkv), M=2 * D, N=D, K=B * Lk, lda=3 * D, a_mn=True, ldb=D, b_mn=True, ldc=D,
              accumulate=True)
        C.colsum(dkv, _grad(blk.bkv), 1, B * Lk, 2 * D, 3 * D, 0, 1.0)
        del dqkv
        dX = _ln_bwd(dxk, X.view(B * Lk, D), mean_k, rstd_k, blk.lnk_w, blk.lnk_b).view(B, Lk, D)
        dxq_in = _ln_bwd(dxq, xq_in, mean_q, rstd_q, blk.lnq_w, blk.lnq_b, res=dh).view(B, Lq, D)
        dX[:, Lk - Lq:] += dxq_in
        return dX, None, None, None, None, None, None, None


class LongerBlock(nn.Module):
    """Parameters of ``LongerSequenceAttentionBlock`` (names follow the reference)."""

    def __init__(self, token_dim: int, hidden_dim: int, device=None) -> None:
        super().__init__()
        D, H = token_dim, hidden_dim
        self.token_dim, self.hidden_dim, self.eps = D, H, 1e-5
        self.lnq_w = nn.Parameter(torch.ones(D, device=device))
        self.lnq_b = nn.Parameter(torch.zeros(D, device=device))
        self.lnk_w = nn.Parameter(torch.ones(D, device=device))
        self.lnk_b = nn.Parameter(torch.zeros(D, device=device))
        self.wq = gemm_param(torch.empty(D, D, device=device))
        self.bq = nn.Parameter(torch.empty(D, device=device))
        self.wkv = gemm_param(torch.empty(2 * D, D, device=device))
        self.bkv = nn.Parameter(torch.empty(2 * D, device=device))
        self.wo = gemm_param(torch.empty(D, D, device=device))
        self.bo = nn.Parameter(torch.empty(D, device=device))
        self.lnf_w = nn.Parameter(torch.ones(D, device=device))
        self.lnf_b = nn.Parameter(torch.zeros(D, device=device))
        self.w1 = gemm_param(torch.empty(H, D, device=device))
        self.b1 = nn.Parameter(torch.empty(H, device=device))
        self.w2 = gemm_param(torch.empty(D, H, device=device))
        self.b2 = nn.Parameter(torch.empty(D, device=device))
        for w, b, fan in ((self.wq, self.bq, D), (self.wkv, self.bkv, D), (self.wo, self.bo, D), (self.w1, self.b1, D),
                          (self.w2, self.b2, H)):
            _kaiming_uniform_(w.data, fan)
            _kaiming_uniform_(b.data, fan)

    def forward_reference(self, X, kstart, Lq, heads, causal, ktail, kexcl=0):
        B, Lk, D = X.shape
        X = X.float()
        xk = F.layer_norm(X, (D,), self.lnk_w, self.lnk_b, self.eps)
        xq = F.layer_norm(X[:, Lk - Lq:], (D,), self.lnq_w, self.lnq_b, self.eps)
        q = xq @ self.wq.t() + self.bq
        kv = xk @ self.wkv.t() + self.bkv
        qfull = torch.cat([torch.zeros(B, Lk - Lq, D, device=X.device), q], dim=1)
        att = suffix_attention_reference(torch.cat([qfull, kv], dim=-1), kstart, heads, Lq, causal, ktail=ktail,
                                         kexcl=kexcl)
        h = X[:, Lk - Lq:] + att @ self.wo.t() + self.bo
        hn = F.layer_norm(h, (D,), self.lnf_w, self.lnf_b, self.eps)
        return h + F.gelu(hn @ self.w1.t() + self.b1) @ self.w2.t() + self.b2

    def request_kv(self, X: torch.Tensor) -> torch.Tensor:
        """fp32 K | V ``[B, Lk, 2d]`` of request-side tokens (cached for candidate queries)."""

        xk = F.layer_norm(X.float(), (self.token_dim,), self.lnk_w, self.lnk_b, self.eps)
        return xk @ self.wkv.float().t() + self.bkv

    def candidate_forward(self, C: torch.Tensor, kv_req: torch.Tensor, kstart: torch.Tensor,
                          heads: int) -> torch.Tensor:
        """Candidate global tokens ``C [B, Gc, d]`` through the block: they attend to the
        cached request-side keys ``kv_req [B, Lk, 2d]`` (key ``j`` valid from ``kstart``)
        and to every candidate token; no request-side token sees them."""

        B, Gc, D = C.shape
        X = C.float()
        hd = D // heads
        xq = F.layer_norm(X, (D,), self.lnq_w, self.lnq_b, self.eps)
        q = (xq @ self.wq.float().t() + self.bq).view(B, Gc, heads, hd).transpose(1, 2)
        kv = torch.cat([kv_req.float(), self.request_kv(X)], dim=1)                     # [B, Lk + Gc, 2D]
        Lk = kv.shape[1]
        k = kv[..., :D].reshape(B, Lk, heads, hd).transpose(1, 2)
        v = kv[..., D:].reshape(B, Lk, heads, hd).transpose(1, 2)
        valid = torch.arange(Lk, device=X.device).view(1, Lk) >= kstart.to(X.device).long().view(B, 1)
        valid[:, Lk - Gc:] = True
        s = (q @ k.transpose(-1, -2)) / (hd ** 0.5)
        s = s.masked_fill(~valid.view(B, 1, 1, Lk), float("-inf"))
        att = (torch.softmax(s, dim=-1) @ v).transpose(1, 2).reshape(B, Gc, D)
        h = X + att @ self.wo.float().t() + self.bo
        hn = F.layer_norm(h, (D,), self.lnf_w, self.lnf_b, self.eps)
        return h + F.gelu(hn @ self.w1.float().t() + self.b1) @ self.w2.float().t() + self.b2

    def forward(self, X, kstart, Lq, heads, causal, ktail, native: bool, kexcl: int = 0):
        if native:
            return LongerBlockFn.apply(X, kstart, self, Lq, heads, causal, ktail, kexcl)
        return self.forward_reference(X, kstart, Lq, heads, causal, ktail, kexcl)

    def reference_state_dict(self, prefix: str) -> dict[str, torch.Tensor]:
        sd = {prefix + "query_norm.weight": self.lnq_w, prefix + "query_norm.bias": self.lnq_b,
              prefix + "key_norm.weight": self.lnk_w, prefix + "key_norm.bias": self.lnk_b,
              prefix + "query_projection.weight": self.wq, prefix + "query_projection.bias": self.bq,
              prefix + "kv_projection.weight": self.wkv, prefix + "kv_projection.bias": self.bkv,
              prefix + "output_projection.weight": self.wo, prefix + "output_projection.bias": self.bo,
              prefix + "ffn_norm.weight": self.lnf_w, prefix + "ffn_norm.bias": self.lnf_b,
              prefix + "ffn.0.weight": self.w1, prefix + "ffn.0.bias": self.b1,
              prefix + "ffn.3.weight": self.w2, prefix + "ffn.3.bias": self.b2}
        return {k: v.detach().clone() for k, v in sd.items()}


class _MLP(nn.Module):
    """``Linear -> GELU -> Linear`` (reference ``_projection_mlp`` ``src/model.py:753-760``); weights
    stored with a leading group axis of 1 so the CUDA path is the grouped per-token FFN."""

    def __init__(self, k_in: int, k_log: int, hidden: int, out: int, device=None) -> None:
        super().__init__()
        self.k_in, self.k_log, self.hidden, self.out_dim = k_in, k_log, hidden, out
        self.w1 = gemm_param(torch.zeros(1, hidden, k_in, device=device))
        self.b1 = nn.Parameter(torch.empty(1, hidden, device=device))
        self.w2 = gemm_param(torch.empty(1, out, hidden, device=device))
        self.b2 = nn.Parameter(torch.empty(1, out, device=device))
        _kaiming_uniform_(self.w1.data[0, :, :k_log], k_log)  # padded input columns stay zero
        _kaiming_uniform_(self.b1.data, k_log)
        _kaiming_uniform_(self.w2.data, hidden)
        _kaiming_uniform_(self.b2.data, hidden)

    def forward(self, x: torch.Tensor, native: bool) -> torch.Tensor:
        if native:
            from ..ops.layers import PerTokenFFNFn

            y = PerTokenFFNFn.apply(x.to(torch.bfloat16).view(x.shape[0], 1, self.k_in), self.w1, self.b1, self.w2,
                                    self.b2, False)
            return y.view(x.shape[0], self.out_dim)
        h = F.gelu(x.float()[:, :self.k_log] @ self.w1[0, :, :self.k_log].t() + self.b1[0])
        return h @ self.w2[0].t() + self.b2[0]


class LongerEncoder(nn.Module):
    """Sequence tokens + global tokens -> cross block -> self blocks -> ``[B, R + G, d]``.

    Global tokens, in order: user globals (``longer_user_global_inputs``), ``extra_globals``
    learned tokens passed to ``forward`` (the CLS tokens of a feature-encoder LONGER),
    candidate globals (``target_inputs``). With ``time_delta = (c0, c1)`` (the event
    columns of ``time_delta_field``) a learned position embedding is added to the other
    event columns before the step projector (reference ``_longer_sequence_projector_inputs``
    ``src/model.py:3393-3436``). The tcgen05 attention kernels take head_dim 32; other
    head widths run the PyTorch definition (``runtime.kernel_backend: torch``)."""

    def __init__(self, config: AppConfig, seq, encoder: FeatureEncoder, target_plan, user_plan, device=None,
                 extra_globals: int = 0, time_delta: tuple[int, int] | None = None) -> None:
        super().__init__()
        m = config.model
        Din = int(seq.longer_dim)
        self.merge = int(seq.longer_token_merge)
        if self.merge < 1 or int(seq.longer_inner_layers) < 0:
            raise ValueError(f"LONGER sequence {seq.name!r}: longer_token_merge >= 1 and longer_inner_layers >= 0")
        D = Din * self.merge           # merged token width: every block after the merger runs at it
        self.Din, self.D = Din, D
        heads = seq.longer_num_heads  # reference SequenceConfig.resolved_longer_num_heads
        if heads is None:
            heads = int(m.num_heads) if Din % int(m.num_heads) == 0 else next(h for h in (8, 4, 2, 1) if Din % h == 0)
        self.heads = int(heads)
        if Din % self.heads:
            raise ValueError(f"LONGER sequence {seq.name!r}: longer_dim {Din} not divisible by {self.heads} heads")
        self.head_dim = D // self.heads
        hidden_in = int(seq.longer_hidden_dim or 4 * Din)
        hidden = hidden_in * self.merge
        self.R = int(seq.longer_query_tokens)
        self.L = int(seq.max_length)
        plan = encoder.seq_plans[seq.name]
        self.step = _MLP(plan.out_ld, plan.out_width, hidden_in, Din, device=device)
        # token merger (reference LongerTokenMerger): inner blocks at the event width over
        # each group of `merge` consecutive events, then each group's slots side by side
        self.inner = nn.ModuleList(LongerBlock(Din, hidden_in, device=device)
                                   for _ in range(int(seq.longer_inner_layers)))
        self.Gu = int(seq.longer_user_global_tokens) if user_plan is not None else 0
        self.Gx = int(extra_globals)
        cand = seq.longer_candidate_global_tokens
        if target_plan is None:
            self.Gc = 0
        elif cand is not None:
            self.Gc = int(cand)
        elif extra_globals or self.Gu:
            self.Gc = max(0, int(seq.rankmixer_summary_tokens) - self.Gu - self.Gx)
        else:
            self.Gc = 1
        self.G = self.Gu + self.Gx + self.Gc
        self.cand_mlp = (_MLP(target_plan.out_ld, target_plan.out_width, hidden, self.Gc * D, device=device)
                         if self.Gc else None)
        self.user_mlp = (_MLP(user_plan.out_ld, user_plan.out_width, hidden, self.Gu * D, device=device)
                         if self.Gu else None)
        self.cross = LongerBlock(D, hidden, device=device)
        self.selfs = nn.ModuleList(LongerBlock(D, hidden, device=device) for _ in range(int(seq.longer_self_layers)))
        self.output_tokens = self.R + self.G
        self.pos = None
        self.pos_cols = 0
        if time_delta is not None:
            c0, c1 = time_delta
            if c1 != plan.out_width:
                raise NotImplementedError("LONGER positions expect the time delta as the last event columns")
            self.pos_cols = c0
            self.pos = nn.Parameter(torch.randn(self.L, c0, device=device) * float(m.init_std))
            self._pad_cols = plan.out_ld - c0

    def merge_tokens(self, tokens: torch.Tensor, kst: torch.Tensor, native: bool):
        """``[B, L, d]`` event tokens with ``kst`` leading padding events -> ``[B, ceil(L/m), m*d]``
        merged tokens and their padding count (reference ``LongerTokenMerger.forward``
        ``src/model.py:1489-1517``): left-pad to a multiple of ``m``, run the inner blocks
        over each group of ``m`` tokens (full attention among the group's valid tokens),
        zero the padding slots, lay each group's slots side by side."""

        m = self.merge
        B, L, Din = tokens.shape
        pad = (-L) % m
        if pad:
            tokens = F.pad(tokens, (0, 0, pad, 0))
            kst = kst + pad
        Lp = L + pad
        ng = Lp // m
        if len(self.inner):
            h = tokens.reshape(B * ng, m, Din)
            starts = torch.arange(ng, device=kst.device, dtype=kst.dtype) * m
            gk = (kst.view(B, 1) - starts.view(1, ng)).clamp(0, m).reshape(B * ng).to(torch.int32)
            for blk in self.inner:
                h = blk(h, gk, m, self.heads, False, 0, native)
            tokens = h.reshape(B, Lp, Din)
        valid = torch.arange(Lp, device=tokens.device).view(1, Lp) >= kst.view(B, 1)
        tokens = tokens * valid.unsqueeze(-1).to(tokens.dtype)
        return tokens.reshape(B, ng, m * Din), torch.div(kst, m, rounding_mode="floor")

    def project(self, seq_in, lengths, native: bool) -> torch.Tensor:
        """Event tokens ``[rows, L, longer_dim]`` (positions added to the event values first)."""

        rows, L = lengths.shape[0], self.L
        if self.pos is not None:
            from .sequence_encoders import positions

            pe = self.pos[positions(lengths, L)].view(rows * L, self.pos_cols)
            pe = F.pad(pe, (0, self._pad_cols)) if self._pad_cols else pe
            seq_in = seq_in + pe.to(seq_in.dtype)
        return self.step(seq_in, native).view(rows, L, self.Din)

    def forward(self, seq_in, lengths, target_in, user_in, native: bool, cls_tokens=None,
                tokens=None, summary_only: bool = False, user_tokens=None, cand_tokens=None) -> torch.Tensor:
        """``tokens``: event tokens already projected (``project``), else ``seq_in`` is projected here.
        ``summary_only``: return only the ``G`` global tokens; the last block then runs only
        their queries (reference ``forward_request_summary`` ``src/model.py:1906-2004``: the
        recent outputs of the last layer cannot reach the summary)."""

        B, L, D, R, G = lengths.shape[0], self.L, self.D, self.R, self.G
        if native and (self.head_dim not in NATIVE_HEAD_DIMS
                       or (len(self.inner) and self.Din // self.heads not in NATIVE_HEAD_DIMS)):
            raise NotImplementedError(f"LONGER head_dim {self.head_dim} (inner {self.Din // self.heads}): the native "
                                      f"attention kernels take {NATIVE_HEAD_DIMS} (or set runtime.kernel_backend: "
                                      "torch)")
        if tokens is None:
            tokens = self.project(seq_in, lengths, native)
        kst = (L - lengths.clamp(0, L)).to(torch.int32)
        if self.merge > 1 or len(self.inner):
            tokens, kst = self.merge_tokens(tokens, kst, native)
            L = tokens.shape[1]
        if L < R:  # fewer (merged) tokens than recent queries: left-pad, the padding is masked
            tokens = F.pad(tokens, (0, 0, R - L, 0))
            kst = kst + (R - L)
            L = R
        parts = [tokens]
        # user_tokens / cand_tokens: global tokens given directly ([B, Gu, D] / [B, Gc, D])
        # instead of projected from user_in / target_in
        if self.Gu:
            parts.append(user_tokens.to(tokens.dtype) if user_tokens is not None
                         else self.user_mlp(user_in, native).view(B, self.Gu, D))
        if self.Gx:
            if cls_tokens is None:
                raise ValueError("LONGER encoder built with extra global tokens needs cls_tokens")
            parts.append(cls_tokens.to(tokens.dtype).expand(B, -1, -1))
        if self.Gc:
            parts.append(cand_tokens.to(tokens.dtype) if cand_tokens is not None
                         else self.cand_mlp(target_in, native).view(B, self.Gc, D))
        X = torch.cat(parts, dim=1) if len(parts) > 1 else tokens
        # [B, R + G, D]: [recent; globals]. Recent queries: bottom-right causal; user / CLS globals:
        # every valid key; the candidate globals (last Gc) are seen by nobody else, so every
        # output except theirs is candidate-independent (reference LongerSequenceEncoder: the
        # request-side keys exclude the candidate globals, src/model.py:1706-1730, 2036-2296)
        nblk = 1 + len(self.selfs)
        summary_only = summary_only and G > 0
        lq = G if (summary_only and nblk == 1) else R + G
        X = self.cross(X, kst, lq, self.heads, True, G, native, kexcl=self.Gc)
        kst = (kst - (L - R)).clamp(min=0)
        # recent rows of padding (sequences shorter than R) are zeroed after every block,
        # as the reference masks its recent outputs (src/model.py:1782-1785, 1874-1877)
        keep = self._recent_keep(kst, R, G, X)
        if keep is not None and X.shape[1] == R + G:
            X = X * keep
        for i, blk in enumerate(self.selfs):
            # self blocks: the same visibility over [recent; globals] (reference mixed mask
            # over [user; recent], candidates over everything)
            lq = G if (summary_only and i == nblk - 2) else R + G
            X = blk(X, kst, lq, self.heads, True, G, native, kexcl=self.Gc)
            if keep is not None and X.shape[1] == R + G:
                X = X * keep
        return X

    @staticmethod
    def _recent_keep(kst, R, G, X):
        """``[B, R + G, 1]`` row mask (0 for padded recent rows), or None when no sample is
        shorter than ``R`` (a host-side check is avoided: the mask is always applied when
        any padding row can exist, i.e. kst > 0 is possible)."""

        if R == 0:
            return None
        rows = torch.arange(R + G, device=X.device).view(1, -1)
        keep = (rows >= kst.to(X.device).view(-1, 1)) | (rows >= R)
        return keep.unsqueeze(-1).to(X.dtype)

    def _request_tokens(self, tokens, lengths, user_in, cls_tokens, native: bool):
        """Request-side rows ``[sequence; user; CLS]`` and their padding count."""

        B, L, R = lengths.shape[0], self.L, self.R
        kst = (L - lengths.clamp(0, L)).to(torch.int32)
        if self.merge > 1 or len(self.inner):
            tokens, kst = self.merge_tokens(tokens, kst, native)
            L = tokens.shape[1]
        if L < R:
            tokens = F.pad(tokens, (0, 0, R - L, 0))
            kst = kst + (R - L)
            L = R
        parts = [tokens.float()]
        if self.Gu:
            parts.append(self.user_mlp(user_in, native).float().view(B, self.Gu, self.D))
        if self.Gx:
            if cls_tokens is None:
                raise ValueError("LONGER encoder built with extra global tokens needs cls_tokens")
            parts.append(cls_tokens.float().expand(B, -1, -1))
        return torch.cat(parts, dim=1), kst, L

    @torch.no_grad()
    def request_cache(self, lengths, user_in=None, *, seq_in=None, tokens=None, cls_tokens=None,
                      native: bool = False) -> dict:
        """Candidate-independent LONGER state of each request (reference
        ``LongerSequenceEncoder.precompute_cache`` ``src/model.py:1632-1800``): per block the
        fp32 K/V of its request-side keys and their padding count, and the request-side
        outputs ``[recent; user; CLS]`` after the last block. Rows are requests."""

        if tokens is None:
            tokens = self.project(seq_in, lengths, native)
        X, kst, L = self._request_tokens(tokens, lengths, user_in, cls_tokens, native)
        R, Gr = self.R, self.Gu + self.Gx
        kv, ksts = [], []
        kv.append(self.cross.request_kv(X))
        ksts.append(kst)
        X = self.cross.forward_reference(X, kst, R + Gr, self.heads, True, Gr)
        kst = (kst - (L - R)).clamp(min=0)
        keep = self._recent_keep(kst, R, Gr, X)
        if keep is not None:
            X = X * keep
        for blk in self.selfs:
            kv.append(blk.request_kv(X))
            ksts.append(kst)
            X = blk.forward_reference(X, kst, R + Gr, self.heads, True, Gr)
            if keep is not None:
                X = X * keep
        return {"kv": kv, "kstart": ksts, "out": X, "lengths": lengths}

    @torch.no_grad()
    def forward_candidates(self, cache: dict, target_in, row_indices=None, native: bool = False) -> torch.Tensor:
        """LONGER output ``[C, R + G, d]`` (order ``[recent; globals]``) of candidate rows whose
        request is ``row_indices[c]`` (identity when None), from a ``request_cache``: only the
        candidate global tokens run through the blocks, against the cached request keys
        (reference ``LongerSequenceEncoder.forward`` with a cache ``src/model.py:2036-2296``)."""

        out = cache["out"]
        ri = (torch.arange(out.shape[0], device=out.device) if row_indices is None
              else row_indices.to(out.device).long())
        req = out.index_select(0, ri)
        if not self.Gc:
            return req
        C = ri.shape[0]
        c = self.cand_mlp(target_in, native).float().view(C, self.Gc, self.D)
        blocks = [self.cross, *self.selfs]
        for blk, kv, kst in zip(blocks, cache["kv"], cache["kstart"]):
            c = blk.candidate_forward(c, kv.index_select(0, ri), kst.index_select(0, ri), self.heads)
        return torch.cat([req, c], dim=1)

    @staticmethod
    def reference_order(X: torch.Tensor, G: int) -> torch.Tensor:
        """``[recent; globals]`` (here) -> ``[globals; recent]`` (reference output order)."""

        return torch.cat([X[:, X.shape[1] - G:], X[:, :X.shape[1] - G]], dim=1)


class LongerModel(nn.Module):
    """``model.name: longer``: one ``encoder: longer`` sequence -> flattened tokens -> heads.

    With ``model.sequence_head: mixformer`` the LONGER tokens are the behaviour
    sequence of a MixFormer head whose ``num_ns_tokens`` feature heads (width
    ``token_dim``) come from the scalar feature-token inputs; the flattened heads
    feed the task heads.
    """

    def __init__(self, config: AppConfig, *, device: torch.device, rank: int = 0, world: int = 1, process_group=None,
                 vocab_sizes: dict[str, int] | None = None, base_seed: int | None = None) -> None:
        super().__init__()
        if len(config.sequences) != 1 or config.sequences[0].encoder != "longer":
            raise ValueError("LongerModel requires exactly one encoder=longer sequence")
        self.config = config
        m = config.model
        seq = config.sequences[0]
        self.seq = seq
        by_name = {f.name: f for f in config.features}
        target = [n for n in seq.target_inputs if n in by_name]
        user = [n for n in seq.longer_user_global_inputs if n in by_name] if seq.longer_user_global_tokens else []
        self.mix = m.sequence_head == "mixformer"
        ns_inputs = [n for n in config.resolved.tokenization.feature_token_inputs if n in by_name] if self.mix else []
        groups = [g for g in (target, user) if g]
        self.encoder = FeatureEncoder(config, device=device, rank=rank, world=world, process_group=process_group,
                                      vocab_sizes=vocab_sizes, input_names=ns_inputs, slice_tokens=1 if ns_inputs else 0,
                                      base_seed=base_seed, sequences=[seq], domain_tokens=groups or None)
        self.has_target, self.has_user = bool(target), bool(user)
        kp = self.encoder.domain_k_pad
        gplan = _SlicePlan(kp, kp)
        self.longer = LongerEncoder(config, seq, self.encoder, gplan if target else None, gplan if user else None,
                                    device=device)
        self.ntask = len(config.task_names)
        if self.mix:
            N, Dh = int(m.num_ns_tokens or 32), int(m.token_dim)
            self.mixer = MixFormerHead(self.encoder.plan.out_ld, self.encoder.plan.out_width, self.longer.D, N, Dh,
                                       int(m.hidden_dim), int(m.hidden_dim), max(1, int(m.num_layers)), device=device)
            out_dim = self.mixer.output_dim
        else:
            out_dim = self.longer.output_tokens * self.longer.D
        self.heads_mod = TaskHeads(self.ntask, out_dim, int(m.task_head_hidden_dim or 4 * self.longer.D),
                                   m.task_head_activation, device=device)

    def gemm_param_names(self) -> set[str]:
        return {n for n, p in self.named_parameters() if getattr(p, "_mdl_gemm", False)}

    def dense_buckets(self) -> list[list[str]]:
        names = [n for n, _ in self.named_parameters()]
        return [[n for n in names if n.startswith("heads_mod.")], [n for n in names if not n.startswith("heads_mod.")]]

    @property
    def store(self):
        return self.encoder.store

    def encode(self, batch):
        """LONGER output ``[B, R + G, d]`` (token order ``[recent; globals]``), the
        event validity of those tokens, the scalar-feature matrix (MixFormer head)."""

        from ..ops.embedding import fused_lookup

        native = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
        anchor = torch.zeros(0, device=batch.ids.device, requires_grad=True)
        from .features import lookup_sequence

        B, L = batch.rows, self.longer.L
        seq_in, lengths = lookup_sequence(self.encoder, batch, self.seq.name, B, L, anchor)
        target_in = user_in = None
        if self.has_target or self.has_user:
            g = fused_lookup(self.store, self.encoder.domain_plan, batch.ids, batch.offsets, batch.dense, B, anchor)
            kp = self.encoder.domain_k_pad
            target_in = g[:, :kp] if self.has_target else None
            user_in = g[:, (kp if self.has_target else 0):][:, :kp] if self.has_user else None
        feat_in = (fused_lookup(self.store, self.encoder.plan, batch.ids, batch.offsets, batch.dense, B, anchor)
                   if self.mix else None)
        X = self.longer(seq_in, lengths, target_in, user_in, native)
        R, G = self.longer.R, self.longer.G
        e = torch.arange(R + G, device=X.device)
        valid = (e.view(1, -1) >= (R - lengths.clamp(0, R)).view(-1, 1)) | (e.view(1, -1) >= R)
        return X, valid, feat_in, native

    @torch.no_grad()
    def precompute_request_cache(self, batch) -> dict:
        """Request-side LONGER state of a batch's requests (reference
        ``LongerModel.precompute_request_cache`` ``src/model.py:6596-6599``): one row per
        request of the sequence payload (``row_indices`` maps candidates to requests; every
        candidate row is its own request without it). User-global inputs are read from each
        request's first candidate row."""

        from ..ops.embedding import fused_lookup
        from .features import lookup_sequence

        native = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
        anchor = torch.zeros(0, device=batch.ids.device)
        seq_in, lengths, ri = lookup_sequence(self.encoder, batch, self.seq.name, batch.rows, self.longer.L, anchor,
                                              expand=False)
        nreq = lengths.numel()
        user_in = None
        if self.has_user:
            g = fused_lookup(self.store, self.encoder.domain_plan, batch.ids, batch.offsets, batch.dense,
                             batch.rows, anchor)
            kp = self.encoder.domain_k_pad
            user_rows = g[:, (kp if self.has_target else 0):][:, :kp]
            if ri is not None:
                first = torch.full((nreq,), -1, dtype=torch.long, device=user_rows.device)
                idx = torch.arange(ri.numel(), device=user_rows.device)
                first.scatter_reduce_(0, ri.long().to(user_rows.device), idx, reduce="amin", include_self=False)
                user_rows = user_rows.index_select(0, first.clamp(min=0))
            user_in = user_rows
        return self.longer.request_cache(lengths.to(seq_in.device), user_in, seq_in=seq_in, native=native)

    @torch.no_grad()
    def forward_with_cache(self, batch, request_cache: dict) -> torch.Tensor:
        """Logits ``[rows, tasks]`` of a candidate batch from a request cache: only the
        candidate global tokens (and the heads) are computed per candidate."""

        from ..ops.embedding import fused_lookup

        if self.mix:
            raise NotImplementedError("request caches cover the flattened LONGER readout (sequence_head: none)")
        native = batch.ids.is_cuda and self.config.runtime.kernel_backend == "native"
        anchor = torch.zeros(0, device=batch.ids.device)
        target_in = None
        if self.has_target:
            g = fused_lookup(self.store, self.encoder.domain_plan, batch.ids, batch.offsets, batch.dense,
                             batch.rows, anchor)
            target_in = g[:, :self.encoder.domain_k_pad]
        ri = (batch.sequences.get(self.seq.name) or {}).get("row_indices")
        X = self.longer.forward_candidates(request_cache, target_in, ri, native)
        readout = LongerEncoder.reference_order(X, self.longer.G).reshape(batch.rows, -1).contiguous()
        scale = torch.ones(self.ntask, device=readout.device)
        return self.heads_mod.forward_shared(readout.float(), None, None, scale)["logits"]

    def forward(self, batch, task_scale: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        X, valid, feat_in, native = self.encode(batch)
        if task_scale is None:
            task_scale = torch.full((self.ntask,), 1.0 / max(1, batch.rows), device=X.device)
        if self.mix:
            readout = self.mixer(feat_in, X, valid, native)
        else:
            readout = LongerEncoder.reference_order(X, self.longer.G).reshape(batch.rows, -1).contiguous()
        return self.heads_mod.forward_shared(readout, batch.labels, batch.label_mask, task_scale)


class _SlicePlan:
    """Width of one global-token input slice (``out_ld`` columns, ``out_width`` used)."""

    def __init__(self, out_ld: int, out_width: int) -> None:
        self.out_ld, self.out_width = out_ld, out_width
