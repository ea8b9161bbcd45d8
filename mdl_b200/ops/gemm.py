"""Batched GEMM with fused epilogues (bias, GELU / GELU-with-derivative / dGELU, ReLU, column sums).

On CUDA tensors this calls the persistent tcgen05 kernel in ``csrc/gemm.cu``;
on CPU tensors it evaluates the same contract with PyTorch in fp32, which is
also the oracle the GPU tests compare against.

Layout contract (elements, not bytes), for group ``g``:

* ``A`` is ``M x K``: K-major ``A[m,k] = a[g*gsA + m*lda + k]``, MN-major
  ``A[m,k] = a[g*gsA + k*lda + m]``.
* ``B`` is ``N x K``: K-major ``B[n,k] = b[g*gsB + n*ldb + k]``, MN-major
  ``B[n,k] = b[g*gsB + k*ldb + n]``.
* ``C`` is ``M x N`` row-major at ``out[g*gsC + m*ldc + n]``.

The reference runs the corresponding products as cuBLAS strided-batched
GEMMs (``src/modules/mlp.py:187-207``, ``src/modules/mlp.py:30-42``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import error_word, ext

ACT_NONE = 0
ACT_GELU = 1
ACT_DGELU = 2
ACT_RELU = 3
ACT_DRELU = 4
ACT_GELU_GRAD = 5  # x = bf16(acc): out = gelu'(x), out2 = gelu(x)  (saves the derivative for the backward)
ACT_DMUL = 6       # out = acc * aux
ACT_ADD = 7        # out = acc + aux (fused residual add)


def _view(t: torch.Tensor, g: int, rows: int, cols: int, gs: int, ld: int, mn_major: bool) -> torch.Tensor:
    if mn_major:
        return t.as_strided((g, rows, cols), (gs, 1, ld))
    return t.as_strided((g, rows, cols), (gs, ld, 1))


def gelu_grad(x: torch.Tensor) -> torch.Tensor:
    """Derivative of the erf GELU."""

    cdf = 0.5 * (1.0 + torch.erf(x * 0.7071067811865476))
    pdf = torch.exp(-0.5 * x * x) * 0.3989422804014327
    return cdf + x * pdf


def bgemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    M: int,
    N: int,
    K: int,
    G: int = 1,
    lda: int,
    gsA: int = 0,
    a_mn: bool = False,
    ldb: int,
    gsB: int = 0,
    b_mn: bool = False,
    ldc: int,
    gsC: int = 0,
    out2: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    gs_bias: int = 0,
    aux: torch.Tensor | None = None,
    ld_aux: int = 0,
    gs_aux: int = 0,
    colsum: torch.Tensor | None = None,
    gs_colsum: int = 0,
    act: int = ACT_NONE,
    alpha: float = 1.0,
    accumulate: bool = False,
    kg: int = 1,
    ksA: int = 0,
    ksB: int = 0,
) -> torch.Tensor:
    """``out[g] = epilogue(alpha * A[g] @ B[g]^T)``; see the module docstring.

    ``gsA == 0`` / ``gsB == 0`` with ``G > 1`` shares that operand across groups;
    ``kg > 1`` (``G == 1``) sums ``kg`` products over K ranges ``ksA`` / ``ksB``
    elements apart.
    """

    if out.is_cuda:
        ext().gemm(
            a, lda, gsA, a_mn, b, ldb, gsB, b_mn, M, N, K, G, out, ldc, gsC,
            out2, bias, gs_bias, aux, ld_aux, gs_aux, colsum, gs_colsum,
            act, float(alpha), accumulate, error_word(out.device), 0, kg, ksA, ksB,
        )
        return out
    if kg > 1:
        av = _view(a, kg, M, K, ksA, lda, a_mn).float()
        bv = _view(b, kg, N, K, ksB, ldb, b_mn).float()
        acc = torch.bmm(av, bv.transpose(1, 2)).sum(0, keepdim=True) * alpha
    else:
        av = _view(a, G, M, K, gsA, lda, a_mn).float()
        bv = _view(b, G, N, K, gsB, ldb, b_mn).float()
        acc = torch.bmm(av, bv.transpose(1, 2)) * alpha
    if bias is not None:
        acc = acc + bias.as_strided((G, 1, N), (gs_bias, 0, 1)).float()
    if act in (ACT_DGELU, ACT_DRELU, ACT_DMUL):
        auxv = aux.as_strided((G, M, N), (gs_aux, ld_aux, 1)).float()
        acc = acc * {ACT_DGELU: gelu_grad, ACT_DRELU: lambda a: (a > 0).float(), ACT_DMUL: lambda a: a}[act](auxv)
    if act == ACT_ADD:
        acc = acc + aux.as_strided((G, M, N), (gs_aux, ld_aux, 1)).float()
    if act == ACT_RELU:
        acc = F.relu(acc)
    outv = out.as_strided((G, M, N), (gsC, ldc, 1))
    if act == ACT_GELU_GRAD:
        x = acc.to(torch.bfloat16).float()
        outv.copy_(gelu_grad(x).to(out.dtype))
        out2.as_strided((G, M, N), (gsC, ldc, 1)).copy_(F.gelu(x).to(out2.dtype))
    elif accumulate:
        outv.copy_(outv.float() + acc)
    else:
        outv.copy_(acc.to(out.dtype))
    if act == ACT_GELU:
        out2.as_strided((G, M, N), (gsC, ldc, 1)).copy_(F.gelu(acc).to(out2.dtype))
    if colsum is not None:
        cs = colsum.as_strided((G, N), (gs_colsum, 1))
        cs.add_(acc.sum(dim=1))
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           act: int = ACT_NONE, out_dtype: torch.dtype = torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``x @ weight^T + bias`` for 2D bf16 ``x [M,K]`` and ``weight [N,K]``.

    With ``act=ACT_GELU`` returns ``(pre, gelu(pre))``; otherwise ``(out, None)``.
    """

    M, K = x.shape
    N = weight.shape[0]
    out = torch.empty(M, N, dtype=out_dtype, device=x.device)
    out2 = torch.empty(M, N, dtype=torch.bfloat16, device=x.device) if act == ACT_GELU else None
    bgemm(x, weight, out, M=M, N=N, K=K, lda=x.stride(0), ldb=weight.stride(0), ldc=N,
          out2=out2, bias=bias, act=act)
    return out, out2
