"""Numerics of the tcgen05 batched GEMM against a plain PyTorch fp32 reference."""

import pytest
import torch

from mdl_b200.ops import gemm as G


@pytest.fixture(params=["auto", "single", "pair"])
def pair_mode(request):
    """Runs a GPU test with the GEMM's CTA-pair tiles chosen by shape, off, and forced on."""

    from mdl_b200.ops._ext import ext

    mode = {"auto": -1, "single": 0, "pair": 1}[request.param]
    prev = ext().gemm_pair_mode(mode)
    yield request.param
    ext().gemm_pair_mode(prev)


def _ref(a, b, M, N, K, Gn, lda, gsA, a_mn, ldb, gsB, b_mn):
    av = G._view(a, Gn, M, K, gsA, lda, a_mn).float()
    bv = G._view(b, Gn, N, K, gsB, ldb, b_mn).float()
    return torch.bmm(av, bv.transpose(1, 2))


def _operands(M, N, K, Gn, a_mn, b_mn, device):
    torch.manual_seed(0)
    if a_mn:
        a = torch.randn(Gn, K, M, device=device).bfloat16()
        lda, gsA = M, K * M
    else:
        a = torch.randn(Gn, M, K, device=device).bfloat16()
        lda, gsA = K, M * K
    if b_mn:
        b = torch.randn(Gn, K, N, device=device).bfloat16()
        ldb, gsB = N, K * N
    else:
        b = torch.randn(Gn, N, K, device=device).bfloat16()
        ldb, gsB = K, N * K
    return a, lda, gsA, b, ldb, gsB


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", [(128, 256, 64, 1), (256, 512, 192, 3), (200, 296, 136, 2)])
def test_gemm_cpu_reference_matches_bmm(a_mn, b_mn, shape):
    M, N, K, Gn = shape
    a, lda, gsA, b, ldb, gsB = _operands(M, N, K, Gn, a_mn, b_mn, "cpu")
    out = torch.empty(Gn, M, N)
    G.bgemm(a, b, out, M=M, N=N, K=K, G=Gn, lda=lda, gsA=gsA, a_mn=a_mn, ldb=ldb, gsB=gsB, b_mn=b_mn,
            ldc=N, gsC=M * N)
    ref = _ref(a, b, M, N, K, Gn, lda, gsA, a_mn, ldb, gsB, b_mn)
    torch.testing.assert_close(out, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", [(128, 256, 64, 1), (256, 512, 192, 3), (200, 296, 136, 2), (1024, 768, 1024, 4)])
def test_gemm_tcgen05_layouts(a_mn, b_mn, shape, pair_mode):
    M, N, K, Gn = shape
    a, lda, gsA, b, ldb, gsB = _operands(M, N, K, Gn, a_mn, b_mn, "cuda")
    out = torch.empty(Gn, M, N, device="cuda", dtype=torch.float32)
    G.bgemm(a, b, out, M=M, N=N, K=K, G=Gn, lda=lda, gsA=gsA, a_mn=a_mn, ldb=ldb, gsB=gsB, b_mn=b_mn,
            ldc=N, gsC=M * N)
    torch.cuda.synchronize()
    ref = _ref(a, b, M, N, K, Gn, lda, gsA, a_mn, ldb, gsB, b_mn)
    torch.testing.assert_close(out, ref, atol=2e-3 * K ** 0.5, rtol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("act", [G.ACT_NONE, G.ACT_GELU, G.ACT_DGELU, G.ACT_RELU, G.ACT_DRELU, G.ACT_GELU_GRAD,
                                 G.ACT_DMUL])
def test_gemm_tcgen05_epilogues(act, pair_mode):
    M, N, K, Gn = 384, 512, 256, 2
    a, lda, gsA, b, ldb, gsB = _operands(M, N, K, Gn, False, True, "cuda")
    bias = torch.randn(Gn, N, device="cuda")
    aux = torch.randn(Gn, M, N, device="cuda").bfloat16()
    out = torch.empty(Gn, M, N, device="cuda", dtype=torch.bfloat16)
    out2 = torch.empty_like(out)
    colsum = torch.zeros(Gn, N, device="cuda")
    G.bgemm(a, b, out, M=M, N=N, K=K, G=Gn, lda=lda, gsA=gsA, ldb=ldb, gsB=gsB, b_mn=True, ldc=N, gsC=M * N,
            out2=out2, bias=bias, gs_bias=N, aux=aux, ld_aux=N, gs_aux=M * N, colsum=colsum, gs_colsum=N,
            act=act, alpha=0.5)
    ref_out = torch.empty(Gn, M, N, dtype=torch.bfloat16)
    ref_out2 = torch.empty_like(ref_out)
    ref_cs = torch.zeros(Gn, N)
    G.bgemm(a.cpu(), b.cpu(), ref_out, M=M, N=N, K=K, G=Gn, lda=lda, gsA=gsA, ldb=ldb, gsB=gsB, b_mn=True, ldc=N,
            gsC=M * N, out2=ref_out2, bias=bias.cpu(), gs_bias=N, aux=aux.cpu(), ld_aux=N, gs_aux=M * N,
            colsum=ref_cs, gs_colsum=N, act=act, alpha=0.5)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ref_out.float(), atol=0.05, rtol=0.02)
    if act in (G.ACT_GELU, G.ACT_GELU_GRAD):
        torch.testing.assert_close(out2.cpu().float(), ref_out2.float(), atol=0.05, rtol=0.02)
    torch.testing.assert_close(colsum.cpu(), ref_cs, atol=0.5, rtol=0.02)


@pytest.mark.gpu
def test_gemm_tcgen05_accumulate_fp32(pair_mode):
    M, N, K = 256, 256, 128
    a, lda, gsA, b, ldb, gsB = _operands(M, N, K, 1, True, True, "cuda")
    out = torch.ones(M, N, device="cuda")
    G.bgemm(a, b, out, M=M, N=N, K=K, lda=lda, a_mn=True, ldb=ldb, b_mn=True, ldc=N, accumulate=True)
    ref = _ref(a, b, M, N, K, 1, lda, gsA, True, ldb, gsB, True)[0] + 1.0
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=1e-3)


def _shared_and_krange(device):
    """A shared weight over a batch of row groups, and the weight gradient that sums
    per-sample row ranges (the OneTrans S-token products)."""

    torch.manual_seed(1)
    B, L, s, K, N = 3, 200, 136, 128, 320
    x = torch.randn(B, L, K, device=device).bfloat16()
    w = torch.randn(N, K, device=device).bfloat16()
    out = torch.zeros(B, L, N, device=device, dtype=torch.float32)
    G.bgemm(x, w, out, M=s, N=N, K=K, G=B, lda=K, gsA=L * K, ldb=K, gsB=0, ldc=N, gsC=L * N)
    ref = torch.zeros(B, L, N, device=device)
    ref[:, :s] = x[:, :s].float() @ w.float().t()
    dy = torch.randn(B, L, N, device=device).bfloat16()
    gw = torch.zeros(N, K, device=device)
    G.bgemm(dy, x, gw, M=N, N=K, K=s, lda=N, a_mn=True, ldb=K, b_mn=True, ldc=K, accumulate=True, kg=B,
            ksA=L * N, ksB=L * K)
    gref = torch.einsum("bln,blk->nk", dy[:, :s].float(), x[:, :s].float())
    aux = torch.randn(B, L, N, device=device).bfloat16()
    add = torch.zeros(B, L, N, device=device, dtype=torch.bfloat16)
    G.bgemm(x, w, add, M=s, N=N, K=K, G=B, lda=K, gsA=L * K, ldb=K, gsB=0, ldc=N, gsC=L * N, aux=aux, ld_aux=N,
            gs_aux=L * N, act=G.ACT_ADD)
    add_ref = torch.zeros(B, L, N, device=device)
    add_ref[:, :s] = ref[:, :s] + aux[:, :s].float()
    return out, ref, gw, gref, add, add_ref, K, s


def test_gemm_shared_operand_and_k_ranges_cpu():
    out, ref, gw, gref, add, add_ref, _, _ = _shared_and_krange("cpu")
    torch.testing.assert_close(out, ref)
    torch.testing.assert_close(gw, gref, atol=1e-3, rtol=1e-4)
    torch.testing.assert_close(add.float(), add_ref, atol=0.05, rtol=0.01)


@pytest.mark.gpu
def test_gemm_shared_operand_and_k_ranges_tcgen05(pair_mode):
    out, ref, gw, gref, add, add_ref, K, s = _shared_and_krange("cuda")
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, atol=2e-3 * K ** 0.5, rtol=1e-3)
    torch.testing.assert_close(gw, gref, atol=2e-3 * (3 * s) ** 0.5, rtol=1e-3)
    torch.testing.assert_close(add.float(), add_ref, atol=0.1, rtol=0.02)
