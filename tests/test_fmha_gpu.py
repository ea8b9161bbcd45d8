"""tcgen05 flash attention (causal query suffix, per-sample padding prefix) against
the fp32 PyTorch definition, forward and backward."""

import pytest
import torch

from mdl_b200.ops.attention import suffix_attention, suffix_attention_reference


def _case(B, Lk, Lq, H, kstart, causal, device, seed=0, hd=32):
    g = torch.Generator(device="cpu").manual_seed(seed)
    D = hd * H
    qkv = (torch.randn(B, Lk, 3 * D, generator=g) * 1.5).bfloat16().to(device)
    ks = torch.tensor(kstart, dtype=torch.int32).to(device)
    dout = torch.randn(B, Lq, D, generator=g).bfloat16().to(device)
    return qkv, ks, dout


def test_suffix_attention_ktail_matches_longer_mask():
    """Globals after the sequence with ktail == globals before it with the reference's
    mixed mask (globals see all keys; recent queries are causal and see the globals)."""

    torch.manual_seed(0)
    B, L, G, R, H = 2, 30, 3, 10, 2
    D = 32 * H
    qkv = torch.randn(B, L + G, 3 * D)
    ks = torch.tensor([0, 7])
    out = suffix_attention_reference(qkv, ks, H, R + G, True, ktail=G)
    # reference layout: [globals; sequence], queries [globals; last R], mixed mask
    ref_qkv = torch.cat([qkv[:, L:], qkv[:, :L]], dim=1)
    hd = 32
    q = ref_qkv[:, :, :D].reshape(B, L + G, H, hd).transpose(1, 2)
    k = ref_qkv[:, :, D:2 * D].reshape(B, L + G, H, hd).transpose(1, 2)
    v = ref_qkv[:, :, 2 * D:].reshape(B, L + G, H, hd).transpose(1, 2)
    qi = torch.cat([torch.arange(G), torch.arange(L + G - R, L + G)])
    kpos = torch.arange(L + G)
    key_valid = (kpos.view(1, -1) < G) | (kpos.view(1, -1) >= G + ks.view(-1, 1))
    glob = key_valid.unsqueeze(1).expand(B, G, L + G)
    rec = key_valid.unsqueeze(1) & (kpos.view(1, 1, -1) <= torch.arange(L + G - R, L + G).view(1, R, 1))
    rec = rec & (torch.arange(L + G - R, L + G).view(1, R, 1) >= G + ks.view(-1, 1, 1))
    allowed = torch.cat([glob, rec], dim=1)
    s = (q[:, :, qi] @ k.transpose(-1, -2)) / hd ** 0.5
    s = s.masked_fill(~allowed.unsqueeze(1), float("-inf"))
    p = torch.nan_to_num(torch.softmax(s, -1))
    o = (p @ v).transpose(1, 2).reshape(B, G + R, D)
    # ours: queries [last R sequence tokens; globals]
    torch.testing.assert_close(out[:, R:], o[:, :G], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(out[:, :R], o[:, G:], atol=1e-5, rtol=1e-4)


def test_suffix_attention_kexcl_matches_request_candidate_split():
    """ktail = G globals after the sequence, the last Gc of them excluded: equal to the
    reference's two-part LONGER attention -- user globals and recent queries over
    [user; sequence] (mixed mask), candidate globals over [candidate; user; sequence]."""

    torch.manual_seed(1)
    B, L, Gu, Gc, R, H = 2, 30, 2, 3, 10, 2
    G, D, hd = Gu + Gc, 32 * H, 32
    qkv = torch.randn(B, L + G, 3 * D)
    ks = torch.tensor([0, 9])
    out = suffix_attention_reference(qkv, ks, H, R + G, True, ktail=G, kexcl=Gc)

    def heads(x, part):
        return x[..., part * D:(part + 1) * D].reshape(x.shape[0], x.shape[1], H, hd).transpose(1, 2)

    def attend(q_rows, k_rows, allowed):
        q, k, v = heads(q_rows, 0), heads(k_rows, 1), heads(k_rows, 2)
        s = (q @ k.transpose(-1, -2)) / hd ** 0.5
        p = torch.nan_to_num(torch.softmax(s.masked_fill(~allowed.unsqueeze(1), float("-inf")), -1))
        return (p @ v).transpose(1, 2).reshape(q_rows.shape[0], q_rows.shape[1], D)

    seq, user, cand = qkv[:, :L], qkv[:, L:L + Gu], qkv[:, L + Gu:]
    # request side: keys [user; sequence]
    rk = torch.cat([user, seq], dim=1)
    kpos = torch.arange(Gu + L)
    kvalid = (kpos.view(1, -1) < Gu) | (kpos.view(1, -1) >= Gu + ks.view(-1, 1))
    qpos = torch.arange(Gu + L - R, Gu + L)
    rec_allowed = kvalid.unsqueeze(1) & (kpos.view(1, 1, -1) <= qpos.view(1, R, 1))
    rec_allowed = rec_allowed & (qpos.view(1, R, 1) >= Gu + ks.view(-1, 1, 1))
    o_user = attend(user, rk, kvalid.unsqueeze(1).expand(B, Gu, -1))
    o_rec = attend(seq[:, L - R:], rk, rec_allowed)
    # candidate side: keys [candidate; user; sequence], all valid keys
    ck = torch.cat([cand, user, seq], dim=1)
    cvalid = torch.cat([torch.ones(B, Gc, dtype=torch.bool), kvalid], dim=1)
    o_cand = attend(cand, ck, cvalid.unsqueeze(1).expand(B, Gc, -1))
    torch.testing.assert_close(out[:, :R], o_rec, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(out[:, R:R + Gu], o_user, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(out[:, R + Gu:], o_cand, atol=1e-5, rtol=1e-4)


def test_suffix_attention_reference_matches_loop():
    B, Lk, Lq, H = 2, 20, 9, 2
    qkv, ks, _ = _case(B, Lk, Lq, H, [0, 6], True, "cpu")
    out = suffix_attention_reference(qkv, ks, H, Lq)
    D, hd = 32 * H, 32
    x = qkv.float()
    for b in range(B):
        for i in range(Lq):
            p = Lk - Lq + i
            for h in range(H):
                q = x[b, p, h * hd:(h + 1) * hd]
                keys = [j for j in range(Lk) if int(ks[b]) <= j <= p]
                if not keys or p < int(ks[b]):
                    assert out[b, i, h * hd:(h + 1) * hd].abs().max() == 0
                    continue
                k = x[b, keys, D + h * hd:D + (h + 1) * hd]
                v = x[b, keys, 2 * D + h * hd:2 * D + (h + 1) * hd]
                w = torch.softmax(k @ q / hd ** 0.5, 0)
                torch.testing.assert_close(out[b, i, h * hd:(h + 1) * hd], w @ v, atol=1e-5, rtol=1e-4)


CASES = [
    # B, Lk, Lq, H, kstart, causal
    (2, 544, 544, 8, [0, 37], True),        # OneTrans layer 0: all tokens query
    (3, 544, 288, 8, [0, 300, 530], True),  # pyramid layer 1: suffix queries, padded prefixes
    (2, 160, 96, 8, [0, 150], True),        # last layers (queries before kstart output zero)
    (2, 300, 300, 2, [5, 129], False),      # non-causal
    (1, 64, 40, 4, [0], True),              # shorter than one tile
    (2, 300, 280, 8, [0, 120], True, 1),    # LONGER cross block: 1 trailing global token
    (2, 433, 300, 4, [7, 200], True, 24),   # 24 trailing globals, padded prefixes
    (2, 300, 280, 8, [0, 120], True, 6, 2),  # 6 globals, the last 2 (candidates) hidden from the others
    (3, 433, 300, 4, [7, 200, 420], True, 24, 8),
    (2, 40, 40, 2, [0, 12], True, 8, 3),    # LONGER self block: every token a query
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_fmha_forward_backward(case):
    B, Lk, Lq, H, kstart, causal = case[:6]
    ktail = case[6] if len(case) > 6 else 0
    kexcl = case[7] if len(case) > 7 else 0
    qkv, ks, dout = _case(B, Lk, Lq, H, kstart, causal, "cuda")
    q1 = qkv.clone().requires_grad_(True)
    out = suffix_attention(q1, ks, H, Lq, causal, ktail, kexcl)
    out.backward(dout)
    torch.cuda.synchronize()
    q2 = qkv.float().clone().requires_grad_(True)
    ref = suffix_attention_reference(q2, ks, H, Lq, causal, ktail=ktail, kexcl=kexcl)
    ref.backward(dout.float())
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, f"forward max error {err}"
    g, gr = q1.grad.float(), q2.grad
    rel = ((g - gr).norm() / gr.norm().clamp_min(1e-6)).item()
    assert rel < 2e-2, f"backward relative error {rel}"
    for part in range(3):  # Q, K and V gradients each
        sl = slice(part * 32 * H, (part + 1) * 32 * H)
        pr = ((g[..., sl] - gr[..., sl]).norm() / gr[..., sl].norm().clamp_min(1e-6)).item()
        assert pr < 3e-2, f"part {part} relative error {pr}"


@pytest.mark.parametrize("B,L,N,D", [(3, 17, 4, 16), (5, 70, 8, 64), (2, 40, 3, 100)])
def test_single_query_attention_cpu_reference_matches_masked_softmax(B, L, N, D):
    from mdl_b200.ops.attention import single_query_attention_reference

    torch.manual_seed(0)
    q, hist = torch.randn(B, N, D), torch.randn(B, L, N, D)
    ks = torch.randint(0, L + 1, (B,))
    out = single_query_attention_reference(q, hist, ks, 0.3)
    for b in range(B):
        for n in range(N):
            if ks[b] >= L:
                assert not out[b, n].any()
                continue
            h = hist[b, ks[b]:, n]
            w = torch.softmax(0.3 * h @ q[b, n], 0)
            torch.testing.assert_close(out[b, n], w @ h, atol=1e-5, rtol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("B,L,N,D", [(3, 17, 4, 16), (64, 257, 32, 64), (7, 90, 3, 100), (4, 33, 2, 128)])
def test_single_query_attention_kernel_matches_fp32(B, L, N, D):
    from mdl_b200.ops.attention import SingleQueryAttentionFn, single_query_attention_reference

    torch.manual_seed(1)
    dev = torch.device("cuda")
    q = torch.randn(B, N, D, device=dev, requires_grad=True)
    hist = torch.randn(B, L, N, D, device=dev).bfloat16().requires_grad_(True)
    ks = torch.randint(0, L, (B,), device=dev)
    ks[0] = L  # a sample without a valid event
    out = SingleQueryAttentionFn.apply(q, hist, ks, 0.25)
    ref_q = q.detach().clone().requires_grad_(True)
    ref_h = hist.detach().float().requires_grad_(True)
    ref = single_query_attention_reference(ref_q, ref_h, ks, 0.25)
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)
    g = torch.randn_like(ref)
    out.backward(g)
    ref.backward(g)
    torch.cuda.synchronize()
    torch.testing.assert_close(q.grad, ref_q.grad, atol=5e-3, rtol=5e-3)
    torch.testing.assert_close(hist.grad.float(), ref_h.grad, atol=2e-2, rtol=2e-2)
    assert not hist.grad[0].any()


SIMT_CASES = [
    # hd, B, Lk, Lq, H, kstart, causal, ktail, kexcl
    (8, 3, 300, 40, 4, [0, 120, 299], True, 6, 2),    # LONGER cross block, production widths (32 = 4 x 8)
    (8, 2, 40, 40, 4, [0, 12], True, 8, 3),           # LONGER self block
    (16, 2, 200, 200, 2, [5, 150], False, 0, 0),      # non-causal
    (16, 2, 257, 130, 2, [0, 64], True, 0, 0),        # OneTrans-style suffix
    (64, 2, 180, 100, 4, [3, 90], True, 0, 0),        # OneTrans d=256 / 4 heads
    (8, 700, 2, 2, 4, [0, 1] * 350, False, 0, 0),     # LONGER inner blocks: many tiny groups
    (8, 3, 2051, 35, 4, [0, 1500, 2050], True, 3, 1),  # production LONGER cross block: key-split kernels
    (16, 2, 700, 64, 2, [0, 650], False, 0, 0),       # key-split, non-causal, two 32-row blocks
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", SIMT_CASES)
def test_simt_attention_forward_backward(case):
    """The CUDA-core suffix attention (head widths 8, 16, 64) against the fp32 definition."""

    hd, B, Lk, Lq, H, kstart, causal, ktail, kexcl = case
    qkv, ks, dout = _case(B, Lk, Lq, H, kstart, causal, "cuda", hd=hd)
    q1 = qkv.clone().requires_grad_(True)
    out = suffix_attention(q1, ks, H, Lq, causal, ktail, kexcl)
    out.backward(dout)
    torch.cuda.synchronize()
    q2 = qkv.float().clone().requires_grad_(True)
    ref = suffix_attention_reference(q2, ks, H, Lq, causal, ktail=ktail, kexcl=kexcl)
    ref.backward(dout.float())
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, f"forward max error {err}"
    g, gr = q1.grad.float(), q2.grad
    for part in range(3):  # Q, K and V gradients each
        sl = slice(part * hd * H, (part + 1) * hd * H)
        pr = ((g[..., sl] - gr[..., sl]).norm() / gr[..., sl].norm().clamp_min(1e-6)).item()
        assert pr < 3e-2, f"part {part} relative error {pr}"


@pytest.mark.parametrize("B,L,G,D", [(3, 17, 2, 16), (4, 40, 4, 64)])
def test_shared_query_reference_matches_per_query_softmax(B, L, G, D):
    from mdl_b200.ops.attention import shared_query_attention_reference

    torch.manual_seed(0)
    q, hist = torch.randn(B, G, D), torch.randn(B, L, D)
    ks = torch.randint(0, L + 1, (B,))
    out = shared_query_attention_reference(q, hist, ks, 0.3)
    for b in range(B):
        for g in range(G):
            if ks[b] >= L:
                assert not out[b, g].any()
                continue
            h = hist[b, ks[b]:]
            w = torch.softmax(0.3 * h @ q[b, g], 0)
            torch.testing.assert_close(out[b, g], w @ h, atol=1e-5, rtol=1e-5)


def test_shared_query_supported_shapes():
    from mdl_b200.ops.attention import shared_query_supported

    assert shared_query_supported(2, 256) and shared_query_supported(4, 256) and shared_query_supported(8, 128)
    assert not shared_query_supported(8, 256) and not shared_query_supported(2, 258)
    assert not shared_query_supported(9, 64) and not shared_query_supported(2, 63)


@pytest.mark.gpu
@pytest.mark.parametrize("B,L,G,D", [(3, 17, 1, 16), (64, 257, 2, 256), (9, 90, 3, 100), (5, 33, 8, 128),
                                     (17, 64, 4, 256), (2, 5, 6, 62)])
def test_shared_query_attention_kernel_matches_fp32(B, L, G, D):
    from mdl_b200.ops.attention import SharedQueryAttentionFn, shared_query_attention_reference

    torch.manual_seed(2)
    dev = torch.device("cuda")
    q = (0.3 * torch.randn(B, G, D, device=dev)).requires_grad_(True)
    hist = torch.randn(B, L, D, device=dev).bfloat16().requires_grad_(True)
    ks = torch.randint(0, L, (B,), device=dev)
    ks[0] = L  # a sample without a valid event
    out = SharedQueryAttentionFn.apply(q, hist, ks, 0.25)
    ref_q = q.detach().clone().requires_grad_(True)
    ref_h = hist.detach().float().requires_grad_(True)
    ref = shared_query_attention_reference(ref_q, ref_h, ks, 0.25)
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)
    g = torch.randn_like(ref)
    out.backward(g)
    ref.backward(g)
    torch.cuda.synchronize()
    torch.testing.assert_close(q.grad, ref_q.grad, atol=5e-3, rtol=5e-3)
    torch.testing.assert_close(hist.grad.float(), ref_h.grad, atol=2e-2, rtol=2e-2)
    assert not hist.grad[0].any()
    for b in range(1, B):  # padding events get zero gradient
        assert not hist.grad[b, :int(ks[b])].any()

