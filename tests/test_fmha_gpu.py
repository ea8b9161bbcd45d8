"""tcgen05 flash attention (causal query suffix, per-sample padding prefix) against
the fp32 PyTorch definition, forward and backward."""

import pytest
import torch

from mdl_b200.ops.attention import suffix_attention, suffix_attention_reference


def _case(B, Lk, Lq, H, kstart, causal, device, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    D = 32 * H
    qkv = (torch.randn(B, Lk, 3 * D, generator=g) * 1.5).bfloat16().to(device)
    ks = torch.tensor(kstart, dtype=torch.int32).to(device)
    dout = torch.randn(B, Lq, D, generator=g).bfloat16().to(device)
    return qkv, ks, dout


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
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_fmha_forward_backward(case):
    B, Lk, Lq, H, kstart, causal = case
    qkv, ks, dout = _case(B, Lk, Lq, H, kstart, causal, "cuda")
    q1 = qkv.clone().requires_grad_(True)
    out = suffix_attention(q1, ks, H, Lq, causal)
    out.backward(dout)
    torch.cuda.synchronize()
    q2 = qkv.float().clone().requires_grad_(True)
    ref = suffix_attention_reference(q2, ks, H, Lq, causal)
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
