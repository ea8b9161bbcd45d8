"""STCA with request-level batching: the history transforms run once per request and
each candidate attends to its request's transformed history; equal to expanding the
history to every candidate first, and to a cached ``transform_histories`` (CPU)."""

import torch

from mdl_b200.models.stca import STCAEncoder


def test_request_major_stca_matches_expanded():
    torch.manual_seed(0)
    enc = STCAEncoder(16, 2, 3, 2)
    R, L, C = 3, 12, 7
    hist = torch.randn(R, L, 16, requires_grad=True)
    lengths = torch.tensor([12, 5, 0])
    valid = torch.arange(L).view(1, L) >= (L - lengths).view(R, 1)
    ri = torch.tensor([0, 0, 1, 2, 1, 0, 2])
    target = torch.randn(C, 16)
    out = enc(hist, valid, target, False, row_indices=ri)
    hist2 = hist.detach().clone().requires_grad_(True)
    ref = enc(hist2.index_select(0, ri), valid.index_select(0, ri), target, False)
    torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)
    out.sum().backward()
    ref.sum().backward()
    torch.testing.assert_close(hist.grad, hist2.grad, atol=1e-5, rtol=1e-5)
    with torch.no_grad():
        cache = enc.transform_histories(hist, False)
        cached = enc(None, valid, target, False, row_indices=ri, transformed=cache)
    torch.testing.assert_close(cached, out.detach(), atol=1e-6, rtol=1e-6)
