"""The allocation-free LayerNorm backward, called through its exported C symbol.

``mdl_layernorm_bwd_noalloc`` is for callers that may not allocate device memory
while they run (code inside host callbacks or allocator-locked hooks, runtimes that
plan all memory in advance, plain C programs without an allocator). It keeps its
partial sums in a fixed device array inside the library. This test calls it through
ctypes, exactly as such a caller would, and checks that two calls in a row match the
regular entry point (which takes a caller-allocated scratch buffer) within the
tolerances of the other LayerNorm tests. This file is named so that pytest collects
it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from mdl_b200.ops._ext import _lib_path, ext

    ext()  # make sure the library is built and loaded with its torch dependencies
    lib = ctypes.CDLL(str(_lib_path()))
    fn = lib.mdl_layernorm_bwd_noalloc
    fn.restype = ctypes.c_int
    vp, f32, i32 = ctypes.c_void_p, ctypes.c_float, ctypes.c_int
    fn.argtypes = [vp, vp, f32, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
    lib.mdl_noalloc_last_error.restype = ctypes.c_char_p
    return lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _case(B, T, D, mix, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, T, D, device="cuda", generator=g).bfloat16()
    r = torch.randn(B, T, D, device="cuda", generator=g).bfloat16()
    gamma = torch.randn(D, device="cuda", generator=g)
    beta = torch.randn(D, device="cuda", generator=g)
    dy = torch.randn(B, T, D, device="cuda", generator=g).bfloat16()
    from mdl_b200.ops._ext import ext

    out = torch.empty_like(x)
    mean = torch.empty(B * T, device="cuda")
    rstd = torch.empty_like(mean)
    ext().ln_fwd(x, None if mix else r, gamma, beta, out, mean, rstd, B, T, D, mix, 1e-5)
    return x, (None if mix else r), gamma, dy, mean, rstd


def _regular(x, r, gamma, dy, mean, rstd, B, T, D, mix, bcast=None, scale=1.0, want_dx2=False):
    from mdl_b200.ops._ext import ext

    C = ext()
    dx = torch.empty_like(x)
    dx2 = torch.empty_like(x) if want_dx2 else None
    dg = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    grid = C.ln_bwd_grid(B)
    partials = torch.empty(grid, 2 * D, device="cuda")
    C.ln_bwd(None if bcast is not None else dy, bcast, scale, x, r, mean, rstd, gamma, dx, dx2, partials, dg, db,
             B, T, D, mix, grid)
    return dx, dg, db, dx2


def _noalloc(lib, x, r, gamma, dy, mean, rstd, B, T, D, mix, bcast=None, scale=1.0, want_dx2=False):
    dx = torch.empty_like(x)
    dx2 = torch.empty_like(x) if want_dx2 else None
    dg = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mdl_layernorm_bwd_noalloc(_ptr(None if bcast is not None else dy), _ptr(bcast), scale, _ptr(x), _ptr(r),
                                       _ptr(mean), _ptr(rstd), _ptr(gamma), _ptr(dx), _ptr(dx2), _ptr(dg), _ptr(db),
                                       B, T, D, int(mix), stream)
    assert rc == 0, lib.mdl_noalloc_last_error().decode()
    return dx, dg, db, dx2


def _check(got, ref):
    torch.cuda.synchronize()
    torch.testing.assert_close(got[0].float(), ref[0].float(), atol=8e-2, rtol=3e-2)
    torch.testing.assert_close(got[1], ref[1], atol=0.5, rtol=2e-2)
    torch.testing.assert_close(got[2], ref[2], atol=0.5, rtol=2e-2)
    if ref[3] is not None:
        torch.testing.assert_close(got[3].float(), ref[3].float(), atol=8e-2, rtol=3e-2)


@pytest.mark.parametrize("mix", [True, False])
def test_noalloc_matches_regular_entry_point_twice(mix):
    lib = _lib()
    T, D = 16, 768
    # Two calls in a row. The first (B=2048) fills every row of the array the CTA
    # cap allows (341 CTAs at D=768); the second uses fewer CTAs (B=300), so a call
    # that read rows it did not write would pick up the first call's partial sums.
    for seed, B in ((1, 2048), (2, 300)):
        x, r, gamma, dy, mean, rstd = _case(B, T, D, mix, seed)
        ref = _regular(x, r, gamma, dy, mean, rstd, B, T, D, mix)
        got = _noalloc(lib, x, r, gamma, dy, mean, rstd, B, T, D, mix)
        _check(got, ref)


def test_noalloc_cta_cap_at_wide_rows():
    # D=2048 leaves room for 128 CTAs in the array; B=600 would otherwise take 600 or more
    lib = _lib()
    T, D = 16, 2048
    for seed, B in ((3, 600), (4, 50)):
        x, r, gamma, dy, mean, rstd = _case(B, T, D, False, seed)
        ref = _regular(x, r, gamma, dy, mean, rstd, B, T, D, False)
        got = _noalloc(lib, x, r, gamma, dy, mean, rstd, B, T, D, False)
        _check(got, ref)


def test_noalloc_broadcast_gradient_and_second_copy():
    # dy[b, t, :] = dy_bcast[b, :] * scale (backward of a token mean), plus the dx2 copy
    lib = _lib()
    B, T, D = 700, 16, 768
    x, r, gamma, dy, mean, rstd = _case(B, T, D, True, 5)
    bcast = torch.randn(B, D, device="cuda").bfloat16()
    ref = _regular(x, r, gamma, dy, mean, rstd, B, T, D, True, bcast=bcast, scale=1.0 / T, want_dx2=True)
    got = _noalloc(lib, x, r, gamma, dy, mean, rstd, B, T, D, True, bcast=bcast, scale=1.0 / T, want_dx2=True)
    _check(got, ref)


def test_noalloc_rejects_sizes_beyond_its_limits():
    lib = _lib()
    x = torch.zeros(1, device="cuda")
    rc = lib.mdl_layernorm_bwd_noalloc(_ptr(x), None, 1.0, _ptr(x), None, _ptr(x), _ptr(x), None, _ptr(x), None,
                                       None, None, 4, 1, 4096, 0, None)
    assert rc == -1
    assert b"2048" in lib.mdl_noalloc_last_error()
    # token mixing of 32 tokens x 2048 columns needs (32 + 16) * 2048 * 4 = 384 KB of shared
    # memory per CTA, above the device limit
    rc = lib.mdl_layernorm_bwd_noalloc(_ptr(x), None, 1.0, _ptr(x), None, _ptr(x), _ptr(x), None, _ptr(x), None,
                                       None, None, 4, 32, 2048, 1, None)
    assert rc == -1
    assert b"shared memory" in lib.mdl_noalloc_last_error()
