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


def _regular(x, r, gamma, dy, mean, rstd, B, T, D, mix):
    from mdl_b200.ops._ext import ext

    C = ext()
    dx = torch.empty_like(x)
    dg = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    grid = C.ln_bwd_grid(B)
    partials = torch.empty(grid, 2 * D, device="cuda")
    C.ln_bwd(dy, None, 1.0, x, r, mean, rstd, gamma, dx, None, partials, dg, db, B, T, D, mix, grid)
    return dx, dg, db


def _noalloc(lib, x, r, gamma, dy, mean, rstd, B, T, D, mix):
    dx = torch.empty_like(x)
    dg = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mdl_layernorm_bwd_noalloc(_ptr(dy), None, 1.0, _ptr(x), _ptr(r), _ptr(mean), _ptr(rstd), _ptr(gamma),
                                       _ptr(dx), None, _ptr(dg), _ptr(db), B, T, D, int(mix), stream)
    assert rc == 0, lib.mdl_noalloc_last_error().decode()
    return dx, dg, db


@pytest.mark.parametrize("mix", [True, False])
def test_noalloc_matches_regular_entry_point_twice(mix):
    lib = _lib()
    B, T, D = 300, 16, 768
    for seed in (1, 2):  # two calls in a row: the second must not see the first's leftovers
        x, r, gamma, dy, mean, rstd = _case(B, T, D, mix, seed)
        ref = _regular(x, r, gamma, dy, mean, rstd, B, T, D, mix)
        got = _noalloc(lib, x, r, gamma, dy, mean, rstd, B, T, D, mix)
        torch.cuda.synchronize()
        torch.testing.assert_close(got[0].float(), ref[0].float(), atol=8e-2, rtol=3e-2)
        torch.testing.assert_close(got[1], ref[1], atol=0.5, rtol=2e-2)
        torch.testing.assert_close(got[2], ref[2], atol=0.5, rtol=2e-2)


def test_noalloc_rejects_sizes_beyond_its_limits():
    lib = _lib()
    x = torch.zeros(1, device="cuda")
    rc = lib.mdl_layernorm_bwd_noalloc(_ptr(x), None, 1.0, _ptr(x), None, _ptr(x), _ptr(x), None, _ptr(x), None,
                                       None, None, 4, 1, 4096, 0, None)
    assert rc == -1
    assert b"2048" in lib.mdl_noalloc_last_error()
