"""Micro-benchmark of the suffix attention (``ops.attention.suffix_attention``: the tcgen05
flash attention for head width 32, the CUDA-core kernels for 8, 16 and 64) against its
PyTorch definition, forward and backward, on LONGER / OneTrans shapes.

    python -m mdl_b200.benchmark.attention_widths [--reps R] [--no-reference] [--shape NAME ...]
                                                  [--batch B]

``--shape`` keeps the named shapes, ``--batch`` overrides their batch (small profiler cases).

Device time with CUDA events (after two warm-ups); random padding starts in [0, Lk/2).
"""

from __future__ import annotations

import argparse

import torch

from ..ops.attention import suffix_attention, suffix_attention_reference

# B, Lk, Lq, heads, head width, causal, ktail, kexcl
SHAPES = {
    "longer_production_cross": (1280, 2051, 35, 4, 8, True, 3, 1),
    "longer_workload5_cross": (512, 2001, 257, 8, 32, True, 1, 1),
    "onetrans_d256_h4": (256, 545, 545, 4, 64, True, 0, 0),
}


def _time(fn, shape, reps: int) -> tuple[float, float]:
    B, Lk, Lq, H, hd, causal, ktail, kexcl = shape
    D = H * hd
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn(B, Lk, 3 * D, device="cuda", generator=g).bfloat16().requires_grad_(True)
    ks = torch.randint(0, Lk // 2, (B,), device="cuda", dtype=torch.int32, generator=g)
    dout = torch.randn(B, Lq, D, device="cuda", generator=g).bfloat16()
    for _ in range(2):
        fn(qkv, ks, H, Lq, causal, ktail, kexcl).backward(dout)
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    f = b = 0.0
    for _ in range(reps):
        e[0].record()
        o = fn(qkv, ks, H, Lq, causal, ktail, kexcl)
        e[1].record()
        o.backward(dout)
        e[2].record()
        torch.cuda.synchronize()
        f += e[0].elapsed_time(e[1])
        b += e[1].elapsed_time(e[2])
    return f / reps, b / reps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--no-reference", action="store_true")
    ap.add_argument("--shape", action="append", choices=sorted(SHAPES), default=None)
    ap.add_argument("--batch", type=int, default=None)
    args = ap.parse_args(argv)

    def ref(qkv, ks, H, Lq, c, kt, ke):
        return suffix_attention_reference(qkv, ks, H, Lq, c, ktail=kt, kexcl=ke)

    for name, shape in SHAPES.items():
        if args.shape and name not in args.shape:
            continue
        if args.batch:
            shape = (args.batch,) + shape[1:]
        nf, nb = _time(suffix_attention, shape, args.reps)
        line = f"{name:26s} {shape}: native fwd {nf:.3f} ms bwd {nb:.3f} ms"
        if not args.no_reference:
            try:
                rf, rb = _time(ref, shape, max(1, args.reps // 3))
                line += f" | PyTorch definition fwd {rf:.3f} ms bwd {rb:.3f} ms"
            except torch.cuda.OutOfMemoryError:
                line += " | PyTorch definition: out of memory"
            torch.cuda.empty_cache()
        print(line, flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
