"""Device time of the flash attention (forward, backward) on a OneTrans layer shape.

    python -m mdl_b200.benchmark.attention [--batch 1024] [--lk 544] [--lq 544] [--heads 8]
                                           [--padding 0] [--non-causal] [--iters 20]

Inputs are random bf16 ``qkv [B, Lk, 3*32*H]`` (larger than L2 at the default
size); ``--padding`` gives every sample that many leading padded keys. Reports,
per call: milliseconds (CUDA events over ``--iters`` calls after warm-up), the
128 x 128 score tiles visited, the exponentials evaluated and the tensor-core
FLOPs of those tiles, and the rates they imply. Rank-0 JSON line.
"""

from __future__ import annotations

import argparse
import json

import torch

from ..ops.attention import SuffixAttentionFn


def visited_tiles(lk: int, lq: int, kstart: int, causal: bool) -> int:
    """128 x 128 (query tile, key tile) pairs the kernels process per (sample, head)."""

    nq = (lq + 127) // 128
    tmax = (lk - kstart + 127) // 128 - 1
    total = 0
    for i in range(nq):
        t0 = i if causal else 0
        total += max(0, tmax - t0 + 1)
    return total


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--lk", type=int, default=544)
    ap.add_argument("--lq", type=int, default=544)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--padding", type=int, default=0)
    ap.add_argument("--non-causal", action="store_true")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    B, Lk, Lq, H = args.batch, args.lk, args.lq, args.heads
    causal = not args.non_causal
    D = 32 * H
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(B, Lk, 3 * D, device=dev, generator=g).bfloat16().requires_grad_(True)
    ks = torch.full((B,), args.padding, dtype=torch.int32, device=dev)
    dout = torch.randn(B, Lq, D, device=dev, generator=g).bfloat16()

    def fwd():
        return SuffixAttentionFn.apply(qkv, ks, H, Lq, causal)

    out = fwd()
    for _ in range(3):
        out = fwd()
        torch.autograd.grad(out, qkv, dout)
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record()
    for _ in range(args.iters):
        out = fwd()
    e[1].record()
    e[2].record()
    for _ in range(args.iters):
        torch.autograd.grad(out, qkv, dout, retain_graph=True)
    e[3].record()
    torch.cuda.synchronize()
    fwd_ms = e[0].elapsed_time(e[1]) / args.iters
    bwd_ms = e[2].elapsed_time(e[3]) / args.iters
    tiles = visited_tiles(Lk, Lq, args.padding, causal) * B * H
    exps = tiles * 128 * 128
    flops_fwd = tiles * 2 * (2 * 128 * 128 * 32)          # S = QK^T, O += PV
    flops_bwd = tiles * 5 * (2 * 128 * 128 * 32)          # S^T, dP^T, dV, dK, dQ
    print(json.dumps({
        "shape": {"B": B, "Lk": Lk, "Lq": Lq, "heads": H, "head_dim": 32, "causal": causal, "padding": args.padding},
        "tiles_128x128": tiles,
        "fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
        "fwd_exp_per_s": round(exps / fwd_ms / 1e9, 3), "bwd_exp_per_s": round(exps / bwd_ms / 1e9, 3),
        "fwd_tflops": round(flops_fwd / fwd_ms / 1e9, 1), "bwd_tflops": round(flops_bwd / bwd_ms / 1e9, 1),
        "units": "exp_per_s in 1e12/s (Texp/s), tflops of the visited tiles",
    }), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
