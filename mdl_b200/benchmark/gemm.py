"""Micro-benchmark of the tcgen05 grouped GEMM and its fused epilogues on the
per-token FFN shapes of the RankMixer workload (B=2048 rows, D=768, H=3072, one
group per token).

    python -m mdl_b200.benchmark.gemm [--groups G] [--reps R] [--only NAME]

Prints device time (CUDA events, after two warm-up launches) and TFLOP/s per
epilogue kind. ``--only`` runs one case, so a profiler can capture exactly its
launches.
"""

from __future__ import annotations

import argparse

import torch

from ..ops.gemm import ACT_DMUL, ACT_GELU, ACT_GELU_GRAD, ACT_NONE, ACT_RELU, bgemm


def cases(G: int, B: int = 2048, H: int = 3072, D: int = 768, device: str = "cuda") -> dict:
    dev = torch.device(device)
    x = torch.randn(B, G, D, device=dev).to(torch.bfloat16)
    w1 = (torch.randn(G, H, D, device=dev) * 0.03).to(torch.bfloat16)
    b1 = torch.zeros(G, H, device=dev)
    pre = torch.empty(G, B, H, device=dev, dtype=torch.bfloat16)
    act = torch.empty_like(pre)
    w2 = (torch.randn(G, D, H, device=dev) * 0.02).to(torch.bfloat16)
    y = torch.empty(B, G, D, device=dev, dtype=torch.bfloat16)
    dpre = torch.empty_like(pre)
    dw = torch.zeros(G, H, D, device=dev)
    cs = torch.zeros(G, H, device=dev)
    f1 = dict(M=B, N=H, K=D, G=G, lda=G * D, gsA=D, ldb=D, gsB=H * D, ldc=H, gsC=B * H)
    return {
        "fwd1_plain": lambda: bgemm(x, w1, pre, **f1),
        "fwd1_bias_relu": lambda: bgemm(x, w1, pre, **f1, bias=b1, gs_bias=H, act=ACT_RELU),
        "fwd1_bias_gelu": lambda: bgemm(x, w1, pre, **f1, out2=act, bias=b1, gs_bias=H, act=ACT_GELU),
        "fwd1_bias_gelu_grad": lambda: bgemm(x, w1, pre, **f1, out2=act, bias=b1, gs_bias=H, act=ACT_GELU_GRAD),
        "fwd2": lambda: bgemm(act, w2, y, M=B, N=D, K=H, G=G, lda=H, gsA=B * H, ldb=H, gsB=D * H, ldc=G * D, gsC=D),
        "dpre_dmul_colsum": lambda: bgemm(y, w2, dpre, M=B, N=H, K=D, G=G, lda=G * D, gsA=D, ldb=H, gsB=D * H,
                                          b_mn=True, ldc=H, gsC=B * H, aux=pre, ld_aux=H, gs_aux=B * H, colsum=cs,
                                          gs_colsum=H, act=ACT_DMUL),
        "dw_fp32_acc": lambda: bgemm(dpre, x, dw, M=H, N=D, K=B, G=G, lda=H, gsA=B * H, a_mn=True, ldb=G * D,
                                     gsB=D, b_mn=True, ldc=D, gsC=H * D, accumulate=True),
        "dx": lambda: bgemm(dpre, w1, y, M=B, N=D, K=H, G=G, lda=H, gsA=B * H, ldb=D, gsB=H * D, b_mn=True,
                            ldc=G * D, gsC=D),
    }, 2.0 * B * H * D * G


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--groups", type=int, default=16)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--only", default=None)
    args = ap.parse_args(argv)
    table, flops = cases(args.groups)
    for name, fn in table.items():
        if args.only and name != args.only:
            continue
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / args.reps * 1e3
        print(f"{name:24s} {us:9.1f} us {flops / us / 1e6:8.1f} TFLOP/s", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
