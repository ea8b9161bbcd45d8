"""Benchmark matrix: ``bench.py`` over GPU counts and workloads, plus a scaling summary.

    python -m mdl_b200.benchmark.matrix --gpus 1 2 4 8 --configs 2 4 [--steps 20] [--warmup 5]
                                        [--impl ours|reference|both] [--out matrix.jsonl]
    python -m mdl_b200.benchmark.matrix --summarize matrix.jsonl

Counterpart of the reference's ``scripts/run_benchmark_matrix.sh`` and
``scripts/summarize_benchmarks.py``: every (workload, arm, N) runs as one
``torch.distributed.run`` job on one node (rendezvous on 127.0.0.1) under a
hard ``timeout``; each job's JSON line is appended to ``--out``. The summary
gives, per workload and arm, the samples/s at each N, the per-GPU rate and the
weak-scaling efficiency ``value_N / (N * value_1)``, and the ratio of this
framework to the reference arm where both ran.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def bench_command(n: int, config: int, impl: str, steps: int, warmup: int, port: int) -> list[str]:
    args = ["bench.py", "--gpus", str(n), "--steps", str(steps), "--warmup", str(warmup), "--config", str(config),
            "--impl", impl]
    if n == 1:
        return [sys.executable, *args]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
            "--master-addr=127.0.0.1", f"--master-port={port}", *args]


def run_one(n: int, config: int, impl: str, steps: int, warmup: int, port: int, timeout_s: int) -> dict:
    cmd = ["timeout", "-k", "60", str(timeout_s), *bench_command(n, config, impl, steps, warmup, port)]
    proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    line = None
    for text in reversed(proc.stdout.splitlines()):
        text = text.strip()
        if text.startswith("{"):
            try:
                line = json.loads(text)
                break
            except json.JSONDecodeError:
                continue
    if line is None:
        line = {"error": f"exit {proc.returncode}", "stderr_tail": proc.stderr[-2000:]}
    line.setdefault("impl", impl)
    line.update({"matrix_config": config, "matrix_gpus": n})
    return line


def summarize(rows: list[dict]) -> str:
    table: dict[tuple[int, str], dict[int, float]] = {}
    for r in rows:
        if "value" in r and r.get("value"):
            table.setdefault((r["matrix_config"], r.get("impl", "ours")), {})[r["matrix_gpus"]] = float(r["value"])
    out = ["| workload | arm | GPUs | samples/s | per GPU | weak-scaling efficiency | ours / reference |",
           "|---|---|---|---|---|---|---|"]
    for (cfg, impl), by_n in sorted(table.items()):
        base = by_n.get(1)
        ref = table.get((cfg, "reference"), {})
        for n in sorted(by_n):
            v = by_n[n]
            eff = f"{v / (n * base):.3f}" if base else "-"
            ratio = f"{v / ref[n]:.2f}" if impl == "ours" and ref.get(n) else "-"
            out.append(f"| {cfg} | {impl} | {n} | {v:,.0f} | {v / n:,.0f} | {eff} | {ratio} |")
    return "\n".join(out)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, nargs="+", default=[1, 2, 4, 8])
    ap.add_argument("--configs", type=int, nargs="+", default=[2, 4])
    ap.add_argument("--impl", choices=["ours", "reference", "both"], default="ours")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--timeout", type=int, default=900, help="seconds per job")
    ap.add_argument("--port", type=int, default=29611)
    ap.add_argument("--out", default="benchmark_matrix.jsonl")
    ap.add_argument("--summarize", metavar="JSONL", help="only print the summary of an existing result file")
    args = ap.parse_args(argv)
    if args.summarize:
        with open(args.summarize) as fh:
            rows = [json.loads(x) for x in fh if x.strip()]
        print(summarize(rows))
        return 0
    impls = ["reference", "ours"] if args.impl == "both" else [args.impl]
    rows = []
    for config in args.configs:
        for n in args.gpus:
            for impl in impls:
                r = run_one(n, config, impl, args.steps, args.warmup, args.port, args.timeout)
                rows.append(r)
                with open(args.out, "a") as fh:
                    fh.write(json.dumps(r) + "\n")
                print(json.dumps({k: r.get(k) for k in ("matrix_config", "matrix_gpus", "impl", "value",
                                                        "ms_per_step", "error")}), flush=True)
    print(summarize(rows))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
