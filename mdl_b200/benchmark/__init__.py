"""Benchmark and profiling entry points (kernel micro-benchmarks, single-step
runs for kernel launch lists). The headline training benchmark is ``bench.py``
at the repository root."""
