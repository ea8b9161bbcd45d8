"""Reference-arm harness for bench.py (the reference itself is installed under baseline/_ref)."""
