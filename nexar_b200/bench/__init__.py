"""Benchmarks shipped with nexar_b200 (run with python -m / torchrun -m)."""
