"""Benchmarks: connector microbenchmark (decode benchmark lives in bench.py)."""
