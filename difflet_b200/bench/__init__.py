"""Benchmark harnesses: kernel microbenchmarks and end-to-end pipeline timing."""
