"""Parallel runtime: mesh math, process groups, symmetric peer memory, sequence / tensor / CFG parallelism."""
