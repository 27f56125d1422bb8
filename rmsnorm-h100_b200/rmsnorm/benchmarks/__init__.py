# SPDX-License-Identifier: MIT
"""Benchmark command line of the package (python -m rmsnorm.benchmarks.benchmark_rmsnorm)."""
