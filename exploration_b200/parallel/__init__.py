"""Parallelism: DP x CP contexts, Ulysses exchanges, gradient reduction."""
from .context import ParallelContext, init_distributed, process_group_timeout, sum_all

__all__ = ["ParallelContext", "init_distributed", "process_group_timeout", "sum_all"]
