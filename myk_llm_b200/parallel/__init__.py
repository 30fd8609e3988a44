"""Process groups, data-parallel runtimes and peer-memory collectives."""

from .distributed import DistInfo, all_reduce_sum, barrier, init_distributed, parallelize, shutdown

__all__ = ["DistInfo", "all_reduce_sum", "barrier", "init_distributed", "parallelize", "shutdown"]
