"""Host-side utilities: rank/env helpers, profiling, routing capture, metrics, clocks."""
from .dist import get_rank_and_world_size, init_distributed, print0, shutdown_comm

__all__ = ["get_rank_and_world_size", "init_distributed", "print0", "shutdown_comm"]
