"""Multi-GPU fold: independent context windows dealt to the GPUs of one node.

Fold windows are independent units (crates/taco/src/gpu_fold.rs:128-186: each window restarts its
context), so each GPU runs its own windows with no collective on the data path; the host gathers
the coded chunks in window order. `deal` is that round-robin split, and `max_over_ranks` the one
collective the benchmark needs: the slowest rank's device time (torch.distributed, NCCL on GPUs,
gloo in the CPU tests).
"""

from __future__ import annotations

import numpy as np


def deal(n_windows: int, world: int, rank: int) -> np.ndarray:
    """The window indices of `rank`: windows rank, rank + world, rank + 2 world, ..."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    return np.arange(rank, n_windows, world, dtype=np.int64)


def gather_order(n_windows: int, world: int) -> np.ndarray:
    """For the concatenation of every rank's windows (rank 0's first), the window index of each
    position: the host's gather back into window order inverts it."""
    return np.concatenate([deal(n_windows, world, r) for r in range(world)])


def max_over_ranks(values: list[float], device=None) -> list[float]:
    """The element-wise max over the ranks of the default process group (identity without one)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]
