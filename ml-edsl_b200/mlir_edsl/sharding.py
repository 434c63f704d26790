"""Row sharding of the dense layer across GPUs (one process per GPU).

Y[r] = act(X[r] @ W + b) depends only on row r, so rows split into
contiguous shards with no exchange; W and b are replicated. The partition is
the one the C runtime uses for its multi-device host calls (run_sharded in
csrc/runtime.cu): M // n rows each, the first M % n shards one row more.
"""
from typing import List, Tuple


def row_shards(M: int, n: int) -> List[Tuple[int, int]]:
    """(first_row, rows) for each of n shards of M rows."""
    if n < 1:
        raise ValueError("n must be >= 1")
    base, rem = divmod(M, n)
    out, r0 = [], 0
    for i in range(n):
        rows = base + (1 if i < rem else 0)
        out.append((r0, rows))
        r0 += rows
    return out


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a per-rank float over the process group (identity without one).
    Used for timings: a multi-GPU step takes as long as its slowest rank."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
