"""Token (M) sharding of the quantized linear-layer path across ranks.

Every row of the GEMM, the norm/mod/quant and the SwiGLU/quant is independent,
so a DiT step shards over tokens with the weights, scales, bias and modulation
vectors replicated and no collective on the data path.  These helpers give each
rank its contiguous slice of tokens, the modulation row of every token in that
slice (a slice may straddle the boundary between two batch elements), and the
max-over-ranks reduction used for timing.
"""
from __future__ import annotations

import numpy as np


def token_range(M: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's tokens: contiguous, sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def mod_rows(start: int, stop: int, rows_per_mod: int | None = None,
             mod_index: np.ndarray | None = None) -> np.ndarray:
    """Modulation row (batch element) of each token in [start, stop), as int32.

    Either tokens are laid out batch-major with `rows_per_mod` tokens per batch
    element (token t uses row t // rows_per_mod), or a full per-token map is
    given and sliced."""
    if mod_index is not None:
        return np.ascontiguousarray(np.asarray(mod_index, dtype=np.int32)[start:stop])
    if not rows_per_mod or rows_per_mod < 1:
        raise ValueError("rows_per_mod must be >= 1 without mod_index")
    return (np.arange(start, stop, dtype=np.int64) // rows_per_mod).astype(np.int32)


def max_over_ranks(value: float, device=None) -> float:
    """Max of a float over all ranks of the default process group (identity without one)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
