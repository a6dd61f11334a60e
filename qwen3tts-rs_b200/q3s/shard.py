"""Row sharding across GPUs (one process per GPU) and the cross-rank timing
reduction.

Rows are independent in the reference sampler: each call owns its seed,
subsequence counter and history (src/talker/sampling.rs:144-170, 247-334),
and the only coupling between rows is the order of calls within one stream
(talker.rs:500-566: codebook 0, then codebooks 1..15 of the same frame).
So a batch is split into contiguous ranges of whole streams, one per rank,
and no data crosses GPUs.  The only collective is the MAX reduction of each
rank's device time.
"""
from __future__ import annotations

from typing import Tuple


def row_range(total_rows: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [begin, end) of `total_rows` for `rank` (sizes differ by at
    most one row; earlier ranks take the extra rows)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if total_rows < 0:
        raise ValueError("total_rows must be >= 0")
    base, extra = divmod(total_rows, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def stream_range(streams: int, rows_per_stream: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [begin, end) of `rank` when every stream of `rows_per_stream`
    consecutive rows (one talker row and its code-predictor rows) must stay on
    one GPU."""
    s0, s1 = row_range(streams, world, rank)
    return s0 * rows_per_stream, s1 * rows_per_stream


def max_over_ranks(value: float, device=None) -> float:
    """MAX of `value` over the default process group (the value itself when
    torch.distributed is not initialised).  `device` is where the reduction
    tensor lives: a CUDA device under NCCL, None (CPU) under gloo."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(rows_per_rank: int, world: int, steps: int, elapsed_ms: float) -> float:
    """Rows per second of the whole job: every rank processed `rows_per_rank`
    rows per step, timed as the slowest rank (`elapsed_ms` over `steps`)."""
    if elapsed_ms <= 0:
        raise ValueError("elapsed_ms must be > 0")
    return world * rows_per_rank * steps / (elapsed_ms / 1e3)
