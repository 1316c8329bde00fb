"""M-row panel sharding of D = A * B over ranks (one process per GPU).

D's rows are independent, so rank r of W computes rows [r*M/W, (r+1)*M/W) with all of B
replicated: no data-path collective. These helpers are shared by bench.py and the tests; the
optional all-gather of the D panels uses torch.distributed (NCCL on GPUs, gloo on CPU).
The reference has no multi-GPU code; this follows the sharding BASELINE configs[4] asks for.
"""
from __future__ import annotations


def panel(M: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of `rank` when M rows are split as evenly as possible."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return M * rank // world, M * (rank + 1) // world


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank float (e.g. elapsed ms) over the default process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_panels(local, rows_per_rank: int):
    """All-gather equal-height D panels (rows_per_rank x N) into the full matrix on every
    rank. Requires M divisible by the world size (bench.py's sharded workload is)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size()
    if local.shape[0] != rows_per_rank:
        raise ValueError("panels must all have rows_per_rank rows")
    full = torch.empty((rows_per_rank * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                       device=local.device)
    dist.all_gather_into_tensor(full, local.contiguous())
    return full
