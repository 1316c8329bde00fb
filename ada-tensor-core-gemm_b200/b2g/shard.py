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


def mean_over_ranks(value: float, device=None) -> float:
    """Mean of a per-rank float (e.g. the SM clock a kernel ran at) over the process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item()) / dist.get_world_size()


def strong_scaling(flop: float, ms_n: float, world: int, ms_1: float | None = None,
                   mhz_n: float | None = None, mhz_1: float | None = None,
                   gather_bytes_per_gpu: float | None = None, link_gbs: float | None = None,
                   gemm_peak_tflops: float | None = None) -> dict:
    """Strong-scaling figures of one GEMM of `flop` FLOP split over `world` GPUs that took
    ms_n (max over ranks), against ms_1 on one GPU: speed-up, efficiency (speed-up / world)
    and the clock-normalised speed-up (time x SM MHz, so a run that clocked higher does not
    look superlinear). With the all-gather's bytes received per GPU and a link bandwidth it
    also names what bounds the fused GEMM + all-gather step: the larger of the GEMM time at
    the tensor peak and the gather time at the link bandwidth."""
    out = {"tflops": flop / (ms_n * 1e-3) / 1e12, "tflops_per_gpu": flop / (ms_n * 1e-3) / 1e12 / world}
    if ms_1:
        out["speedup_vs_1gpu"] = ms_1 / ms_n
        out["efficiency"] = ms_1 / ms_n / world
        if mhz_n and mhz_1:
            out["speedup_clock_normalised"] = (ms_1 * mhz_1) / (ms_n * mhz_n)
    if gather_bytes_per_gpu is not None and link_gbs and gemm_peak_tflops:
        t_gemm = flop / world / (gemm_peak_tflops * 1e12) * 1e3
        t_link = gather_bytes_per_gpu / (link_gbs * 1e9) * 1e3
        out["fused_step_bound"] = {"gemm_ms_at_peak": t_gemm, "gather_ms_at_link": t_link,
                                   "limit": "all-gather (NVLink)" if t_link > t_gemm else "GEMM",
                                   "roofline_ms": max(t_gemm, t_link)}
    return out


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
