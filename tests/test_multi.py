"""Multi-rank host logic on CPU: two gloo ranks shard a GEMM by M-row panels (the oracle
computes each rank's panel), gather the panels and check the result equals the full product;
the max-over-ranks timing reduction; panel arithmetic."""
import os
import socket

import numpy as np
import pytest

from b2g.shard import gather_panels, max_over_ranks, panel


def test_panels_cover_rows_exactly():
    for M in (1, 7, 4096, 32768, 4097):
        for W in (1, 2, 3, 4, 8):
            if W > M:
                continue
            spans = [panel(M, W, r) for r in range(W)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        panel(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_q):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [os.path.join(root, "ada-tensor-core-gemm_b200"), os.path.join(root, "oracle")]
    import torch
    import torch.distributed as dist

    import oracle as O
    from b2g.shard import gather_panels, max_over_ranks, mean_over_ranks, panel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, N, K = 64, 40, 48
        r0, r1 = panel(M, world, rank)
        # every rank generates only its own rows of A (counter-based generator) and all of B
        A_panel = O.fill_uniform((r1 - r0, K), 3, 0, first=r0 * K)
        B = O.fill_uniform((N, K), 3, 1)
        D_panel = torch.from_numpy(O.gemm_f64(A_panel, B))
        full = gather_panels(D_panel, M // world)
        slowest = max_over_ranks(10.0 + rank)
        mean = mean_over_ranks(1000.0 + 10.0 * rank)
        if rank == 0:
            A = O.fill_uniform((M, K), 3, 0)
            ref = O.gemm_f64(A, B)
            result_q.put((float(np.max(np.abs(full.numpy() - ref))), slowest, mean))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    err, slowest, mean = q.get()
    assert err == 0.0  # row panels of an FP64 product are exactly the full product's rows
    assert slowest == 11.0  # max over ranks
    assert mean == 1005.0  # mean over ranks (e.g. the SM clock each rank's kernel ran at)


def test_single_process_helpers():
    assert max_over_ranks(3.5) == 3.5


def test_strong_scaling_summary():
    """The `sharded` object's arithmetic: speed-up and efficiency against the same run's
    1-GPU time, the clock-normalised speed-up, and what bounds the fused GEMM + all-gather."""
    from b2g.shard import strong_scaling

    flop = 2.0 * 32768 * 32768 * 8192
    s = strong_scaling(flop, 1.5, 8, ms_1=12.0, mhz_n=1350.0, mhz_1=1170.0,
                       gather_bytes_per_gpu=7 * 4096 * 32768 * 2, link_gbs=770.0,
                       gemm_peak_tflops=1376.0)
    assert s["speedup_vs_1gpu"] == 8.0 and s["efficiency"] == 1.0
    assert abs(s["speedup_clock_normalised"] - 8.0 * 1170.0 / 1350.0) < 1e-12
    assert abs(s["tflops"] - flop / 1.5e-3 / 1e12) < 1e-6
    fb = s["fused_step_bound"]
    assert fb["limit"] == "all-gather (NVLink)"  # 1.88 GB at 770 GB/s > 2.2 TFLOP at peak
    assert abs(fb["gather_ms_at_link"] - 7 * 4096 * 32768 * 2 / 770e9 * 1e3) < 1e-9
    assert fb["roofline_ms"] == fb["gather_ms_at_link"]
    one = strong_scaling(flop, 12.0, 1)
    assert "efficiency" not in one and "fused_step_bound" not in one
