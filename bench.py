#!/usr/bin/env python
"""Benchmark of the B200 FP16 GEMM hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload headline|f16acc|sharded] [--tile T] [--stages S] [--group G]

A step is one GEMM D = A * B over one batch of synthetic FP16 input (seeded uniform,
BASELINE.json configs). Workloads:
  headline  configs[1]: 4096^3, seed 1, U[-1,1], FP32 accumulate. Under torchrun every rank
            multiplies its own 4096-row M-panel of a (4096*N) x 4096 x 4096 GEMM with B
            replicated (no data-path collective): weak scaling.
  f16acc    configs[2]: 4096^3, seed 2, U[-0.5,0.5], FP16 accumulate (same sharding).
  sharded   configs[4]: 32768 x 32768 x 8192, seed 3, U[-1,1], FP32 accumulate; the M rows
            are split over the ranks (strong scaling); --allgather adds a timed NCCL
            all-gather of the D panels and the same gather fused into the GEMM
            (b2g_gemm_peers over CUDA IPC mappings), reported separately (any workload).

Unless --no-sharded, the bench line also carries a `sharded` object: configs[4] with its M
rows split over the ranks (strong scaling), the same run's 1-GPU time of the whole problem,
an NCCL all-gather of the D panels and the fused GEMM + all-gather (b2g_gemm_peers), each
device-timed as the max over ranks. Under torchrun NCCL's init log goes to a per-process
file and rank 0 quotes its `Init COMPLETE` line (`nccl_comm`).

`value` is whole-job TFLOP/s with inputs resident in HBM, timed with CUDA events on the
launching stream, max over ranks. Between timed iterations the inputs rotate over enough
buffer sets that the working set exceeds the 126 MB L2. `e2e` is the same metric through
the C-ABI with pinned host buffers: every step copies A and B host->device and D back
(steps pipelined over two device buffer sets on H2D, compute and D2H streams).
--impl reference times the reference's own implementation on the same workload: its CPU
GEMM code (the FP64 dot products of cpu_spot_check, src/gemm_bench.cu:672-696, compiled
from its source) on all host cores, plus its sm_89 kernel JIT-run on this B200 as an extra
column.
"""
from __future__ import annotations

import argparse
import datetime
import glob
import json
import math
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "ada-tensor-core-gemm_b200")
sys.path.insert(0, PKG)

METRIC = "TFLOP/s (4096³ FP16→FP32acc) and % of B200 dense FP16 peak; 1/2/4/8-GPU"
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    "headline": dict(M=4096, N=4096, K=4096, seed=1, lo=-1.0, hi=1.0, acc="f32", split=False,
                     name="configs[1]: 4096x4096x4096 FP16 in, FP32 acc, per GPU (M-panels)"),
    "f16acc": dict(M=4096, N=4096, K=4096, seed=2, lo=-0.5, hi=0.5, acc="f16", split=False,
                   name="configs[2]: 4096x4096x4096 FP16 in, FP16 acc, per GPU (M-panels)"),
    "sharded": dict(M=32768, N=32768, K=8192, seed=3, lo=-1.0, hi=1.0, acc="f32", split=True,
                    name="configs[4]: 32768x32768x8192 FP16 in, FP32 acc, M split over GPUs"),
}

# BASELINE configs[3] shape sweep (FP16 in, FP32 acc, U[-1,1], seed = 100 + index), and the
# reference's Phase 6 decode sweep (docs/RESULTS.md:249-265: M = 1..4096, N = K = 4096).
SWEEPS = {
    "config4": [(256, 256, 256), (512, 512, 512), (1024, 1024, 1024), (2048, 2048, 2048),
                (4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384),
                (4095, 4095, 4095), (5000, 3000, 2000), (16384, 16384, 256),
                (256, 16384, 16384)],
    "decode": [(m, 4096, 4096) for m in (1, 8, 32, 128, 512, 2048, 4096)],
}
SWEEPS["all"] = SWEEPS["config4"] + SWEEPS["decode"]
# extra shapes in the default bench line, each with its configs[3] / decode sweep seed
# (the decode shape first: the 8192^3 GEMM runs the GPU at its power cap and lowers the clock)
BENCH_SHAPES = [((128, 4096, 4096), 103), ((8192, 8192, 8192), 105)]

NVML_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
                0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
                0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
                0x100: "display_clock_setting"}


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=tuple(WORKLOADS), default="headline")
    p.add_argument("--tile", type=int, default=-1)
    p.add_argument("--stages", type=int, default=0)
    p.add_argument("--group", type=int, default=0, help="0 = chosen from the L2 size")
    p.add_argument("--e2e-steps", type=int, default=0, help="0 = min(steps, 20)")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="target CPU time of the bounded cpu_baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--allgather", action="store_true")
    p.add_argument("--no-shapes", action="store_true",
                   help="leave out the 8192^3 and decode comparisons with cuBLAS")
    p.add_argument("--no-sharded", action="store_true",
                   help="skip the configs[4] strong-scaling object (`sharded`) of the bench line")
    p.add_argument("--sweep", choices=tuple(SWEEPS), default=None,
                   help="per-shape table (one JSON line per shape, then a markdown table) "
                        "instead of the single bench line")
    p.add_argument("--soak", type=float, default=0.0,
                   help="seconds of back-to-back GEMMs of --workload in windows, with clock, "
                        "power and temperature telemetry (SOAK, lines + a summary line)")
    p.add_argument("--window", type=float, default=2.0, help="soak window seconds")
    return p.parse_args()


# ---------------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------------

def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def traffic_from_profiles(kernel_key: str):
    """DRAM bytes per launch from a committed ncu summary line
    `dram_bytes_per_launch[<kernel_key>]: <bytes>` under profiles/."""
    pat = re.compile(r"dram_bytes_per_launch\[" + re.escape(kernel_key) + r"\]:\s*([0-9.eE+]+)")
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
        with open(path) as fh:
            m = pat.search(fh.read())
        if m:
            return float(m.group(1)), os.path.relpath(path, ROOT)
    return None, None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a background thread."""

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples = []  # (t, sm_mhz, reasons_bits)
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = None
            try:
                import torch

                uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
                if not uuid.startswith("GPU-"):
                    uuid = "GPU-" + uuid
                self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode())
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[cuda_index]) if vis else cuda_index
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.err = str(e)

    def _reasons(self):
        nv = self.nv
        for fn in ("nvmlDeviceGetCurrentClocksEventReasons",
                   "nvmlDeviceGetCurrentClocksThrottleReasons"):
            if hasattr(nv, fn):
                return getattr(nv, fn)(self.h)
        return 0

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append((time.perf_counter(),
                                     self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM),
                                     self._reasons()))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def start(self):
        if not self.ok:
            return
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def mark(self, name):
        setattr(self, name, time.perf_counter())

    def stop(self):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self, t0, t1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": "NVML unavailable: " + getattr(self, "err", "?")}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside and self.samples:  # timed region shorter than the sampling period
            inside = [min(self.samples, key=lambda s: abs(s[0] - t1))]
        bits = 0
        for s in inside:
            bits |= s[2]
        reasons = sorted(n for b, n in NVML_REASONS.items() if bits & b and b != 0x1)
        return {"sm_mhz": statistics.median(s[1] for s in inside) if inside else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(inside)}


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------
def fused_allgather(full, rows, N, acc, dA, dB, stream, sptr, dev, rank, world,
                    sequential_ms, barrier, tile=-1, stages=0, group=0, reps=5):
    """GEMM and all-gather in one kernel per rank: every rank maps every other rank's full D
    through CUDA IPC and runs b2g_gemm_peers, whose epilogue stores each D box into its own
    rows of every rank's full D over NVLink. Timed like the rest (CUDA events, max over ranks)
    and checked bit for bit against an NCCL all-gather of the same GEMM's panels. `full` is
    filled with NaN on every rank before the timed steps and again before the checked step,
    so every compared byte was written by that step's TMA stores or peer stores."""
    import torch
    import torch.distributed as dist

    import b2g
    from b2g.shard import max_over_ranks

    handles = [None] * world
    dist.all_gather_object(handles, b2g.ipc_handle(full))
    bases, peers = [], []
    for p, (h, off) in enumerate(handles):
        if p != rank:
            base = b2g.ipc_open(h)
            bases.append(base)
            peers.append(base + off + rank * rows * N * 2)
    own = full[rank * rows:(rank + 1) * rows]

    def step():
        b2g.gemm_peers(dA, dB, own, peers, acc=acc, tile=tile, stages=stages, group=group,
                       stream=sptr)

    def nan_everywhere():
        full.fill_(float("nan"))
        torch.cuda.synchronize()
        barrier()  # no rank pushes into a `full` that is still being filled

    nan_everywhere()
    for _ in range(2):
        step()
    b2g.sync_status(sptr)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    b2g.sync_status(sptr)
    barrier()  # every rank's pushes into `full` have completed
    fused_ms = max_over_ranks(e0.elapsed_time(e1) / reps, dev)
    nan_everywhere()
    step()
    b2g.sync_status(sptr)
    barrier()  # the checked step's pushes have landed everywhere
    panel = torch.empty_like(own)
    b2g.gemm(dA, dB, panel, acc=acc, tile=tile, stages=stages, group=group, stream=sptr)
    b2g.sync_status(sptr)
    ref = torch.empty_like(full)
    dist.all_gather_into_tensor(ref, panel)
    torch.cuda.synchronize()
    same = torch.tensor([1 if torch.equal(ref, full) else 0], device=dev)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    barrier()  # no rank still writes through a mapping
    for base in bases:
        b2g.ipc_close(base)
    del ref
    return {"ms": fused_ms, "vs_gemm_then_allgather": round(fused_ms / sequential_ms, 4),
            "equal_to_nccl_gather": bool(same.item()),
            "check": "full D NaN-filled on every rank before the checked step",
            "how": "b2g_gemm_peers: epilogue stores each D box into every rank's D (CUDA IPC)"}


NCCL_LOG = "/tmp/b2g_nccl_{pid}.log"


def nccl_log_setup():
    """NCCL's communicator-init log (NCCL_DEBUG=INFO, subsystem INIT) goes to a per-process
    file, not to stdout, which carries the JSON line; rank 0 quotes its `Init COMPLETE` lines
    (rank, nranks) in the output. Set before the first NCCL call of the process."""
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
    os.environ["NCCL_DEBUG_FILE"] = NCCL_LOG.format(pid=os.getpid())


def nccl_log_summary(world):
    """The communicator as NCCL and torch report it (read after the process group is gone,
    so NCCL has flushed its log)."""
    import torch
    import torch.distributed as dist

    out = {"ranks_torch": world, "backend": "nccl"}
    try:
        v = torch.cuda.nccl.version()
        out["nccl_version_torch"] = ".".join(str(x) for x in v) if isinstance(v, tuple) else v
    except Exception:  # noqa: BLE001
        pass
    path = os.environ.get("NCCL_DEBUG_FILE", "")
    if path and os.path.exists(path):
        with open(path, errors="replace") as fh:
            lines = fh.read().splitlines()
        out["init_complete"] = [ln.split("NCCL INFO", 1)[-1].strip() for ln in lines
                                if "Init COMPLETE" in ln][:4]
        ver = [ln.split("NCCL INFO", 1)[-1].strip() for ln in lines if "NCCL version" in ln]
        out["version_line"] = ver[0] if ver else None
        out["log_file"] = path
    else:
        out["log_file"] = None
    return out


def sharded_leg(args, world, rank, dev, stream, sptr, barrier):
    """BASELINE configs[4] strong scaling: the 32768 x 32768 x 8192 GEMM with its M rows split
    over the ranks (B replicated), device-timed as the max over ranks; the same run's 1-GPU
    figure (rank 0 alone with the whole problem, the other ranks waiting); an NCCL
    all-gather of the D panels; and the all-gather fused into the GEMM (b2g_gemm_peers).
    No cuBLAS or end-to-end legs here, so every N fits the driver's per-run limit."""
    import torch
    import torch.distributed as dist

    import b2g
    from b2g.shard import max_over_ranks, mean_over_ranks, panel, strong_scaling

    wl = WORKLOADS["sharded"]
    M, N, K = wl["M"], wl["N"], wl["K"]
    r0, r1 = panel(M, world, rank)
    rows = r1 - r0
    f16 = torch.float16
    flop = 2.0 * M * N * K
    host = torch.empty((max(M, N), K), dtype=f16, pin_memory=True)
    dB = torch.empty((N, K), dtype=f16, device=dev)
    if rank == 0:  # B is generated once and broadcast (set-up, outside any timed region)
        b2g.fill_uniform(N * K, wl["seed"], 1, wl["lo"], wl["hi"], out=host.data_ptr())
        dB.copy_(host[:N])
    if world > 1:
        dist.broadcast(dB, src=0)
    solo = rank == 0 and world > 1
    if solo:  # rank 0 keeps all of A for the 1-GPU run; its panel is the first rows
        b2g.fill_uniform(M * K, wl["seed"], 0, wl["lo"], wl["hi"], out=host.data_ptr())
        dA_full = torch.empty((M, K), dtype=f16, device=dev)
        dA_full.copy_(host[:M])
        dA = dA_full[:rows]
    else:
        b2g.fill_uniform(rows * K, wl["seed"], 0, wl["lo"], wl["hi"], out=host.data_ptr(),
                         first=r0 * K)
        dA = torch.empty((rows, K), dtype=f16, device=dev)
        dA.copy_(host[:rows])
    del host
    dD = torch.empty((rows, N), dtype=f16, device=dev)
    torch.cuda.synchronize()
    steps, warm = max(3, min(args.steps, 10)), 2

    def time_gemm(a, d, m):
        def go():
            b2g.gemm_raw(a.data_ptr(), dB.data_ptr(), d.data_ptr(), None, m, N, K, K, K, N,
                         b2g.B_NK, b2g.ACC_F32, b2g.EPI_NONE, 1.0, b2g.TILE_AUTO, 0, 0, sptr)
        for _ in range(warm):
            go()
        b2g.sync_status(sptr)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            go()
        e1.record(stream)
        torch.cuda.synchronize()
        b2g.sync_status(sptr)
        return e0.elapsed_time(e1) / steps, b2g.kernel_clock()[0], b2g.last_launch()

    ms1 = mhz1 = None
    if solo:
        dD_full = torch.empty((M, N), dtype=f16, device=dev)
        ms1, mhz1, _ = time_gemm(dA_full, dD_full, M)
        del dD_full, dA_full
        torch.cuda.empty_cache()
    barrier()
    ms_local, mhz_local, launch = time_gemm(dA, dD, rows)
    barrier()
    ms_n = max_over_ranks(ms_local, dev)
    mhz_n = mean_over_ranks(mhz_local, dev)
    if world == 1:
        ms1, mhz1 = ms_n, mhz_n
    peaks, _ = measured_peaks()
    out = {"workload": wl["name"], "M": M, "N": N, "K": K, "rows_per_gpu": rows,
           "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": round(ms_n, 4),
           "kernel_sm_mhz_mean": round(mhz_n, 1), "launch_rank0": launch,
           "one_gpu_same_run": {"ms_per_step": round(ms1, 4) if ms1 else None,
                                "tflops": round(flop / (ms1 * 1e-3) / 1e12, 2) if ms1 else None,
                                "kernel_sm_mhz": round(mhz1, 1) if mhz1 else None},
           "timing": "CUDA events per rank around back-to-back launches, max over ranks; "
                     "inputs > L2 (B alone is 512 MiB)"}
    recv = (world - 1) * rows * N * 2
    scal = strong_scaling(flop, ms_n, world, ms1, mhz_n, mhz1,
                          recv if world > 1 else None, 770.0, peaks["bf16_tflops_sustained"])
    out.update({k: (round(v, 4) if isinstance(v, float) else v) for k, v in scal.items()})
    if world > 1:
        full = torch.empty((M, N), dtype=f16, device=dev)
        for _ in range(2):
            dist.all_gather_into_tensor(full, dD)
        torch.cuda.synchronize()
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 3
        a0.record(stream)
        for _ in range(reps):
            dist.all_gather_into_tensor(full, dD)
        a1.record(stream)
        torch.cuda.synchronize()
        ag = max_over_ranks(a0.elapsed_time(a1) / reps, dev)
        out["allgather_nccl"] = {"ms": round(ag, 4), "bytes_received_per_gpu": recv,
                                 "gbs_per_gpu": round(recv / (ag * 1e-3) / 1e9, 1),
                                 "gemm_then_allgather_ms": round(ms_n + ag, 4)}
        out["fused_gemm_allgather"] = fused_allgather(full, rows, N, b2g.ACC_F32, dA, dB,
                                                      stream, sptr, dev, rank, world, ms_n + ag,
                                                      barrier, reps=3)
        fb = out.get("fused_step_bound")
        if fb:
            out["fused_gemm_allgather"]["frac_of_roofline"] = round(
                fb["roofline_ms"] / out["fused_gemm_allgather"]["ms"], 4)
        del full
    del dA, dB, dD
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import b2g
    from b2g.shard import max_over_ranks, panel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        nccl_log_setup()
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    wl = WORKLOADS[args.workload]
    Mg, N, K = wl["M"] * (1 if wl["split"] else world), wl["N"], wl["K"]
    r0, r1 = panel(Mg, world, rank)
    rows = r1 - r0
    acc = b2g.ACC_F32 if wl["acc"] == "f32" else b2g.ACC_F16
    flop_rank = 2.0 * rows * N * K
    flop_job = 2.0 * Mg * N * K

    # pinned host inputs of this rank (its M-panel of A, all of B)
    hA = torch.empty((rows, K), dtype=torch.float16, pin_memory=True)
    hB = torch.empty((N, K), dtype=torch.float16, pin_memory=True)
    hD = torch.empty((rows, N), dtype=torch.float16, pin_memory=True)
    b2g.fill_uniform(rows * K, wl["seed"], 0, wl["lo"], wl["hi"], out=hA.data_ptr(),
                     first=r0 * K)
    b2g.fill_uniform(N * K, wl["seed"], 1, wl["lo"], wl["hi"], out=hB.data_ptr())

    set_bytes = 2 * (rows * K + N * K + rows * N)
    nbuf = max(1, min(4, math.ceil(2 * L2_BYTES / set_bytes)))
    sets = []
    for _ in range(nbuf):
        dA = torch.empty((rows, K), dtype=torch.float16, device=dev)
        dB = torch.empty((N, K), dtype=torch.float16, device=dev)
        dA.copy_(hA)
        dB.copy_(hB)
        sets.append((dA, dB, torch.empty((rows, N), dtype=torch.float16, device=dev)))
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream

    def launch(i, which="ours"):
        dA, dB, dD = sets[i % nbuf]
        if which == "ours":
            b2g.gemm_raw(dA.data_ptr(), dB.data_ptr(), dD.data_ptr(), None, rows, N, K, K, K, N,
                         b2g.B_NK, acc, b2g.EPI_NONE, 1.0, args.tile, args.stages, args.group,
                         sptr)
        else:
            b2g.cublas_gemm(dA, dB, dD, sptr)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def timed(which, steps, warmup, sampler=None):
        for i in range(warmup):
            launch(i, which)
        b2g.sync_status(sptr)
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if sampler:
            sampler.mark("t0")
        e0.record(stream)
        for i in range(steps):
            launch(i, which)
        e1.record(stream)
        torch.cuda.synchronize()
        if sampler:
            sampler.mark("t1")
        barrier()
        b2g.sync_status(sptr)
        return max_over_ranks(e0.elapsed_time(e1), dev)

    # tcgen05 issue-rate probe (FLOP/clk/SM), for the %-of-peak column
    probe_kind = 1 if acc == b2g.ACC_F16 else 0
    probe_fpc1, _ = b2g.probe_tcgen05(probe_kind, 1, 256, 4096)
    probe_fpc2, _ = b2g.probe_tcgen05(probe_kind, 2, 256, 4096)

    sampler = ClockSampler(local)
    sampler.start()
    ms = timed("ours", args.steps, args.warmup, sampler)
    sampler.stop()
    clocks = sampler.summary(sampler.t0, sampler.t1)
    # the SM clock the last timed launch actually ran at (clock64 / globaltimer in CTA 0)
    kmhz, _ = b2g.kernel_clock()
    clocks["kernel_sm_mhz"] = round(kmhz, 1)
    headline_launch = b2g.last_launch()
    # the denominator of %-of-peak is the probe of the MMA the timed kernel issues: the pair
    # MMA (cta_group::2) for the 2-CTA tiles, the one-SM MMA otherwise
    pair_kernel = headline_launch["tile"] in (b2g.TILE_256x256_2SM, b2g.TILE_256x512_2SM,
                                              b2g.TILE_256x128_2SM)
    probe_fpc = probe_fpc2 if pair_kernel else probe_fpc1

    # correctness of the timed output against cuBLAS (device max-rel, reference metric)
    dA, dB, dD = sets[(args.steps - 1) % nbuf]
    dRef = torch.empty_like(dD)
    b2g.cublas_gemm(dA, dB, dRef, sptr)
    err = torch.zeros(1, dtype=torch.float32, device=dev)
    b2g.max_rel_diff(dD, dRef, err, sptr)
    maxrel = float(err.item())
    del dRef
    ms_cublas = timed("cublas", args.steps, args.warmup)

    # e2e through the C-ABI with pinned host buffers: every step copies its A and B host ->
    # device, runs the GEMM and copies D device -> host. The steps are pipelined over two
    # device buffer sets and three streams: step i's inputs go up on the H2D stream while
    # step i - 1 computes and step i - 2's D comes down on the D2H stream (PCIe is full
    # duplex), each copy ordered after the last use of its buffer by events.
    e2e_steps = args.e2e_steps or min(args.steps, 20)
    bufs = [sets[0], sets[1 % nbuf]]
    hDs = [hD, torch.empty_like(hD, pin_memory=True)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = {k: [torch.cuda.Event(), torch.cuda.Event()] for k in ("in", "gemm", "out")}
    used = [False, False]

    def e2e_step(i):
        b = i % 2
        dA, dB, dD = bufs[b]
        if used[b]:
            s_in.wait_event(ev["gemm"][b])  # the GEMM two steps back has read these inputs
        with torch.cuda.stream(s_in):
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)
            ev["in"][b].record(s_in)
        stream.wait_event(ev["in"][b])
        if used[b]:
            stream.wait_event(ev["out"][b])  # D of two steps back has been read out
        b2g.gemm_raw(dA.data_ptr(), dB.data_ptr(), dD.data_ptr(), None, rows, N, K, K, K, N,
                     b2g.B_NK, acc, b2g.EPI_NONE, 1.0, args.tile, args.stages, args.group, sptr)
        ev["gemm"][b].record(stream)
        s_out.wait_event(ev["gemm"][b])
        with torch.cuda.stream(s_out):
            hDs[b].copy_(dD, non_blocking=True)
            ev["out"][b].record(s_out)
        used[b] = True

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    b2g.sync_status(sptr)
    barrier()
    used[0] = used[1] = False
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    for i in range(e2e_steps):
        e2e_step(i)
    for b in range(2):
        stream.wait_event(ev["out"][b])  # the timed region ends when the last D is on the host
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    b2g.sync_status(sptr)
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), dev)

    allgather = None
    if args.allgather and world > 1:
        full = torch.empty((rows * world, N), dtype=torch.float16, device=dev)
        src = sets[0][2]
        for _ in range(2):
            dist.all_gather_into_tensor(full, src)
        torch.cuda.synchronize()
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        reps = 5
        for _ in range(reps):
            dist.all_gather_into_tensor(full, src)
        a1.record(stream)
        torch.cuda.synchronize()
        ag = max_over_ranks(a0.elapsed_time(a1) / reps, dev)
        recv = (world - 1) * rows * N * 2
        allgather = {"ms": ag, "bytes_received_per_gpu": recv, "gbs_per_gpu": recv / (ag * 1e-3) / 1e9}
        allgather["fused"] = fused_allgather(full, rows, N, acc, sets[0][0], sets[0][1], stream,
                                             sptr, dev, rank, world, ms / args.steps + ag,
                                             barrier, args.tile, args.stages, args.group)
        del full

    # configs[4] strong scaling next to the (unchanged) headline; every rank takes part
    sharded = None
    if args.workload != "sharded" and not args.no_sharded:
        del sets
        torch.cuda.empty_cache()
        sharded = sharded_leg(args, world, rank, dev, stream, sptr, barrier)

    # the north star's other square (8192^3) and a decode shape, each against the reference's
    # cuBLAS call in the same run (1 GPU only: the scaling runs keep their per-N time)
    shapes = None
    if world == 1 and not args.no_shapes:
        side = torch.cuda.Stream(device=dev)  # graphs are captured on a non-default stream
        shapes = []
        with torch.cuda.stream(side):
            for (M, N, K), seed in BENCH_SHAPES:
                row, _, _ = shape_vs_cublas(M, N, K, seed, 50, 10, side)
                shapes.append({k: row[k] for k in (
                    "M", "N", "K", "seed", "ms", "tflops", "cublas_tflops", "ours_over_cublas",
                    "maxrel_vs_cublas", "roofline", "hbm_gbs_algorithmic", "launch",
                    "kernel_sm_mhz")})
        torch.cuda.synchronize()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(hA.numpy().view(np.uint16), hB.numpy().view(np.uint16), N, K,
                           args.cpu_seconds, wl)

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    nccl = nccl_log_summary(world) if world > 1 else None

    peaks, peak_src = measured_peaks()
    per_launch_ms = ms / args.steps
    achieved = flop_rank / (per_launch_ms * 1e-3) / 1e12
    sustained = ms > 1000.0
    peak = peaks["bf16_tflops_sustained" if sustained else "bf16_tflops"]
    kernel_key = f"gemm_sm100_{args.workload}"
    traffic, traffic_src = traffic_from_profiles(kernel_key)
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    sm_mhz = (clocks.get("kernel_sm_mhz") or clocks.get("sm_mhz")
              or peaks.get("clocks_under_load", {}).get("sm_mhz_median"))
    probe_peak = probe_fpc * sms * sm_mhz * 1e6 / 1e12 if sm_mhz else None
    value = flop_job * args.steps / (ms * 1e-3) / 1e12
    h2d = 2 * (rows * K + N * K)
    d2h = 2 * rows * N
    out = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "strong" if wl["split"] else "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic: seeded counter-based uniform FP16 (BASELINE.json seeds/ranges)",
        "config": {
            "workload": wl["name"], "M_total": Mg, "M_per_gpu": rows, "N": N, "K": K,
            "acc": wl["acc"], "seed": wl["seed"], "dist": [wl["lo"], wl["hi"]],
            "tile": args.tile, "stages": args.stages, "group": args.group,
            "parallelism": f"M-row panels x{world}, B replicated, no data-path collective",
            "l2": f"{nbuf} rotating input sets of {set_bytes / 2**20:.0f} MiB "
                  f"({nbuf * set_bytes / 2**20:.0f} MiB > 126 MiB L2)",
        },
        "roofline": {
            "bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
            "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "peak_source": f"{peak_src} cuBLAS bf16 "
                           f"{'sustained' if sustained else 'burst'} (MEASURED_PEAKS.json)",
            "traffic": traffic, "traffic_source": traffic_src,
            "algorithmic_flop_per_launch": flop_rank,
            "algorithmic_bytes_per_launch": 2 * (rows * K + N * K + rows * N),
        },
        "pct_probe_peak": round(100 * achieved / probe_peak, 2) if probe_peak else None,
        "probe": {"flop_per_clk_sm": round(probe_fpc, 1),
                  "cta_group": 2 if pair_kernel else 1,
                  "flop_per_clk_sm_cta_group_1": round(probe_fpc1, 1),
                  "flop_per_clk_sm_cta_group_2": round(probe_fpc2, 1),
                  "timed_launch": headline_launch, "sms": sms, "sm_mhz": sm_mhz,
                  "peak_tflops": round(probe_peak, 1) if probe_peak else None},
        "cublas_tflops": round(flop_job * args.steps / (ms_cublas * 1e-3) / 1e12, 3),
        "maxrel_vs_cublas": maxrel,
        "e2e": {"value": round(flop_job * e2e_steps / (ms_e2e * 1e-3) / 1e12, 3),
                "unit": "TFLOP/s", "h2d_bytes_per_step": h2d * world,
                "d2h_bytes_per_step": d2h * world, "steps": e2e_steps,
                "how": "every step: pinned H2D of A and B, the GEMM through the C-ABI, D2H of "
                       "D; steps pipelined over 2 buffer sets on H2D / compute / D2H streams"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "shapes_vs_cublas": shapes,
    }
    if cpu:
        out["cpu_baseline"] = cpu
    if allgather:
        out["allgather"] = allgather
    if sharded:
        out["sharded"] = sharded
    if nccl:
        out["nccl_comm"] = nccl
    print(json.dumps(out), flush=True)


def cpu_baseline(A, B, N, K, seconds, wl):
    """Blocked FP32 CPU GEMM (the oracle's, all OpenMP threads) on a bounded row sample."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    O.lib()
    t = time.perf_counter()
    O.gemm_f32_blocked(A, B, 0, 0, 16)
    dt = max(time.perf_counter() - t, 1e-6)
    rows = int(min(A.shape[0], max(16, 16 * seconds / dt)))
    t = time.perf_counter()
    _, threads = O.gemm_f32_blocked(A, B, 0, 0, rows)
    dt = time.perf_counter() - t
    return {"value": round(2.0 * rows * N * K / dt / 1e12, 5), "unit": "TFLOP/s",
            "cores": threads, "kind": "port",
            "sample": f"{rows} of {A.shape[0]} rows of the {wl['M']}x{N}x{K} GEMM, blocked "
                      f"FP32 (oracle/oracle.c orc_gemm_f32_blocked), {dt:.1f} s"}


# ---------------------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------------------
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import oracle as O

    wl = WORKLOADS[args.workload]
    M, N, K = wl["M"], wl["N"], wl["K"]
    if not O.ref_available():
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref/libref.so was not built (needs the "
                                         "reference checkout at build time)"}))
        return
    R = O.ref()
    A = O.fill_uniform((M, K), wl["seed"], 0, wl["lo"], wl["hi"])
    B = O.fill_uniform((N, K), wl["seed"], 1, wl["lo"], wl["hi"])
    D = np.zeros((M, N), np.uint16)
    try:
        threads = len(os.sched_getaffinity(0))
    except AttributeError:
        threads = os.cpu_count() or 1
    # calibrate: one row per thread
    t = R.ref_cpu_rows(A, B, D, M, N, K, 0, threads, threads)
    rate = 2.0 * threads * N * K / max(t, 1e-6)  # FLOP/s
    budget = 90.0
    t_step = budget / max(1, args.steps + args.warmup)
    rows = int(max(threads, min(M, rate * t_step / (2.0 * N * K))))
    for i in range(args.warmup):
        R.ref_cpu_rows(A, B, D, M, N, K, (i * rows) % max(1, M - rows + 1), rows, threads)
    tot = 0.0
    for i in range(args.steps):
        tot += R.ref_cpu_rows(A, B, D, M, N, K, (i * rows) % max(1, M - rows + 1), rows, threads)
    value = 2.0 * rows * N * K * args.steps / tot / 1e12
    sample = (f"{rows} of {M} output rows per step (every element of those rows, FP64 dot "
              f"products), {threads} host threads")
    out = {
        "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tot / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if wl["split"] else "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic: seeded counter-based uniform FP16 (BASELINE.json seeds/ranges)",
        "config": {"workload": wl["name"], "M": M, "N": N, "K": K, "acc": wl["acc"],
                   "seed": wl["seed"], "dist": [wl["lo"], wl["hi"]]},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads,
                         "kind": "reference",
                         "sample": sample + "; cpu_spot_check from src/gemm_bench.cu "
                                            "compiled from the reference's source"},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    try:
        out["ref_sm89_on_b200"] = ref_kernel_on_gpu(R, A, B, M, N, K, wl, args)
    except Exception as e:  # noqa: BLE001
        out["ref_sm89_on_b200"] = {"unavailable": str(e)[:200]}
    print(json.dumps(out), flush=True)


def ref_kernel_on_gpu(R, A, B, M, N, K, wl, args):
    """The reference's own sm_89 kernel (README best config: tile 3, 3 stages, swizzle,
    group 2, MMA_K8; or its FP16-accumulate build) JIT-run on this B200."""
    import numpy as np
    import torch

    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    variant = 2 if wl["acc"] == "f16" else 3
    dA = torch.from_numpy(A.view(np.float16)).cuda()
    dB = torch.from_numpy(B.view(np.float16)).cuda()
    nbuf = 3
    Ds = [torch.empty((M, N), dtype=torch.float16, device="cuda") for _ in range(nbuf)]
    As = [dA] + [dA.clone() for _ in range(nbuf - 1)]
    Bs = [dB] + [dB.clone() for _ in range(nbuf - 1)]
    s = torch.cuda.current_stream()

    def launch(i):
        rc = R.ref_gemm_launch(variant, As[i % nbuf].data_ptr(), Bs[i % nbuf].data_ptr(),
                               Ds[i % nbuf].data_ptr(), None, M, N, K, 1.0, 2, 3, 3, 2,
                               s.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"reference kernel launch failed: cudaError {rc}")

    for i in range(max(3, args.warmup)):
        launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(args.steps):
        launch(i)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    return {"tflops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 3), "ms_per_step": ms,
            "kernel": "gemm_kernel<128,128,32,2,2,3,SWZ> MMA_K8" if variant == 3
            else "gemm_kernel<128,128,32,2,2,3,SWZ> ACC_F16",
            "build": "compute_89 PTX from src/gemm_bench.cu, JIT by the driver"}


# ---------------------------------------------------------------------------------------
# shape sweep and soak -- single GPU, rank 0
# ---------------------------------------------------------------------------------------
def _ld8(k):
    return (k + 7) // 8 * 8  # TMA row strides are multiples of 16 bytes: pad odd K


def _time_launches(launch, steps, warmup, stream):
    """Mean device ms per launch of back-to-back launches; launch(i) uses input set i % n,
    the sets together larger than L2, so no launch finds its inputs in L2."""
    import torch

    for i in range(warmup):
        launch(i + 7919)  # sets far from the first timed ones
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        launch(i)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _capture(launch, n, stream):
    """n launches (input set i % sets, as in _time_launches) captured in one CUDA graph."""
    import torch

    for i in range(3):
        launch(i + 7919)  # any lazily sized scratch exists before the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n):
            launch(i)
    g.replay()
    torch.cuda.synchronize()
    return g


def _replay_ms(g, n, stream, replays=5):
    """Device ms per launch of `replays` back-to-back replays of a graph of n launches."""
    import torch

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(replays):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / (replays * n)


def _time_graph(launch, n, stream, replays=5):
    """Device time per launch: n launches captured in one CUDA graph, replayed back to back.
    Unlike a host loop of C-ABI calls, whose ~6-12 us of host work per call can exceed a small
    GEMM's device time, this times only the GPU."""
    g = _capture(launch, n, stream)
    ms = _replay_ms(g, n, stream, replays)
    del g
    return ms


def shape_vs_cublas(M, N, K, seed, steps, warmup, stream, tile=-1, stages=0, group=0):
    """One GEMM shape, ours and the reference's cuBLAS call on the same inputs: device time per
    launch from CUDA-graph replay (input sets rotated, together > 2 x L2), the host-loop time
    through each C-ABI beside it, max-rel vs cuBLAS, roofline fraction against
    min(measured tensor peak, AI x measured HBM bandwidth) and the algorithmic HBM GB/s.
    Returns (row, hA, hB); `stream` must be a non-default stream (graphs are captured on it)."""
    import numpy as np
    import torch

    import b2g

    sptr = stream.cuda_stream
    peaks, _ = measured_peaks()
    bw = peaks["hbm_gbs"]
    ptc = peaks["bf16_tflops"]
    ld = _ld8(K)
    hA = np.zeros((M, ld), np.uint16)
    hB = np.zeros((N, ld), np.uint16)
    hA[:, :K] = b2g.fill_uniform(M * K, seed, 0, -1.0, 1.0).reshape(M, K)
    hB[:, :K] = b2g.fill_uniform(N * K, seed, 1, -1.0, 1.0).reshape(N, K)
    # rotating input sets whose total exceeds twice the L2 (at least 2 sets)
    set_bytes = 2 * (M * ld + N * ld + M * N)
    nbuf = max(2, min(4096, math.ceil(2 * L2_BYTES / set_bytes)))
    dA0 = torch.from_numpy(hA.view(np.float16)).cuda()
    dB0 = torch.from_numpy(hB.view(np.float16)).cuda()
    sets = [(dA0.clone(), dB0.clone(), torch.empty((M, N), dtype=torch.float16,
                                                   device="cuda")) for _ in range(nbuf)]
    del dA0, dB0
    flop = 2.0 * M * N * K
    # every set at least once per timed run (a set comes round again only after sets
    # totalling > 2 x L2 have been read), and about a second of GPU time at most
    steps = max(5, min(steps, int(2e15 / max(flop, 1) / 1000) + 5), min(nbuf, 4096))
    warm = max(3, min(warmup, steps))

    def ours(i):
        dA, dB, dD = sets[i % nbuf]
        b2g.gemm_raw(dA.data_ptr(), dB.data_ptr(), dD.data_ptr(), None, M, N, K, ld, ld, N,
                     b2g.B_NK, b2g.ACC_F32, b2g.EPI_NONE, 1.0, tile, stages, group, sptr)

    # device time (graph replay) is the figure; the host loop through the C-ABI is kept
    # beside it, since at decode sizes its host work per call can bound the loop
    ms_loop = _time_launches(ours, steps, warm, stream)
    n_graph = min(steps, 1024)
    g_ours = _capture(ours, n_graph, stream)
    b2g.sync_status(sptr)
    launch = b2g.last_launch()
    kmhz, _ = b2g.kernel_clock()
    # the reference's cuBLAS call takes lda = ldb = K: unpadded copies when K % 8 != 0
    csets = sets if ld == K else [(a[:, :K].contiguous(), b[:, :K].contiguous(), d)
                                  for a, b, d in sets]

    def cub(i):
        dA, dB, dD = csets[i % nbuf]
        b2g.cublas_gemm(dA, dB, dD, sptr)

    dRef = torch.empty((M, N), dtype=torch.float16, device="cuda")
    b2g.cublas_gemm(csets[0][0], csets[0][1], dRef, sptr)
    ours(0)
    err = torch.zeros(1, dtype=torch.float32, device="cuda")
    b2g.max_rel_diff(sets[0][2], dRef, err, sptr)
    maxrel = float(err.item())
    del dRef
    cublas_ms_loop = _time_launches(cub, steps, warm, stream)
    g_cub = _capture(cub, n_graph, stream)
    # the two arms' replays alternate, three rounds, best of each: the SM clock drifts under
    # the 1 kW cap (e.g. after a power-heavy shape), and alternation gives both arms the same
    ms, cublas_ms = float("inf"), float("inf")
    for _ in range(3):
        ms = min(ms, _replay_ms(g_ours, n_graph, stream))
        cublas_ms = min(cublas_ms, _replay_ms(g_cub, n_graph, stream))
    b2g.sync_status(sptr)
    del g_ours, g_cub, csets
    alg_bytes = 2.0 * (M * K + N * K + M * N)
    ai = flop / alg_bytes
    roof = min(ptc, ai * bw / 1e3)  # TFLOP/s
    tf = flop / (ms * 1e-3) / 1e12
    ctf = flop / (cublas_ms * 1e-3) / 1e12 if cublas_ms else None
    row = {
        "M": M, "N": N, "K": K, "seed": seed, "ms": round(ms, 5), "tflops": round(tf, 2),
        "cublas_tflops": round(ctf, 2) if ctf else None,
        "ours_over_cublas": round(tf / ctf, 4) if ctf else None,
        "timing": "device time per launch: CUDA-graph replay of the launches, the two arms' "
                  "replays alternating, best of 3 each",
        "ms_api_loop": round(ms_loop, 5),
        "cublas_ms_api_loop": round(cublas_ms_loop, 5),
        "maxrel_vs_cublas": maxrel,
        "roofline": {"bound": "tensor" if ai * bw / 1e3 >= ptc else "hbm",
                     "ai_flop_per_byte": round(ai, 1), "peak_tflops": round(roof, 1),
                     "frac": round(tf / roof, 4)},
        "hbm_gbs_algorithmic": round(alg_bytes / (ms * 1e-3) / 1e9, 1),
        "launch": launch, "kernel_sm_mhz": round(kmhz),
        "l2": f"{nbuf} rotating input sets, {nbuf * set_bytes / 2**20:.0f} MiB > 2 x L2",
    }
    del sets
    torch.cuda.empty_cache()
    return row, hA, hB


def sweep_ours(args):
    """Per shape: our kernel and cuBLAS (shape_vs_cublas) and a blocked FP32 CPU GEMM on a
    bounded row sample (the cpu_baseline leg)."""
    import torch

    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()  # CUDA graphs are captured on a non-default stream
    torch.cuda.set_stream(stream)
    peaks, peak_src = measured_peaks()
    bw = peaks["hbm_gbs"]
    ptc = peaks["bf16_tflops"]
    rows_out = []
    for idx, (M, N, K) in enumerate(SWEEPS[args.sweep]):
        row, hA, hB = shape_vs_cublas(M, N, K, 100 + idx, args.steps, args.warmup, stream,
                                      args.tile, args.stages, args.group)
        if not args.no_cpu_baseline:
            row["cpu_baseline"] = cpu_baseline(hA[:, :K].copy(), hB[:, :K].copy(), N, K,
                                               min(args.cpu_seconds, 2.0),
                                               {"M": M})
        print(json.dumps(row), flush=True)
        rows_out.append(row)
        del hA, hB
    print(f"\n| M | N | K | ours TFLOP/s | cuBLAS | ours/cuBLAS | bound | frac of roofline "
          f"({peak_src} {ptc:.0f} TF/s, {bw:.0f} GB/s) | HBM GB/s | us ours / cuBLAS (host "
          f"loop) | CPU FP32 TFLOP/s |")
    print("|---:|---:|---:|---:|---:|---:|---|---:|---:|---:|---:|")
    for r in rows_out:
        c = r["cublas_tflops"]
        cpu = r.get("cpu_baseline", {}).get("value")
        print(f"| {r['M']} | {r['N']} | {r['K']} | {r['tflops']:.1f} | "
              f"{c if c is not None else '-'} | "
              f"{(r['tflops'] / c) if c else float('nan'):.3f} | {r['roofline']['bound']} | "
              f"{r['roofline']['frac']:.3f} | {r['hbm_gbs_algorithmic']:.0f} | "
              f"{r['ms_api_loop'] * 1e3:.1f} / {r['cublas_ms_api_loop'] * 1e3:.1f} | "
              f"{cpu if cpu is not None else '-'} |")


def sweep_reference(args):
    """Per shape: the reference's sm_89 kernel JIT-run on this B200 (README best config) and
    its CPU code (cpu_spot_check's FP64 dot products) on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref.so not built"}))
        return
    R = O.ref()
    try:
        threads = len(os.sched_getaffinity(0))
    except AttributeError:
        threads = os.cpu_count() or 1
    for idx, (M, N, K) in enumerate(SWEEPS[args.sweep]):
        seed = 100 + idx
        row = {"impl": "reference", "M": M, "N": N, "K": K, "seed": seed}
        if K % 32 or N % 2:  # the reference's own requirement (src/gemm_bench.cu:746)
            row["ref_sm89_on_b200"] = {"skip": "the reference requires K % 32 == 0"}
        else:
            A = O.fill_uniform((M, K), seed, 0, -1.0, 1.0)
            B = O.fill_uniform((N, K), seed, 1, -1.0, 1.0)
            wl = {"acc": "f32"}
            a2 = argparse.Namespace(steps=max(3, min(args.steps, 20)), warmup=3)
            try:
                row["ref_sm89_on_b200"] = ref_kernel_on_gpu(R, A, B, M, N, K, wl, a2)
            except Exception as e:  # noqa: BLE001
                row["ref_sm89_on_b200"] = {"unavailable": str(e)[:200]}
            import numpy as np

            D = np.zeros((M, N), np.uint16)
            rows = min(M, threads)
            t = R.ref_cpu_rows(A, B, D, M, N, K, 0, rows, threads)
            row["reference_cpu"] = {"tflops": round(2.0 * rows * N * K / max(t, 1e-9) / 1e12, 6),
                                    "cores": threads, "sample": f"{rows} output rows"}
        print(json.dumps(row), flush=True)


class Telemetry(ClockSampler):
    """ClockSampler plus memory clock, power, temperature and utilisation (soak)."""

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append((
                    time.perf_counter(), nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                    self._reasons(), nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_MEM),
                    nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0,
                    nv.nvmlDeviceGetTemperature(self.h, nv.NVML_TEMPERATURE_GPU),
                    nv.nvmlDeviceGetUtilizationRates(self.h).gpu))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)


def soak_ours(args):
    """Back-to-back GEMMs of --workload for --soak seconds in --window windows (the
    reference's soak mode, src/gemm_bench.cu SOAK lines and scripts/soak.ps1 telemetry)."""
    import torch

    import b2g

    wl = WORKLOADS[args.workload]
    M, N, K = wl["M"], wl["N"], wl["K"]
    acc = b2g.ACC_F32 if wl["acc"] == "f32" else b2g.ACC_F16
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    nbuf = 3
    sets = []
    hA = b2g.fill_uniform(M * K, wl["seed"], 0, wl["lo"], wl["hi"]).reshape(M, K)
    hB = b2g.fill_uniform(N * K, wl["seed"], 1, wl["lo"], wl["hi"]).reshape(N, K)
    import numpy as np

    for _ in range(nbuf):
        sets.append((torch.from_numpy(hA.view(np.float16)).cuda(),
                     torch.from_numpy(hB.view(np.float16)).cuda(),
                     torch.empty((M, N), dtype=torch.float16, device="cuda")))
    flop = 2.0 * M * N * K

    def launch(i):
        dA, dB, dD = sets[i % nbuf]
        b2g.gemm_raw(dA.data_ptr(), dB.data_ptr(), dD.data_ptr(), None, M, N, K, K, K, N,
                     b2g.B_NK, acc, b2g.EPI_NONE, 1.0, args.tile, args.stages, args.group, sptr)

    for i in range(max(3, args.warmup)):
        launch(i)
    b2g.sync_status(sptr)
    tel = Telemetry(0, period_s=0.2)
    tel.start()
    print(f"# soak {args.soak:.0f} s, window {args.window:.1f} s, {wl['name']}")
    print("SOAK,elapsed_s,window_ms,iters,tflops,ms_per_iter", flush=True)
    t_start = time.perf_counter()
    wins = []
    i = 0
    while time.perf_counter() - t_start < args.soak:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        n = 0
        w0 = time.perf_counter()
        while time.perf_counter() - w0 < args.window:
            launch(i)
            i += 1
            n += 1
            if n % 64 == 0:
                e1.record(stream)
                e1.synchronize()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        tf = flop * n / (ms * 1e-3) / 1e12
        wins.append(tf)
        print(f"SOAK,{time.perf_counter() - t_start:.2f},{ms:.1f},{n},{tf:.2f},{ms / n:.5f}",
              flush=True)
    tel.stop()
    b2g.sync_status(sptr)
    busy = [s for s in tel.samples if len(s) > 6 and s[6] >= 50]

    def stat(k):
        v = [s[k] for s in busy]
        return {"avg": round(statistics.mean(v), 1), "min": min(v), "max": max(v)} if v else None

    def drift(vals):
        k = len(vals) // 3
        if k < 1:
            return None
        a, b = statistics.mean(vals[:k]), statistics.mean(vals[-k:])
        return {"first_third": round(a, 2), "last_third": round(b, 2),
                "pct": round(100 * (b - a) / a, 2) if a else None}

    bits = [s[2] for s in busy]
    reasons = {n: sum(1 for b in bits if b & m) for m, n in NVML_REASONS.items() if m != 0x1}
    out = {"soak": {
        "workload": wl["name"], "seconds": args.soak, "window_s": args.window,
        "windows": len(wins), "sustained_tflops": round(statistics.mean(wins), 2) if wins else None,
        "tflops_min": round(min(wins), 2) if wins else None,
        "tflops_max": round(max(wins), 2) if wins else None,
        "tflops_drift": drift(wins),
        "busy_samples": len(busy), "sm_mhz": stat(1), "mem_mhz": stat(3), "power_w": stat(4),
        "temp_c": stat(5),
        "sm_mhz_drift": drift([s[1] for s in busy]), "power_drift": drift([s[4] for s in busy]),
        "temp_drift": drift([s[5] for s in busy]),
        "reason_samples": {k: v for k, v in reasons.items() if v},
    }}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        if args.sweep:
            sweep_reference(args)
        else:
            run_reference(args)
    elif args.sweep:
        sweep_ours(args)
    elif args.soak > 0:
        soak_ours(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
