"""Nsight Compute collection for one kernel configuration of the gemm_bench CLI.

Port of the reference's scripts/profile.ps1 (:28-104) to B200:
  1. a section pass (SpeedOfLight, compute and memory workload, occupancy, scheduler, warp
     state, launch and instruction statistics; or --full for `--set full`) exported to
     <out-dir>/<tag>.ncu-rep;
  2. a metrics pass with a curated list (below) printed as CSV and parsed;
  3. the reference's clock-free cross-check of tensor utilisation (docs/RESULTS.md:330-366):
         busy tensor cycles = FLOP / (FLOP per clock per SM x SMs)
         dense occupancy    = busy tensor cycles / sm__cycles_elapsed.avg
     with FLOP = 2MNK and FLOP per clock per SM from the tcgen05 issue-rate probe
     (b2g_probe_tcgen05, cta_group 2 for the pair kernels), next to ncu's own
     `_sparsity_off` dense tensor metric on the elapsed basis, the one the reference trusts;
  4. a markdown summary <out-dir>/<tag>.md with the commands that made it.

On a shared GPU pool the collection is bounded: the same command line first runs without
ncu and must exit 0; every ncu command passes --clock-control none (ncu otherwise locks the
GPU clocks), one kernel (-k) and one launch (-c 1) after `skip` warm-up launches. Size the
problem so a capture ends by itself in a minute or two (a few GB on the device at most).

    python -m b2g.profile --m 4096 --n 4096 --k 4096 --tag gemm_sm100_2cta_4096
    python -m b2g.profile --m 128 --n 4096 --k 4096 --tag splitk_decode --metrics-only
    python -m b2g.profile --cublas --tag cublas_4096
"""
from __future__ import annotations

import argparse
import csv
import io
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_EXE = os.path.join(os.path.dirname(HERE), "lib", "gemm_bench")

SECTIONS = ["SpeedOfLight", "ComputeWorkloadAnalysis", "MemoryWorkloadAnalysis",
            "MemoryWorkloadAnalysis_Tables", "Occupancy", "SchedulerStats", "WarpStateStats",
            "LaunchStats", "InstructionStats"]

# The reference's metric list (scripts/profile.ps1:48-90), restated for B200. Its dense tensor
# counters (sm__ops_path_tensor_op_hmma_*_sparsity_off, scripts/profile.ps1:49-58) count
# mma.sync work only and read 0 for tcgen05 kernels (measured: ours and cuBLAS's alike), so
# the tensor pipe is read from sm__pipe_tensor_cycles_active and cross-checked, clock-free, by
# the dense occupancy from the probe's FLOP per clock per SM (which agreed with it to 0.1% on
# the 4096^3 capture). Then TMA traffic, L2 and DRAM bytes, the stall reasons of the
# reference's list, and NVLink bytes for the fused all-gather kernels.
METRICS = [
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__inst_executed_pipe_tc.sum",
    "sm__cycles_elapsed.avg",
    "sm__cycles_active.avg",
    "gpu__time_duration.sum",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "lts__throughput.avg.pct_of_peak_sustained_elapsed",
    "lts__t_sector_hit_rate.pct",
    "l1tex__m_l1tex2xbar_write_bytes_mem_global_op_tma_st.sum",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "launch__registers_per_thread",
    "launch__grid_size",
    "launch__block_size",
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_wait_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_membar_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_sleeping_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_math_pipe_throttle_per_issue_active.ratio",
    "smsp__issue_active.avg.pct_of_peak_sustained_active",
]
NVLINK_METRICS = ["nvltx__bytes_data_user.sum", "nvlrx__bytes_data_user.sum"]


def app_args(M, N, K, tile=-1, stages=0, group=0, acc="f32", splits=-1, skip=3, seed=1,
             cublas=False, extra=(), b_layout="nk"):
    """gemm_bench arguments of one profiled configuration: `skip` + 2 warm-up launches and
    one timed launch (the reference's --warmup (Skip + 2) --iters 1), uniform seeded inputs."""
    a = ["--m", str(M), "--n", str(N), "--k", str(K), "--tile", str(tile), "--stages",
         str(stages), "--group", str(group), "--acc", acc, "--warmup", str(skip + 2),
         "--iters", "1", "--init", "uniform", "--seed", str(seed), "--dist", "-1,1"]
    if splits >= 0:
        a += ["--splits", str(splits)]
    if b_layout != "nk":
        a += ["--b-layout", b_layout]
    if not cublas:
        a.append("--noref")
    return a + list(extra)


def commands(exe, args, kernel, skip, rep_path, full=False, nvlink=False, kernel_base=None):
    """(plain run, section pass, metrics pass) command lines. Every ncu command keeps the
    GPU clocks alone (--clock-control none) and captures one launch of one kernel.
    kernel_base="demangled" matches `kernel` against the full name with template arguments
    (e.g. to pick the fused all-gather instantiation `gemm_sm100_2cta<256, true>`)."""
    plain = [exe] + list(args)
    base = ["ncu", "--clock-control", "none", "--target-processes", "all"]
    if kernel_base:
        base += ["--kernel-name-base", kernel_base]
    base += ["-k", kernel, "-s", str(skip), "-c", "1"]
    sections = ["--set", "full"] if full else [x for s in SECTIONS for x in ("--section", s)]
    section_cmd = base + sections + ["--force-overwrite", "-o", rep_path] + plain
    metrics = METRICS + (NVLINK_METRICS if nvlink else [])
    metric_cmd = base + ["--csv", "--metrics", ",".join(metrics)] + plain
    return plain, section_cmd, metric_cmd


def parse_metrics_csv(text: str) -> dict:
    """ncu --csv --metrics output -> {metric name: float} for the (single) captured launch.
    Lines before the CSV header (the application's own output, ==PROF== lines) are skipped;
    values use ',' thousands separators in some ncu versions."""
    lines = text.splitlines()
    start = next((i for i, ln in enumerate(lines) if ln.startswith('"ID"')), None)
    if start is None:
        return {}
    out = {}
    for row in csv.DictReader(io.StringIO("\n".join(lines[start:]))):
        name, val = row.get("Metric Name"), row.get("Metric Value")
        if not name or val is None:
            continue
        try:
            out[name] = float(val.replace(",", ""))
        except ValueError:
            continue
    return out


def dense_occupancy(flop: float, flop_per_clk_sm: float, sms: int, cycles_elapsed: float):
    """The reference's clock-free tensor utilisation: the cycles the tensor cores of `sms`
    SMs need for `flop` at the probed rate, over the elapsed SM cycles."""
    busy = flop / (flop_per_clk_sm * sms)
    return busy, busy / cycles_elapsed


def summarize(m: dict, M: int, N: int, K: int, fpc: float | None, sms: int | None,
              gpus: int = 1) -> dict:
    """Derived figures of one captured launch; with gpus > 1 the launch is one device's
    M / gpus-row panel (gemm_bench --gpus), so FLOP and compulsory bytes are per panel."""
    Mp = M / gpus
    flop = 2.0 * Mp * N * K
    s = {"flop": flop, "compulsory_bytes": 2.0 * (Mp * K + N * K + Mp * N)}
    get = m.get
    if get("gpu__time_duration.sum"):
        t = get("gpu__time_duration.sum") * 1e-9
        s["tflops_under_ncu"] = flop / t / 1e12
    rd, wr = get("dram__bytes_read.sum"), get("dram__bytes_write.sum")
    if rd is not None and wr is not None:
        s["dram_bytes"] = rd + wr
        if get("gpu__time_duration.sum"):
            s["dram_gbs"] = (rd + wr) / (get("gpu__time_duration.sum") * 1e-9) / 1e9
    ce = get("sm__cycles_elapsed.avg")
    if fpc and sms and ce:
        busy, occ = dense_occupancy(flop, fpc, sms, ce)
        s["busy_tensor_cycles"] = busy
        s["dense_occupancy_elapsed"] = occ
        ca = get("sm__cycles_active.avg")
        if ca:
            s["dense_occupancy_active"] = busy / ca
    ta = get("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed")
    if ta is not None and "dense_occupancy_elapsed" in s:
        s["tensor_pipe_vs_dense_occupancy"] = ta / 100.0 / s["dense_occupancy_elapsed"]
    return s


def markdown(tag, cmds, m, s, M, N, K, fpc, sms) -> str:
    plain, section_cmd, metric_cmd = cmds
    cwd = os.getcwd() + os.sep
    q = lambda c: " ".join(x.replace(cwd, "") for x in c)  # noqa: E731  (paths as run)
    lines = [f"# {tag}: {M} x {N} x {K} -- ncu summary (b2g.profile)", "",
             "Commands (one GPU; the plain run exited 0 first):", "", "```", q(plain),
             q(section_cmd), q(metric_cmd), "```", "",
             "One captured launch; ncu serialises launches and runs this one from a cold L2, "
             "so compare ratios and shares, not the time.", "", "| metric | value |",
             "|---|---|"]
    for k in METRICS + NVLINK_METRICS:
        if k in m:
            lines.append(f"| {k} | {m[k]:,.4g} |")
    lines += ["", "| derived | value |", "|---|---|"]
    for k, v in s.items():
        lines.append(f"| {k} | {v:,.4g} |" if isinstance(v, float) else f"| {k} | {v} |")
    if fpc and sms:
        lines += ["", f"Dense occupancy = 2MNK / ({fpc:.1f} FLOP/clk/SM x {sms} SMs) / "
                      "sm__cycles_elapsed.avg (docs/RESULTS.md:330-366 method; FLOP/clk/SM "
                      "from b2g_probe_tcgen05)."]
    return "\n".join(lines) + "\n"


def run(M, N, K, tag, out_dir, exe=DEFAULT_EXE, tile=-1, stages=0, group=0, acc="f32",
        splits=-1, skip=3, seed=1, full=False, cublas=False, nvlink=False, kernel=None,
        metrics_only=False, fpc=None, sms=None, log=print, runner=subprocess.run,
        b_layout="nk", extra=(), kernel_base=None):
    os.makedirs(out_dir, exist_ok=True)
    kernel = kernel or ("regex:nvjet" if cublas else "regex:gemm_sm100")
    args = app_args(M, N, K, tile, stages, group, acc, splits, skip, seed, cublas, extra,
                    b_layout)
    rep = os.path.join(out_dir, tag)
    cmds = commands(exe, args, kernel, skip, rep, full, nvlink, kernel_base)
    plain, section_cmd, metric_cmd = cmds
    log("==> plain run: " + " ".join(plain))
    r = runner(plain, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"plain run exited {r.returncode}; not profiling:\n{r.stdout[-2000:]}"
                           f"{r.stderr[-2000:]}")
    if not metrics_only:
        log("==> section report -> " + rep + ".ncu-rep")
        r = runner(section_cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"ncu section pass failed ({r.returncode}):\n{r.stderr[-2000:]}")
    log("==> metric summary")
    r = runner(metric_cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ncu metrics pass failed ({r.returncode}):\n{r.stderr[-2000:]}")
    m = parse_metrics_csv(r.stdout)
    if not m:
        raise RuntimeError("ncu metrics pass printed no metric rows:\n" + r.stdout[-2000:])
    gpus = int(extra[list(extra).index("--gpus") + 1]) if "--gpus" in extra else 1
    s = summarize(m, M, N, K, fpc, sms, gpus)
    md = markdown(tag, cmds, m, s, M, N, K, fpc, sms)
    with open(rep + ".md", "w") as fh:
        fh.write(md)
    log(md)
    return {"metrics": m, "summary": s, "report": rep + ".ncu-rep", "markdown": rep + ".md"}


def probe_rate(tile: int, acc: str) -> float:
    """FLOP/clk/SM of the tcgen05 probe for the kernel family a tile uses: the pair MMA
    (cta_group 2) for the 2-CTA tiles and the automatic choice, else cta_group 1."""
    sys.path.insert(0, os.path.dirname(HERE))
    import b2g

    cg = 2 if tile in (-1, 2, 4, 6) else 1
    fpc, _ = b2g.probe_tcgen05(1 if acc == "f16" else 0, cg, 256, 4096)
    return fpc


def device_sms() -> int:
    import torch

    return torch.cuda.get_device_properties(0).multi_processor_count


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--tile", type=int, default=-1)
    p.add_argument("--stages", type=int, default=0)
    p.add_argument("--group", type=int, default=0)
    p.add_argument("--acc", choices=("f32", "f16"), default="f32")
    p.add_argument("--splits", type=int, default=-1)
    p.add_argument("--seed", type=int, default=1)
    p.add_argument("--skip", type=int, default=3, help="warm-up launches of the kernel skipped")
    p.add_argument("--tag", default="run")
    p.add_argument("--out-dir", default="ncu_out")
    p.add_argument("--exe", default=DEFAULT_EXE)
    p.add_argument("--kernel", default=None, help="ncu -k filter (default regex:gemm_sm100)")
    p.add_argument("--kernel-base", default=None, choices=("function", "demangled", "mangled"),
                   help="ncu --kernel-name-base for the -k filter")
    p.add_argument("--full", action="store_true", help="--set full instead of the sections")
    p.add_argument("--cublas", action="store_true", help="profile the cuBLAS column's kernel")
    p.add_argument("--nvlink", action="store_true", help="add NVLink tx/rx byte counters")
    p.add_argument("--metrics-only", action="store_true", help="skip the section pass")
    p.add_argument("--b-layout", choices=("nk", "kn"), default="nk")
    p.add_argument("--gpus", type=int, default=1,
                   help="gemm_bench --gpus N (M-panels over N devices of this one process)")
    p.add_argument("--allgather", action="store_true", help="gemm_bench --allgather")
    p.add_argument("--fpc", type=float, default=None,
                   help="FLOP/clk/SM for the dense-occupancy check (default: run the probe)")
    a = p.parse_args(argv)
    fpc = a.fpc or probe_rate(a.tile, a.acc)
    sms = device_sms()
    extra = (["--gpus", str(a.gpus)] if a.gpus > 1 else []) + (["--allgather"] if a.allgather else [])
    run(a.m, a.n, a.k, a.tag, a.out_dir, a.exe, a.tile, a.stages, a.group, a.acc, a.splits,
        a.skip, a.seed, a.full, a.cublas, a.nvlink, a.kernel, a.metrics_only, fpc, sms,
        b_layout=a.b_layout, extra=extra, kernel_base=a.kernel_base)
    return 0


if __name__ == "__main__":
    sys.exit(main())
