"""Sustained-load soak of the gemm_bench CLI with clock / power / temperature telemetry.

Port of the reference's scripts/soak.ps1: runs ``gemm_bench --soak SECONDS --window W`` (its
``SOAK,`` lines go to <out-dir>/<tag>.throughput.txt) while sampling nvidia-smi every
--sample-ms into <out-dir>/<tag>.telemetry.csv with the reference's columns (t, smMHz,
memMHz, powerW, tempC, utilPct and the five throttle-reason flags), then prints the same
correlation: statistics over busy samples (utilisation >= 50%), first-third vs last-third
drift of clock / power / temperature, how often each throttle reason was active, the
throughput windows and their first-third vs last-third change.

    python -m b2g.soak --seconds 180 --tag fp32acc
    python -m b2g.soak --seconds 180 --acc f16 --tag f16acc

Nothing else may use the GPU while this runs.
"""
from __future__ import annotations

import argparse
import csv
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_EXE = os.path.join(os.path.dirname(HERE), "lib", "gemm_bench")

TELEMETRY_COLUMNS = ["t", "smMHz", "memMHz", "powerW", "tempC", "utilPct", "swPowerCap",
                     "hwSlowdown", "hwThermal", "swThermal", "hwPowerBrake"]
_QUERY = ("clocks.sm,clocks.mem,power.draw,temperature.gpu,utilization.gpu,"
          "clocks_event_reasons.sw_power_cap,clocks_event_reasons.hw_slowdown,"
          "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
          "clocks_event_reasons.hw_power_brake_slowdown")
_REASONS = ("swPowerCap", "hwSlowdown", "hwThermal", "swThermal", "hwPowerBrake")


def device_uuid(cuda_index: int):
    """UUID ("GPU-...") of CUDA device `cuda_index` of this process's visible devices, or
    None. nvidia-smi numbers GPUs its own way (PCI order), which need not be CUDA's order
    (CUDA_DEVICE_ORDER, CUDA_VISIBLE_DEVICES), so the soaked GPU is named by its UUID."""
    try:
        import torch

        u = str(torch.cuda.get_device_properties(cuda_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:  # noqa: BLE001 -- no torch / no device
        return None


def sample(ident="0"):
    """One telemetry sample (values in TELEMETRY_COLUMNS order after `t`) of the GPU that
    nvidia-smi's -i names `ident` (a UUID, or an nvidia-smi index), or None."""
    try:
        out = subprocess.run(["nvidia-smi", f"--query-gpu={_QUERY}",
                              "--format=csv,noheader,nounits", "-i", str(ident)],
                             capture_output=True, text=True, timeout=20)
        f = [v.strip() for v in out.stdout.strip().splitlines()[0].split(",")]
        if out.returncode != 0 or len(f) != 10:
            return None
        return {"smMHz": int(float(f[0])), "memMHz": int(float(f[1])), "powerW": float(f[2]),
                "tempC": int(float(f[3])), "utilPct": int(float(f[4])),
                **dict(zip(_REASONS, f[5:]))}
    except Exception:  # noqa: BLE001 -- no nvidia-smi: no telemetry
        return None


def throughput_rows(lines):
    """SOAK,elapsed_s,window_ms,iters,tflops,ms_per_iter lines -> dicts (header skipped)."""
    rows = []
    for ln in lines:
        if not ln.startswith("SOAK,") or "elapsed_s" in ln:
            continue
        f = ln.strip().split(",")
        rows.append({"t": float(f[1]), "ms": float(f[2]), "iters": int(f[3]),
                     "tflops": float(f[4]), "msPerIter": float(f[5])})
    return rows


def report(samples, rows, header_lines, sample_ms, log=print):
    """The reference's summary: telemetry over busy samples, drift, throttle reasons,
    throughput windows and first vs last third. Returns the summary as a dict."""
    busy = [s for s in samples if s["utilPct"] >= 50]
    out = {"busy_samples": len(busy)}
    log(f"\n=== telemetry over {len(busy)} busy samples ({sample_ms} ms apart) ===")
    for p in ("smMHz", "memMHz", "powerW", "tempC"):
        if busy:
            v = [s[p] for s in busy]
            out[p] = (statistics.fmean(v), min(v), max(v))
            log(f"{p:<8} avg {out[p][0]:8.1f}   min {out[p][1]:8.1f}   max {out[p][2]:8.1f}")
    n = len(busy)
    if n >= 9:
        a, b = busy[: n // 3], busy[int(2 * n / 3):]
        log("\nfirst third vs last third (drift check):")
        for p in ("smMHz", "powerW", "tempC"):
            av, bv = statistics.fmean(s[p] for s in a), statistics.fmean(s[p] for s in b)
            out[f"drift_{p}"] = bv - av
            log(f"{p:<8} {av:8.1f} -> {bv:8.1f}   delta {bv - av:+7.1f}")
    log("\nthrottle reasons asserted at any point while busy:")
    for p in _REASONS:
        hits = sum(1 for s in busy if s[p] == "Active")
        out[f"active_{p}"] = hits
        log(f"  {p:<14} {hits:5d} / {len(busy)} samples")
    log("\n=== throughput windows ===")
    for r in rows:
        log(f"{r['t']:8.2f} {r['ms']:10.2f} {r['iters']:7d} {r['tflops']:10.3f} {r['msPerIter']:9.4f}")
    for ln in header_lines:
        log(ln.rstrip())
    if len(rows) >= 6:
        k = len(rows) // 3
        fa = statistics.fmean(r["tflops"] for r in rows[:k])
        la = statistics.fmean(r["tflops"] for r in rows[-k:])
        out["throughput_first_last"] = (fa, la, 100 * (la - fa) / fa)
        log(f"\nthroughput first third {fa:.2f} -> last third {la:.2f} TFLOP/s  "
            f"({100 * (la - fa) / fa:.2f}%)")
    return out


def run(seconds, window, M, N, K, tile, stages, layout, group, acc, tag, out_dir, sample_ms,
        exe=DEFAULT_EXE, gpu=0, log=print):
    os.makedirs(out_dir, exist_ok=True)
    stdout_path = os.path.join(out_dir, f"{tag}.throughput.txt")
    smi_path = os.path.join(out_dir, f"{tag}.telemetry.csv")
    args = [exe, "--m", str(M), "--n", str(N), "--k", str(K), "--tile", str(tile), "--stages",
            str(stages), "--layout", str(layout), "--group", str(group), "--acc", acc, "--noref",
            "--warmup", "20", "--soak", str(seconds), "--window", str(window)]
    # the CLI runs on its CUDA device 0: make that the soaked GPU, and sample the same GPU
    uuid = device_uuid(gpu)
    env = dict(os.environ)
    if uuid:
        env["CUDA_VISIBLE_DEVICES"] = uuid
    ident = uuid or str(gpu)
    log(f"soaking {seconds} s on {ident}: {' '.join(args)}")
    t0 = time.monotonic()
    samples = []
    with open(stdout_path, "w") as fh:
        proc = subprocess.Popen(args, stdout=fh, stderr=subprocess.STDOUT, env=env)
        while proc.poll() is None:
            s = sample(ident)
            if s is not None:
                samples.append({"t": round(time.monotonic() - t0, 2), **s})
            time.sleep(sample_ms / 1000.0)
        rc = proc.wait()
    with open(smi_path, "w", newline="", encoding="utf-8") as fh:
        w = csv.DictWriter(fh, fieldnames=TELEMETRY_COLUMNS, quoting=csv.QUOTE_ALL)
        w.writeheader()
        for s in samples:
            w.writerow(s)
    with open(stdout_path) as fh:
        lines = fh.readlines()
    summary = report(samples, throughput_rows(lines), [ln for ln in lines if ln.startswith("#")],
                     sample_ms, log)
    log(f"\nwrote {stdout_path} and {smi_path}")
    summary["returncode"] = rc
    return summary


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--seconds", type=float, default=180)
    p.add_argument("--window", type=float, default=2.0)
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--tile", type=int, default=-1)
    p.add_argument("--stages", type=int, default=0)
    p.add_argument("--layout", type=int, default=2)
    p.add_argument("--group", type=int, default=0)
    p.add_argument("--acc", choices=("f32", "f16"), default="f32")
    p.add_argument("--tag", default="soak")
    p.add_argument("--out-dir", default="data")
    p.add_argument("--sample-ms", type=int, default=250)
    p.add_argument("--exe", default=DEFAULT_EXE)
    p.add_argument("--gpu", type=int, default=0,
                   help="CUDA ordinal (of the visible devices) to soak and sample")
    a = p.parse_args(argv)
    s = run(a.seconds, a.window, a.m, a.n, a.k, a.tile, a.stages, a.layout, a.group, a.acc,
            a.tag, a.out_dir, a.sample_ms, a.exe, a.gpu)
    return s["returncode"]


if __name__ == "__main__":
    sys.exit(main())
