"""Configuration sweep of the gemm_bench CLI, GPU state logged around every run, as CSV.

Port of the reference's scripts/sweep.ps1 (its tuning phases 2-4): for every tile x layout it
runs ``gemm_bench --sweep --check`` (stages 2..8 at that tile), reads the result rows, and
samples nvidia-smi (SM and memory clock, power, temperature) before and after each run so
that a thermal drift is not mistaken for a kernel effect. The CSV has the columns of the
reference's data/sweep_results.csv in the same order; columns it does not have (the
rasterization group, the SM clock the kernel ran at, the split-K factor) follow them.

    python -m b2g.sweep --m 4096 --n 4096 --k 4096 --tiles 0 1 2 --layouts 2 --out sweep.csv

Rows are read by position in the CLI's table (tile CTA layout stages grp thr reg/thr smem
CTA/SM ms TFLOP/s %SoL maxrel, then key=value fields); the automatic tile (-1) counts as a
row, and SKIP rows are reported, not written.
"""
from __future__ import annotations

import argparse
import csv
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_EXE = os.path.join(os.path.dirname(HERE), "lib", "gemm_bench")

# data/sweep_results.csv of the reference, in its order, then this build's additions
REF_COLUMNS = ["M", "N", "K", "tile", "cta", "layout", "stages", "threads", "regs", "smem",
               "ctaPerSm", "ms", "tflops", "pctSoL", "maxrel", "solTflops", "smMHz0", "smMHz1",
               "powerW1", "tempC0", "tempC1"]
EXTRA_COLUMNS = ["group", "kernelSmMHz", "splits"]
COLUMNS = REF_COLUMNS + EXTRA_COLUMNS

_ROW = re.compile(r"^\s*-?\d+\s")


def gpu_state(index: int = 0) -> dict:
    """SM / memory clock, power, temperature and utilisation from nvidia-smi (empty strings
    where nvidia-smi is missing or fails)."""
    q = "clocks.sm,clocks.mem,power.draw,temperature.gpu,utilization.gpu"
    keys = ("smMHz", "memMHz", "powerW", "tempC", "utilPct")
    try:
        out = subprocess.run(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                              "-i", str(index)], capture_output=True, text=True, timeout=20)
        vals = [v.strip() for v in out.stdout.strip().splitlines()[0].split(",")]
        if out.returncode != 0 or len(vals) != len(keys):
            raise ValueError(out.stderr)
        return dict(zip(keys, vals))
    except Exception:  # noqa: BLE001 -- no GPU tools: the state columns stay empty
        return {k: "" for k in keys}


def sol_tflops(text: str) -> str:
    """The cuBLAS (speed-of-light) TFLOP/s the CLI prints in its header, or ''."""
    m = re.search(r"cuBLAS \(SoL\)\s*:.*?([\d.]+) TFLOP/s", text)
    return m.group(1) if m else ""


def parse_rows(text: str):
    """(rows, skipped) from the CLI's table: rows are dicts keyed by COLUMNS names (those the
    table itself gives), skipped are (tile, layout, stages, reason) of SKIP rows."""
    rows, skipped = [], []
    for line in text.splitlines():
        if not _ROW.match(line):
            continue
        f = line.split()
        if "SKIP:" in line:
            skipped.append((f[0], f[2], f[3], line.split("SKIP:", 1)[1].strip()))
            continue
        if len(f) < 13:
            continue
        row = {"tile": f[0], "cta": f[1], "layout": f[2], "stages": f[3], "group": f[4],
               "threads": f[5], "regs": f[6], "smem": f[7], "ctaPerSm": f[8], "ms": f[9],
               "tflops": f[10], "pctSoL": f[11], "maxrel": f[12]}
        kv = dict(t.split("=", 1) for t in f[13:] if "=" in t)
        row["kernelSmMHz"] = kv.get("sm_mhz", "")
        row["splits"] = kv.get("splits", "")
        rows.append(row)
    return rows, skipped


def run(M, N, K, tiles, layouts, iters, warmup, out, exe=DEFAULT_EXE, gpu=0, log=print):
    rows = []
    for t in tiles:
        for lay in layouts:
            before = gpu_state(gpu)
            cmd = [exe, "--m", str(M), "--n", str(N), "--k", str(K), "--tile", str(t),
                   "--layout", str(lay), "--sweep", "--iters", str(iters), "--warmup",
                   str(warmup), "--check"]
            p = subprocess.run(cmd, capture_output=True, text=True)
            text = p.stdout + p.stderr
            after = gpu_state(gpu)
            sol = sol_tflops(text)
            got, skipped = parse_rows(text)
            for tile, layout, stages, why in skipped:
                log(f"  skip tile={tile} layout={layout} stages={stages}: {why}")
            for r in got:
                r.update(M=M, N=N, K=K, solTflops=sol, smMHz0=before["smMHz"],
                         smMHz1=after["smMHz"], powerW1=after["powerW"],
                         tempC0=before["tempC"], tempC1=after["tempC"])
                rows.append(r)
            if p.returncode != 0 and not got:
                log(f"  tile={t} layout={lay}: gemm_bench exited {p.returncode}: "
                    f"{text.strip().splitlines()[-1] if text.strip() else ''}")
            log(f"done tile={t} layout={lay}  (SM {after['smMHz']} MHz, {after['powerW']} W, "
                f"{after['tempC']} C)")
    d = os.path.dirname(os.path.abspath(out))
    os.makedirs(d, exist_ok=True)
    with open(out, "w", newline="", encoding="utf-8") as fh:
        w = csv.DictWriter(fh, fieldnames=COLUMNS, quoting=csv.QUOTE_ALL, extrasaction="ignore")
        w.writeheader()
        for r in rows:
            w.writerow({k: r.get(k, "") for k in COLUMNS})
    log(f"\nwrote {out} ({len(rows)} rows)\n")
    best = sorted(rows, key=lambda r: float(r["tflops"]), reverse=True)
    cols = ("cta", "layout", "stages", "group", "regs", "smem", "ctaPerSm", "ms", "tflops",
            "pctSoL", "maxrel")
    if best:
        log("  ".join(f"{c:>10}" for c in cols))
        for r in best:
            log("  ".join(f"{r[c]:>10}" for c in cols))
    return rows


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--tiles", type=int, nargs="+", default=[0, 1, 2])
    p.add_argument("--layouts", type=int, nargs="+", default=[0, 1, 2])
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--warmup", type=int, default=30)
    p.add_argument("--out", default=os.path.join("data", "sweep_results.csv"))
    p.add_argument("--exe", default=DEFAULT_EXE)
    p.add_argument("--gpu", type=int, default=0, help="nvidia-smi index for the state columns")
    a = p.parse_args(argv)
    rows = run(a.m, a.n, a.k, a.tiles, a.layouts, a.iters, a.warmup, a.out, a.exe, a.gpu)
    return 0 if rows else 1


if __name__ == "__main__":
    sys.exit(main())
