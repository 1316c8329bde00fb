"""CPU tests of the experiment tools that port the reference's sweep.ps1, soak.ps1 and
profile.ps1: b2g.sweep (configuration sweep -> CSV with the reference's columns), b2g.soak
(SOAK windows + nvidia-smi telemetry) and b2g.profile (ncu passes + the dense-occupancy
check). A fake gemm_bench prints lines in the real CLI's formats; a stand-in runner plays
ncu."""
import csv
import os
import stat
import sys
import textwrap

import pytest

from b2g import profile, soak, sweep

# header of the reference's data/sweep_results.csv, in order
REFERENCE_SWEEP_HEADER = ["M", "N", "K", "tile", "cta", "layout", "stages", "threads", "regs",
                          "smem", "ctaPerSm", "ms", "tflops", "pctSoL", "maxrel", "solTflops",
                          "smMHz0", "smMHz1", "powerW1", "tempC0", "tempC1"]
REFERENCE_TELEMETRY_HEADER = ["t", "smMHz", "memMHz", "powerW", "tempC", "utilPct",
                              "swPowerCap", "hwSlowdown", "hwThermal", "swThermal",
                              "hwPowerBrake"]

FAKE_CLI = textwrap.dedent('''\
    #!{python}
    # Stand-in for gemm_bench: prints the real CLI's header, table rows and SOAK lines.
    import sys, time
    a = sys.argv[1:]
    opt = lambda k, d: a[a.index(k) + 1] if k in a else d
    tile, layout = int(opt("--tile", "-1")), int(opt("--layout", "2"))
    print("# device        : fake B200  sm_100  148 SMs")
    if "--soak" in a:
        print("SOAK,elapsed_s,window_ms,iters,tflops,ms_per_iter")
        for i in range(9):
            print("SOAK,%.2f,%.2f,%d,%.3f,%.4f" % (2.0 * (i + 1), 2000.0, 20000, 1400.0 - i, 0.1))
        time.sleep(0.3)
        print("# soak summary: windows=9")
        sys.exit(0)
    print("# cuBLAS (SoL)  :    0.095 ms  1447.69 TFLOP/s")
    print("%-6s %-12s %-8s %6s %5s %5s %7s %6s %6s %10s %9s %8s %s" % (
        "tile", "CTA", "layout", "stages", "grp", "thr", "reg/thr", "smem", "CTA/SM", "ms",
        "TFLOP/s", "%SoL", "maxrel"))
    for st in range(2, 9):
        if layout != 2:
            print("%-6d %-12s %-8s %6d %5d %5s %7s %6s %6s %10s %9s %8s  SKIP: %s" % (
                tile, "256x256x64", "sw128", st, 0, "-", "-", "-", "-", "-", "-", "-",
                "layout not applicable on sm_100a"))
            continue
        print("%-6d %-12s %-8s %6d %5d %5d %7d %6d %6d %10.3f %9.2f %8s %s  sm_mhz=%.0f  splits=%d"
              % (tile, "256x256x64", "sw128", st, 8, 192, 136, 230584, 1, 0.1 + st * 1e-3,
                 1400.0 + st, "96.7%", "0.00e+00 OK", 1700, 1))
''')


def _fake_exe(tmp_path):
    p = tmp_path / "gemm_bench_fake"
    p.write_text(FAKE_CLI.format(python=sys.executable))
    p.chmod(p.stat().st_mode | stat.S_IEXEC)
    return str(p)


def test_sweep_columns_are_the_references_then_extras():
    assert sweep.REF_COLUMNS == REFERENCE_SWEEP_HEADER
    assert sweep.COLUMNS[:len(REFERENCE_SWEEP_HEADER)] == REFERENCE_SWEEP_HEADER


def test_sweep_parses_rows_by_position_and_reports_skips():
    text = "\n".join([
        "# cuBLAS (SoL)  :    0.095 ms  1447.69 TFLOP/s",
        "tile   CTA          layout   stages   grp   thr reg/thr   smem CTA/SM         ms   "
        "TFLOP/s     %SoL maxrel",
        "-1     auto         sw128         6     0   192     136 230584      1      0.095   "
        "1447.69   100.2% 1.2e-05 OK  cpu=4.5e-04 OK (worst m=1 n=2)  sm_mhz=1430  splits=1",
        "0      128x128x64   sw128         2     0     -       -      -      -          -         "
        "-        -  SKIP: smem over per-block opt-in limit",
    ])
    rows, skipped = sweep.parse_rows(text)
    assert sweep.sol_tflops(text) == "1447.69"
    assert len(rows) == 1 and len(skipped) == 1
    r = rows[0]
    assert (r["tile"], r["stages"], r["group"], r["threads"], r["regs"]) == \
        ("-1", "6", "0", "192", "136")
    assert (r["ms"], r["tflops"], r["pctSoL"], r["maxrel"]) == \
        ("0.095", "1447.69", "100.2%", "1.2e-05")
    assert (r["kernelSmMHz"], r["splits"]) == ("1430", "1")
    assert skipped[0][0] == "0" and "smem" in skipped[0][3]


def test_sweep_end_to_end_with_a_fake_cli(tmp_path):
    out = tmp_path / "data" / "sweep_results.csv"
    logs = []
    rows = sweep.run(4096, 4096, 4096, [0, 2], [0, 2], 5, 2, str(out), _fake_exe(tmp_path),
                     log=logs.append)
    assert len(rows) == 2 * 7  # layout 0 rows are all SKIP rows
    with open(out, newline="", encoding="utf-8") as fh:
        data = list(csv.reader(fh))
    assert data[0] == sweep.COLUMNS
    body = [dict(zip(data[0], r)) for r in data[1:]]
    assert len(body) == 14
    assert {b["tile"] for b in body} == {"0", "2"}
    assert all(b["solTflops"] == "1447.69" and b["M"] == "4096" for b in body)
    assert [b["stages"] for b in body[:7]] == [str(s) for s in range(2, 9)]
    assert any("skip tile=0 layout=sw128" in ln or "skip tile=0" in ln for ln in logs)


def test_soak_report_drift_and_reasons():
    samples = [{"t": i * 0.25, "smMHz": 1400 - i, "memMHz": 3996, "powerW": 990.0 + i,
                "tempC": 55 + i // 3, "utilPct": 100 if i else 10,
                "swPowerCap": "Active", "hwSlowdown": "Not Active", "hwThermal": "Not Active",
                "swThermal": "Not Active", "hwPowerBrake": "Not Active"} for i in range(13)]
    rows = soak.throughput_rows(["SOAK,elapsed_s,window_ms,iters,tflops,ms_per_iter\n"] +
                                ["SOAK,%d,2000,100,%d,0.1\n" % (i, 1300 + i) for i in range(6)])
    s = soak.report(samples, rows, [], 250, log=lambda *_: None)
    assert s["busy_samples"] == 12
    assert s["active_swPowerCap"] == 12 and s["active_hwThermal"] == 0
    assert s["drift_smMHz"] < 0 and s["drift_powerW"] > 0
    fa, la, pct = s["throughput_first_last"]
    assert (fa, la) == (1300.5, 1304.5) and pct > 0


def test_soak_end_to_end_with_a_fake_cli(tmp_path):
    s = soak.run(1, 2.0, 4096, 4096, 4096, -1, 0, 2, 0, "f32", "fake", str(tmp_path / "data"),
                 20, _fake_exe(tmp_path), log=lambda *_: None)
    assert s["returncode"] == 0
    thr = tmp_path / "data" / "fake.throughput.txt"
    tel = tmp_path / "data" / "fake.telemetry.csv"
    assert thr.exists() and tel.exists()
    with open(tel, newline="", encoding="utf-8") as fh:
        assert next(csv.reader(fh)) == REFERENCE_TELEMETRY_HEADER
    assert len(soak.throughput_rows(open(thr).readlines())) == 9
    assert "throughput_first_last" in s
    assert os.path.getsize(thr) > 0


def test_soak_names_the_gpu_by_uuid(tmp_path, monkeypatch):
    """The soaked GPU and the sampled GPU are the same one: the CLI is pinned to the device's
    UUID through CUDA_VISIBLE_DEVICES and nvidia-smi is asked about that UUID."""
    seen = {}
    monkeypatch.setattr(soak, "device_uuid", lambda i: f"GPU-fake-{i}")

    def fake_sample(ident):
        seen.setdefault("ident", ident)
        return None

    monkeypatch.setattr(soak, "sample", fake_sample)
    real_popen = soak.subprocess.Popen

    def spy_popen(args, **kw):
        seen["cvd"] = kw.get("env", {}).get("CUDA_VISIBLE_DEVICES")
        return real_popen(args, **kw)

    monkeypatch.setattr(soak.subprocess, "Popen", spy_popen)
    s = soak.run(1, 2.0, 64, 64, 64, -1, 0, 2, 0, "f32", "uuid", str(tmp_path / "data"), 20,
                 _fake_exe(tmp_path), gpu=3, log=lambda *_: None)
    assert s["returncode"] == 0
    assert seen["cvd"] == "GPU-fake-3" and seen["ident"] == "GPU-fake-3"


# ---------------------------------------------------------------------------------------
# b2g.profile: port of scripts/profile.ps1
# ---------------------------------------------------------------------------------------

_FAKE_NCU_CSV = '''==PROF== Connected to process 1234
M N K ...
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","gemm_bench","h","b2g::gemm_sm100_2cta<256, 0>","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","sm__cycles_elapsed.avg","cycle","153,016"
"0","1","gemm_bench","h","b2g::gemm_sm100_2cta<256, 0>","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","sm__cycles_active.avg","cycle","134,428"
"0","1","gemm_bench","h","b2g::gemm_sm100_2cta<256, 0>","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ns","96,400"
"0","1","gemm_bench","h","b2g::gemm_sm100_2cta<256, 0>","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_read.sum","byte","69,190,000"
"0","1","gemm_bench","h","b2g::gemm_sm100_2cta<256, 0>","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_write.sum","byte","17,440,000"
"0","1","gemm_bench","h","b2g::gemm_sm100_2cta<256, 0>","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed","%","74.58"
'''


def test_profile_commands_keep_clocks_and_bound_the_capture():
    args = profile.app_args(4096, 4096, 4096, skip=3)
    assert args[args.index("--warmup") + 1] == "5" and args[args.index("--iters") + 1] == "1"
    assert "--noref" in args  # our kernel only; --cublas keeps the cuBLAS column instead
    assert "--noref" not in profile.app_args(64, 64, 64, cublas=True)
    plain, sec, met = profile.commands("exe", args, "regex:gemm_sm100", 3, "out/x")
    for c in (sec, met):
        assert c[:3] == ["ncu", "--clock-control", "none"]
        assert c[c.index("-c") + 1] == "1" and c[c.index("-s") + 1] == "3"
        assert c[c.index("-k") + 1] == "regex:gemm_sm100"
        assert c[-len(plain):] == plain
    assert "--set" not in sec and sec.count("--section") == len(profile.SECTIONS)
    _, full, _ = profile.commands("exe", args, "k", 3, "out/x", full=True)
    assert full[full.index("--set") + 1] == "full"
    _, _, nv = profile.commands("exe", args, "k", 3, "out/x", nvlink=True)
    assert "nvltx__bytes_data_user.sum" in nv[nv.index("--metrics") + 1]


def test_profile_parse_and_dense_occupancy():
    m = profile.parse_metrics_csv(_FAKE_NCU_CSV)
    assert m["sm__cycles_elapsed.avg"] == 153016.0 and m["dram__bytes_read.sum"] == 69.19e6
    s = profile.summarize(m, 4096, 4096, 4096, fpc=8187.0, sms=148)
    busy = 2.0 * 4096 ** 3 / (8187.0 * 148)  # the reference's hand calculation
    assert abs(s["busy_tensor_cycles"] - busy) < 1e-6
    assert abs(s["dense_occupancy_elapsed"] - busy / 153016.0) < 1e-12
    assert abs(s["dense_occupancy_active"] - busy / 134428.0) < 1e-12
    assert abs(s["dram_bytes"] - 86.63e6) < 1
    assert abs(s["tflops_under_ncu"] - 2.0 * 4096 ** 3 / 96.4e-6 / 1e12) < 1e-6
    # the pipe counter against the clock-free figure (1.0: they agree)
    assert abs(s["tensor_pipe_vs_dense_occupancy"] - 0.7458 / (busy / 153016.0)) < 1e-12
    assert profile.parse_metrics_csv("no csv here") == {}


def test_profile_run_with_a_stand_in_ncu(tmp_path):
    """The whole flow with a fake runner: plain run first, then the two ncu passes, then
    the markdown summary; a failing plain run stops before any ncu command."""
    calls = []

    class R:
        def __init__(self, rc, out=""):
            self.returncode, self.stdout, self.stderr = rc, out, ""

    def runner(cmd, **_):
        calls.append(cmd)
        return R(0, _FAKE_NCU_CSV if "--metrics" in cmd else "ok")

    out = profile.run(4096, 4096, 4096, "t", str(tmp_path), exe="gb", fpc=8187.0, sms=148,
                      log=lambda *_: None, runner=runner)
    assert calls[0][0] == "gb" and calls[1][0] == "ncu" and "--metrics" in calls[2]
    md = open(out["markdown"]).read()
    assert "dense_occupancy_elapsed" in md and "--clock-control none" in md
    calls.clear()
    with pytest.raises(RuntimeError):
        profile.run(64, 64, 64, "u", str(tmp_path), exe="gb", log=lambda *_: None,
                    runner=lambda cmd, **_: (calls.append(cmd), R(1))[1])
    assert len(calls) == 1  # no ncu after a failed plain run
