"""Scan-only benchmark in the reference's result format.

    python -m mamba_ssm_benchmark_b200.bench_scan [--lengths 256,1024,...] [--out results/bench/scan.json]
                                                  [--csv results/csv/bench_scan.csv]

The same measurement and record layout as the reference's benchmarks/bench_scan.py:43-66 (one
Mamba layer's scan, B=1, D=512, N=16, growing L; forward under no_grad and forward+backward of
``y.sum()``), written as ``{"env": ..., "config": {"B", "D", "N"}, "runs": [{"scan", "L", "fwd",
"fwd_bwd"}]}`` with each measurement ``{"ms", "q25", "q75", "peak_mb"}`` or ``{"oom": true}``
(benchmarks/common.py:36-46), so the reference's plotting and CSV export read it unchanged.  The
CSV has the columns of analysis/export_csv.py:40-43 (scan, L, fwd_*, fwd_bwd_*).  The scan name
recorded is "b200".  Times are CUDA-event medians over repeats after warm-up.
"""

import argparse
import csv
import datetime
import json
import os
import platform
import statistics
import subprocess
import sys

import torch

SCAN_NAME = "b200"
CONFIG = {"B": 1, "D": 512, "N": 16}


def make_inputs(L, B=1, D=512, N=16, device="cuda"):
    """The reference benchmark's inputs (benchmarks/bench_scan.py:25-32): x, Bm, Cm ~ N(0, 1),
    delta ~ U[1e-3, 0.101), A[d, n] = -(n + 1); drawn on the CPU from seed 0 in the order
    x, delta, Bm, Cm; all leaves require grad."""
    g = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randn(B, L, D, generator=g)
    delta = torch.rand(B, L, D, generator=g) * 0.1 + 1e-3
    A = -torch.arange(1, N + 1, dtype=torch.float32).expand(D, N).contiguous()
    Bm = torch.randn(B, L, N, generator=g)
    Cm = torch.randn(B, L, N, generator=g)
    return [t.to(device).requires_grad_() for t in (x, delta, A, Bm, Cm)]


def environment():
    """What makes a measurement comparable to another one (the reference's runtime.environment keys
    that apply here)."""
    def run(cmd):
        try:
            return subprocess.run(cmd, capture_output=True, text=True, timeout=10).stdout.strip()
        except (OSError, subprocess.SubprocessError):
            return None

    env = {"timestamp": datetime.datetime.now().astimezone().isoformat(timespec="seconds"),
           "python": sys.version.split()[0], "platform": platform.platform(), "cpu": platform.processor(),
           "torch": torch.__version__, "cuda": torch.version.cuda, "scan_library": "libssm_b200 (sm_100a)"}
    if torch.cuda.is_available():
        props = torch.cuda.get_device_properties(0)
        env.update(gpu=props.name, vram_gib=props.total_memory / 2**30,
                   driver=run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"]),
                   gpu_clocks_mhz=run(["nvidia-smi", "--query-gpu=clocks.sm,clocks.mem", "--format=csv,noheader"]))
    return env


def time_ms(fn, warmup=2, min_repeats=3, max_repeats=20, budget_ms=500.0):
    """Median, q25, q75 of fn()'s device time in ms (CUDA events on the current stream)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    while len(times) < max_repeats and (len(times) < min_repeats or sum(times) < budget_ms):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    q = statistics.quantiles(times, n=4) if len(times) >= 2 else [times[0]] * 3
    return statistics.median(times), q[0], q[2]


class DevicePeak:
    """Context manager: the most device memory (MiB) allocated inside the block above what was held
    when it was entered."""

    def __enter__(self):
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        self.held = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        self.mib = None
        return self

    def __exit__(self, *exc):
        torch.cuda.synchronize()
        self.mib = (torch.cuda.max_memory_allocated() - self.held) / 2**20
        return False


def measure(fn, **kw):
    """One record of the result format: one untimed call under the memory probe, then the timed
    repeats; an out-of-memory error anywhere turns the record into {"oom": true}."""
    try:
        with DevicePeak() as peak:
            fn()
        ms, q25, q75 = time_ms(fn, **kw)
    except torch.OutOfMemoryError:
        torch.cuda.empty_cache()
        return {"oom": True}
    return {"ms": ms, "q25": q25, "q75": q75, "peak_mb": peak.mib}


def csv_rows(results):
    """Rows of analysis/export_csv.py's bench_scan table."""
    def flat(prefix, d):
        return {f"{prefix}_{k}": v for k, v in (d or {}).items()}
    return [{"scan": r["scan"], "L": r["L"], **flat("fwd", r["fwd"]), **flat("fwd_bwd", r["fwd_bwd"])}
            for r in results["runs"]]


def write_csv(results, path):
    rows = csv_rows(results)
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    keys = list(dict.fromkeys(k for r in rows for k in r))
    with open(path, "w", newline="", encoding="utf-8") as f:
        w = csv.DictWriter(f, fieldnames=keys)
        w.writeheader()
        w.writerows(rows)


def run(lengths, measure_fn=measure):
    from . import selective_scan
    results = {"env": environment(), "config": dict(CONFIG), "runs": []}
    for L in lengths:
        ins = make_inputs(L, **CONFIG)

        def fwd():
            with torch.no_grad():
                selective_scan(*ins, scan=SCAN_NAME)

        def fwd_bwd():
            selective_scan(*ins, scan=SCAN_NAME)[0].sum().backward()

        rec = {"scan": SCAN_NAME, "L": L, "fwd": measure_fn(fwd), "fwd_bwd": measure_fn(fwd_bwd)}
        results["runs"].append(rec)
        fm, bm = rec["fwd"], rec["fwd_bwd"]
        print(f"{SCAN_NAME:14s} L={L:6d}  fwd {fm.get('ms', float('nan')):9.3f} ms {fm.get('peak_mb', 0):8.1f} MB"
              f"   fwd+bwd {bm.get('ms', float('nan')):9.3f} ms {bm.get('peak_mb', 0):8.1f} MB", flush=True)
        del ins
        torch.cuda.empty_cache()
    return results


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--lengths", default="256,1024,4096,16384,65536")
    ap.add_argument("--out", default="results/bench/scan.json")
    ap.add_argument("--csv", default=None, help="also write the flattened CSV table here")
    args = ap.parse_args(argv)
    results = run([int(v) for v in args.lengths.split(",")])
    os.makedirs(os.path.dirname(args.out) or ".", exist_ok=True)
    with open(args.out, "w") as f:
        json.dump(results, f, indent=2)
    print(f"saved {args.out}")
    if args.csv:
        write_csv(results, args.csv)
        print(f"saved {args.csv}")


if __name__ == "__main__":
    main()
