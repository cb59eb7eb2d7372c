#!/usr/bin/env python
"""Selective-scan (Mamba S6) fwd+bwd throughput on B200 — the BASELINE config-1 workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|3]

One step = the fused selective scan forward + backward over one batch (B=16, L=512, D=512,
N=16, fp32, with the mixer's D-skip and SiLU(z) gate) through the C ABI of libssm_b200.so.
Prints one JSON line (rank 0).

value  : whole-job tokens/s with inputs resident in HBM (CUDA events around exactly K steps,
         barrier + synchronize on both sides, max over ranks).  Input/output sets rotate so
         that every step touches buffers evicted from the 126 MB L2 (4 sets, ~0.5 GB).
e2e    : the same metric through the public Python API (selective_scan_fused + autograd
         backward) with host (pinned) inputs and outputs: H2D copies, fwd, bwd and D2H copies
         of every output inside the timed region (copies on their own streams, overlapping the
         neighbouring steps' compute).
N > 1  : one process per GPU (torchrun).  Channel sharding, weak scaling: every rank owns a
         512-channel shard of a (512 N)-channel layer; B and C are shared, so the backward
         ends with an NCCL all-reduce of dB|dC (the real exchange of channel sharding).
         A token is one (batch, position) row through 512 channels, so the job processes
         N x B x L tokens per step.
--config 2 : the long-context forward (B=1, L=131072, D=512): the sequence is split into N
         contiguous shards (strong scaling); each rank summarises its shard, the summaries are
         all-gathered over NCCL and composed, and each rank finishes its shard from its
         carried-in state (mamba_ssm_benchmark_b200/sharding.py).
--config 4 : the full byte-level Mamba LM (11 blocks, d_model 256) built on these ops
         (mamba_ssm_benchmark_b200/mixer.py): training step on 16 x 512 Markov bytes including
         clipping and AdamW (value: tokens/s), and 256-token generation through CUDA-graph
         decode steps at batch 1 and 64 ("decode": ms/token).
--impl reference : the reference's CPU scan (the oracle port of models/scan.py, chunked scan +
         recomputing backward) on the host cores, bounded samples of the same workload.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "selective-scan fwd+bwd tokens/s and achieved HBM GB/s (% of peak) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, choices=(1, 2, 3, 4), default=1)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(workload):
    """dram read+write bytes per launch of the backward kernel, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", f"bwd_kernel_{workload}.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def mufu_bound(cfg, bwd_ms, clk):
    """The backward's other roofline: special-function (MUFU) throughput.  Every (t, d, n) needs
    exp(delta A) twice (state recompute and reverse pass) and every (t, d) the gate's sigmoid (ex2 +
    rcp), at 16 MUFU results per clock per SM (measured on this B200 pool)."""
    ops = 2 * cfg.B * cfg.L * cfg.D * cfg.N + 2 * cfg.B * cfg.L * cfg.D
    mhz = clk.get("sm_mhz") or 1965.0
    peak = 16 * 148 * mhz * 1e6
    achieved = ops / (bwd_ms / 1e3)
    return {"ops_per_launch": ops, "unit": "MUFU ops/s", "achieved": achieved, "peak": peak, "frac": achieved / peak,
            "peak_source": "16 ops/clk/SM (measured ex2 throughput) x 148 SMs x median SM clock"}


# --------------------------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 7]
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if "Active" in v and "Not" not in v})
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------------------------
# the GPU arm
# --------------------------------------------------------------------------------------------
class ScanStep:
    """Pre-marshalled C-ABI calls of one fused fwd+bwd step over one buffer set."""

    def __init__(self, cfg, device, seed, shared_seed, B_rows=None):
        from mamba_ssm_benchmark_b200 import _native as nat
        from mamba_ssm_benchmark_b200.workloads import make_inputs
        self.nat = nat
        B, L, D, N = cfg.B, cfg.L, cfg.D, cfg.N
        dt = cfg.dtype
        ins = make_inputs(B, L, D, N, seed=seed, dist="config", dtype=dt)
        shared = make_inputs(B, L, D, N, seed=shared_seed, dist="config", dtype=dt)
        ins["Bm"], ins["Cm"] = shared["Bm"], shared["Cm"]
        t = {k: (v.to(device) if v is not None else None) for k, v in ins.items()}
        self.t = t
        f32 = dict(dtype=torch.float32, device=device)
        self.y = torch.empty(B, L, D, dtype=dt, device=device)
        self.last = torch.empty(B, D, N, **f32)
        self.cs = torch.empty(B, -(-L // 16), D, N, **f32)
        self.yg = torch.empty(B, L, D, dtype=dt, device=device)
        self.du = torch.empty(B, L, D, dtype=dt, device=device)
        self.ddelta = torch.empty_like(self.du)
        self.dz = torch.empty_like(self.du)
        self.dBC = torch.empty(B, L, 2 * N, dtype=dt, device=device)   # dB | dC in one buffer
        self.dA = torch.empty(D, N, **f32)
        self.dD = torch.empty(D, **f32)
        self.fws = nat.fwd_workspace_bytes(B, L, D, N)
        self.bws = nat.bwd_workspace_bytes(B, L, D, N)
        self.fw = torch.empty(max(self.fws, 1), dtype=torch.uint8, device=device)
        self.bw = torch.empty(self.bws, dtype=torch.uint8, device=device)
        v3, p = nat.view3, nat.ptr
        self.lib = nat.lib()
        stream = nat.stream_of(device)
        self.fwd_args = (B, L, D, N, 0, v3(t["u"]), v3(t["delta"]), p(t["A"]), v3(t["Bm"]), v3(t["Cm"]),
                         p(t["Dskip"]), v3(t["z"]), None, v3(self.y), v3(self.yg), p(self.last), p(self.cs),
                         self.fw.data_ptr(),
                         self.fws, stream)
        self.bwd_args = (B, L, D, N, 0, v3(t["u"]), v3(t["delta"]), p(t["A"]), v3(t["Bm"]), v3(t["Cm"]),
                         p(t["Dskip"]), v3(t["z"]), None, p(self.cs), v3(self.yg), v3(t["dy"]), None, v3(self.du),
                         v3(self.ddelta), p(self.dA), v3(self.dBC[..., :N]), v3(self.dBC[..., N:]), p(self.dD),
                         v3(self.dz), None, self.bw.data_ptr(), self.bws, stream)
        self.launches = (1 if self.fws == 0 else 3) + 2

    def fwd(self):
        rc = self.lib.ssm_scan_fwd(*self.fwd_args)
        if rc:
            self.nat.check(rc, "ssm_scan_fwd")

    def bwd(self):
        rc = self.lib.ssm_scan_bwd(*self.bwd_args)
        if rc:
            self.nat.check(rc, "ssm_scan_bwd")


def e2e_run(cfg, device, steps, world, seed):
    """Public API with host buffers: every step copies its inputs from pinned host memory, runs the
    forward and backward through selective_scan_fused + autograd, and copies every output back to
    pinned host memory.  The copies run on their own streams with double-buffered device inputs, so
    step i's device-to-host copy and step i+1's host-to-device copy overlap step i's compute.
    Each direction is one copy per step: the inputs sit in one pinned staging buffer (one
    256-byte-aligned slot per tensor, the device tensors are views of its device twin), and the
    outputs are gathered on the device into one contiguous byte buffer before their download.
    Measured on a B200, one copy each way instead of one per tensor (9 up, 10 down) took
    1.48-1.64 ms per config-1 step against 1.71-2.01 ms.
    A step's outputs are held until the step two later, whose compute first waits for their
    device-to-host copy, so the allocator reuses their blocks in stream order (recording them
    on the copy stream instead kept the allocator growing with fresh device allocations)."""
    from mamba_ssm_benchmark_b200 import selective_scan_fused, sharding
    from mamba_ssm_benchmark_b200.workloads import make_inputs
    ins = make_inputs(cfg.B, cfg.L, cfg.D, cfg.N, seed=seed, dist="config", dtype=cfg.dtype)
    names = [k for k, v in ins.items() if v is not None]
    offs, total = {}, 0
    for n in names:
        offs[n] = total
        total += (ins[n].numel() * ins[n].element_size() + 255) // 256 * 256
    staging = torch.empty(total, dtype=torch.uint8).pin_memory()

    def views(buf):
        return {n: buf[offs[n]:offs[n] + ins[n].numel() * ins[n].element_size()].view(ins[n].dtype).view(ins[n].shape)
                for n in names}

    for n, v in views(staging).items():
        v.copy_(ins[n])
    h2d = total                                   # the whole staging buffer, alignment padding included
    compute = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    dev_bufs = [torch.empty(total, dtype=torch.uint8, device=device) for _ in range(2)]
    dev_sets = [views(buf) for buf in dev_bufs]
    up_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    down_done = [torch.cuda.Event() for _ in range(2)]
    held = [None, None]                           # outputs whose device-to-host copies may still run
    outs_host = [None, None]
    d2h = 0

    def upload(k):
        up.wait_event(comp_done[k])               # the compute that last read this set is done
        with torch.cuda.stream(up):
            dev_bufs[k].copy_(staging, non_blocking=True)
        up_done[k].record(up)

    def compute_step(k):
        nonlocal d2h
        compute.wait_event(up_done[k])
        compute.wait_event(down_done[k])          # slot k's previous outputs are copied out ...
        held[k] = None                            # ... so this step may reuse their blocks
        dv = dev_sets[k]
        leaves = [dv[n].detach().requires_grad_() for n in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")]
        y, last = selective_scan_fused(leaves[0], leaves[1], leaves[2], leaves[3], leaves[4], D=leaves[5],
                                       z=leaves[6])
        grads = list(torch.autograd.grad(y, leaves, dv["dy"]))
        if world > 1:
            sharding.reduce_shared_grads(grads[3:5])          # dBm, dCm: partial sums over channel shards
        res = [y.detach(), last.detach()] + grads
        packed = torch.cat([r.contiguous().view(-1).view(torch.uint8) for r in res])   # one download
        comp_done[k].record(compute)
        if outs_host[k] is None:
            outs_host[k] = torch.empty(packed.numel(), dtype=torch.uint8, pin_memory=True)
        down.wait_event(comp_done[k])
        with torch.cuda.stream(down):
            outs_host[k].copy_(packed, non_blocking=True)
        down_done[k].record(down)
        held[k] = packed
        d2h = packed.numel()

    def run(n):
        upload(0)
        for i in range(n):
            k = i % 2
            if i + 1 < n:
                upload(1 - k)
            compute_step(k)
        compute.wait_stream(up)
        compute.wait_stream(down)

    run(3)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    run(steps)
    e1.record(compute)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    return ms / steps, h2d, d2h


def host_link(device, h2d, d2h, tokens_step, e2e_value, world, reps=8):
    """The host link's floor for the e2e step: device time to copy h2d bytes from pinned host
    memory to the device and d2h bytes back at the same time (one copy each way per repetition,
    on two streams), max over ranks.  Returns the e2e "link" record: that time, the bandwidth,
    the tokens/s the copies alone would allow and the e2e value's fraction of it."""
    hu = torch.empty(h2d, dtype=torch.uint8).pin_memory()
    du = torch.empty(h2d, dtype=torch.uint8, device=device)
    hd = torch.empty(d2h, dtype=torch.uint8).pin_memory()
    dd = torch.zeros(d2h, dtype=torch.uint8, device=device)
    cur = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def burst(n):
        up.wait_stream(cur)
        down.wait_stream(cur)
        for _ in range(n):
            with torch.cuda.stream(up):
                du.copy_(hu, non_blocking=True)
            with torch.cuda.stream(down):
                hd.copy_(dd, non_blocking=True)
        cur.wait_stream(up)
        cur.wait_stream(down)

    burst(2)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    burst(reps)
    e1.record(cur)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / reps
    if world > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    bound = tokens_step / (ms / 1e3)
    return {"ms_per_step": ms, "gbs": (h2d + d2h) / (ms / 1e3) / 1e9, "bound_value": bound,
            "frac": e2e_value / bound,
            "what": "pinned H2D of the step's input bytes and D2H of its output bytes, at the same time"}


def cpu_model():
    """The host CPU's model name (from /proc/cpuinfo), for the CPU baseline records."""
    try:
        with open("/proc/cpuinfo") as f:
            for row in f:
                if row.startswith("model name"):
                    return row.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference_sample(cfg, budget_s, d_slice=None, b_rows=None, repeats_min=3, backward=True):
    """Oracle port (the reference's chunked CPU scan + recomputing backward) on a slice of the
    workload; returns (tokens/s in 512-channel token units, description, samples)."""
    from mamba_ssm_benchmark_b200.workloads import make_inputs
    from oracle import scan_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    b = b_rows or cfg.B
    d = d_slice or cfg.D
    ins = make_inputs(b, cfg.L, d, cfg.N, seed=0, dist="config", dtype=torch.float32)

    def one():
        lv = [ins[k].clone().requires_grad_() for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")]
        y, _ = O.selective_scan_fused(lv[0], lv[1], lv[2], lv[3], lv[4], Dskip=lv[5], z=lv[6])
        if backward:
            torch.autograd.grad(y, lv, ins["dy"])

    one()
    times = []
    t_start = time.perf_counter()
    while len(times) < repeats_min or time.perf_counter() - t_start < budget_s:
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > 3 * budget_s:
            break
    med = statistics.median(times)
    tokens = b * cfg.L * d / 512.0
    desc = (f"B={b} of {cfg.B} rows, L={cfg.L}, {d} of {cfg.D} channels, N={cfg.N}, fused "
            f"{'fwd+bwd' if backward else 'fwd'}; median of {len(times)}")
    return tokens / med, desc, times


def run_reference(args, cfg, workload):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    # size one "step" so that warmup + steps fit in ~150 s of host time
    from mamba_ssm_benchmark_b200.workloads import make_inputs  # noqa: F401
    budget = 150.0 / max(1, args.steps + args.warmup)
    probe_rate, _, probe = cpu_reference_sample(cfg, 0.0, d_slice=min(cfg.D, 64), b_rows=1, repeats_min=1,
                                                backward=cfg.backward)
    t_probe = statistics.median(probe)
    d_s = int(max(8, min(cfg.D, 64 * budget / max(t_probe, 1e-6))) // 8 * 8)
    b_s = 1
    if d_s >= cfg.D:
        d_s = cfg.D
        b_s = int(max(1, min(cfg.B, budget / max(t_probe * cfg.D / 64, 1e-6))))
    from oracle import scan_oracle as O
    from mamba_ssm_benchmark_b200.workloads import make_inputs as mk
    ins = mk(b_s, cfg.L, d_s, cfg.N, seed=0, dist="config", dtype=torch.float32)

    def step():
        lv = [ins[k].clone().requires_grad_() for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")]
        y, _ = O.selective_scan_fused(lv[0], lv[1], lv[2], lv[3], lv[4], Dskip=lv[5], z=lv[6])
        if cfg.backward:
            torch.autograd.grad(y, lv, ins["dy"])

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    tokens = b_s * cfg.L * d_s / 512.0
    value = tokens * args.steps / dt
    sample = f"per step: B={b_s} of {cfg.B} rows, L={cfg.L}, {d_s} of {cfg.D} channels, N={cfg.N}, fused " \
             f"{'fwd+bwd' if cfg.backward else 'fwd'} (tokens counted in 512-channel units)"
    cores = torch.get_num_threads()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong" if args.config == 2 else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload, "B": cfg.B, "L": cfg.L, "D": cfg.D, "N": cfg.N},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "cpu_model": cpu_model(),
                             "kind": "port",
                             "sample": sample + "; oracle/scan_oracle.py restates models/scan.py (chunked)"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_sequence_shards(args, cfg, workload, rank, world, device):
    """Config 2: one long sequence split into ``world`` contiguous shards (strong scaling).

    Per step and rank: summary pass over the shard, NCCL all-gather of the (decay, hend)
    summaries, prefix composition, finish pass from the carried-in state.  On one GPU the step
    is a single ssm_scan_fwd over the whole sequence (which splits it into segments itself)."""
    from mamba_ssm_benchmark_b200 import _native as nat
    from mamba_ssm_benchmark_b200 import selective_scan_fused, sharding
    from mamba_ssm_benchmark_b200.workloads import algorithmic_bytes, make_inputs
    lo, hi = sharding.shard_range(cfg.L, world, rank)
    Ls = hi - lo
    B, D, N = cfg.B, cfg.D, cfg.N
    sets = 1 if world == 1 else 2        # at 8 shards one set is ~130 MB: rotate two to stay above L2
    stream = torch.cuda.current_stream(device)
    lib = nat.lib()
    data = []
    for s_ in range(sets):
        ins = make_inputs(B, Ls, D, N, seed=100 * s_ + rank, dist="config", dtype=cfg.dtype, device=device)
        data.append(ins)
    if world == 1:
        outs = [(torch.empty(B, Ls, D, dtype=cfg.dtype, device=device),
                 torch.empty(B, D, N, dtype=torch.float32, device=device)) for _ in range(sets)]
        wsb = nat.fwd_workspace_bytes(B, Ls, D, N)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=device)
        launches = 1 if wsb == 0 else 3

        def step(i, ev=None):
            d, (y, last) = data[i % sets], outs[i % sets]
            if ev is not None:
                ev[0].record(stream)
            rc = lib.ssm_scan_fwd(B, Ls, D, N, 0, nat.view3(d["u"]), nat.view3(d["delta"]), nat.ptr(d["A"]),
                                  nat.view3(d["Bm"]), nat.view3(d["Cm"]), nat.ptr(d["Dskip"]), nat.view3(d["z"]),
                                  None, nat.view3(y), nat.NULL_VIEW, nat.ptr(last), None, ws.data_ptr(), wsb,
                                  nat.stream_of(device))
            nat.check(rc, "ssm_scan_fwd")
            if ev is not None:
                ev[1].record(stream)
    else:
        shards = [sharding.SequenceShard(d["u"], d["delta"], d["A"], d["Bm"], d["Cm"], "zoh", D=d["Dskip"], z=d["z"])
                  for d in data]
        launches = 2 if shards[0].wsb == 0 else 4

        def step(i, ev=None):
            sh = shards[i % sets]
            decay, hend = sh.summary()
            decays, hends = sharding.exchange_summaries(decay, hend)
            h_in, _ = sharding.compose_prefix(decays, hends)
            if ev is not None:
                ev[0].record(stream)
            sh.finish(h_in[rank])
            if ev is not None:
                ev[1].record(stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(device)
    K = args.steps
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    clocks = ClockSampler(device.index)
    clocks.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        step(i, kev[i])
    e1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    k_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    if world > 1:
        t = torch.tensor([ms, k_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, k_ms = t.tolist()
    ms_step = ms / K
    tokens_step = B * cfg.L
    value = tokens_step / (ms_step / 1e3)
    eb = 4 if cfg.dtype == torch.float32 else 2
    fwd_bytes, _ = algorithmic_bytes(B, Ls, D, N, eb, fused=True, backward=False)
    peak, peak_kind = measured_peak()
    achieved = fwd_bytes / (k_ms / 1e3) / 1e9

    # e2e: public API with this rank's shard in pinned host memory
    host = {k: data[0][k].cpu().pin_memory() for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")}
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    y_host = torch.empty(B, Ls, D, dtype=cfg.dtype, pin_memory=True)
    last_host = torch.empty(B, D, N, dtype=torch.float32, pin_memory=True)
    d2h = y_host.numel() * y_host.element_size() + last_host.numel() * 4

    def e2e_step():
        dv = {k: v.to(device, non_blocking=True) for k, v in host.items()}
        scan = sharding.sequence_sharded_scan if world > 1 else selective_scan_fused
        y, last = scan(dv["u"], dv["delta"], dv["A"], dv["Bm"], dv["Cm"], D=dv["Dskip"], z=dv["z"])
        y_host.copy_(y, non_blocking=True)
        last_host.copy_(last, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    a1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = a0.elapsed_time(a1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = t.item()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc, _ = cpu_reference_sample(cfg, budget_s=12.0, b_rows=1, d_slice=16, backward=False)
        cpu = {"value": rate, "unit": "tokens/s", "cores": torch.get_num_threads(), "cpu_model": cpu_model(),
               "kind": "port",
               "sample": desc + "; tokens counted in 512-channel units; oracle/scan_oracle.py restates "
                                "models/scan.py (chunked scan)"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload, "B": B, "L": cfg.L, "L_per_gpu": Ls, "D": D, "N": N,
                       "activations": str(cfg.dtype).replace("torch.", ""), "fused_gate": True,
                       "parallelism": f"sequence-sharded x{world} (strong)" if world > 1 else "single GPU",
                       "l2": f"{sets} rotating input set(s), inputs > 126 MB L2",
                       "token": "one (batch, position) row through 512 channels"},
            "roofline": {"kernel": "ssm_scan_fwd" if world == 1 else "ssm_scan_fwd_finish", "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s", "traffic": None,
                         "algorithmic_bytes_per_launch": fwd_bytes, "avg_launch_ms": k_ms},
            "e2e": {"value": tokens_step / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": args.e2e_steps},
            "gpu_launches": K * launches,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_lm(args, rank, world, device):
    """Config 4: training step and graph decode of the Mamba LM on the sm_100a ops (1 GPU)."""
    from mamba_ssm_benchmark_b200.mixer import GraphDecoder, MambaLM
    from mamba_ssm_benchmark_b200.workloads import markov_bytes
    if world > 1:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "config": {"workload": "cfg4_mamba_lm"},
                              "unavailable": "config 4 is a single-GPU workload"}), flush=True)
        return
    torch.manual_seed(0)
    model = MambaLM(n_layers=11, d_model=256, d_state=16, expand=2, d_conv=4).to(device)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    host = markov_bytes(16, 513, seed=0).pin_memory()
    data = host.to(device)
    stream = torch.cuda.current_stream(device)

    def train_step(batch):
        logits = model(batch[:, :-1])
        loss = F.cross_entropy(logits.reshape(-1, 256), batch[:, 1:].reshape(-1))
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(args.warmup):
        train_step(data)
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        train_step(data)
    e1.record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    tokens = 16 * 512
    # e2e: the batch comes from pinned host memory and the loss goes back every step
    loss_host = torch.empty((), dtype=torch.float32, pin_memory=True)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(args.e2e_steps):
        loss = train_step(host.to(device, non_blocking=True))
        loss_host.copy_(loss.detach(), non_blocking=True)
    a1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = a0.elapsed_time(a1) / args.e2e_steps

    decode = {}
    model.eval()
    for bsz in (1, 64):
        with torch.no_grad():
            prompt = markov_bytes(bsz, 16, seed=bsz).to(device)
            states = model.init_state(bsz, 16 + 256, device)
            model(prompt, states, 0)
            step = GraphDecoder(model, states)
            tok = prompt[:, -1:]
            for _ in range(5):
                step(tok)
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            d0.record(stream)
            for _ in range(256):
                tok = step(tok)[:, -1].argmax(-1, keepdim=True)
            d1.record(stream)
            torch.cuda.synchronize(device)
            decode[f"batch{bsz}_ms_per_token"] = d0.elapsed_time(d1) / 256
            del step, states
    per_layer = 2 + 4       # conv fwd + scan fwd; scan bwd + finalize + conv bwd + finalize
    line = {"metric": "Mamba LM training tokens/s (16 x 512, incl. AdamW) and decode ms/token", "value": tokens / ms * 1e3,
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded order-2 Markov bytes)",
            "config": {"workload": "cfg4_mamba_lm_L11_d256_B16_T512", "layers": 11, "d_model": 256, "d_state": 16,
                       "global_batch": 16, "seq_len": 512, "optimizer": "AdamW (fused) + clip 1.0"},
            "decode": decode,
            "e2e": {"value": tokens / e2e_ms * 1e3, "unit": "tokens/s", "h2d_bytes_per_step": host.numel() * 8,
                    "d2h_bytes_per_step": 4, "steps": args.e2e_steps},
            "gpu_launches": args.steps * 11 * per_layer,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    from mamba_ssm_benchmark_b200.workloads import CONFIGS, algorithmic_bytes
    cfg = CONFIGS.get(args.config)
    workload = cfg.name if cfg is not None else "cfg4_mamba_lm_L11_d256_B16_T512"
    if args.impl == "reference":
        if cfg is None:
            if dist_env()[0] == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the scan path; "
                                  "config 4 (full LM) has no CPU-reference arm here"}), flush=True)
            return
        run_reference(args, cfg, workload)
        return
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    if args.config == 2:
        run_sequence_shards(args, cfg, workload, rank, world, device)
        return
    if args.config == 4:
        run_lm(args, rank, world, device)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    from mamba_ssm_benchmark_b200 import sharding
    sets = 4 if args.config == 1 else 1
    steps = [ScanStep(cfg, device, seed=1000 * s + rank, shared_seed=1000 * s) for s in range(sets)]
    stream = torch.cuda.current_stream(device)
    dBC_bufs = [st.dBC for st in steps]

    # N > 1: the dB|dC all-reduce of step i runs on a side stream while step i + 1's forward runs;
    # a set's next backward (which rewrites its dB|dC buffer) waits for that set's all-reduce.
    comm = torch.cuda.Stream(device) if world > 1 else None
    bwd_done = [torch.cuda.Event() for _ in range(sets)]
    comm_done = [torch.cuda.Event() for _ in range(sets)]

    def one(i, ev=None):
        k = i % sets
        st = steps[k]
        st.fwd()
        if ev is not None:
            ev[0].record(stream)
        if world > 1 and i >= sets:
            stream.wait_event(comm_done[k])
        st.bwd()
        if ev is not None:
            ev[1].record(stream)
        if world > 1:
            bwd_done[k].record(stream)
            comm.wait_event(bwd_done[k])
            with torch.cuda.stream(comm):
                sharding.reduce_shared_grads([dBC_bufs[k]])
            comm_done[k].record(comm)

    def drain():
        if comm is not None:
            stream.wait_stream(comm)

    for i in range(args.warmup):
        one(i)
    drain()
    torch.cuda.synchronize(device)
    K = args.steps
    bev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        one(i, bev[i])
    drain()
    e1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in bev)
    if world > 1:
        t = torch.tensor([ms, bwd_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, bwd_ms = t.tolist()
    ms_step = ms / K
    tokens_step = cfg.B * cfg.L * world
    value = tokens_step / (ms_step / 1e3)
    eb = 4 if cfg.dtype == torch.float32 else 2
    fwd_bytes, bwd_bytes = algorithmic_bytes(cfg.B, cfg.L, cfg.D, cfg.N, eb, fused=True, backward=True)
    peak, peak_kind = measured_peak()
    achieved = bwd_bytes / (bwd_ms / 1e3) / 1e9
    step_gbs = (fwd_bytes + bwd_bytes) / (ms_step / 1e3) / 1e9
    traffic = ncu_traffic(workload)

    e2e_ms, h2d, d2h = e2e_run(cfg, device, args.e2e_steps, world, seed=77 + rank)
    e2e_value = tokens_step / (e2e_ms / 1e3)
    link = host_link(device, h2d, d2h, tokens_step, e2e_value, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc, _ = cpu_reference_sample(cfg, budget_s=12.0, b_rows=max(1, cfg.B // 8) if cfg.B > 1 else 1,
                                             d_slice=cfg.D if args.config == 1 else 128)
        cpu = {"value": rate, "unit": "tokens/s", "cores": torch.get_num_threads(), "cpu_model": cpu_model(),
               "kind": "port",
               "sample": desc + "; oracle/scan_oracle.py restates models/scan.py (chunked scan)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload, "B": cfg.B, "L": cfg.L, "D_per_gpu": cfg.D, "N": cfg.N,
                       "activations": str(cfg.dtype).replace("torch.", ""), "fused_gate": True,
                       "parallelism": f"channel-sharded x{world} (weak)" if world > 1 else "single GPU",
                       "l2": f"{sets} rotating buffer sets" + (" (>126 MB L2)" if sets > 1 else
                                                                " (inputs > 126 MB L2)"),
                       "token": "one (batch, position) row through a 512-channel shard"},
            "hbm_gbs_step": step_gbs, "hbm_frac_step": step_gbs / peak,
            "roofline": {"kernel": "ssm_scan_bwd (ssm_bwd_kernel + ssm_bwd_finalize)", "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s", "traffic": traffic,
                         "algorithmic_bytes_per_launch": bwd_bytes, "avg_launch_ms": bwd_ms,
                         "mufu": mufu_bound(cfg, bwd_ms, clk)},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": args.e2e_steps, "link": link},
            "gpu_launches": K * steps[0].launches,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
