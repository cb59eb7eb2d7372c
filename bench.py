#!/usr/bin/env python
"""Selective-scan (Mamba S6) fwd+bwd throughput on B200 — the BASELINE workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 0|1|2|3|4]

Default (--config 1): one JSON line (rank 0) whose headline is config 1 -- the fused selective
scan forward + backward over B=16, L=512, D=512, N=16, fp32, with the mixer's D-skip and SiLU(z)
gate, through the C ABI of libssm_b200.so -- and whose "sub_records" time the other scan
configurations in the same run, each with its own rooflines, e2e and (1 GPU) CPU baseline:
    cfg3  fwd+bwd, bf16, B=8, L=8192, D=5120 (1 GPU: the whole layer; N GPUs: the same layer
          channel-sharded, D/N channels per GPU, NCCL all-reduce of dB|dC: strong scaling)
    cfg2  forward, fp32, B=1, L=131072, D=512 (N GPUs: the sequence split into N contiguous
          shards, summaries all-gathered over NCCL: strong scaling)
    cfg0  forward, fp32, B=1, L=4096, D=512 (1 GPU only)

value  : whole-job tokens/s with inputs resident in HBM (CUDA events around exactly K steps,
         barrier + synchronize on both sides, max over ranks).  A token is one (batch, position)
         row through all D channels of the workload's layer.  Config 1 rotates 4 input/output sets
         (~0.5 GB) so that every step touches buffers evicted from the 126 MB L2; the other
         workloads' inputs are larger than L2.
e2e    : the same metric through the public Python API (selective_scan_fused + autograd
         backward) with pinned host inputs and outputs: H2D copies, fwd, bwd and D2H copies of
         every output inside the timed region.
N > 1  : one process per GPU (torchrun).  Headline (config 1), weak scaling: every rank owns a
         512-channel shard of a (512 N)-channel layer; B and C are shared, so the backward ends
         with an NCCL all-reduce of dB|dC, overlapped with the next step's forward.  The job
         processes N x B x L 512-channel tokens per step.  After the timed region every record
         checks its own results (parity_ok): the all-reduced dB|dC against the sum of the
         gathered per-rank partials, and a slice of every rank's outputs and gradients against
         the CPU oracle; per_rank gives each rank's forward, backward and all-reduce times.
--config 2|3|0 : that workload alone, as the headline.
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


def parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, choices=(0, 1, 2, 3, 4), default=1)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="headline only (no sub-records)")
    ap.add_argument("--shape", default=None,
                    help="B,L,D overriding the workload's shape (a smaller case of it, for profiling)")
    return ap.parse_args(argv)


def workload_config(args, cfg_id):
    """CONFIGS[cfg_id], with --shape applied when it names this workload (the headline)."""
    import dataclasses
    from mamba_ssm_benchmark_b200.workloads import CONFIGS
    cfg = CONFIGS[cfg_id]
    if args.shape and cfg_id == args.config:
        B, L, D = (int(v) for v in args.shape.split(","))
        cfg = dataclasses.replace(cfg, B=B, L=L, D=D, name=f"{cfg.name}_shape{B}x{L}x{D}")
    return cfg


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def dtype_name(dt):
    return {torch.float32: "f32", torch.bfloat16: "bf16"}[dt]


def config_of(cfg):
    """The workload's `config` object, identical in both arms (this one and --impl reference)."""
    return {"workload": cfg.name, "B": cfg.B, "L": cfg.L, "D": cfg.D, "N": cfg.N,
            "activations": dtype_name(cfg.dtype), "pass": "fwd+bwd" if cfg.backward else "fwd",
            "fused_gate": True}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def hbm_roofline(kernel, workload, alg_bytes, avg_ms):
    """The HBM roofline object of one kernel: algorithmic bytes per launch / CUDA-event duration,
    against the measured copy bandwidth; traffic = ncu DRAM bytes per launch (None if not captured)."""
    from mamba_ssm_benchmark_b200.workloads import NCU_TRAFFIC
    peak, kind = measured_peak()
    achieved = alg_bytes / (avg_ms / 1e3) / 1e9
    return {"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else "fallback 6.65 TB/s",
            "traffic": NCU_TRAFFIC.get((kernel, workload)), "algorithmic_bytes_per_launch": alg_bytes,
            "avg_launch_ms": avg_ms}


def mufu_bound(B, L, D, N, exps_per_state, ms, clk):
    """Special-function (MUFU) roofline: exps_per_state ex2 per (t, d, n) plus the gate's sigmoid
    (ex2 + rcp) per (t, d), at 16 MUFU results per clock per SM (measured on this B200 pool)."""
    ops = exps_per_state * B * L * D * N + 2 * B * L * D
    mhz = clk.get("sm_mhz") or 1965.0
    peak = 16 * 148 * mhz * 1e6
    achieved = ops / (ms / 1e3)
    return {"ops_per_launch": ops, "unit": "MUFU ops/s", "achieved": achieved, "peak": peak, "frac": achieved / peak,
            "peak_source": "16 ops/clk/SM (measured ex2 throughput) x 148 SMs x median SM clock"}


def max_over_ranks(vals, world, device):
    """Element-wise max over ranks of a list of floats (identity at world 1)."""
    if world == 1:
        return list(vals)
    t = torch.tensor(list(vals), dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


def gather_ranks(vals, world, device):
    """Every rank's list of floats, indexed by rank."""
    if world == 1:
        return [list(vals)]
    t = torch.tensor(list(vals), dtype=torch.float64, device=device)
    parts = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(parts, t)
    return [p.tolist() for p in parts]


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


def clocks_record(clk):
    return {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
            "samples": clk["samples"]}


# --------------------------------------------------------------------------------------------
# the GPU arm: channel-sharded fwd+bwd (configs 1 and 3)
# --------------------------------------------------------------------------------------------
class ChannelStep:
    """Pre-marshalled C-ABI calls of one fused fwd+bwd step over one buffer set: this rank's
    channel shard (D_local channels) of the workload, B and C shared by all shards."""

    def __init__(self, cfg, D_local, device, seed, shared_seed, on_device):
        from mamba_ssm_benchmark_b200 import _native as nat
        from mamba_ssm_benchmark_b200.workloads import make_inputs
        self.nat = nat
        B, L, N = cfg.B, cfg.L, cfg.N
        D = D_local
        dt = cfg.dtype
        ins = make_inputs(B, L, D, N, seed=seed, dist="config", dtype=dt, device=device, draw_on_device=on_device)
        shared = make_inputs(B, L, 1, N, seed=shared_seed, dist="config", dtype=dt, device=device,
                             draw_on_device=on_device)
        ins["Bm"], ins["Cm"] = shared["Bm"], shared["Cm"]
        self.t = t = ins
        f32 = dict(dtype=torch.float32, device=device)
        self.shape = (B, L, D, N)
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
                         self.fw.data_ptr(), self.fws, stream)
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


def time_channel_steps(steps_sets, K, warmup, world, device):
    """K fused fwd+bwd steps rotating over the buffer sets; at world > 1 the dB|dC all-reduce of
    step i runs on a side stream under step i+1's forward (a set's next backward waits for it).
    Returns (ms per step, mean fwd ms, mean bwd ms, mean all-reduce ms), each max over ranks, the
    same per rank (list), and the clocks seen during the timed region."""
    from mamba_ssm_benchmark_b200 import sharding
    sets = len(steps_sets)
    stream = torch.cuda.current_stream(device)
    comm = torch.cuda.Stream(device) if world > 1 else None
    bwd_done = [torch.cuda.Event() for _ in range(sets)]
    comm_done = [torch.cuda.Event() for _ in range(sets)]
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def one(i, rec=None):
        k = i % sets
        st = steps_sets[k]
        if rec is not None:
            rec[0].record(stream)
        st.fwd()
        if rec is not None:
            rec[1].record(stream)
        if world > 1 and i >= sets:
            stream.wait_event(comm_done[k])
        st.bwd()
        if rec is not None:
            rec[2].record(stream)
        if world > 1:
            bwd_done[k].record(stream)
            comm.wait_event(bwd_done[k])
            if rec is not None:
                rec[3].record(comm)
            with torch.cuda.stream(comm):
                sharding.reduce_shared_grads([st.dBC])
            if rec is not None:
                rec[4].record(comm)
            comm_done[k].record(comm)

    def drain():
        if comm is not None:
            stream.wait_stream(comm)

    for i in range(warmup):
        one(i)
    drain()
    torch.cuda.synchronize(device)
    recs = [[ev() for _ in range(5)] for _ in range(K)]
    clocks = ClockSampler(device.index)
    clocks.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = ev(), ev()
    e0.record(stream)
    for i in range(K):
        one(i, recs[i])
    drain()
    e1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / K
    fwd_ms = statistics.mean(r[0].elapsed_time(r[1]) for r in recs)
    bwd_ms = statistics.mean(r[1].elapsed_time(r[2]) for r in recs)
    ar_ms = statistics.mean(r[3].elapsed_time(r[4]) for r in recs) if world > 1 else 0.0
    mine = [ms, fwd_ms, bwd_ms, ar_ms]
    per_rank = gather_ranks(mine, world, device)
    worst = max_over_ranks(mine, world, device)
    return worst, per_rank, clk


def e2e_channel(cfg, ins, device, steps, world):
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
    on the copy stream instead kept the allocator growing with fresh device allocations).
    ``ins``: this rank's inputs (any device); returns (ms per step max over ranks, h2d, d2h)."""
    from mamba_ssm_benchmark_b200 import selective_scan_fused, sharding
    names = [k for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "dy") if ins.get(k) is not None]
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
    ms = max_over_ranks([e0.elapsed_time(e1) / steps], world, device)[0]
    return ms, h2d, d2h


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
    ms = max_over_ranks([e0.elapsed_time(e1) / reps], world, device)[0]
    bound = tokens_step / (ms / 1e3)
    return {"ms_per_step": ms, "gbs": (h2d + d2h) / (ms / 1e3) / 1e9, "bound_value": bound,
            "frac": e2e_value / bound,
            "what": "pinned H2D of the step's input bytes and D2H of its output bytes, at the same time"}


# --------------------------------------------------------------------------------------------
# the CPU baseline (oracle port of the reference's chunked scan) and the reference arm
# --------------------------------------------------------------------------------------------
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


def cpu_reference_sample(cfg, budget_s, d_slice=None, b_rows=None, l_len=None, repeats_min=3):
    """Oracle port (the reference's chunked CPU scan + recomputing backward) on a slice of the
    workload (bf16 workloads: the same bf16-rounded values in fp32, as the reference promotes
    them); returns (tokens/s with a token = one (batch, position) row through the workload's D
    channels, description, samples).  Channels and rows are independent in the scan, so the rate
    scales linearly to the full workload."""
    from mamba_ssm_benchmark_b200.workloads import make_inputs
    from oracle import scan_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    b = b_rows or cfg.B
    d = d_slice or cfg.D
    L = l_len or cfg.L
    ins = make_inputs(b, L, d, cfg.N, seed=0, dist="config", dtype=cfg.dtype)
    ins = {k: (v.float() if v is not None else None) for k, v in ins.items()}

    def one():
        lv = [ins[k].clone().requires_grad_() for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")]
        y, _ = O.selective_scan_fused(lv[0], lv[1], lv[2], lv[3], lv[4], Dskip=lv[5], z=lv[6])
        if cfg.backward:
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
    tokens = b * L * d / cfg.D
    desc = (f"B={b} of {cfg.B} rows, L={L}{'' if L == cfg.L else f' of {cfg.L}'}, {d} of {cfg.D} channels, "
            f"N={cfg.N}, fused {'fwd+bwd' if cfg.backward else 'fwd'}; median of {len(times)}; tokens counted "
            f"through all {cfg.D} channels (linear in channels); oracle/scan_oracle.py restates models/scan.py "
            f"(chunked scan)")
    return tokens / med, desc, times


# CPU-baseline slices per workload: (rows, channels, seconds of sampling)
CPU_SLICES = {0: (1, 512, 6.0), 1: (2, 512, 12.0), 2: (1, 16, 8.0), 3: (1, 64, 8.0)}


def cpu_baseline(cfg_id, cfg):
    rows, chans, budget = CPU_SLICES[cfg_id]
    rate, desc, _ = cpu_reference_sample(cfg, budget_s=budget, d_slice=chans, b_rows=rows)
    return {"value": rate, "unit": "tokens/s", "cores": torch.get_num_threads(), "cpu_model": cpu_model(),
            "kind": "port", "sample": desc}


def run_reference(args, cfg):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    # size one "step" so that warmup + steps fit in ~150 s of host time
    budget = 150.0 / max(1, args.steps + args.warmup)
    _, _, probe = cpu_reference_sample(cfg, 0.0, d_slice=min(cfg.D, 64), b_rows=1, repeats_min=1)
    t_probe = statistics.median(probe)
    d_s = int(max(8, min(cfg.D, 64 * budget / max(t_probe, 1e-6))) // 8 * 8)
    b_s = 1
    if d_s >= cfg.D:
        d_s = cfg.D
        b_s = int(max(1, min(cfg.B, budget / max(t_probe * cfg.D / 64, 1e-6))))
    from oracle import scan_oracle as O
    from mamba_ssm_benchmark_b200.workloads import make_inputs
    ins = make_inputs(b_s, cfg.L, d_s, cfg.N, seed=0, dist="config", dtype=cfg.dtype)
    ins = {k: (v.float() if v is not None else None) for k, v in ins.items()}

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
    tokens = b_s * cfg.L * d_s / cfg.D
    value = tokens * args.steps / dt
    sample = (f"per step: B={b_s} of {cfg.B} rows, L={cfg.L}, {d_s} of {cfg.D} channels, N={cfg.N}, fused "
              f"{'fwd+bwd' if cfg.backward else 'fwd'} (tokens counted through all {cfg.D} channels)")
    cores = torch.get_num_threads()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong" if args.config in (2, 3) else "weak", "vs_baseline": None,
            "dtype": dtype_name(cfg.dtype), "data": "synthetic", "config": config_of(cfg),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "cpu_model": cpu_model(),
                             "kind": "port",
                             "sample": sample + "; oracle/scan_oracle.py restates models/scan.py (chunked)"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------
# self-checks after the timed region (parity_ok)
# --------------------------------------------------------------------------------------------
def oracle_slice_errors(ins, lo, d_n, l_n, device, dtype):
    """This rank's GPU op vs the CPU oracle on a slice of its own inputs (batch row 0, the first
    l_n steps, channels [lo, lo + d_n)): max normwise error of y and of every gradient."""
    from mamba_ssm_benchmark_b200 import selective_scan_fused
    from oracle import scan_oracle as O
    sl = {k: ins[k][:1, :l_n, lo:lo + d_n] for k in ("u", "delta", "z", "dy")}
    sl.update(Bm=ins["Bm"][:1, :l_n], Cm=ins["Cm"][:1, :l_n], A=ins["A"][lo:lo + d_n], Dskip=ins["Dskip"][lo:lo + d_n])
    names = ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")

    def run(dev, dt):
        lv = [sl[k].to(dev, dt if k not in ("A", "Dskip") else torch.float32).clone().requires_grad_() for k in names]
        if dev == "cpu":
            y, _ = O.selective_scan_fused(lv[0], lv[1], lv[2], lv[3], lv[4], Dskip=lv[5], z=lv[6])
        else:
            y, _ = selective_scan_fused(lv[0], lv[1], lv[2], lv[3], lv[4], D=lv[5], z=lv[6])
        g = torch.autograd.grad(y, lv, sl["dy"].to(dev, dt))
        return [y] + list(g)

    got = run(device, dtype)
    ref = run("cpu", torch.float32)
    errs = [O.normwise_error(a.float(), b.float()) for a, b in zip(got, ref)]
    return errs[0], max(errs[1:])


def channel_parity(st, cfg, world, device):
    """Checks after the timed region: (1) the all-reduced dB|dC equals the sum of every rank's
    partial (gathered, summed in rank order); (2) a slice of this rank's outputs and gradients
    matches the CPU oracle.  Returns the record's parity object (same on every rank)."""
    from mamba_ssm_benchmark_b200 import sharding
    st.fwd()
    st.bwd()
    part = st.dBC.float().clone()
    if world > 1:
        sharding.reduce_shared_grads([st.dBC])
        parts = [torch.empty_like(part) for _ in range(world)]
        torch.distributed.all_gather(parts, part)
        ref = parts[0].clone()
        for p_ in parts[1:]:
            ref += p_
        ar_err = ((st.dBC.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
    else:
        ar_err = 0.0
    y_err, g_err = oracle_slice_errors(st.t, 0, min(64, st.shape[2]), min(256, cfg.L), device, cfg.dtype)
    bf = cfg.dtype == torch.bfloat16
    # bf16: every partial is rounded to bf16 and NCCL adds in bf16 (a few bf16 roundings)
    tol_ar, tol_y, tol_g = (2e-2, 1e-2, 1e-2) if bf else (1e-5, 1e-4, 1e-3)
    worst = max_over_ranks([ar_err, y_err, g_err], world, device)
    ok = worst[0] <= tol_ar and worst[1] <= tol_y and worst[2] <= tol_g
    return {"parity_ok": bool(ok),
            "parity": {"allreduce_max_rel": worst[0], "oracle_y_normwise": worst[1], "oracle_grad_normwise": worst[2],
                       "tol": {"allreduce": tol_ar, "y": tol_y, "grads": tol_g},
                       "what": "all-reduced dB|dC vs the rank-order sum of the gathered partials; every rank's "
                               "outputs and gradients on a slice (batch row 0, 256 steps, 64 channels) vs the "
                               "CPU oracle; max over ranks"}}


# --------------------------------------------------------------------------------------------
# records
# --------------------------------------------------------------------------------------------
def channel_record(args, cfg_id, scaling, rank, world, device, sets, cpu):
    """Configs 1 (weak: every rank a full D-channel layer shard) and 3 (strong: D split over the
    ranks).  Returns the record (meaningful on rank 0)."""
    from mamba_ssm_benchmark_b200 import sharding
    from mamba_ssm_benchmark_b200.workloads import algorithmic_bytes
    cfg = workload_config(args, cfg_id)
    if scaling == "strong":
        lo, hi = sharding.shard_range(cfg.D, world, rank)
    else:
        lo, hi = 0, cfg.D
    D_local = hi - lo
    big = cfg.B * cfg.L * cfg.D > (1 << 26)
    steps = [ChannelStep(cfg, D_local, device, seed=1000 * s + rank, shared_seed=1000 * s, on_device=big)
             for s in range(sets)]
    K = args.steps
    worst, per_rank, clk = time_channel_steps(steps, K, args.warmup, world, device)
    ms, fwd_ms, bwd_ms, ar_ms = worst
    tokens_step = cfg.B * cfg.L * (world if scaling == "weak" else 1)
    value = tokens_step / (ms / 1e3)
    eb = 4 if cfg.dtype == torch.float32 else 2
    fwd_bytes, bwd_bytes = algorithmic_bytes(cfg.B, cfg.L, D_local, cfg.N, eb, fused=True, backward=True)
    rec = {"workload": cfg.name, "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
           "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling,
           "dtype": dtype_name(cfg.dtype), "config": config_of(cfg),
           "setup": {"D_per_gpu": D_local,
                     "parallelism": (f"channel-sharded x{world} ({scaling})" if world > 1 else "single GPU"),
                     "l2": f"{sets} rotating buffer sets (> 126 MB L2)" if sets > 1 else "inputs > 126 MB L2",
                     "token": f"one (batch, position) row through {'a ' if scaling == 'weak' and world > 1 else ''}"
                              f"{cfg.D} channels{' per rank' if scaling == 'weak' and world > 1 else ''}"},
           "hbm_gbs_step": (fwd_bytes + bwd_bytes) / (ms / 1e3) / 1e9,
           "roofline": dict(hbm_roofline("ssm_scan_bwd", cfg.name, bwd_bytes, bwd_ms),
                            mufu=mufu_bound(cfg.B, cfg.L, D_local, cfg.N, 1, bwd_ms, clk)),
           "roofline_fwd": dict(hbm_roofline("ssm_scan_fwd", cfg.name, fwd_bytes, fwd_ms),
                                mufu=mufu_bound(cfg.B, cfg.L, D_local, cfg.N, 1, fwd_ms, clk)),
           "gpu_launches": K * steps[0].launches, "clocks": clocks_record(clk)}
    rec["hbm_frac_step"] = rec["hbm_gbs_step"] / measured_peak()[0]
    if world > 1:
        rec["per_rank"] = [{"rank": r, "ms_per_step": v[0], "fwd_ms": v[1], "bwd_ms": v[2], "allreduce_ms": v[3]}
                           for r, v in enumerate(per_rank)]
    rec.update(channel_parity(steps[0], cfg, world, device))
    e2e_steps = args.e2e_steps if cfg_id == 1 else min(args.e2e_steps, 4)
    e2e_ms, h2d, d2h = e2e_channel(cfg, steps[0].t, device, e2e_steps, world)
    e2e_value = tokens_step / (e2e_ms / 1e3)
    rec["e2e"] = {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                  "steps": e2e_steps, "link": host_link(device, h2d, d2h, tokens_step, e2e_value, world)}
    if cpu and rank == 0 and world == 1:
        rec["cpu_baseline"] = cpu_baseline(cfg_id, cfg)
    del steps
    torch.cuda.empty_cache()
    return rec


def sequence_record(args, cfg_id, rank, world, device, cpu):
    """Config 2 (and config 0 at one GPU): one long sequence, forward.  At world > 1 the sequence is
    split into ``world`` contiguous shards (strong scaling): per step and rank, summary pass over
    the shard, NCCL all-gather of the (decay, hend) summaries, prefix composition, finish pass from
    the carried-in state.  On one GPU the step is a single ssm_scan_fwd over the whole sequence
    (which splits it into segments itself)."""
    from mamba_ssm_benchmark_b200 import _native as nat
    from mamba_ssm_benchmark_b200 import selective_scan_fused, sharding
    from mamba_ssm_benchmark_b200.workloads import algorithmic_bytes, make_inputs
    cfg = workload_config(args, cfg_id)
    lo, hi = sharding.shard_range(cfg.L, world, rank)
    Ls = hi - lo
    B, D, N = cfg.B, cfg.D, cfg.N
    eb = 4 if cfg.dtype == torch.float32 else 2
    # inputs above L2 per step: rotate sets when one set is smaller than twice the L2
    set_bytes = 4 * B * Ls * D * eb
    sets = max(1, min(8, math.ceil(2 * 126e6 / set_bytes)))
    stream = torch.cuda.current_stream(device)
    lib = nat.lib()
    data = [make_inputs(B, Ls, D, N, seed=100 * s_ + rank, dist="config", dtype=cfg.dtype, device=device,
                        draw_on_device=True) for s_ in range(sets)]
    if world == 1:
        outs = [(torch.empty(B, Ls, D, dtype=cfg.dtype, device=device),
                 torch.empty(B, D, N, dtype=torch.float32, device=device)) for _ in range(sets)]
        wsb = nat.fwd_workspace_bytes(B, Ls, D, N)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=device)
        launches = 1 if wsb == 0 else 3
        kernel = "ssm_scan_fwd"

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
        kernel = "ssm_scan_fwd_finish"

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

    K = args.steps if cfg_id == 2 else max(args.steps, 200)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(device)
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
    mine = [e0.elapsed_time(e1) / K, statistics.mean(a.elapsed_time(b) for a, b in kev)]
    per_rank = gather_ranks(mine, world, device)
    ms_step, k_ms = max_over_ranks(mine, world, device)
    tokens_step = B * cfg.L
    value = tokens_step / (ms_step / 1e3)
    fwd_bytes, _ = algorithmic_bytes(B, Ls, D, N, eb, fused=True, backward=False)

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
    e2e_steps = args.e2e_steps
    a0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    a1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks([a0.elapsed_time(a1) / e2e_steps], world, device)[0]

    rec = {"workload": cfg.name, "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
           "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
           "scaling": "strong" if cfg_id == 2 else "weak", "dtype": dtype_name(cfg.dtype), "config": config_of(cfg),
           "setup": {"L_per_gpu": Ls, "parallelism": f"sequence-sharded x{world} (strong)" if world > 1 else "single GPU",
                     "l2": f"{sets} rotating input set(s), inputs > 126 MB L2 per step",
                     "token": f"one (batch, position) row through {D} channels"},
           "roofline": hbm_roofline(kernel, cfg.name, fwd_bytes, k_ms),
           "e2e": {"value": tokens_step / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "steps": e2e_steps},
           "gpu_launches": K * launches, "clocks": clocks_record(clk)}
    rec["roofline"]["mufu"] = mufu_bound(B, Ls, D, N, 1, k_ms, clk)
    if world > 1:
        rec["per_rank"] = [{"rank": r, "ms_per_step": v[0], "finish_ms": v[1]} for r, v in enumerate(per_rank)]
    rec.update(sequence_parity(cfg, rank, world, device))
    if cpu and rank == 0 and world == 1:
        rec["cpu_baseline"] = cpu_baseline(cfg_id, cfg)
    del data
    torch.cuda.empty_cache()
    return rec


def sequence_parity(cfg, rank, world, device, d_n=8):
    """The sequence path on a channel slice of the whole sequence (every rank draws the same slice
    on the CPU): this rank's shard of y (sharded protocol at world > 1, one call at world 1) against
    the CPU oracle's y over the whole sequence, normwise; max over ranks."""
    from mamba_ssm_benchmark_b200 import selective_scan_fused, sharding
    from mamba_ssm_benchmark_b200.workloads import make_inputs
    from oracle import scan_oracle as O
    ins = make_inputs(cfg.B, cfg.L, d_n, cfg.N, seed=7, dist="config", dtype=cfg.dtype)
    lo, hi = sharding.shard_range(cfg.L, world, rank)
    dv = {k: ins[k].to(device) for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")}
    sl = lambda t: t[:, lo:hi].contiguous()
    if world > 1:
        y, last = sharding.sequence_sharded_scan(sl(dv["u"]), sl(dv["delta"]), dv["A"], sl(dv["Bm"]), sl(dv["Cm"]),
                                                 D=dv["Dskip"], z=sl(dv["z"]))
    else:
        y, last = selective_scan_fused(dv["u"], dv["delta"], dv["A"], dv["Bm"], dv["Cm"], D=dv["Dskip"], z=dv["z"])
    yr, lr = O.selective_scan_fused(*(ins[k].float() for k in ("u", "delta", "A", "Bm", "Cm")),
                                    Dskip=ins["Dskip"], z=ins["z"].float())
    err_y = O.normwise_error(y.float(), yr[:, lo:hi])
    err_l = O.normwise_error(last, lr)
    worst = max_over_ranks([err_y, err_l], world, device)
    tol = 1e-2 if cfg.dtype == torch.bfloat16 else 1e-4
    return {"parity_ok": bool(worst[0] <= tol and worst[1] <= tol),
            "parity": {"oracle_y_normwise": worst[0], "oracle_last_normwise": worst[1], "tol": tol,
                       "what": f"y of every rank's shard and the final state vs the CPU oracle over the whole "
                               f"sequence, {d_n}-channel slice; max over ranks"}}


def headline_line(rec, world):
    """The driver-facing line: the record's keys plus the base contract's."""
    line = {k: v for k, v in rec.items() if k != "workload"}
    line["vs_baseline"] = None
    line["data"] = "synthetic"
    return line


# --------------------------------------------------------------------------------------------
# config 4: the Mamba LM
# --------------------------------------------------------------------------------------------
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
            "gpu_launches": args.steps * 11 * per_layer, "clocks": clocks_record(clk)}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    cfg = workload_config(args, args.config) if args.config != 4 else None
    if args.impl == "reference":
        if cfg is None:
            if dist_env()[0] == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the scan path; "
                                  "config 4 (full LM) has no CPU-reference arm here"}), flush=True)
            return
        run_reference(args, cfg)
        return
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        if args.config == 4:
            run_lm(args, rank, world, device)
            return
        cpu = not args.no_cpu_baseline
        if args.config in (0, 2):
            rec = sequence_record(args, args.config, rank, world, device, cpu)
        elif args.config == 3:
            rec = channel_record(args, 3, "strong" if world > 1 else "weak", rank, world, device, 1, cpu)
        else:
            rec = channel_record(args, 1, "weak", rank, world, device, 4, cpu)
            if not args.no_sub:
                subs = [channel_record(args, 3, "strong" if world > 1 else "weak", rank, world, device, 1, cpu),
                        sequence_record(args, 2, rank, world, device, cpu)]
                if world == 1:
                    subs.append(sequence_record(args, 0, rank, world, device, cpu))
                rec["sub_records"] = subs
        if rank == 0:
            print(json.dumps(headline_line(rec, world)), flush=True)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
