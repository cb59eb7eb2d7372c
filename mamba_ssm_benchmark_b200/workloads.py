"""Seeded synthetic workloads of the selective-scan benchmark (no dataset is involved).

CONFIGS mirrors the scan configurations the benchmark is quoted on (0-3); inputs are drawn on
the CPU from ``torch.Generator().manual_seed(seed)`` in a fixed order, so the CPU oracle and
the GPU see identical values:

    u, delta_raw, Bm, Cm, Dskip, z, dy, (h0), (dlast)

Distributions ("config"):  u, Bm, Cm, Dskip, z, dy ~ N(0, 1);
    delta = softplus(0.5 N(0,1) + log(expm1(0.01)))  (mean ~0.011, as a Mamba dt_proj at init);
    A = -exp(A_log), A_log[d, n] = log(n + 1)  ->  A[d, n] = -(n + 1)  (S4D-real init,
    models/mamba.py:60-64; benchmarks/bench_scan.py:29).
Distributions ("test"): the reference's GPU differential tests (tests/test_triton.py:17-25):
    x, Bm, Cm, h0 ~ N(0,1); delta ~ U[1e-3, 0.301]; A ~ -U[0.05, 4.05].
"""

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ScanConfig:
    name: str
    B: int
    L: int
    D: int
    N: int
    dtype: torch.dtype
    backward: bool
    fused: bool = True


CONFIGS = {
    0: ScanConfig("cfg0_fwd_fp32_B1_L4096_D512_N16", 1, 4096, 512, 16, torch.float32, False),
    1: ScanConfig("cfg1_fwdbwd_fp32_B16_L512_D512_N16", 16, 512, 512, 16, torch.float32, True),
    2: ScanConfig("cfg2_fwd_fp32_B1_L131072_D512_N16", 1, 131072, 512, 16, torch.float32, False),
    3: ScanConfig("cfg3_fwdbwd_bf16_B8_L8192_D5120_N16", 8, 8192, 5120, 16, torch.bfloat16, True),
}


def s4d_real_A(D, N, dtype=torch.float32):
    """A = -exp(log(n + 1)) broadcast over channels (models/mamba.py:60-64)."""
    return -torch.exp(torch.log(torch.arange(1, N + 1, dtype=torch.float32))).repeat(D, 1).to(dtype)


def make_inputs(B, L, D, N, seed=0, dist="config", h0=False, dlast=False, dtype=torch.float32, device="cpu",
                draw_on_device=False):
    """Returns a dict of CPU-drawn inputs moved to ``device`` (A, Dskip, h0 stay float32).

    Keys: u, delta, A, Bm, Cm, Dskip, z, dy, h0 (or None), dlast (or None).
    ``draw_on_device`` draws on ``device`` with its own generator (same distributions, different
    values; for benchmark-sized inputs that would take the CPU tens of seconds to draw).
    """
    g = torch.Generator(device=device if draw_on_device else "cpu").manual_seed(seed)
    on = dict(device=device) if draw_on_device else {}

    def randn(*s):
        return torch.randn(*s, generator=g, **on)

    u = randn(B, L, D)
    if dist == "config":
        delta = torch.nn.functional.softplus(0.5 * randn(B, L, D) + math.log(math.expm1(0.01)))
        A = s4d_real_A(D, N).to(u.device)
    elif dist == "test":
        delta = torch.rand(B, L, D, generator=g, **on) * 0.3 + 1e-3
        A = -torch.rand(D, N, generator=g, **on) * 4 - 0.05
    else:
        raise ValueError(dist)
    Bm, Cm = randn(B, L, N), randn(B, L, N)
    Dskip = randn(D)
    z = randn(B, L, D)
    dy = randn(B, L, D)
    h = randn(B, D, N) if h0 else None
    dl = randn(B, D, N) if dlast else None
    out = dict(u=u, delta=delta, A=A, Bm=Bm, Cm=Cm, Dskip=Dskip, z=z, dy=dy, h0=h, dlast=dl)
    for k in ("u", "delta", "Bm", "Cm", "z", "dy"):
        out[k] = out[k].to(dtype)
    return {k: (v.to(device) if v is not None else None) for k, v in out.items()}


def algorithmic_bytes(B, L, D, N, elem_bytes, fused=True, backward=True):
    """Bytes a perfect kernel must move, per pass (the roofline numerator).

    forward : reads u, delta, B, C (+ z), writes y;         + A, D, last
    backward: reads u, delta, B, C, dy (+ z), writes du, ddelta, dB, dC (+ dz); + A, dA, D, dD
    Chunk checkpoints are implementation traffic and are not counted.
    """
    bld, bln = B * L * D, B * L * N
    fwd = (4 if fused else 3) * bld * elem_bytes + 2 * bln * elem_bytes + D * N * 4 + D * 4 + B * D * N * 4
    bwd = (7 if fused else 5) * bld * elem_bytes + 4 * bln * elem_bytes + 2 * D * N * 4 + 2 * D * 4
    return fwd, (bwd if backward else 0)


# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of each kernel on each
# workload, from the ncu captures summarised under profiles/ (the summary named beside each entry
# gives the command).  bench.py reports it as roofline.traffic; kernels and workloads not listed
# have not been captured on the current build (traffic null).
NCU_TRAFFIC = {
    # profiles/bwd_kernel_cfg1_fwdbwd_fp32_B16_L512_D512_N16.md (the backward kernel; its finalize
    # reads the per-CTA partials mostly from L2)
    ("ssm_scan_bwd", "cfg1_fwdbwd_fp32_B16_L512_D512_N16"): 133680128,
    # profiles/fwd_kernel_cfg1_fwdbwd_fp32_B16_L512_D512_N16.md
    ("ssm_scan_fwd", "cfg1_fwdbwd_fp32_B16_L512_D512_N16"): 60009472,
    # profiles/fwdbwd_kernels_cfg3_bf16_shape3x8192x5120.md: three of the eight batch rows captured,
    # scaled by 8/3 (every byte either kernel moves is proportional to the batch)
    ("ssm_scan_fwd", "cfg3_fwdbwd_bf16_B8_L8192_D5120_N16"): 4765744000,
    ("ssm_scan_bwd", "cfg3_fwdbwd_bf16_B8_L8192_D5120_N16"): 7996509333,
    # profiles/fwd_segmented_cfg2_cfg0.md: one ssm_scan_fwd call = summary pass + carry + main pass
    # (the three kernels' DRAM bytes summed, mean of three calls)
    ("ssm_scan_fwd", "cfg2_fwd_fp32_B1_L131072_D512_N16"): 1653311061,
    ("ssm_scan_fwd", "cfg0_fwd_fp32_B1_L4096_D512_N16"): 46085973,
}


def markov_bytes(batch, length, seed=0, order=2, vocab=256, temperature=0.5):
    """(batch, length) int64 bytes from a seeded random order-2 Markov chain over 256 symbols: the
    next-byte distribution for every (previous, current) pair is a softmax of N(0, 1) / temperature
    logits, i.e. a (256, 256, 256) transition table drawn from ``seed``.  Generated on the CPU, one
    position at a time for all rows.  (The config-4 training data; the reference has no such
    generator and trains on enwik8.)"""
    if order != 2:
        raise ValueError("only the order-2 chain is defined")
    g = torch.Generator().manual_seed(seed)
    table = torch.softmax(torch.randn(vocab, vocab, vocab, generator=g) / temperature, dim=-1)
    cdf = table.cumsum(-1)
    out = torch.empty(batch, length, dtype=torch.long)
    out[:, :2] = torch.randint(0, vocab, (batch, 2), generator=g)
    for t in range(2, length):
        u = torch.rand(batch, 1, generator=g)
        row = cdf[out[:, t - 2], out[:, t - 1]]
        out[:, t] = torch.searchsorted(row, u).squeeze(1).clamp_(max=vocab - 1)
    return out
