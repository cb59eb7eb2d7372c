"""The backward's sequence split: a long sequence over few (batch, 32-channel) tiles is cut into
segments that run at the same time, each starting from the adjoint the later segments hand it
(adjoint summaries composed in reverse).  Checked against the CPU oracle's gradients (the
reference's SelectiveScanFn.backward, models/scan.py:219-255) on shapes the planner splits, with
every method, h0 and dlast, the fused gate, bf16, ragged lengths and the in-kernel softplus."""

import pytest
import torch

import scan_harness as H
from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200 import selective_scan_fused
from mamba_ssm_benchmark_b200.workloads import make_inputs
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = [
    # B, L, D, N, dtype, method, h0
    (1, 4096, 512, 16, torch.float32, "zoh", True),      # the reference benchmark's shape (B=1, D=512)
    (1, 2048, 64, 16, torch.bfloat16, "zoh", False),
    (2, 1000, 96, 8, torch.float32, "euler", True),
    (1, 777, 40, 16, torch.float32, "bilinear", True),
    (3, 520, 33, 4, torch.float32, "zoh", True),
    (1, 600, 64, 32, torch.float32, "zoh", True),
    (1, 600, 40, 64, torch.float32, "euler", False),   # N = 64: coefficients evaluated again, no cache
]


def _ids(c):
    B, L, D, N, dt, m, h0 = c
    return f"{B}x{L}x{D}x{N}-{'bf16' if dt == torch.bfloat16 else 'f32'}-{m}{'-h0' if h0 else ''}"


@pytest.mark.parametrize("case", CASES, ids=[_ids(c) for c in CASES])
def test_split_backward_matches_oracle(case):
    B, L, D, N, dt, method, with_h0 = case
    S, seg_len = nat.bwd_plan(B, L, D, N, dt)
    assert S > 1 and seg_len % 16 == 0 and (S - 1) * seg_len < L <= S * seg_len
    ins = make_inputs(B, L, D, N, seed=11, dist="config", h0=with_h0, dlast=True)
    if dt == torch.bfloat16:   # both sides see the same bf16-rounded inputs
        ins = {k: (v.to(torch.bfloat16).float() if k in ("u", "delta", "Bm", "Cm", "z", "dy") else v)
               for k, v in ins.items()}
    w2 = ins["dlast"]
    got = H.run(H.ours, ins, method, DEV, dt, with_h0, True, w2=w2)
    ref = H.run(H.oracle, ins, method, "cpu", torch.float32, with_h0, True, w2=w2)
    if dt == torch.bfloat16:
        H.compare(got, ref, fwd_tol=H.BF16_TOL, grad_tol=H.BF16_TOL, elementwise=False)
    else:
        H.compare(got, ref, elementwise=False)
    assert nat.read_device_error() == 0


def test_split_backward_with_softplus_matches_oracle():
    """delta = softplus(raw + bias) inside the kernels, in the adjoint summaries too."""
    B, L, D, N = 1, 1536, 64, 16
    assert nat.bwd_plan(B, L, D, N, torch.float32)[0] > 1
    ins = make_inputs(B, L, D, N, seed=5, dist="config", h0=False, dlast=False)
    g = torch.Generator().manual_seed(6)
    raw = torch.randn(B, L, D, generator=g) * 0.5 - 3.0
    bias = torch.randn(D, generator=g) * 0.2

    def leaves(device):
        t = lambda x: x.to(device).clone().requires_grad_()
        return dict(u=t(ins["u"]), raw=t(raw), A=t(ins["A"]), Bm=t(ins["Bm"]), Cm=t(ins["Cm"]),
                    Dskip=t(ins["Dskip"]), z=t(ins["z"]), bias=t(bias))

    a = leaves(DEV)
    y, _ = selective_scan_fused(a["u"], a["raw"], a["A"], a["Bm"], a["Cm"], D=a["Dskip"], z=a["z"],
                                delta_bias=a["bias"], delta_softplus=True)
    order = ("u", "raw", "A", "Bm", "Cm", "Dskip", "z", "bias")
    gg = torch.autograd.grad((y * ins["dy"].to(DEV)).sum(), [a[k] for k in order])
    c = leaves("cpu")
    delta = torch.nn.functional.softplus(c["raw"] + c["bias"])
    yr, _ = O.selective_scan_fused(c["u"], delta, c["A"], c["Bm"], c["Cm"], Dskip=c["Dskip"], z=c["z"])
    gr = torch.autograd.grad((yr * ins["dy"]).sum(), [c[k] for k in order])
    assert O.normwise_error(y.detach().cpu(), yr.detach()) <= H.FWD_TOL
    for k, x, r in zip(order, gg, gr):
        assert O.normwise_error(x.cpu(), r) <= H.GRAD_TOL, k
    assert nat.read_device_error() == 0


def test_split_backward_is_bitwise_reproducible():
    B, L, D, N = 1, 2048, 96, 16
    assert nat.bwd_plan(B, L, D, N, torch.float32)[0] > 1
    ins = make_inputs(B, L, D, N, seed=2, dist="config", h0=True, dlast=True)
    runs = [H.run(H.ours, ins, "zoh", DEV, torch.float32, True, True, w2=ins["dlast"]) for _ in range(2)]
    for k in runs[0]:
        assert torch.equal(runs[0][k], runs[1][k]), k


def test_plans_keep_full_grids_whole():
    """Grids that fill the GPU (config 1: 256 CTAs, config 3: 1280) are not split."""
    assert nat.bwd_plan(16, 512, 512, 16, torch.float32) == (1, 512)
    assert nat.bwd_plan(8, 8192, 5120, 16, torch.bfloat16)[0] == 1
    assert nat.bwd_plan(1, 128, 512, 16, torch.float32)[0] == 1   # too short to split
