"""In-kernel step-size activation: selective_scan_fused(..., delta_bias, delta_softplus=True) uses
softplus(delta + bias) (models/mamba.py:77) inside the scan kernels.  Checked against the oracle
fed with the activated step size, forward and every gradient (raw delta and bias included)."""

import pytest
import torch

from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200 import selective_scan_fused
from mamba_ssm_benchmark_b200.workloads import make_inputs
from oracle import scan_oracle as O
from scan_harness import FWD_TOL, GRAD_TOL

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert nat.read_device_error() == 0


def _case(B, L, D, N, seed, dtype=torch.float32, spread=1.0):
    ins = make_inputs(B, L, D, N, seed=seed, dist="config", h0=True, dlast=True, dtype=dtype)
    g = torch.Generator().manual_seed(seed + 1)
    # raw step sizes around the usual dt_proj output (softplus^-1 of ~0.01) with some spread
    raw = (torch.randn(B, L, D, generator=g) * spread - 4.6).to(dtype)
    bias = torch.randn(D, generator=g) * 0.5
    return ins, raw, bias


def _grads(fn, ins, raw, bias, device, with_bias=True):
    keys = ("u", "A", "Bm", "Cm", "h0", "Dskip", "z")
    lv = {k: ins[k].to(device).clone().requires_grad_() for k in keys}
    r = raw.to(device).clone().requires_grad_()
    b = bias.to(device).clone().requires_grad_() if with_bias else None
    y, last = fn(lv, r, b)
    outs = [y, last]
    leaves = [lv[k] for k in keys] + [r] + ([b] if with_bias else [])
    gr = torch.autograd.grad((y * ins["dy"].to(device)).sum() + (last * ins["dlast"].to(device)).sum(), leaves)
    return outs + list(gr)


@pytest.mark.parametrize("method", ["zoh", "euler", "bilinear"])
@pytest.mark.parametrize("L", [64, 37, 1])
@pytest.mark.parametrize("with_bias", [True, False])
def test_softplus_fused_matches_oracle(method, L, with_bias):
    B, D, N = 2, 48, 16
    ins, raw, bias = _case(B, L, D, N, seed=L)

    def ours(lv, r, b):
        return selective_scan_fused(lv["u"], r, lv["A"], lv["Bm"], lv["Cm"], h0=lv["h0"], method=method,
                                    D=lv["Dskip"], z=lv["z"], delta_bias=b, delta_softplus=True)

    def ref(lv, r, b):
        delta = torch.nn.functional.softplus(r + (b if b is not None else 0.0))
        return O.selective_scan_fused(lv["u"], delta, lv["A"], lv["Bm"], lv["Cm"], h0=lv["h0"], method=method,
                                      Dskip=lv["Dskip"], z=lv["z"])

    got = _grads(ours, ins, raw, bias, DEV, with_bias)
    want = _grads(ref, {k: (v.double() if v is not None else None) for k, v in ins.items()}, raw.double(),
                  bias.double(), "cpu", with_bias)
    names = ["y", "last", "du", "dA", "dB", "dC", "dh0", "dD", "dz", "draw"] + (["dbias"] if with_bias else [])
    for n, a, b in zip(names, got, want):
        tol = FWD_TOL if n in ("y", "last") else GRAD_TOL
        assert O.normwise_error(a.detach().cpu().double(), b) < tol, n


def test_softplus_threshold_and_extremes():
    """Raw values past softplus's threshold (x > 20 returns x) and far negative (delta ~ 0)."""
    B, L, D, N = 1, 48, 32, 16
    ins, raw, bias = _case(B, L, D, N, seed=3, spread=12.0)
    raw[0, :8] = 25.0
    raw[0, 8:16] = -30.0
    lv = {k: ins[k].to(DEV) for k in ("u", "A", "Bm", "Cm", "Dskip", "z")}
    y, last = selective_scan_fused(lv["u"], raw.to(DEV), lv["A"], lv["Bm"], lv["Cm"], D=lv["Dskip"], z=lv["z"],
                                   delta_bias=bias.to(DEV), delta_softplus=True)
    delta = torch.nn.functional.softplus(raw.double() + bias.double())
    yr, lr = O.selective_scan_fused(ins["u"].double(), delta, ins["A"].double(), ins["Bm"].double(),
                                    ins["Cm"].double(), Dskip=ins["Dskip"].double(), z=ins["z"].double())
    assert O.normwise_error(y.cpu().double(), yr) < FWD_TOL
    assert O.normwise_error(last.cpu().double(), lr) < FWD_TOL


def test_softplus_bf16_and_config1_shape():
    B, L, D, N = 16, 512, 512, 16
    ins, raw, bias = _case(B, L, D, N, seed=9, dtype=torch.bfloat16)
    lv = {k: ins[k].to(DEV) for k in ("u", "A", "Bm", "Cm", "Dskip", "z")}
    y, _ = selective_scan_fused(lv["u"], raw.to(DEV), lv["A"], lv["Bm"], lv["Cm"], D=lv["Dskip"], z=lv["z"],
                                delta_bias=bias.to(DEV), delta_softplus=True)
    delta = torch.nn.functional.softplus(raw.float() + bias)
    y2, _ = selective_scan_fused(lv["u"].float(), delta.to(DEV), lv["A"], lv["Bm"].float(), lv["Cm"].float(),
                                 D=lv["Dskip"], z=lv["z"].float())
    assert O.normwise_error(y.float(), y2) < 1e-2
