"""Parity at the benchmark configurations' own sizes, against the CPU oracle (models/scan.py
restated; models/scan.py:193-255 for the backward, :277-299 for the dispatcher).

* config 3 at its full channel width: bf16 activations, D = 5120, N = 16, on a (B = 1, L = 1024)
  slice of its (8, 8192) rows (channels and rows are independent in the scan; the full width
  exercises the 160 channel tiles the backward's finalize sums for dB and dC).  Compared with the
  oracle on the same bf16-rounded inputs in float32, normwise within the bf16 tolerance (1e-2:
  outputs are rounded to bf16, 2^-8 relative per element).
* config 2 at its full length: the forward over L = 131072 with D = 512 (the sequence split into
  segments by the kernel itself), y and the final state normwise within 1e-4.
"""

import pytest
import torch

import scan_harness as H
from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200 import selective_scan_fused
from mamba_ssm_benchmark_b200.workloads import CONFIGS, make_inputs
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
KEYS = ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert nat.read_device_error() == 0


def test_config3_full_width_bf16_forward_backward():
    cfg = CONFIGS[3]
    B, L, D, N = 1, 1024, cfg.D, cfg.N
    ins = make_inputs(B, L, D, N, seed=3, dist="config", h0=True, dlast=True, dtype=torch.bfloat16)
    lv = {k: ins[k].to(DEV).clone().requires_grad_() for k in KEYS + ("h0",)}
    y, last = selective_scan_fused(lv["u"], lv["delta"], lv["A"], lv["Bm"], lv["Cm"], h0=lv["h0"], D=lv["Dskip"],
                                   z=lv["z"])
    assert y.dtype == torch.bfloat16
    g = torch.autograd.grad((y, last), [lv[k] for k in KEYS + ("h0",)], (ins["dy"].to(DEV), ins["dlast"].to(DEV)))
    cpu = {k: ins[k].float().clone().requires_grad_() for k in KEYS + ("h0",)}
    yr, lr = O.selective_scan_fused(cpu["u"], cpu["delta"], cpu["A"], cpu["Bm"], cpu["Cm"], h0=cpu["h0"],
                                    Dskip=cpu["Dskip"], z=cpu["z"])
    gr = torch.autograd.grad((yr, lr), [cpu[k] for k in KEYS + ("h0",)], (ins["dy"].float(), ins["dlast"]))
    assert O.normwise_error(y.float(), yr) < H.BF16_TOL
    assert O.normwise_error(last, lr) < H.BF16_TOL
    for name, a, b in zip(KEYS + ("h0",), g, gr):
        assert torch.isfinite(a.float()).all(), name
        assert O.normwise_error(a.float(), b) < H.BF16_TOL, name


def test_config2_full_length_forward():
    cfg = CONFIGS[2]
    B, L, D, N = cfg.B, cfg.L, cfg.D, cfg.N
    ins = make_inputs(B, L, D, N, seed=2, dist="config")
    y, last = selective_scan_fused(*(ins[k].to(DEV) for k in KEYS[:5]), D=ins["Dskip"].to(DEV),
                                   z=ins["z"].to(DEV))
    torch.set_num_threads(max(1, torch.get_num_threads()))
    yr, lr = O.selective_scan_fused(*(ins[k] for k in KEYS[:5]), Dskip=ins["Dskip"], z=ins["z"])
    assert O.normwise_error(y, yr) < H.FWD_TOL
    assert O.normwise_error(last, lr) < H.FWD_TOL
