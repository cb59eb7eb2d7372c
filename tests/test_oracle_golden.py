"""Pins the CPU oracle (oracle/scan_oracle.py) to the reference: every golden vector in
tests/golden was produced by the reference's own models/scan.py (tests/golden/make_golden.py)."""

import pytest
import torch

from conftest import golden_names, load_golden
from oracle import scan_oracle as O

SCAN = golden_names("scan_")
LOOP = golden_names("loop_")


def _method(name):
    return next(m for m in O.METHODS if f"_{m}" in name)


def _run(case, method, dtype, scan):
    leaves = [case[k].to(dtype).clone().requires_grad_() for k in ("u", "delta", "A", "Bm", "Cm")]
    h0 = case["h0"].to(dtype).clone().requires_grad_() if "h0" in case else None
    if h0 is not None:
        leaves.append(h0)
    y, last = O.selective_scan(*leaves[:5], h0=h0, method=method, scan=scan)
    w1, w2 = case["w1"].to(dtype), case["w2"].to(dtype)
    grads = torch.autograd.grad((y * w1).sum() + (last * w2).sum(), leaves)
    return y, last, grads


@pytest.mark.parametrize("name", SCAN)
def test_oracle_chunked_matches_reference_fp32(name):
    case = load_golden(name)
    y, last, grads = _run(case, _method(name), torch.float32, "chunked")
    torch.testing.assert_close(y, case["y"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(last, case["last"], rtol=1e-5, atol=1e-5)
    for n, g in zip(("du", "ddelta", "dA", "dBm", "dCm", "dh0"), grads):
        assert O.normwise_error(g, case[n]) < 1e-5, n


@pytest.mark.parametrize("name", LOOP)
def test_oracle_matches_reference_ground_truth_fp64(name):
    case = load_golden(name)
    method = _method(name)
    for scan in ("reference", "chunked"):
        y, last, grads = _run(case, method, torch.float64, scan)
        torch.testing.assert_close(y, case["y"], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(last, case["last"], rtol=1e-10, atol=1e-10)
        for n, g in zip(("du", "ddelta", "dA", "dBm", "dCm", "dh0"), grads):
            torch.testing.assert_close(g, case[n], rtol=1e-9, atol=1e-9, msg=lambda m: f"{scan} {n}: {m}")


def test_oracle_two_level_scan_matches_reference():
    case = load_golden("chunked_scan.npz")
    for c in (1, 3, 8, 64):
        torch.testing.assert_close(O.scan_chunked(case["a"], case["b"], None, c), case[f"h_c{c}"])
        torch.testing.assert_close(O.scan_chunked(case["a"], case["b"], case["h0"], c), case[f"h_c{c}_h0"])
    torch.testing.assert_close(O.scan_chunked(case["a"], case["b"], case["h0"]), case["h_default"])
    torch.testing.assert_close(O.scan_sequential(case["a"], case["b"], case["h0"]), case["h_c1_h0"])


@pytest.mark.parametrize("name", ["sequential", "hillis_steele", "blelloch"])
def test_oracle_alternative_scans_match_reference(name):
    """models/scan.py:70-135 on random affine maps (float64), L = 50 (padded inside Blelloch) and
    L = 64, with and without h0."""
    case = load_golden("scans.npz")
    fn = O.SCANS[name]
    for L in (50, 64):
        a, b, h0 = case[f"a{L}"], case[f"b{L}"], case[f"h0_{L}"]
        torch.testing.assert_close(fn(a, b), case[f"{name}{L}"], rtol=1e-12, atol=1e-12)
        torch.testing.assert_close(fn(a, b, h0), case[f"{name}{L}_h0"], rtol=1e-12, atol=1e-12)


def test_oracle_blelloch_selective_scan_matches_reference():
    """selective_scan(scan="blelloch") in float32 with its recomputing backward."""
    case = {k[4:]: v for k, v in load_golden("scans.npz").items() if k.startswith("sel_")}
    y, last, grads = _run(case, "zoh", torch.float32, "blelloch")
    torch.testing.assert_close(y, case["y"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(last, case["last"], rtol=1e-5, atol=1e-5)
    for n, g in zip(("du", "ddelta", "dA", "dBm", "dCm", "dh0"), grads):
        assert O.normwise_error(g, case[n]) < 1e-5, n


def test_oracle_fused_gate_matches_reference():
    case = load_golden("fused_cfg.npz")
    out, last = O.selective_scan_fused(case["u"], case["delta"], case["A"], case["Bm"], case["Cm"],
                                       Dskip=case["Dskip"], z=case["z"])
    torch.testing.assert_close(out, case["out"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(last, case["last"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("method", O.METHODS)
def test_oracle_decode_step_matches_reference(method):
    case = load_golden("decode.npz")
    y, h = O.state_update(case["state"], case["x"][:, 0], case["delta"][:, 0], case["A"], case["Bm"][:, 0],
                          case["Cm"][:, 0], method=method)
    torch.testing.assert_close(y, case[f"y_{method}"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(h, case[f"state_{method}"], rtol=1e-5, atol=1e-5)


def test_oracle_decode_equals_full_scan():
    """Stepping the decode update over a sequence reproduces the scan (tests/test_models.py:37-48)."""
    torch.manual_seed(0)
    B, L, D, N = 2, 12, 6, 4
    x, delta = torch.randn(B, L, D, dtype=torch.float64), torch.rand(B, L, D, dtype=torch.float64) * 0.3 + 0.01
    A = -torch.rand(D, N, dtype=torch.float64) - 0.1
    Bm, Cm = torch.randn(B, L, N, dtype=torch.float64), torch.randn(B, L, N, dtype=torch.float64)
    y_full, last = O.selective_scan(x, delta, A, Bm, Cm)
    state = torch.zeros(B, D, N, dtype=torch.float64)
    ys = []
    for t in range(L):
        yt, state = O.state_update(state, x[:, t], delta[:, t], A, Bm[:, t], Cm[:, t])
        ys.append(yt)
    torch.testing.assert_close(torch.stack(ys, 1), y_full)
    torch.testing.assert_close(state, last)
