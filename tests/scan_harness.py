"""Shared helpers of the GPU parity tests: run the sm_100a op (through the C ABI) and the CPU
oracle on the same seeded inputs and compare.

Tolerances (normwise, max|err| / max|ref|, against the float32 oracle = the reference's own
algorithm in float32):
    FWD_TOL  = 1e-4   y and last             (north-star bound for y)
    GRAD_TOL = 1e-3   every gradient         (north-star bound for gradients)
    BF16_TOL = 1e-2   bf16 activations: outputs are rounded to bf16 (2^-8 relative per
                      element), so the bound is a few bf16 ulps
Elementwise checks use the reference's own GPU test tolerances (tests/test_triton.py:180-186):
rtol = atol = 1e-4 forward, 2e-3 gradients.
"""

import torch

from mamba_ssm_benchmark_b200 import selective_scan_fused
from oracle import scan_oracle as O

FWD_TOL = 1e-4
GRAD_TOL = 1e-3
BF16_TOL = 1e-2
GRAD_NAMES = ("du", "ddelta", "dA", "dBm", "dCm", "dh0", "dD", "dz")


def leaves_of(ins, device, dtype, with_h0, fused):
    act = lambda t: t.to(device=device, dtype=dtype).clone().requires_grad_()
    f32 = lambda t: t.to(device=device, dtype=torch.float32).clone().requires_grad_()
    L = dict(u=act(ins["u"]), delta=act(ins["delta"]), A=f32(ins["A"]), Bm=act(ins["Bm"]), Cm=act(ins["Cm"]))
    L["h0"] = f32(ins["h0"]) if with_h0 else None
    L["Dskip"] = f32(ins["Dskip"]) if fused else None
    L["z"] = act(ins["z"]) if fused else None
    return L


def run(fn, ins, method, device, dtype, with_h0, fused, w1=None, w2=None, grads=True):
    """Returns outputs and gradients of sum(y*w1) + sum(last*w2) for either implementation."""
    lv = leaves_of(ins, device, dtype, with_h0, fused)
    y, last = fn(lv["u"], lv["delta"], lv["A"], lv["Bm"], lv["Cm"], lv["h0"], method, lv["Dskip"], lv["z"])
    out = {"y": y.detach(), "last": last.detach()}
    if grads:
        w1 = ins["dy"] if w1 is None else w1
        w2 = torch.zeros_like(last) if w2 is None else w2
        loss = (y.float() * w1.to(device)).sum() + (last * w2.to(device)).sum()
        names = [n for n in ("u", "delta", "A", "Bm", "Cm", "h0", "Dskip", "z") if lv[n] is not None]
        gs = torch.autograd.grad(loss, [lv[n] for n in names])
        tr = dict(u="du", delta="ddelta", A="dA", Bm="dBm", Cm="dCm", h0="dh0", Dskip="dD", z="dz")
        out.update({tr[n]: g.detach() for n, g in zip(names, gs)})
    return out


def ours(u, delta, A, Bm, Cm, h0, method, Dskip, z):
    return selective_scan_fused(u, delta, A, Bm, Cm, h0=h0, method=method, D=Dskip, z=z)


def oracle(u, delta, A, Bm, Cm, h0, method, Dskip, z):
    return O.selective_scan_fused(u, delta, A, Bm, Cm, h0=h0, method=method, Dskip=Dskip, z=z)


def compare(got, ref, fwd_tol=FWD_TOL, grad_tol=GRAD_TOL, elementwise=True):
    errs = {}
    for k, r in ref.items():
        if k not in got:
            continue
        g = got[k].detach().float().cpu()
        r = r.detach().float().cpu()
        assert g.shape == r.shape, (k, g.shape, r.shape)
        assert torch.isfinite(g).all(), f"{k} has non-finite values"
        e = O.normwise_error(g, r)
        errs[k] = e
        tol = fwd_tol if k in ("y", "last") else grad_tol
        assert e <= tol, f"{k}: normwise error {e:.3e} > {tol:.0e}"
        if elementwise:
            t = 1e-4 if k in ("y", "last") else 2e-3
            torch.testing.assert_close(g, r, rtol=t, atol=t,
                                       msg=lambda m: f"{k}: {m}")
    return errs
