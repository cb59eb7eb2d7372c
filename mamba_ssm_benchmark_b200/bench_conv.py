"""Times the causal conv1d + SiLU kernels against the reference's torch path (models/mamba.py:100-107:
transpose, F.pad, depthwise F.conv1d, F.silu) on one shape.

    python -m mamba_ssm_benchmark_b200.bench_conv [--B 8 --L 8192 --D 1024 --dtype float32 --reps 50]

x is the first half of a (B, L, 2D) in_proj-like output, as in the mixer.  Prints one JSON line:
device times (CUDA events, median) of forward and forward+backward for both, and the forward's and
backward's achieved bytes per second against the algorithmic bytes (2 and 3 passes over B·L·D).
"""

import argparse
import json
import statistics

import torch
import torch.nn.functional as F

from . import causal_conv1d


def _median_us(fn, reps):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in ev:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in ev) * 1e3


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--L", type=int, default=8192)
    ap.add_argument("--D", type=int, default=1024)
    ap.add_argument("--K", type=int, default=4)
    ap.add_argument("--dtype", choices=("float32", "bfloat16"), default="float32")
    ap.add_argument("--reps", type=int, default=50)
    args = ap.parse_args(argv)
    dt = getattr(torch, args.dtype)
    B, L, D, K = args.B, args.L, args.D, args.K
    g = torch.Generator(device="cuda").manual_seed(0)
    xz = torch.randn(B, L, 2 * D, device="cuda", dtype=dt, generator=g)
    x = xz[..., :D].detach().requires_grad_()
    w = (torch.randn(D, 1, K, device="cuda", generator=g) * 0.3).requires_grad_()
    b = torch.randn(D, device="cuda", generator=g).requires_grad_()
    dout = torch.randn(B, L, D, device="cuda", dtype=dt, generator=g)
    wr, br = w.detach().to(dt).requires_grad_(), b.detach().to(dt).requires_grad_()

    def ours_fwd():
        with torch.no_grad():
            causal_conv1d(x, w, b)

    def ours_fwd_bwd():
        torch.autograd.grad(causal_conv1d(x, w, b), (x, w, b), dout)

    def ref(xx):
        return F.silu(F.conv1d(F.pad(xx.transpose(1, 2), (K - 1, 0)), wr, br, groups=D)).transpose(1, 2)

    def ref_fwd():
        with torch.no_grad():
            ref(x)

    def ref_fwd_bwd():
        torch.autograd.grad(ref(x), (x, wr, br), dout)

    t = {name: _median_us(fn, args.reps) for name, fn in (("fwd_us", ours_fwd), ("fwd_bwd_us", ours_fwd_bwd),
                                                           ("torch_fwd_us", ref_fwd),
                                                           ("torch_fwd_bwd_us", ref_fwd_bwd))}
    nbytes = B * L * D * x.element_size()
    t["fwd_gbs"] = 2 * nbytes / (t["fwd_us"] * 1e-6) / 1e9
    t["bwd_gbs"] = 3 * nbytes / ((t["fwd_bwd_us"] - t["fwd_us"]) * 1e-6) / 1e9
    print(json.dumps({"shape": {"B": B, "L": L, "D": D, "K": K, "dtype": args.dtype}, **t}), flush=True)


if __name__ == "__main__":
    main()
