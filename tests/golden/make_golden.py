"""Generates tests/golden/*.npz by running the REFERENCE implementation's own code.

    python tests/golden/make_golden.py [--ref /path/to/mamba-ssm-benchmark]

Runs only where the reference checkout exists (it does not travel with this repository);
the .npz files it writes are committed and are what the tests read.  Every case records the
seeded inputs and the reference's outputs:

  scan_<shape>_<method>_<h0>.npz   models/scan.py:selective_scan(scan="chunked", fp32):
                                   y, last and the gradients of sum(y*w1) + sum(last*w2)
  loop_<shape>_<method>.npz        models/scan.py:selective_scan_reference in float64
                                   (the autograd ground truth), same cotangents
  chunked_scan.npz                 models/scan.py:scan_chunked on random (a, b) for several
                                   chunk sizes, with and without h0
  scans.npz                        models/scan.py:scan_sequential, scan_hillis_steele and
                                   scan_blelloch on random (a, b), L = 50 and L = 64, +- h0, and
                                   selective_scan with scan="blelloch" (y, last, gradients)
  fused_cfg.npz                    config-distribution inputs through selective_scan + the
                                   mixer gate (y + x*D)*silu(z) (models/mamba.py:124)
  decode.npz                       the inline decode step of models/mamba.py:113-118
  bench_inputs.npz                 benchmarks/bench_scan.py:make_inputs (the scan benchmark's
                                   inputs) at L = 8, for the benchmark in the reference's format
  lm_small.npz                     models/lm.py:LM with layers "MM", d_model 32: parameters,
                                   logits, cross-entropy loss and its parameter gradients on a
                                   byte batch, and prefill + 4 decode steps with states
"""

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from mamba_ssm_benchmark_b200.workloads import make_inputs  # noqa: E402

SCAN_SHAPES = [(2, 1, 32, 16), (2, 37, 50, 16), (1, 64, 24, 8), (2, 19, 5, 4)]
LOOP_SHAPES = [(2, 37, 50, 16), (2, 19, 5, 4)]
METHODS = ("zoh", "euler", "bilinear")


def _np(t):
    return None if t is None else t.detach().cpu().numpy()


def _save(name, **arrays):
    arrays = {k: v for k, v in arrays.items() if v is not None}
    np.savez_compressed(os.path.join(HERE, name), **arrays)


def scan_case(ref_scan, shape, method, with_h0, dtype, scan, seed):
    B, L, D, N = shape
    ins = make_inputs(B, L, D, N, seed=seed, dist="test", h0=with_h0)
    leaves = [ins[k].to(dtype).clone().requires_grad_() for k in ("u", "delta", "A", "Bm", "Cm")]
    h0 = ins["h0"].to(dtype).clone().requires_grad_() if with_h0 else None
    if h0 is not None:
        leaves.append(h0)
    g = torch.Generator().manual_seed(seed + 1000)
    y, last = ref_scan(*leaves[:5], h0=h0, method=method, scan=scan)
    w1 = torch.randn(y.shape, generator=g).to(dtype)
    w2 = torch.randn(last.shape, generator=g).to(dtype)
    grads = torch.autograd.grad((y * w1).sum() + (last * w2).sum(), leaves)
    names = ["du", "ddelta", "dA", "dBm", "dCm", "dh0"]
    out = dict(u=ins["u"], delta=ins["delta"], A=ins["A"], Bm=ins["Bm"], Cm=ins["Cm"], h0=ins["h0"],
               w1=w1.float(), w2=w2.float(), y=y, last=last)
    out.update({n: gr for n, gr in zip(names, grads)})
    return {k: _np(v) for k, v in out.items()}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SSM_REFERENCE_ROOT", "/root/reference"))
    ap.add_argument("--only", default=None, help="write only this fixture group (e.g. bench_inputs)")
    args = ap.parse_args(argv)
    sys.dont_write_bytecode = True            # never write into the reference checkout
    sys.path.insert(0, args.ref)
    from models import scan as ref             # the reference's models/scan.py

    if args.only == "bench_inputs" or args.only is None:
        bench_inputs()
    if args.only == "lm_small" or args.only is None:
        lm_small()
    if args.only == "scans" or args.only is None:
        scans(ref)
    if args.only is not None:
        return

    torch.manual_seed(0)
    for si, shape in enumerate(SCAN_SHAPES):
        for mi, method in enumerate(METHODS):
            for h0 in (False, True):
                arr = scan_case(ref.selective_scan, shape, method, h0, torch.float32, "chunked",
                                seed=100 * si + 10 * mi + int(h0))
                _save("scan_{}x{}x{}x{}_{}_{}.npz".format(*shape, method, "h0" if h0 else "noh0"), **arr)
    for si, shape in enumerate(LOOP_SHAPES):
        for mi, method in enumerate(METHODS):
            arr = scan_case(ref.selective_scan, shape, method, True, torch.float64, "reference",
                            seed=5000 + 100 * si + 10 * mi)
            _save("loop_{}x{}x{}x{}_{}.npz".format(*shape, method), **arr)

    # two-level scan with explicit chunk sizes (models/scan.py:142-165)
    g = torch.Generator().manual_seed(7)
    a = torch.rand(2, 50, 3, 4, generator=g, dtype=torch.float64) * 0.9 + 0.05
    b = torch.randn(2, 50, 3, 4, generator=g, dtype=torch.float64)
    h0 = torch.randn(2, 3, 4, generator=g, dtype=torch.float64)
    res = {"a": _np(a), "b": _np(b), "h0": _np(h0)}
    for c in (1, 3, 8, 64):
        res[f"h_c{c}"] = _np(ref.scan_chunked(a, b, None, c))
        res[f"h_c{c}_h0"] = _np(ref.scan_chunked(a, b, h0, c))
    res["h_default"] = _np(ref.scan_chunked(a, b, h0))
    _save("chunked_scan.npz", **res)

    # config-0 distributions at a reduced length, fused with the mixer gate
    ins = make_inputs(1, 256, 64, 16, seed=0, dist="config")
    y, last = ref.selective_scan(ins["u"], ins["delta"], ins["A"], ins["Bm"], ins["Cm"], scan="chunked")
    out = (y + ins["u"] * ins["Dskip"]) * torch.nn.functional.silu(ins["z"])
    _save("fused_cfg.npz", **{k: _np(v) for k, v in ins.items()}, y=_np(y), out=_np(out), last=_np(last))

    # decode step (models/mamba.py:113-118), float32 state as Mamba.init_state allocates it
    g = torch.Generator().manual_seed(11)
    Bsz, D, N = 3, 40, 16
    x = torch.randn(Bsz, 1, D, generator=g)
    delta = torch.rand(Bsz, 1, D, generator=g) * 0.2 + 1e-3
    A = -torch.rand(D, N, generator=g) * 4 - 0.05
    Bm, Cm = torch.randn(Bsz, 1, N, generator=g), torch.randn(Bsz, 1, N, generator=g)
    state = torch.randn(Bsz, D, N, generator=g)
    res = {"x": x, "delta": delta, "A": A, "Bm": Bm, "Cm": Cm, "state": state}
    for method in METHODS:
        a_, b_ = ref.discretize(delta, A, Bm, x, method)
        h = a_[:, 0] * state + b_[:, 0]
        res[f"y_{method}"] = torch.einsum("bdn,bn->bd", h, Cm[:, 0])
        res[f"state_{method}"] = h
    _save("decode.npz", **{k: _np(v) for k, v in res.items()})
    print("wrote", len([f for f in os.listdir(HERE) if f.endswith(".npz")]), "fixtures to", HERE)


def scans(ref):
    """The reference's alternative scan algorithms (models/scan.py:70-135) on random affine maps."""
    g = torch.Generator().manual_seed(17)
    res = {}
    for L in (50, 64):
        a = torch.rand(2, L, 3, 4, generator=g, dtype=torch.float64) * 0.9 + 0.05
        b = torch.randn(2, L, 3, 4, generator=g, dtype=torch.float64)
        h0 = torch.randn(2, 3, 4, generator=g, dtype=torch.float64)
        res[f"a{L}"], res[f"b{L}"], res[f"h0_{L}"] = _np(a), _np(b), _np(h0)
        for name in ("sequential", "hillis_steele", "blelloch"):
            fn = getattr(ref, f"scan_{name}")
            res[f"{name}{L}"] = _np(fn(a, b))
            res[f"{name}{L}_h0"] = _np(fn(a, b, h0))
    arr = scan_case(ref.selective_scan, (2, 37, 50, 16), "zoh", True, torch.float32, "blelloch", seed=77)
    res.update({f"sel_{k}": v for k, v in arr.items()})
    _save("scans.npz", **res)


def lm_small():
    """A two-block Mamba LM of the reference, seeded, in float32 on the CPU."""
    from models.lm import LM, LMConfig
    torch.manual_seed(0)
    model = LM(LMConfig(layers="MM", d_model=32, d_state=16, expand=2, d_conv=4, scan="chunked"))
    g = torch.Generator().manual_seed(1)
    idx = torch.randint(0, 256, (2, 24), generator=g)
    logits = model(idx)
    loss = torch.nn.functional.cross_entropy(logits.view(-1, 256), idx.view(-1))
    names = [n for n, _ in model.named_parameters()]
    grads = torch.autograd.grad(loss, [p for _, p in model.named_parameters()])
    res = {"idx": idx, "logits": logits, "loss": loss.reshape(1)}
    res.update({"p." + k: v for k, v in model.state_dict().items()})
    res.update({"g." + n: gr for n, gr in zip(names, grads)})
    with torch.no_grad():
        states = model.init_state(2, 40, "cpu")
        res["prefill_logits"] = model(idx[:, :16], states, 0)
        for i in range(4):
            res[f"step{i}_logits"] = model(idx[:, 16 + i:17 + i], states, 16 + i)
    _save("lm_small.npz", **{k: _np(v) for k, v in res.items()})


def bench_inputs():
    """The reference scan benchmark's seeded inputs (benchmarks/bench_scan.py:25-32) at L = 8."""
    from benchmarks.bench_scan import make_inputs as ref_bench_inputs
    x, delta, A, Bm, Cm = ref_bench_inputs(8, device="cpu")
    _save("bench_inputs.npz", x=_np(x), delta=_np(delta), A=_np(A), Bm=_np(Bm), Cm=_np(Cm))


if __name__ == "__main__":
    main()
