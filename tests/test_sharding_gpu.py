"""GPU parity of the sharded scan (mamba_ssm_benchmark_b200/sharding.py).

On one GPU the sequence-shard protocol is emulated shard by shard with the package's own
summary / compose / finish functions; with two or more GPUs the NCCL rank program
(tests/sharding_nccl_worker.py) runs under torchrun.
"""

import os
import subprocess
import sys

import pytest
import torch

import scan_harness as H
from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200 import selective_scan_fused, sharding
from mamba_ssm_benchmark_b200.workloads import make_inputs
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert nat.read_device_error() == 0


@pytest.mark.parametrize("shards", [1, 2, 5])
@pytest.mark.parametrize("method", ["zoh", "euler", "bilinear"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sequence_shards_single_gpu(shards, method, dtype):
    """summary of every shard -> compose_prefix -> finish every shard == one call over the whole
    sequence, and == the oracle."""
    B, L, D, N = 2, 3000, 96, 16
    ins = make_inputs(B, L, D, N, seed=shards, dist="config", h0=True, dtype=dtype)
    dev = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
    u, dl, A, Bm, Cm, Dk, z, h0 = (dev[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "h0"))
    bounds = [sharding.shard_range(L, shards, r) for r in range(shards)]
    pieces = [sharding.SequenceShard(u[:, lo:hi], dl[:, lo:hi], A, Bm[:, lo:hi], Cm[:, lo:hi], method, D=Dk,
                                     z=z[:, lo:hi]) for lo, hi in bounds]
    sums = [p.summary() for p in pieces]
    decays = torch.stack([s[0] for s in sums])
    hends = torch.stack([s[1] for s in sums])
    h_in, last = sharding.compose_prefix(decays, hends, h0)
    ys = []
    for r, (lo, hi) in enumerate(bounds):
        y, lst = pieces[r].finish(h_in[r])
        assert y.dtype == dtype
        want_last = h_in[r + 1] if r + 1 < shards else last
        assert O.normwise_error(lst, want_last) < 1e-5
        ys.append(y)
    y = torch.cat(ys, 1)
    y_one, last_one = selective_scan_fused(u, dl, A, Bm, Cm, h0=h0, method=method, D=Dk, z=z)
    # fp32: the two segmentations agree to rounding; bf16 outputs can differ by one bf16 ulp (2^-8)
    assert O.normwise_error(y, y_one) < (1e-5 if dtype == torch.float32 else 1e-2)
    assert O.normwise_error(last, last_one) < 1e-5
    y_ref, last_ref = O.selective_scan_fused(*(ins[k].float() for k in ("u", "delta", "A", "Bm", "Cm")),
                                             h0=ins["h0"], method=method, Dskip=ins["Dskip"], z=ins["z"].float())
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    assert O.normwise_error(y.float().cpu(), y_ref) < tol
    assert O.normwise_error(last.cpu(), last_ref) < (1e-4 if dtype == torch.float32 else 1e-3)


@pytest.mark.parametrize("method", ["zoh", "euler", "bilinear"])
@pytest.mark.parametrize("with_z", [True, False])
@pytest.mark.parametrize("L", [1, 37, 3000])
def test_adjoint_summary_kernel(method, with_z, L):
    """ssm_scan_bwd_summary == the reverse adjoint dh_{t-1} = a_t (dh_t + C_t dys_t) from zero,
    and the decay product, computed on the CPU."""
    B, D, N = 2, 72, 16
    ins = make_inputs(B, L, D, N, seed=L, dist="config")
    dev = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
    z = dev["z"] if with_z else None
    shard = sharding.SequenceShard(dev["u"], dev["delta"], dev["A"], dev["Bm"], dev["Cm"], method, z=z)
    decay, dstart = shard.adjoint_summary(dev["dy"])
    a, _ = O.discretize(ins["delta"].double(), ins["A"].double(), ins["Bm"].double(), ins["u"].double(), method)
    dys = ins["dy"].double() * (ins["z"].double() * torch.sigmoid(ins["z"].double()) if with_z else 1.0)
    cdys = ins["Cm"].double()[:, :, None, :] * dys[..., None]
    dh = torch.zeros(B, D, N, dtype=torch.float64)
    for t in range(L - 1, -1, -1):
        dh = a[:, t] * (dh + cdys[:, t])
    assert O.normwise_error(dstart.cpu().double(), dh) < 1e-5
    # decay products lie in (0, 1]; over long shards most underflow towards 0, so the error is
    # measured against the scale they multiply (states of order one), not against max|decay|
    assert (decay.cpu().double() - a.prod(1)).abs().max().item() < 1e-6


@pytest.mark.parametrize("shards", [1, 2, 5])
@pytest.mark.parametrize("method", ["zoh", "bilinear"])
def test_sequence_shards_backward_single_gpu(shards, method):
    """Forward and backward of every shard (summary, prefix, finish; adjoint summary, suffix,
    backward) reproduce the single-call autograd gradients."""
    B, L, D, N = 2, 1500, 64, 16
    ins = make_inputs(B, L, D, N, seed=7 + shards, dist="config", h0=True, dlast=True)
    dev = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
    u, dl, A, Bm, Cm, Dk, z, h0, dy, dlast = (dev[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "h0",
                                                               "dy", "dlast"))
    bounds = [sharding.shard_range(L, shards, r) for r in range(shards)]
    pieces = [sharding.SequenceShard(u[:, lo:hi], dl[:, lo:hi], A, Bm[:, lo:hi], Cm[:, lo:hi], method, D=Dk,
                                     z=z[:, lo:hi]) for lo, hi in bounds]
    sums = [p.summary() for p in pieces]
    h_in, last = sharding.compose_prefix(torch.stack([s[0] for s in sums]), torch.stack([s[1] for s in sums]), h0)
    ys = [p.finish(h_in[r], save=True)[0] for r, p in enumerate(pieces)]
    adj = [p.adjoint_summary(dy[:, lo:hi]) for p, (lo, hi) in zip(pieces, bounds)]
    dl_in, dh0 = sharding.compose_suffix(torch.stack([a[0] for a in adj]), torch.stack([a[1] for a in adj]), dlast)
    g = [p.backward(dy[:, lo:hi], dl_in[r]) for r, (p, (lo, hi)) in enumerate(zip(pieces, bounds))]
    got = {"u": torch.cat([x[0] for x in g], 1), "delta": torch.cat([x[1] for x in g], 1),
           "A": sum(x[2] for x in g), "Bm": torch.cat([x[3] for x in g], 1), "Cm": torch.cat([x[4] for x in g], 1),
           "h0": dh0, "Dskip": sum(x[6] for x in g), "z": torch.cat([x[7] for x in g], 1)}
    keys = ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "h0")
    lv = {k: dev[k].clone().requires_grad_() for k in keys}
    y1, last1 = selective_scan_fused(lv["u"], lv["delta"], lv["A"], lv["Bm"], lv["Cm"], h0=lv["h0"], method=method,
                                     D=lv["Dskip"], z=lv["z"])
    want = dict(zip(keys, torch.autograd.grad((y1, last1), [lv[k] for k in keys], (dy, dlast))))
    assert O.normwise_error(torch.cat(ys, 1), y1) < 1e-5
    assert O.normwise_error(last, last1) < 1e-5
    for k in keys:
        assert O.normwise_error(got[k], want[k]) < 1e-4, k
    # and the stitched gradients against the oracle (models/scan.py:219-255 restated) directly
    cpu = {k: ins[k].clone().requires_grad_() for k in keys}
    yr, lr = O.selective_scan_fused(cpu["u"], cpu["delta"], cpu["A"], cpu["Bm"], cpu["Cm"], h0=cpu["h0"],
                                    method=method, Dskip=cpu["Dskip"], z=cpu["z"])
    ref = dict(zip(keys, torch.autograd.grad((yr, lr), [cpu[k] for k in keys], (ins["dy"], ins["dlast"]))))
    assert O.normwise_error(torch.cat(ys, 1), yr) < 1e-4
    for k in keys:
        assert O.normwise_error(got[k], ref[k]) < 1e-3, k


@pytest.mark.parametrize("shards", [2, 3])
def test_sequence_shards_backward_bf16(shards):
    """bf16 activations through the sharded backward (adjoint summaries, suffix, per-shard backward):
    the stitched gradients against the oracle on the same bf16-rounded inputs, at the bf16 tolerance."""
    B, L, D, N = 2, 900, 64, 16
    ins = make_inputs(B, L, D, N, seed=3 + shards, dist="config", h0=True, dlast=True)
    for k in ("u", "delta", "Bm", "Cm", "z", "dy"):
        ins[k] = ins[k].to(torch.bfloat16).float()
    dev = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
    act = {k: dev[k].to(torch.bfloat16) for k in ("u", "delta", "Bm", "Cm", "z", "dy")}
    bounds = [sharding.shard_range(L, shards, r) for r in range(shards)]
    pieces = [sharding.SequenceShard(act["u"][:, lo:hi], act["delta"][:, lo:hi], dev["A"], act["Bm"][:, lo:hi],
                                     act["Cm"][:, lo:hi], "zoh", D=dev["Dskip"], z=act["z"][:, lo:hi])
              for lo, hi in bounds]
    sums = [p.summary() for p in pieces]
    h_in, _ = sharding.compose_prefix(torch.stack([s[0] for s in sums]), torch.stack([s[1] for s in sums]), dev["h0"])
    ys = [p.finish(h_in[r], save=True)[0] for r, p in enumerate(pieces)]
    adj = [p.adjoint_summary(act["dy"][:, lo:hi]) for p, (lo, hi) in zip(pieces, bounds)]
    dl_in, dh0 = sharding.compose_suffix(torch.stack([a[0] for a in adj]), torch.stack([a[1] for a in adj]),
                                         dev["dlast"])
    g = [p.backward(act["dy"][:, lo:hi], dl_in[r]) for r, (p, (lo, hi)) in enumerate(zip(pieces, bounds))]
    got = {"u": torch.cat([x[0] for x in g], 1), "delta": torch.cat([x[1] for x in g], 1), "A": sum(x[2] for x in g),
           "Bm": torch.cat([x[3] for x in g], 1), "Cm": torch.cat([x[4] for x in g], 1), "h0": dh0,
           "Dskip": sum(x[6] for x in g), "z": torch.cat([x[7] for x in g], 1)}
    keys = ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "h0")
    cpu = {k: ins[k].clone().requires_grad_() for k in keys}
    yr, lr = O.selective_scan_fused(cpu["u"], cpu["delta"], cpu["A"], cpu["Bm"], cpu["Cm"], h0=cpu["h0"],
                                    Dskip=cpu["Dskip"], z=cpu["z"])
    ref = dict(zip(keys, torch.autograd.grad((yr, lr), [cpu[k] for k in keys], (ins["dy"], ins["dlast"]))))
    assert O.normwise_error(torch.cat(ys, 1).float().cpu(), yr.detach()) < H.BF16_TOL
    for k in keys:
        assert O.normwise_error(got[k].float().cpu(), ref[k]) < H.BF16_TOL, k


@pytest.mark.parametrize("W", [1, 3, 8])
def test_compose_kernel_matches_the_walk(W):
    """ssm_compose_shards (CUDA) against the torch walk of compose_prefix / compose_suffix (CPU)."""
    g = torch.Generator().manual_seed(W)
    dec = torch.rand(W, 2, 40, 16, generator=g)
    end = torch.randn(W, 2, 40, 16, generator=g)
    st = torch.randn(2, 40, 16, generator=g)
    for start in (None, st):
        for fn in (sharding.compose_prefix, sharding.compose_suffix):
            want = fn(dec, end, start)
            got = fn(dec.to(DEV), end.to(DEV), None if start is None else start.to(DEV))
            for a, b in zip(got, want):
                assert torch.allclose(a.cpu(), b, rtol=1e-6, atol=1e-6)


def test_sequence_sharded_scan_without_process_group():
    """Outside torch.distributed the sharded scan is the whole-sequence scan."""
    B, L, D, N = 1, 1024, 64, 16
    ins = make_inputs(B, L, D, N, seed=4, dist="config", device=DEV)
    args = [ins[k] for k in ("u", "delta", "A", "Bm", "Cm")]
    y, last = sharding.sequence_sharded_scan(*args, D=ins["Dskip"], z=ins["z"])
    y1, last1 = selective_scan_fused(*args, D=ins["Dskip"], z=ins["z"])
    assert O.normwise_error(y, y1) < 1e-5
    assert O.normwise_error(last, last1) < 1e-5


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharding_over_nccl_two_ranks():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29541", os.path.join(ROOT, "tests", "sharding_nccl_worker.py")]
    res = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
