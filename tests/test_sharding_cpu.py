"""Multi-rank host logic of the sharded scan, on CPU ranks over gloo (world size 2 and 3).

The per-shard compute is the oracle here (CPU); what is under test is the package's exchange
and composition code (mamba_ssm_benchmark_b200/sharding.py), the part that runs unchanged
between GPUs under NCCL:

* sequence shards: every rank summarises its contiguous piece of the sequence, the summaries
  are all-gathered, and the composed carried-in state must equal the full-sequence oracle's
  state at the shard boundary (and the shard's output, finished from it, the oracle's output);
* sequence-shard backward: every rank summarises its shard's reverse adjoint, the summaries are
  all-gathered and composed from the last shard to the first, and the adjoint entering each
  shard (and the gradient of h0) must equal the full-sequence oracle's;
* channel shards: every rank differentiates its channel range; after ``reduce_shared_grads``
  dBm and dCm must equal the full-width oracle's gradients, for separate tensors and for
  dB | dC views of one buffer.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mamba_ssm_benchmark_b200 import sharding
from mamba_ssm_benchmark_b200.workloads import make_inputs
from oracle import scan_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")


def _sequence_worker(rank, world, port, method, with_h0):
    _init(rank, world, port)
    try:
        B, L, D, N = 2, 60, 8, 4
        ins = make_inputs(B, L, D, N, seed=11, dist="test", h0=with_h0)
        u, delta, A, Bm, Cm, h0 = (ins[k] for k in ("u", "delta", "A", "Bm", "Cm", "h0"))
        # full-sequence oracle states
        a, b = O.discretize(delta, A, Bm, u, method)
        states = O.scan_sequential(a, b, h0)
        y_full, last_full = O.selective_scan(u, delta, A, Bm, Cm, h0=h0, method=method)
        bounds = [round(i * L / world) for i in range(world + 1)]
        lo, hi = bounds[rank], bounds[rank + 1]
        # this rank's summary (decay, hend from zero), computed by the oracle
        decay = a[:, lo:hi].prod(1)
        hend = O.scan_sequential(a[:, lo:hi], b[:, lo:hi])[:, -1]
        decays, hends = sharding.exchange_summaries(decay, hend)
        assert decays.shape == (world, B, D, N) and hends.shape == (world, B, D, N)
        h_in, last = sharding.compose_prefix(decays, hends, h0)
        want_in = states[:, lo - 1] if lo > 0 else (h0 if h0 is not None else torch.zeros(B, D, N))
        assert O.normwise_error(h_in[rank], want_in) < 1e-5
        assert O.normwise_error(last, last_full) < 1e-5
        # finishing the shard from its carried-in state reproduces the full output
        y_sh, last_sh = O.selective_scan(u[:, lo:hi], delta[:, lo:hi], A, Bm[:, lo:hi], Cm[:, lo:hi],
                                         h0=h_in[rank], method=method)
        assert O.normwise_error(y_sh, y_full[:, lo:hi]) < 1e-5
        assert O.normwise_error(last_sh, states[:, hi - 1]) < 1e-5
    finally:
        dist.destroy_process_group()


def _adjoint(a, cdys, dl=None):
    """Reverse adjoint over dim 1 from dl (zeros if None): dh_{t-1} = a_t (dh_t + C_t dys_t).
    Returns the adjoint entering every step from the right, index t -> after step t."""
    L = a.shape[1]
    dh = torch.zeros_like(a[:, 0]) if dl is None else dl.clone()
    out = torch.empty_like(a)
    for t in range(L - 1, -1, -1):
        out[:, t] = dh
        dh = a[:, t] * (dh + cdys[:, t])
    return out, dh


def _sequence_bwd_worker(rank, world, port, method):
    _init(rank, world, port)
    try:
        B, L, D, N = 2, 48, 6, 4
        ins = make_inputs(B, L, D, N, seed=13, dist="test", h0=True, dlast=True)
        u, delta, A, Bm, Cm, h0, z, dy, dlast = (ins[k] for k in ("u", "delta", "A", "Bm", "Cm", "h0", "z", "dy",
                                                                 "dlast"))
        a, _ = O.discretize(delta, A, Bm, u, method)
        dys = dy * z * torch.sigmoid(z)
        cdys = Cm[:, :, None, :] * dys[..., None]
        after, dh_first = _adjoint(a, cdys, dlast)         # full-sequence reverse adjoint
        bounds = [round(i * L / world) for i in range(world + 1)]
        lo, hi = bounds[rank], bounds[rank + 1]
        decay = a[:, lo:hi].prod(1)
        _, dstart = _adjoint(a[:, lo:hi], cdys[:, lo:hi])
        decays, dstarts = sharding.exchange_summaries(decay, dstart)
        dl_in, dh0 = sharding.compose_suffix(decays, dstarts, dlast)
        assert O.normwise_error(dl_in[rank], after[:, hi - 1]) < 1e-5
        assert O.normwise_error(dh0, dh_first) < 1e-5
        # and dh0 is autograd's gradient of the gated output + dlast . last w.r.t. h0
        lv = {k: ins[k].clone().requires_grad_(k == "h0") for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "h0")}
        y, last = O.selective_scan_fused(lv["u"], lv["delta"], lv["A"], lv["Bm"], lv["Cm"], h0=lv["h0"],
                                         method=method, Dskip=lv["Dskip"], z=lv["z"])
        (g,) = torch.autograd.grad((y * dy).sum() + (last * dlast).sum(), lv["h0"])
        assert O.normwise_error(dh0, g) < 1e-5
    finally:
        dist.destroy_process_group()


def _channel_worker(rank, world, port, one_buffer):
    _init(rank, world, port)
    try:
        B, L, D, N = 2, 24, 10, 4
        ins = make_inputs(B, L, D, N, seed=5, dist="test")
        keys = ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")
        lo, hi = sharding.shard_range(D, world, rank)

        def grads(lo, hi):
            lv = {k: ins[k].clone() for k in keys}
            for k in ("u", "delta", "z"):
                lv[k] = lv[k][:, :, lo:hi].contiguous()
            lv["A"], lv["Dskip"] = lv["A"][lo:hi].contiguous(), lv["Dskip"][lo:hi].contiguous()
            for v in lv.values():
                v.requires_grad_()
            y, _ = O.selective_scan_fused(lv["u"], lv["delta"], lv["A"], lv["Bm"], lv["Cm"], Dskip=lv["Dskip"],
                                          z=lv["z"])
            gb, gc = torch.autograd.grad(y, (lv["Bm"], lv["Cm"]), ins["dy"][:, :, lo:hi])
            return gb, gc

        full_b, full_c = grads(0, D)
        gb, gc = grads(lo, hi)
        if one_buffer:
            buf = torch.cat((gb, gc), -1).contiguous()
            gb, gc = buf[..., :N], buf[..., N:]
        sharding.reduce_shared_grads([gb, gc])
        assert O.normwise_error(gb, full_b) < 1e-5
        assert O.normwise_error(gc, full_c) < 1e-5
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,method,with_h0", [(2, "zoh", False), (2, "zoh", True), (3, "bilinear", True),
                                                  (2, "euler", False)])
def test_sequence_shards_gloo(world, method, with_h0):
    mp.spawn(_sequence_worker, args=(world, _free_port(), method, with_h0), nprocs=world, join=True)


@pytest.mark.parametrize("world,method", [(2, "zoh"), (3, "euler")])
def test_sequence_shards_backward_gloo(world, method):
    mp.spawn(_sequence_bwd_worker, args=(world, _free_port(), method), nprocs=world, join=True)


@pytest.mark.parametrize("one_buffer", [False, True])
def test_channel_shards_gloo(one_buffer):
    mp.spawn(_channel_worker, args=(2, _free_port(), one_buffer), nprocs=2, join=True)


def test_shard_range_partitions():
    for channels in (1, 7, 512, 5120):
        for world in (1, 2, 3, 8):
            spans = [sharding.shard_range(channels, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == channels
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)


def test_compose_suffix_single_rank():
    g = torch.Generator().manual_seed(4)
    dec, dst, dl = (torch.rand(1, 2, 3, 4, generator=g) for _ in range(3))
    dl_in, dh0 = sharding.compose_suffix(dec, dst, dl[0])
    assert torch.equal(dl_in[0], dl[0])
    assert torch.allclose(dh0, dst[0] + dec[0] * dl[0])


def test_compose_prefix_single_rank():
    """One shard: its carried-in state is h0 and the last state is its own summary applied to h0."""
    g = torch.Generator().manual_seed(3)
    dec, hend, h0 = (torch.rand(1, 2, 3, 4, generator=g) for _ in range(3))
    h_in, last = sharding.compose_prefix(dec, hend, h0[0])
    assert torch.equal(h_in[0], h0[0])
    assert torch.allclose(last, dec[0] * h0[0] + hend[0])
