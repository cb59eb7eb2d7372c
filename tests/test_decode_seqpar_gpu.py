"""GPU parity of the single-token decode kernel and of the two-phase (sequence-parallel)
forward, both through the C ABI."""

import pytest
import torch

from conftest import load_golden
from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200 import selective_scan_fused, selective_state_update
from mamba_ssm_benchmark_b200.workloads import make_inputs
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
METHODS = ("zoh", "euler", "bilinear")


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert nat.read_device_error() == 0


@pytest.mark.parametrize("method", METHODS)
def test_decode_matches_reference_golden(method):
    """models/mamba.py:113-118 as recorded from the reference."""
    case = load_golden("decode.npz")
    state = case["state"].to(DEV).clone()
    y = selective_state_update(state, *(case[k].to(DEV) for k in ("x", "delta", "A", "Bm", "Cm")), method=method)
    assert y.shape == case["x"].shape
    assert O.normwise_error(y[:, 0], case[f"y_{method}"]) < 1e-5
    assert O.normwise_error(state, case[f"state_{method}"]) < 1e-5


@pytest.mark.parametrize("N", [4, 8, 16, 32, 64])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_stepping_equals_full_scan(N, dtype):
    """Token-by-token decode reproduces the training-path forward (tests/test_gpu.py:49-65)."""
    B, L, D = 3, 24, 40
    ins = make_inputs(B, L, D, N, seed=N, dist="config", h0=True, dtype=dtype)
    dev = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
    full, last = selective_scan_fused(dev["u"], dev["delta"], dev["A"], dev["Bm"], dev["Cm"], h0=dev["h0"],
                                      D=dev["Dskip"], z=dev["z"])
    state = dev["h0"].clone()
    ys = [selective_state_update(state, dev["u"][:, t], dev["delta"][:, t], dev["A"], dev["Bm"][:, t],
                                 dev["Cm"][:, t], D=dev["Dskip"], z=dev["z"][:, t]) for t in range(L)]
    steps = torch.stack(ys, 1)
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    assert O.normwise_error(steps.float(), full.float()) < tol
    assert O.normwise_error(state, last) < 1e-4


def test_decode_is_graph_capturable():
    B, D, N = 64, 512, 16
    ins = make_inputs(B, 1, D, N, seed=3, dist="config", h0=True)
    state = ins["h0"].to(DEV).clone()
    x, dt, A, Bm, Cm = (ins[k][:, 0].to(DEV) if ins[k].dim() == 3 else ins[k].to(DEV)
                        for k in ("u", "delta", "A", "Bm", "Cm"))
    out = torch.empty(B, D, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        selective_state_update(state, x, dt, A, Bm, Cm, out=out)
    torch.cuda.current_stream().wait_stream(s)
    ref_state = state.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        selective_state_update(state, x, dt, A, Bm, Cm, out=out)
    for _ in range(3):
        graph.replay()
        yr, ref_state = O.state_update(ref_state.cpu(), x.cpu(), dt.cpu(), A.cpu(), Bm.cpu(), Cm.cpu())
        ref_state = ref_state.to(DEV)
    torch.cuda.synchronize()
    assert O.normwise_error(state, ref_state) < 1e-5
    assert O.normwise_error(out, yr) < 1e-5


@pytest.mark.parametrize("parts", [2, 3, 8])
@pytest.mark.parametrize("method", METHODS)
def test_two_phase_sequence_parallel_forward(parts, method):
    """Split one sequence into shards; phase 1 gives each shard's (decay, hend) summary,
    shards compose left to right, phase 2 finishes each shard from its carried-in state.
    The stitched output equals the single-call forward (the config-2 protocol on one GPU)."""
    B, L, D, N = 1, 2048, 64, 16
    ins = make_inputs(B, L, D, N, seed=parts, dist="config", h0=True)
    dev = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
    full, last = selective_scan_fused(dev["u"], dev["delta"], dev["A"], dev["Bm"], dev["Cm"], h0=dev["h0"],
                                      method=method, D=dev["Dskip"], z=dev["z"])
    bounds = [round(i * L / parts) for i in range(parts + 1)]
    lib = nat.lib()
    stream = nat.stream_of(torch.device(DEV))
    sums, wss = [], []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        Ls = hi - lo
        wsb = nat.fwd_workspace_bytes(B, Ls, D, N)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=DEV)
        dec = torch.empty(B, D, N, device=DEV)
        hend = torch.empty(B, D, N, device=DEV)
        sl = lambda k: dev[k][:, lo:hi]
        rc = lib.ssm_scan_fwd_summary(B, Ls, D, N, nat.METHODS[method], nat.view3(sl("u")), nat.view3(sl("delta")),
                                      nat.ptr(dev["A"]), nat.view3(sl("Bm")), nat.ptr(dec), nat.ptr(hend),
                                      ws.data_ptr(), wsb, stream)
        nat.check(rc, "summary")
        sums.append((dec, hend))
        wss.append((ws, wsb))
    carry = dev["h0"].clone()
    outs = []
    for i, (lo, hi) in enumerate(zip(bounds[:-1], bounds[1:])):
        Ls = hi - lo
        y = torch.empty(B, Ls, D, device=DEV)
        lst = torch.empty(B, D, N, device=DEV)
        sl = lambda k: dev[k][:, lo:hi]
        rc = lib.ssm_scan_fwd_finish(B, Ls, D, N, nat.METHODS[method], nat.view3(sl("u")), nat.view3(sl("delta")),
                                     nat.ptr(dev["A"]), nat.view3(sl("Bm")), nat.view3(sl("Cm")),
                                     nat.ptr(dev["Dskip"]), nat.view3(sl("z")), nat.ptr(carry), nat.view3(y),
                                     nat.NULL_VIEW, nat.ptr(lst), None, wss[i][0].data_ptr(), wss[i][1], stream)
        nat.check(rc, "finish")
        dec, hend = sums[i]
        carry = dec * carry + hend                       # compose this shard's summary
        assert O.normwise_error(lst, carry) < 1e-5
        outs.append(y)
    torch.cuda.synchronize()
    assert O.normwise_error(torch.cat(outs, 1), full) < 1e-5
    assert O.normwise_error(carry, last) < 1e-5
