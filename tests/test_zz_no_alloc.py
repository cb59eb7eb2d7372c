"""ssm_scan_bwd_noalloc: the backward for callers that cannot allocate device memory when they
run it (a fixed memory pool after start-up, or a plugin host that gives the plugin no
allocator).  It takes no workspace and uses scratch built into the library instead.

Checked through the C ABI against ssm_scan_bwd with a caller workspace, on two calls in a row
(the built-in scratch keeps the previous call's contents).  This file is collected last so a
failure here cannot hide the results of the other tests; it also passes alone in a fresh
process."""

import pytest
import torch

import scan_harness as H
from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200.workloads import make_inputs
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _forward(ins, B, L, D, N):
    """Runs ssm_scan_fwd for training: returns (chunk_states, ygate)."""
    lib = nat.lib()
    dt = ins["u"].dtype
    y = torch.empty(B, L, D, device=DEV, dtype=dt)
    yg = torch.empty(B, L, D, device=DEV, dtype=dt)
    last = torch.empty(B, D, N, device=DEV)
    cs = torch.empty(B, -(-L // 16), D, N, device=DEV)
    wsb = nat.fwd_workspace_bytes(B, L, D, N)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=DEV)
    rc = lib.ssm_scan_fwd(B, L, D, N, 0, nat.view3(ins["u"]), nat.view3(ins["delta"]), nat.ptr(ins["A"]),
                          nat.view3(ins["Bm"]), nat.view3(ins["Cm"]), nat.ptr(ins["Dskip"]), nat.view3(ins["z"]),
                          nat.ptr(ins["h0"]), nat.view3(y), nat.view3(yg), nat.ptr(last), nat.ptr(cs),
                          ws.data_ptr(), wsb, nat.stream_of(torch.device(DEV)))
    nat.check(rc, "ssm_scan_fwd")
    return cs, yg


def _outputs(B, L, D, N, dt):
    a = dict(device=DEV, dtype=dt)
    return dict(du=torch.empty(B, L, D, **a), ddelta=torch.empty(B, L, D, **a),
                dA=torch.empty(D, N, device=DEV), dB=torch.empty(B, L, N, **a),
                dC=torch.empty(B, L, N, **a), dD=torch.empty(D, device=DEV),
                dz=torch.empty(B, L, D, **a), dh0=torch.empty(B, D, N, device=DEV))


def _backward(ins, cs, yg, B, L, D, N, noalloc, out=None):
    lib = nat.lib()
    out = out if out is not None else _outputs(B, L, D, N, ins["u"].dtype)
    common = (B, L, D, N, 0, nat.view3(ins["u"]), nat.view3(ins["delta"]), nat.ptr(ins["A"]), nat.view3(ins["Bm"]),
              nat.view3(ins["Cm"]), nat.ptr(ins["Dskip"]), nat.view3(ins["z"]), nat.ptr(ins["h0"]), nat.ptr(cs),
              nat.view3(yg), nat.view3(ins["dy"]), nat.ptr(ins["dlast"]), nat.view3(out["du"]),
              nat.view3(out["ddelta"]), nat.ptr(out["dA"]), nat.view3(out["dB"]), nat.view3(out["dC"]),
              nat.ptr(out["dD"]), nat.view3(out["dz"]), nat.ptr(out["dh0"]))
    stream = nat.stream_of(torch.device(DEV))
    if noalloc:
        rc = lib.ssm_scan_bwd_noalloc(*common, stream)
    else:
        wsb = nat.bwd_workspace_bytes(B, L, D, N)
        ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
        rc = lib.ssm_scan_bwd(*common, ws.data_ptr(), wsb, stream)
    nat.check(rc, "ssm_scan_bwd_noalloc" if noalloc else "ssm_scan_bwd")
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("shape,dtype", [((2, 100, 64, 16), torch.float32), ((16, 512, 512, 16), torch.float32),
                                         ((3, 37, 50, 8), torch.float32), ((2, 300, 96, 16), torch.bfloat16),
                                         ((1, 2048, 64, 16), torch.float32)],
                         ids=["2x100x64x16", "16x512x512x16", "3x37x50x8", "2x300x96x16-bf16",
                              "1x2048x64x16-split"])
def test_noalloc_backward_matches_workspace_backward_twice(shape, dtype):
    B, L, D, N = shape
    assert nat.bwd_workspace_bytes(B, L, D, N) <= 32 << 20
    results = []
    for seed in (1, 2):                      # two calls in a row on different inputs
        ins = make_inputs(B, L, D, N, seed=seed, dist="config", h0=True, dlast=True, dtype=dtype)
        ins = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
        cs, yg = _forward(ins, B, L, D, N)
        ref = _backward(ins, cs, yg, B, L, D, N, noalloc=False)
        got = _backward(ins, cs, yg, B, L, D, N, noalloc=True)
        for k in ref:
            assert torch.isfinite(got[k].float()).all(), k
            assert O.normwise_error(got[k].float(), ref[k].float()) <= H.GRAD_TOL, k
        results.append(got)
    # the second call did not leave the first call's values behind
    assert not torch.equal(results[0]["dB"], results[1]["dB"])
    assert nat.read_device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    B, L, D, N = 64, 8192, 512, 16           # needs far more than the built-in scratch
    assert nat.bwd_workspace_bytes(B, L, D, N) > 32 << 20
    v = nat.NULL_VIEW
    rc = nat.lib().ssm_scan_bwd_noalloc(B, L, D, N, 0, v, v, None, v, v, None, v, None, None, v, v, None, v, v,
                                        None, v, v, None, v, None, None)
    assert rc == nat.SSM_ERR_WORKSPACE
    assert b"built-in scratch" in nat.lib().ssm_last_error_message()


def test_noalloc_call_allocates_no_device_memory():
    """With its inputs and outputs in place, the call leaves the device's free memory and torch's
    allocator untouched: it uses only the built-in scratch."""
    B, L, D, N = 4, 256, 128, 16
    ins = make_inputs(B, L, D, N, seed=3, dist="config", h0=True, dlast=True)
    ins = {k: (v.to(DEV) if v is not None else None) for k, v in ins.items()}
    cs, yg = _forward(ins, B, L, D, N)
    out = _outputs(B, L, D, N, torch.float32)
    _backward(ins, cs, yg, B, L, D, N, noalloc=True, out=out)       # first call on this device
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    held0, peak0 = torch.cuda.memory_allocated(), torch.cuda.max_memory_allocated()
    for _ in range(3):
        _backward(ins, cs, yg, B, L, D, N, noalloc=True, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == held0 and torch.cuda.max_memory_allocated() == peak0
    assert nat.read_device_error() == 0
