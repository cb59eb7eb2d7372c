"""GPU parity of the causal depthwise conv1d + SiLU kernels (ssm_conv1d_fwd / _bwd) against the
oracle restatement of models/mamba.py:100-107."""

import pytest
import torch

from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200 import causal_conv1d
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert nat.read_device_error() == 0


def _inputs(B, L, D, K, seed, dtype=torch.float32, strided=False):
    g = torch.Generator().manual_seed(seed)
    if strided:   # x as the first half of an in_proj output (row stride 2D)
        xz = torch.randn(B, L, 2 * D, generator=g).to(dtype)
        x = xz.to(DEV)[..., :D]
    else:
        x = torch.randn(B, L, D, generator=g).to(dtype).to(DEV)
    w = (torch.randn(D, 1, K, generator=g) * 0.5).to(DEV)
    b = torch.randn(D, generator=g).to(DEV)
    dout = torch.randn(B, L, D, generator=g).to(dtype).to(DEV)
    return x, w, b, dout


@pytest.mark.parametrize("B,L,D", [(2, 64, 128), (3, 37, 50), (1, 1, 8), (2, 100, 96), (16, 512, 512)])
@pytest.mark.parametrize("K", [4, 3, 2, 1])
@pytest.mark.parametrize("silu", [True, False])
def test_forward_and_backward_match_reference(B, L, D, K, silu):
    x, w, b, dout = _inputs(B, L, D, K, seed=B * 100 + L + K)
    xl, wl, bl = (t.detach().clone().requires_grad_() for t in (x, w, b))
    out = causal_conv1d(xl, wl, bl, activation="silu" if silu else None)
    xr, wr, br = (t.detach().cpu().double().requires_grad_() for t in (x, w, b))
    ref, _ = O.causal_conv1d(xr, wr[:, 0], br, silu=silu)
    assert O.normwise_error(out.detach().cpu().double(), ref) < 1e-5
    got = torch.autograd.grad(out, (xl, wl, bl), dout)
    want = torch.autograd.grad(ref, (xr, wr, br), dout.cpu().double())
    for name, gg, ww in zip(("dx", "dweight", "dbias"), got, want):
        assert gg.shape == ww.shape, name
        assert O.normwise_error(gg.cpu().double(), ww) < 1e-5, name


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_strided_view_and_bf16(dtype):
    """x read through the (B, L, 2D) in_proj output without a copy; bf16 in and out."""
    B, L, D, K = 2, 96, 64, 4
    x, w, b, dout = _inputs(B, L, D, K, seed=7, dtype=dtype, strided=True)
    assert x.stride(1) == 2 * D
    xl = x.detach().requires_grad_()
    out = causal_conv1d(xl, w, b)
    assert out.dtype == dtype
    ref, _ = O.causal_conv1d(x.float().cpu(), w[:, 0].cpu(), b.cpu())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert O.normwise_error(out.float().cpu(), ref) < tol
    (dx,) = torch.autograd.grad(out, xl, dout)
    xr = x.float().cpu().requires_grad_()
    ref, _ = O.causal_conv1d(xr, w[:, 0].cpu(), b.cpu())
    (dxr,) = torch.autograd.grad(ref, xr, dout.float().cpu())
    assert O.normwise_error(dx.float().cpu(), dxr) < tol


def test_no_bias_and_determinism():
    x, w, _, dout = _inputs(4, 300, 256, 4, seed=3)
    runs = []
    for _ in range(2):
        xl, wl = x.detach().requires_grad_(), w.detach().clone().requires_grad_()
        out = causal_conv1d(xl, wl)
        runs.append(torch.autograd.grad(out, (xl, wl), dout))
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])


@pytest.mark.parametrize("L", [1, 2, 5, 40])
def test_decode_state_continues_the_sequence(L):
    """Prefill the first P positions, then continue from the conv state: equals one pass over the
    whole sequence; the state is updated in place like models/mamba.py:104-105."""
    B, P, D, K = 3, 20, 64, 4
    x, w, b, _ = _inputs(B, P + L, D, K, seed=L)
    full = causal_conv1d(x, w, b)
    state = torch.zeros(B, D, K - 1, device=DEV)
    first = causal_conv1d(x[:, :P].contiguous(), w, b, conv_state=state, update_state=True)
    rest = causal_conv1d(x[:, P:].contiguous(), w, b, conv_state=state, update_state=True)
    assert O.normwise_error(torch.cat([first, rest], 1), full) < 1e-6
    _, ref_state = O.causal_conv1d(x.cpu(), w[:, 0].cpu(), b.cpu())
    assert torch.allclose(state.cpu(), ref_state, atol=0, rtol=0)


def test_errors():
    x, w, b, _ = _inputs(1, 8, 16, 4, seed=1)
    with pytest.raises(ValueError, match="weight"):
        causal_conv1d(x, torch.randn(16, 5, device=DEV))
    with pytest.raises(TypeError):
        causal_conv1d(x.double(), w)
    with pytest.raises(RuntimeError, match="CUDA"):
        causal_conv1d(x.cpu(), w.cpu())
