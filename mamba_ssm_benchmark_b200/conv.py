"""Causal depthwise conv1d (+ SiLU) of the Mamba mixer on sm_100a (C ABI: ssm_conv1d_fwd/_bwd).

Replaces models/mamba.py:100-107: ``x.transpose(1, 2)``, left padding with d_conv - 1 zeros (or
the decode state), ``F.conv1d(..., groups=d_inner)``, ``F.silu``, transpose back.  The kernels
work in the (B, L, D) layout directly, read x through its strides (the first half of in_proj's
output needs no copy) and fuse the bias and the SiLU.
"""

import torch

from . import _native as nat

SUPPORTED_K = (1, 2, 3, 4)


def _weight2d(weight, D):
    w = weight.reshape(D, -1)
    return w.to(torch.float32).contiguous()


def _check(x, weight):
    if not x.is_cuda:
        raise RuntimeError("the sm_100a conv1d needs CUDA tensors (this package has no CPU path)")
    if x.dim() != 3:
        raise ValueError(f"x must be (B, L, D), got {tuple(x.shape)}")
    D = x.shape[2]
    K = weight.numel() // D if weight.numel() % D == 0 else -1
    if K not in SUPPORTED_K or weight.shape[0] != D:
        raise ValueError(f"weight must be (D, K) or (D, 1, K) with D={D}, K in {SUPPORTED_K}; got {tuple(weight.shape)}")
    if x.dtype not in nat.DTYPES:
        raise TypeError(f"conv1d supports float32 and bfloat16 activations, got {x.dtype}")
    return K


def _inner_contig(t):
    return t if (t.stride(-1) == 1 or t.shape[-1] == 1) else t.contiguous()


def _fwd(x, w, bias, silu, state=None, new_state=None):
    Bsz, L, D = x.shape
    K = w.shape[1]
    out = torch.empty((Bsz, L, D), dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        rc = nat.lib().ssm_conv1d_fwd(Bsz, L, D, K, nat.view3(x), nat.ptr(w), nat.ptr(bias), nat.ptr(state),
                                      1 if silu else 0, nat.view3(out), nat.ptr(new_state),
                                      nat.stream_of(x.device))
    nat.check(rc, "ssm_conv1d_fwd")
    return out


class CausalConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, bias, silu):
        ctx.save_for_backward(x, w, bias)
        ctx.silu = silu
        return _fwd(x, w, bias, silu)

    @staticmethod
    def backward(ctx, dout):
        x, w, bias = ctx.saved_tensors
        Bsz, L, D = x.shape
        K = w.shape[1]
        dout = _inner_contig(dout.to(x.dtype))
        dx = torch.empty((Bsz, L, D), dtype=x.dtype, device=x.device)
        dw = torch.empty((D, K), dtype=torch.float32, device=x.device)
        db = torch.empty((D,), dtype=torch.float32, device=x.device) if bias is not None else None
        wsb = nat.conv_workspace_bytes(Bsz, L, D, K)
        ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
        with torch.cuda.device(x.device):
            rc = nat.lib().ssm_conv1d_bwd(Bsz, L, D, K, nat.view3(x), nat.ptr(w), nat.ptr(bias), 1 if ctx.silu else 0,
                                          nat.view3(dout), nat.view3(dx), nat.ptr(dw), nat.ptr(db), ws.data_ptr(),
                                          wsb, nat.stream_of(x.device))
        nat.check(rc, "ssm_conv1d_bwd")
        return dx, dw, db, None


def causal_conv1d(x, weight, bias=None, activation="silu", conv_state=None, update_state=False):
    """out = act(causal depthwise conv1d(x)), all in (B, L, D).

    x: (B, L, D) float32 or bfloat16, any batch/row strides; weight: (D, K) or nn.Conv1d's
    (D, 1, K); bias: (D) or None; activation: "silu" or None.  With ``conv_state`` (B, D, K - 1)
    the sequence continues from a decode state (inference, no autograd), and with
    ``update_state=True`` the state is replaced in place by the last K - 1 inputs, as
    models/mamba.py:104-105 does.  Differentiable w.r.t. x, weight and bias without a state."""
    K = _check(x, weight)
    if activation not in ("silu", None):
        raise ValueError(f"activation must be 'silu' or None, got {activation!r}")
    silu = activation == "silu"
    D = x.shape[2]
    x = _inner_contig(x)
    w = _weight2d(weight, D)
    b = None if bias is None else bias.to(torch.float32).contiguous()
    if conv_state is None:
        if torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad or
                                        (bias is not None and bias.requires_grad)):
            out = CausalConv1dFn.apply(x, w, b, silu)
        else:
            out = _fwd(x, w, b, silu)
        return out
    if tuple(conv_state.shape) != (x.shape[0], D, K - 1) or conv_state.dtype != x.dtype:
        raise ValueError(f"conv_state must be ({x.shape[0]}, {D}, {K - 1}) in {x.dtype}")
    state = conv_state.contiguous()
    new_state = None
    if update_state:
        in_place = state.data_ptr() == conv_state.data_ptr() and x.shape[1] <= 4   # one time tile
        new_state = state if in_place else torch.empty_like(state)
    with torch.no_grad():
        out = _fwd(x, w, b, silu, state, new_state)
    if update_state and new_state.data_ptr() != conv_state.data_ptr():
        conv_state.copy_(new_state)
    return out
