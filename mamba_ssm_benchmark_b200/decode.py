"""Single-token selective state update for autoregressive decoding.

The reference has no function for this step; its definition is the inline decode branch of
``Mamba.forward`` for L == 1 with a state (models/mamba.py:113-118, 123-124):

    a, b = discretize(delta, A, Bm, x, method);  h = a * h0 + b
    y = einsum("bdn,bn->bd", h, Cm);  state.ssm.copy_(h);  y = (y + x*D) * silu(z)

``selective_state_update`` does all of it in one sm_100a kernel launch (the reference issues
about ten eager kernels per layer and token, README.md:445-447), updates ``state`` in place
and is CUDA-graph capturable (no allocation besides the output, no synchronisation).
"""

import torch

from . import _native as nat
from .scan import SUPPORTED_N


def selective_state_update(state, x, delta, A, Bm, Cm, D=None, z=None, method="zoh", out=None):
    """state: (B, D, N) float32, updated in place.  x, delta, z: (B, D) or (B, 1, D);
    Bm, Cm: (B, N) or (B, 1, N); A: (D, N); D: (D).  Returns y shaped like x."""
    if method not in nat.METHODS:
        raise ValueError(f"unknown discretization {method!r}")
    squeeze = x.dim() == 3
    if squeeze:
        x, delta = x[:, 0], delta[:, 0]
        Bm, Cm = Bm[:, 0], Cm[:, 0]
        z = None if z is None else z[:, 0]
    Bsz, Dch = x.shape
    N = A.shape[1]
    if N not in SUPPORTED_N:
        raise ValueError(f"d_state must be one of {SUPPORTED_N}, got {N}")
    if state.dtype != torch.float32 or not state.is_contiguous() or tuple(state.shape) != (Bsz, Dch, N):
        raise ValueError("state must be a contiguous float32 (B, D, N) tensor")
    if not x.is_cuda:
        raise RuntimeError("selective_state_update needs CUDA tensors (this package has no CPU path)")
    acts = [t for t in (x, delta, Bm, Cm, z) if t is not None]
    ct = acts[0].dtype if all(t.dtype == acts[0].dtype for t in acts) and acts[0].dtype in nat.DTYPES \
        else torch.float32

    def prep(t):
        if t is None:
            return None
        t = t.to(ct)
        return t if t.stride(-1) == 1 else t.contiguous()

    x, delta, Bm, Cm, z = (prep(t) for t in (x, delta, Bm, Cm, z))
    A = A.to(torch.float32).contiguous()
    D = None if D is None else D.to(torch.float32).contiguous()
    y = out if out is not None else torch.empty((Bsz, Dch), dtype=ct, device=x.device)
    with torch.cuda.device(x.device):
        rc = nat.lib().ssm_state_update(Bsz, Dch, N, nat.METHODS[method], state.data_ptr(), nat.view2(x),
                                        nat.view2(delta), A.data_ptr(), nat.view2(Bm), nat.view2(Cm),
                                        nat.ptr(D), nat.view2(z), nat.view2(y), nat.stream_of(x.device))
    nat.check(rc, "ssm_state_update")
    return y.unsqueeze(1) if squeeze else y
