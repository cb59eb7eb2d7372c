"""The selective-scan op: a drop-in for the reference's fused GPU scan.

Reference interfaces this module keeps (same argument names, meaning and errors):

* ``selective_scan_triton(x, delta, A, Bm, Cm, h0=None, method="zoh", d_block=None)``
  — kernels/triton_scan.py:322-329, the fused-kernel entry point, returning ``(y, last)``.
* ``selective_scan(x, delta, A, Bm, Cm, h0=None, method="zoh", scan="chunked", d_block=None,
  chunk_size=None)`` — models/scan.py:277-299, the dispatcher the Mamba mixer calls
  (models/mamba.py:120-121), with the reference's default.  Every scan name the reference
  accepts ("chunked", "sequential", "hillis_steele", "blelloch", "reference", "triton", "auto")
  names an algorithm for the same function, the selective scan; on CUDA tensors each of them
  runs the sm_100a kernels (there is one implementation here, no dispatch between backends),
  and on CPU tensors every one raises, because this package ships no non-CUDA path.  An
  unknown name raises ValueError.

Extension: ``D=`` and ``z=`` fuse the mixer's skip and gate, ``(y + x*D) * silu(z)``
(models/mamba.py:124), into the same kernels.

Computation: float32 state and accumulation always.  Activations are read in their own
dtype when x, delta, Bm, Cm (and z) all share float32 or bfloat16; any other mix is first
promoted to float32 exactly like models/scan.py:288-291.  Outputs follow the reference:
``y`` in x's dtype, ``last`` in float32 (``ct``), gradients in the dtype of each input.
"""

import math

import torch

from . import _native as nat

# scan names of the reference (models/scan.py:280-282) plus this package's own; all select the fused kernels
SCAN_NAMES = ("chunked", "sequential", "hillis_steele", "blelloch", "reference", "triton", "auto", "b200", "cuda")
SUPPORTED_N = (4, 8, 16, 32, 64)
CHUNK = 16  # checkpoint interval of the forward's saved states (time steps)


def _validate(x, delta, A, Bm, Cm, method):
    if method not in nat.METHODS:
        raise ValueError(f"unknown discretization {method!r}; expected one of {list(nat.METHODS)}")
    if x.dim() != 3 or delta.shape != x.shape:
        raise ValueError(f"x and delta must be (B, L, D) of equal shape, got {tuple(x.shape)} / {tuple(delta.shape)}")
    Bsz, L, D = x.shape
    if min(Bsz, L, D) < 1:
        raise ValueError(f"x must have positive B, L and D, got {tuple(x.shape)} (the reference fails on "
                         f"empty inputs too)")
    if A.dim() != 2 or A.shape[0] != D:
        raise ValueError(f"A must be (D, N) with D={D}, got {tuple(A.shape)}")
    N = A.shape[1]
    if N not in SUPPORTED_N:
        raise ValueError(f"d_state must be a power of two in {SUPPORTED_N} for the sm_100a kernel, got {N}")
    for name, t in (("Bm", Bm), ("Cm", Cm)):
        if tuple(t.shape) != (Bsz, L, N):
            raise ValueError(f"{name} must be (B, L, N) = {(Bsz, L, N)}, got {tuple(t.shape)}")
    if not x.is_cuda:
        raise RuntimeError("the sm_100a selective scan needs CUDA tensors (this package has no CPU path)")
    return Bsz, L, D, N


def _act(t, dtype):
    """Cast to the compute-side activation dtype and make the innermost stride 1."""
    if t is None:
        return None
    if t.dtype != dtype:
        t = t.to(dtype)
    if t.stride(-1) != 1 and t.shape[-1] != 1:
        t = t.contiguous()
    return t


def _f32(t):
    return None if t is None else t.to(torch.float32).contiguous()


class SelectiveScanFn(torch.autograd.Function):
    """(y, last) = scan(x, delta, A, Bm, Cm, h0, D, z) on sm_100a.

    Saves the inputs plus the state entering every 16-step chunk (B, ceil(L/16), D, N) fp32,
    from which the backward kernel recomputes states in registers (the reference recomputes
    all (B, L, D_tile, N) states into HBM instead, kernels/triton_scan.py:305-309), and, when z
    is given, the gate's input y + x*D, which the backward needs for dz.
    """

    @staticmethod
    def forward(ctx, x, delta, A, Bm, Cm, h0, D, z, method, delta_bias=None, delta_softplus=False):
        Bsz, L, Dch = x.shape
        N = A.shape[1]
        dev = x.device
        y = torch.empty((Bsz, L, Dch), dtype=x.dtype, device=dev)
        last = torch.empty((Bsz, Dch, N), dtype=torch.float32, device=dev)
        need_bwd = any(ctx.needs_input_grad[:8])
        nchunks = -(-L // CHUNK)
        cs = torch.empty((Bsz, nchunks, Dch, N), dtype=torch.float32, device=dev) if need_bwd else None
        # the gate's input (y + x D), needed by the backward to form dz
        yg = torch.empty((Bsz, L, Dch), dtype=x.dtype, device=dev) if (need_bwd and z is not None) else None
        wsb = nat.fwd_workspace_bytes(Bsz, L, Dch, N)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            rc = nat.lib().ssm_scan_fwd_ex(
                Bsz, L, Dch, N, nat.METHODS[method], nat.view3(x), nat.view3(delta), nat.ptr(A),
                nat.view3(Bm), nat.view3(Cm), nat.ptr(D), nat.view3(z), nat.ptr(h0),
                nat.view3(y), nat.view3(yg), nat.ptr(last), nat.ptr(cs), nat.delta_opts(delta_bias, delta_softplus),
                ws.data_ptr(), wsb, nat.stream_of(dev))
        nat.check(rc, "ssm_scan_fwd")
        if need_bwd:
            ctx.save_for_backward(x, delta, A, Bm, Cm, h0, D, z, cs, yg, delta_bias)
        ctx.method = method
        ctx.delta_softplus = delta_softplus
        return y, last

    @staticmethod
    def backward(ctx, dy, dlast):
        x, delta, A, Bm, Cm, h0, D, z, cs, yg, delta_bias = ctx.saved_tensors
        grads = scan_backward(x, delta, A, Bm, Cm, h0, D, z, cs, yg, dy, dlast, ctx.method, delta_bias,
                              ctx.delta_softplus)
        return (*grads[:8], None, grads[8], None)


def scan_backward(x, delta, A, Bm, Cm, h0, D, z, cs, yg, dy, dlast, method, delta_bias=None, delta_softplus=False):
    """One ssm_scan_bwd call: returns (du, ddelta, dA, dB, dC, dh0, dD, dz, ddelta_bias), each None
    where the input (h0 for dh0, delta_bias) was None.  cs and yg are what the forward saved
    (chunk_states, the gate input).  With delta_softplus, ddelta is the gradient w.r.t. the raw
    delta (before bias and softplus)."""
    Bsz, L, Dch = x.shape
    N = A.shape[1]
    dev = x.device
    dy = _act(dy, x.dtype)
    dlast = None if dlast is None else dlast.to(torch.float32).contiguous()
    du = torch.empty((Bsz, L, Dch), dtype=x.dtype, device=dev)
    ddelta = torch.empty((Bsz, L, Dch), dtype=x.dtype, device=dev)
    dA = torch.empty((Dch, N), dtype=torch.float32, device=dev)
    dB = torch.empty((Bsz, L, N), dtype=x.dtype, device=dev)
    dC = torch.empty((Bsz, L, N), dtype=x.dtype, device=dev)
    dD = torch.empty((Dch,), dtype=torch.float32, device=dev) if D is not None else None
    dz = torch.empty((Bsz, L, Dch), dtype=x.dtype, device=dev) if z is not None else None
    dh0 = torch.empty((Bsz, Dch, N), dtype=torch.float32, device=dev) if h0 is not None else None
    dbias = torch.empty((Dch,), dtype=torch.float32, device=dev) if (delta_softplus and delta_bias is not None) else None
    wsb = nat.bwd_workspace_bytes(Bsz, L, Dch, N)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = nat.lib().ssm_scan_bwd_ex(
            Bsz, L, Dch, N, nat.METHODS[method], nat.view3(x), nat.view3(delta), nat.ptr(A),
            nat.view3(Bm), nat.view3(Cm), nat.ptr(D), nat.view3(z), nat.ptr(h0), nat.ptr(cs),
            nat.view3(yg), nat.view3(dy), nat.ptr(dlast), nat.view3(du), nat.view3(ddelta), nat.ptr(dA),
            nat.view3(dB), nat.view3(dC), nat.ptr(dD), nat.view3(dz), nat.ptr(dh0),
            nat.delta_opts(delta_bias, delta_softplus, dbias), ws.data_ptr(), wsb, nat.stream_of(dev))
    nat.check(rc, "ssm_scan_bwd")
    return du, ddelta, dA, dB, dC, dh0, dD, dz, dbias


def _prepare(x, delta, A, Bm, Cm, h0, D, z, method):
    _validate(x, delta, A, Bm, Cm, method)
    if any(t is not None and t.dtype == torch.float64 for t in (x, delta, A, Bm, Cm, h0, D, z)):
        raise TypeError("float64 is not supported by the sm_100a kernel; use float32 or bfloat16")
    acts = [t for t in (x, delta, Bm, Cm, z) if t is not None]
    uniform = all(t.dtype == acts[0].dtype for t in acts)
    ct = acts[0].dtype if uniform and acts[0].dtype in nat.DTYPES else torch.float32
    return (_act(x, ct), _act(delta, ct), _f32(A), _act(Bm, ct), _act(Cm, ct), _f32(h0), _f32(D), _act(z, ct))


def selective_scan_fused(x, delta, A, Bm, Cm, h0=None, method="zoh", D=None, z=None, delta_bias=None,
                         delta_softplus=False):
    """Returns (out, last) with out = (scan(x) + x*D) * silu(z) (each term optional).

    x, delta, z: (B, L, D); A: (D, N); Bm, Cm: (B, L, N); h0: (B, D, N); D: (D).
    With ``delta_softplus`` the scan uses softplus(delta + delta_bias) as its step size, computed in
    the kernels (the mixer's ``F.softplus(dt_proj(dt))``, models/mamba.py:77, with ``delta`` the
    projection without its bias); gradients flow to the raw delta and to delta_bias (D).
    out has x's dtype; last is float32.
    """
    in_dtype = x.dtype
    args = _prepare(x, delta, A, Bm, Cm, h0, D, z, method)
    bias = _f32(delta_bias) if delta_softplus else None
    y, last = SelectiveScanFn.apply(*args, method, bias, bool(delta_softplus))
    return y.to(in_dtype), last


def selective_scan_triton(x, delta, A, Bm, Cm, h0=None, method="zoh", d_block=None):
    """Drop-in for kernels/triton_scan.py:selective_scan_triton (same contract).

    ``d_block`` is accepted for signature compatibility; the kernel tiles channels itself.
    """
    del d_block
    return selective_scan_fused(x, delta, A, Bm, Cm, h0=h0, method=method)


def selective_scan(x, delta, A, Bm, Cm, h0=None, method="zoh", scan="chunked", d_block=None, chunk_size=None):
    """Drop-in for models/scan.py:selective_scan: returns (y, h_last).

    x, delta: (B, L, D); A: (D, N); Bm, Cm: (B, L, N); h0: (B, D, N).  ``scan`` may be any name the
    reference accepts; all of them compute the selective scan and run the fused sm_100a kernels.
    ``chunk_size`` and ``d_block`` only tune the reference's PyTorch scans and are ignored.
    """
    del chunk_size
    if scan not in SCAN_NAMES:
        raise ValueError(f"unknown scan {scan!r}; expected one of {SCAN_NAMES}")
    with torch.autocast(device_type="cuda", enabled=False):
        return selective_scan_triton(x, delta, A, Bm, Cm, h0=h0, method=method, d_block=d_block)


def chunk_states_shape(B, L, D, N):
    """Shape of the per-chunk states the forward saves for the backward."""
    return (B, math.ceil(L / CHUNK), D, N)
