"""CPU oracle: a restatement of the reference's selective-scan algorithm in plain torch (CPU).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by __graft_entry__.smoke() and by bench.py's
CPU-baseline leg as the checker / the timed CPU baseline; never by the product path.

It follows the reference (aman078-ai/mamba-ssm-benchmark) step by step:
  discretize            models/scan.py:39-55
  scan_sequential       models/scan.py:70-76
  scan_hillis_steele    models/scan.py:79-98   (with the h0 fold of :79-84)
  scan_blelloch         models/scan.py:101-135 (Blelloch's work-efficient up/down-sweep scan)
  default_chunk         models/scan.py:138-139
  scan_chunked          models/scan.py:142-165
  channel blocks        models/scan.py:180-190
  ChunkedScanFn         models/scan.py:193-255 (forward + recomputing backward, driven by
                        any of the scans; the chain rule through discretize by autograd,
                        as at :249)
  selective_scan_loop   models/scan.py:264-274 (autograd through a time loop: ground truth)
  selective_scan        models/scan.py:277-299 (dtype promotion, autocast off)
  gate                  models/mamba.py:124
  state_update          models/mamba.py:113-118
Parity pin: tests/test_oracle_golden.py checks every function here against golden vectors
that tests/golden/make_golden.py produced by running the reference's own code.
"""

import math

import torch

METHODS = ("zoh", "euler", "bilinear")
# transient (B, L, d_block, N) buffer budget when d_block is not given (models/scan.py:182)
ELEMENT_BUDGET = 1 << 24


def discretize(delta, A, Bm, x, method="zoh"):
    """(B,L,D) delta, x; (D,N) A; (B,L,N) Bm -> a, b (B,L,D,N)."""
    z = delta[..., None] * A
    bx = x[..., None] * Bm[:, :, None, :]
    if method == "zoh":
        return torch.exp(z), torch.expm1(z) / A * bx
    if method == "euler":
        return torch.exp(z), delta[..., None] * bx
    if method == "bilinear":
        w = 1.0 / (1.0 - 0.5 * z)
        return (1.0 + 0.5 * z) * w, delta[..., None] * w * bx
    raise ValueError(f"unknown discretization {method!r}")


def scan_sequential(a, b, h0=None):
    """h_t = a_t h_{t-1} + b_t along dim 1, all states returned."""
    h = torch.zeros_like(b[:, 0]) if h0 is None else h0
    out = torch.empty_like(b)
    for t in range(a.shape[1]):
        h = a[:, t] * h + b[:, t]
        out[:, t] = h
    return out


def scan_hillis_steele(a, b, h0=None):
    """Inclusive scan by recursive doubling over dim 1 (h0 folded into the first element)."""
    if h0 is not None:
        b = b.clone()
        b[:, 0] += a[:, 0] * h0
    n = a.shape[1]
    step = 1
    while step < n:
        b = torch.cat([b[:, :step], b[:, step:] + a[:, step:] * b[:, :-step]], dim=1)
        if 2 * step < n:
            a = torch.cat([a[:, :step], a[:, step:] * a[:, :-step]], dim=1)
        step *= 2
    return b


def scan_blelloch(a, b, h0=None):
    """Work-efficient two-sweep scan (Blelloch 1990) of the affine maps h -> a_t h + b_t along dim 1.

    The sequence is padded to a power of two P with identity maps (a = 1, b = 0).  Up-sweep: at
    stride 2d every node r = 2d k + 2d - 1 becomes "node r - d, then node r" (the total of its
    subtree).  The root is replaced by the identity; down-sweep: at each stride the left child
    takes its parent's prefix and the right child becomes "parent's prefix, then the left
    subtree's total".  Each position then holds the map of all steps before it (an exclusive
    prefix), so the state after step t is a_t (prefix_t(h0)) + b_t."""
    Bsz, L = a.shape[:2]
    rest = tuple(a.shape[2:])
    P = 1 << max(0, (L - 1).bit_length())
    pa = torch.cat([a, a.new_ones((Bsz, P - L) + rest)], dim=1)
    pb = torch.cat([b, b.new_zeros((Bsz, P - L) + rest)], dim=1)
    d = 1
    while d < P:                                   # up-sweep
        r = torch.arange(2 * d - 1, P, 2 * d)
        left = r - d
        pb[:, r] = pa[:, r] * pb[:, left] + pb[:, r]
        pa[:, r] = pa[:, r] * pa[:, left]
        d *= 2
    pa[:, P - 1] = 1.0
    pb[:, P - 1] = 0.0
    d = P // 2
    while d >= 1:                                  # down-sweep
        r = torch.arange(2 * d - 1, P, 2 * d)
        left = r - d
        la, lb = pa[:, left].clone(), pb[:, left].clone()
        pa[:, left], pb[:, left] = pa[:, r], pb[:, r]
        pb[:, r] = la * pb[:, r] + lb
        pa[:, r] = la * pa[:, r]
        d //= 2
    prev = pb[:, :L] if h0 is None else pb[:, :L] + pa[:, :L] * h0.unsqueeze(1)
    return a * prev + b


SCANS = {"sequential": scan_sequential, "hillis_steele": scan_hillis_steele, "blelloch": scan_blelloch}


def default_chunk(L):
    return max(4, 1 << math.ceil(math.log2(max(1.0, math.sqrt(L)))))


def scan_chunked(a, b, h0=None, chunk_size=None):
    """Two-level scan: sequential inside chunks, doubling scan over chunk ends, fix-up."""
    Bsz, L = a.shape[:2]
    rest = tuple(a.shape[2:])
    C = chunk_size or default_chunk(L)
    nc = -(-L // C)
    if nc * C > L:
        padn = (Bsz, nc * C - L) + rest
        a = torch.cat([a, a.new_ones(padn)], dim=1)
        b = torch.cat([b, b.new_zeros(padn)], dim=1)
    a = a.reshape((Bsz, nc, C) + rest)
    b = b.reshape((Bsz, nc, C) + rest)
    local = torch.empty_like(b)
    local[:, :, 0] = b[:, :, 0]
    for t in range(1, C):                          # fused multiply-add per step, into the output
        torch.addcmul(b[:, :, t], a[:, :, t], local[:, :, t - 1], out=local[:, :, t])
    decay = torch.cumprod(a, dim=2)
    ends = scan_hillis_steele(decay[:, :, -1], local[:, :, -1], h0)
    first = torch.zeros_like(ends[:, :1]) if h0 is None else h0[:, None]
    carry = torch.cat([first, ends[:, :-1]], dim=1)
    local.addcmul_(decay, carry[:, :, None])       # fix-up in place
    return local.reshape((Bsz, nc * C) + rest)[:, :L]


def channel_blocks(B, L, D, N, d_block=None):
    if not d_block:
        d_block = max(1, ELEMENT_BUDGET // (B * L * N))
    d_block = min(d_block, D)
    return [(i, min(i + d_block, D)) for i in range(0, D, d_block)]


def _scan_fn(chunk_size, name="chunked"):
    if name != "chunked":
        return SCANS[name]
    return lambda a, b, h0=None: scan_chunked(a, b, h0, chunk_size)


class ChunkedScanFn(torch.autograd.Function):
    """Memory-bounded selective scan: saves only the inputs; the backward recomputes the states
    of one channel block at a time with the chosen scan, runs the adjoint recurrence
    dh_t = g_t + a_{t+1} dh_{t+1} as a reversed scan, and takes the chain rule through the
    discretisation with autograd on (a, b) = discretize(...) (models/scan.py:219-255)."""

    @staticmethod
    def forward(ctx, x, delta, A, Bm, Cm, h0, method, d_block, chunk_size, scan_name="chunked"):
        scan = _scan_fn(chunk_size, scan_name)
        Bsz, L, D = x.shape
        N = A.shape[1]
        y = torch.empty_like(x)
        last = x.new_empty(Bsz, D, N)
        for i, j in channel_blocks(Bsz, L, D, N, d_block):
            a, b = discretize(delta[..., i:j], A[i:j], Bm, x[..., i:j], method)
            h = scan(a, b, None if h0 is None else h0[:, i:j])
            y[..., i:j] = torch.einsum("bldn,bln->bld", h, Cm)
            last[:, i:j] = h[:, -1]
        ctx.save_for_backward(x, delta, A, Bm, Cm, h0)
        ctx.cfg = (method, d_block, chunk_size, scan_name)
        return y, last

    @staticmethod
    def backward(ctx, dy, dlast):
        x, delta, A, Bm, Cm, h0 = ctx.saved_tensors
        method, d_block, chunk_size, scan_name = ctx.cfg
        scan = _scan_fn(chunk_size, scan_name)
        Bsz, L, D = x.shape
        N = A.shape[1]
        grads = dict(x=torch.empty_like(x), delta=torch.empty_like(delta), A=torch.empty_like(A),
                     B=torch.zeros_like(Bm), C=torch.zeros_like(Cm),
                     h0=None if h0 is None else torch.empty_like(h0))
        for i, j in channel_blocks(Bsz, L, D, N, d_block):
            hb0 = None if h0 is None else h0[:, i:j]
            with torch.enable_grad():
                leaves = [t.detach().requires_grad_() for t in (delta[..., i:j], A[i:j], Bm, x[..., i:j])]
                a, b = discretize(leaves[0], leaves[1], leaves[2], leaves[3], method)
            with torch.no_grad():
                ad = a.detach()
                h = scan(ad, b.detach(), hb0)
                dyb = dy[..., i:j]
                grads["C"] += torch.einsum("bld,bldn->bln", dyb, h)
                g = dyb[..., None] * Cm[:, :, None, :]
                if dlast is not None:
                    g[:, -1] += dlast[:, i:j]
                a_shift = torch.cat([ad[:, 1:], torch.ones_like(ad[:, :1])], dim=1)
                dh = scan(a_shift.flip(1), g.flip(1)).flip(1)
                start = torch.zeros_like(h[:, :1]) if hb0 is None else hb0[:, None]
                da = dh * torch.cat([start, h[:, :-1]], dim=1)       # d/da of a_t h_{t-1}
                if hb0 is not None:
                    grads["h0"][:, i:j] = dh[:, 0] * ad[:, 0]
                del h, g, a_shift
            g_delta, g_A, g_B, g_x = torch.autograd.grad((a, b), leaves, (da, dh))
            grads["delta"][..., i:j] = g_delta
            grads["A"][i:j] = g_A
            grads["B"] += g_B
            grads["x"][..., i:j] = g_x
        return (grads["x"], grads["delta"], grads["A"], grads["B"], grads["C"], grads["h0"], None, None, None, None)


def selective_scan_loop(x, delta, A, Bm, Cm, h0=None, method="zoh"):
    """Ground truth: time loop differentiated by autograd (O(B L D N) memory; small shapes)."""
    Bsz, L, D = x.shape
    h = x.new_zeros(Bsz, D, A.shape[1]) if h0 is None else h0
    ys = []
    for t in range(L):
        a, b = discretize(delta[:, t:t + 1], A, Bm[:, t:t + 1], x[:, t:t + 1], method)
        h = a[:, 0] * h + b[:, 0]
        ys.append(torch.einsum("bdn,bn->bd", h, Cm[:, t]))
    return torch.stack(ys, 1), h


def selective_scan(x, delta, A, Bm, Cm, h0=None, method="zoh", scan="chunked", d_block=None, chunk_size=None):
    """(y, last) computed in promote(x.dtype, float32) like the reference; y cast back to x.dtype."""
    dtype = x.dtype
    ct = torch.promote_types(dtype, torch.float32)
    with torch.autocast(device_type=x.device.type, enabled=False):
        args = [None if t is None else t.to(ct) for t in (x, delta, A, Bm, Cm, h0)]
        if scan == "reference":
            y, last = selective_scan_loop(*args, method=method)
        elif scan == "chunked" or scan in SCANS:
            y, last = ChunkedScanFn.apply(*args, method, d_block, chunk_size, scan)
        else:
            raise ValueError(f"oracle implements scan='chunked', {sorted(SCANS)} and 'reference', not {scan!r}")
    return y.to(dtype), last


def gate(y, x, Dskip=None, z=None):
    """Mamba mixer output before out_proj: (y + x D) * silu(z)."""
    if Dskip is not None:
        y = y + x * Dskip.to(x.dtype)
    if z is not None:
        y = y * torch.nn.functional.silu(z)
    return y


def selective_scan_fused(x, delta, A, Bm, Cm, h0=None, method="zoh", Dskip=None, z=None, **kw):
    y, last = selective_scan(x, delta, A, Bm, Cm, h0=h0, method=method, **kw)
    return gate(y, x, Dskip, z), last


def state_update(state, x, delta, A, Bm, Cm, Dskip=None, z=None, method="zoh"):
    """One decode step; returns (y (B, D), new state).  x, delta, z: (B, D); Bm, Cm: (B, N)."""
    ct = state.dtype
    a, b = discretize(delta[:, None].to(ct), A.to(ct), Bm[:, None].to(ct), x[:, None].to(ct), method)
    h = a[:, 0] * state + b[:, 0]
    y = torch.einsum("bdn,bn->bd", h, Cm.to(ct))
    y = gate(y.to(x.dtype), x, Dskip, z)
    return y, h


def normwise_error(got, ref):
    """max |got - ref| / max |ref| (elementwise relative error is meaningless near zeros)."""
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    den = ref.abs().max().item()
    return (got - ref).abs().max().item() / (den if den > 0 else 1.0)


def causal_conv1d(x, weight, bias=None, silu=True, conv_state=None):
    """The mixer's causal depthwise conv (models/mamba.py:100-107), (B, L, D) in and out.

    weight (D, K) (nn.Conv1d's (D, 1, K) squeezed), bias (D) or None; conv_state (B, D, K-1)
    prefixes the inputs when given (decode), else K-1 zeros do.  Returns (out, new_state) with
    new_state the last K-1 inputs of the padded/prefixed sequence (models/mamba.py:104-105)."""
    Bsz, L, D = x.shape
    K = weight.shape[-1]
    xc = x.transpose(1, 2)
    if conv_state is None:
        xc = torch.nn.functional.pad(xc, (K - 1, 0))
    else:
        xc = torch.cat([conv_state.to(xc.dtype), xc], dim=-1)
    new_state = xc[..., xc.shape[-1] - (K - 1):]
    out = torch.nn.functional.conv1d(xc, weight.reshape(D, 1, K).to(xc.dtype),
                                     None if bias is None else bias.to(xc.dtype), groups=D)
    if silu:
        out = torch.nn.functional.silu(out)
    return out.transpose(1, 2), new_state
