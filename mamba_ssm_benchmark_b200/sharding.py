"""Multi-GPU sharding of the selective scan: channel shards and sequence shards.

One process per GPU, ``torch.distributed`` for the exchanges (NCCL on GPUs; the exchange and
composition functions are device-agnostic, so the same code runs on CPU ranks under gloo).

Channel shards (batch-parallel layers, configs 1 and 3).  Channels are independent in the
scan, so every rank runs the forward and backward of its own contiguous channel range with no
communication.  Bm and Cm are shared by all channels: each rank's dBm/dCm is a partial sum over
its channels, and ``reduce_shared_grads`` all-reduces them (one collective over one flat buffer).
dA, dD stay local to the rank that owns the channels.

Sequence shards (long context, config 2).  The recurrence h_t = a_t h_{t-1} + b_t is linear, so a
contiguous shard r of the sequence is summarised by (decay_r, hend_r): the product of its a_t and
its final state when started from zero (``SequenceShard.summary``, ``ssm_scan_fwd_summary``).  The summaries are all-gathered
(2 * B*D*N floats per rank), every rank composes the prefix of the shards before it to get its
carried-in state h_in_r (``compose_prefix``), and finishes its shard from h_in_r
(``SequenceShard.finish``, ``ssm_scan_fwd_finish``).  This is the reference's two-level chunked scan (models/scan.py:142-165:
per-chunk scans, a combine over chunk ends, a fix-up) with one chunk per GPU; the all-gather
replaces a rank-to-rank chain, so no rank waits on its predecessors' finish passes.

The backward of a sequence shard needs the adjoint entering it from the right, which is affine in
the next shard's: every rank computes its adjoint summary (``ssm_scan_bwd_summary``: the gradient
w.r.t. its initial state from a zero adjoint at its end, and its decay product), the summaries are
all-gathered and composed from the last shard to the first (``compose_suffix``), and every rank runs
the full backward of its shard with its incoming adjoint (the reverse adjoint of
models/scan.py:239-240, carried across shards).
"""

import time

import torch
import torch.distributed as dist

from . import _native as nat
from .scan import CHUNK, _act, _prepare, scan_backward


# ------------------------------------------------------------------------------------------------
# partitions and channel shards
# ------------------------------------------------------------------------------------------------
def shard_range(extent, world, rank):
    """[lo, hi) of the piece of an axis of length ``extent`` (channels, or sequence positions) that
    rank ``rank`` owns when it is split over ``world`` ranks: contiguous, sizes differing by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    base, extra = divmod(extent, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def reduce_shared_grads(grads, group=None):
    """Sum the partial gradients of inputs shared by all channel shards (dBm, dCm) over the ranks,
    in place.  All tensors go through one all-reduce: if they are views of one contiguous buffer
    (dBm | dCm stored side by side) that buffer is reduced directly, else they are packed."""
    grads = [g for g in grads if g is not None]
    if not grads or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return grads
    base = grads[0]._base if grads[0]._base is not None else grads[0]
    shared = (base.is_contiguous() and all(g._base is base or g is base for g in grads)
              and sum(g.numel() for g in grads) == base.numel())
    if shared:
        dist.all_reduce(base, group=group)
        return grads
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    off = 0
    for g in grads:
        g.copy_(flat[off:off + g.numel()].view_as(g))
        off += g.numel()
    return grads


# ------------------------------------------------------------------------------------------------
# sequence shards: exchange and composition (host logic, any device)
# ------------------------------------------------------------------------------------------------
def exchange_summaries(decay, hend, group=None):
    """All-gather every rank's (decay, hend) summary: returns (decays, hends), each (W, B, D, N),
    indexed by rank (= shard position along the sequence).  One collective into one (W, 2, B, D, N)
    buffer; the two results are views of it (``compose_prefix`` reads them in place).  A summary
    that is already the (2, B, D, N) pack (``SequenceShard.summary``) is sent without a copy."""
    base = decay._base
    if (base is not None and base is hend._base and base.dim() == decay.dim() + 1 and base.shape[0] == 2
            and base.dtype == torch.float32 and base.is_contiguous()
            and decay.data_ptr() == base.data_ptr() and hend.data_ptr() == base[1].data_ptr()):
        pack = base
    else:
        pack = torch.stack((decay.to(torch.float32), hend.to(torch.float32))).contiguous()
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return pack[0:1], pack[1:2]
    world = dist.get_world_size(group)
    allp = torch.empty((world,) + tuple(pack.shape), dtype=pack.dtype, device=pack.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(allp, pack, group=group)
    else:                                   # gloo (CPU ranks): the list form
        dist.all_gather(list(allp.unbind(0)), pack, group=group)
    return allp[:, 0], allp[:, 1]


def _compose_on_device(decays, ends, start, reverse):
    """One ssm_compose_shards launch over CUDA-resident summaries."""
    W, B, D, N = decays.shape
    blocks_ok = lambda t: t.dtype == torch.float32 and t[0].is_contiguous() and t.stride(0) == decays.stride(0)
    if not (blocks_ok(decays) and blocks_ok(ends) and decays.stride(0) >= B * D * N):
        decays = decays.to(torch.float32).contiguous()
        ends = ends.to(torch.float32).contiguous()
    stride = decays.stride(0) if W > 1 else B * D * N
    start = None if start is None else start.to(torch.float32).contiguous()
    out = torch.empty((W, B, D, N), dtype=torch.float32, device=decays.device)
    last = torch.empty((B, D, N), dtype=torch.float32, device=decays.device)
    with torch.cuda.device(decays.device):
        rc = nat.lib().ssm_compose_shards(W, B, D, N, nat.ptr(decays), nat.ptr(ends), stride, nat.ptr(start),
                                          int(reverse), nat.ptr(out), nat.ptr(last), nat.stream_of(decays.device))
    nat.check(rc, "ssm_compose_shards")
    return out, last


def compose_prefix(decays, hends, h0=None):
    """Carried-in state of every shard and the final state of the whole sequence.

    decays, hends: (W, B, D, N) summaries of shards 0..W-1 in sequence order; h0: (B, D, N) or None.
    h_in[0] = h0, h_in[r] = decays[r-1] * h_in[r-1] + hends[r-1]; last = the same step past shard W-1.
    (The combine of chunk ends in models/scan.py:160-164, written as a left-to-right walk because W
    is at most the number of GPUs.)  CUDA tensors: one ssm_compose_shards launch; CPU tensors (the
    host-side protocol on gloo ranks): the same walk in torch."""
    if decays.is_cuda:
        return _compose_on_device(decays, hends, h0, False)
    W = decays.shape[0]
    h = torch.zeros_like(hends[0]) if h0 is None else h0.to(torch.float32)
    h_in = torch.empty_like(hends)
    for r in range(W):
        h_in[r] = h
        h = torch.addcmul(hends[r], decays[r], h)
    return h_in, h


# ------------------------------------------------------------------------------------------------
# sequence shards: the two kernel phases (CUDA)
# ------------------------------------------------------------------------------------------------
class SequenceShard:
    """The kernel phases over one contiguous shard of a sequence.

    ``summary()`` scans the shard from a zero state (``ssm_scan_fwd_summary``) and returns
    (decay, hend), each (B, D, N) float32: the product of the shard's per-step decays and its end
    state from zero.  ``finish(h_in)`` scans it again from the carried-in state
    (``ssm_scan_fwd_finish``) and returns (y, last) like ``selective_scan_fused`` with h0 = h_in;
    with ``save=True`` it also keeps what the backward needs.  Both phases share one workspace,
    through which the kernels pass per-block summaries from the first phase to the second, so they
    must run in this order on the same stream.  ``adjoint_summary(dy)`` (``ssm_scan_bwd_summary``)
    is the backward's first phase: the gradient with respect to the shard's initial state when no
    adjoint enters from the right, and the decay product."""

    def __init__(self, x, delta, A, Bm, Cm, method="zoh", D=None, z=None):
        self.in_dtype = x.dtype
        self.method = method
        (self.x, self.delta, self.A, self.Bm, self.Cm, _, self.D,
         self.z) = _prepare(x, delta, A, Bm, Cm, None, D, z, method)
        Bsz, L, Dch = self.x.shape
        self.shape = (Bsz, L, Dch, self.A.shape[1])
        self.dev = self.x.device
        self.wsb = nat.fwd_workspace_bytes(*self.shape)
        self.ws = torch.empty(max(self.wsb, 1), dtype=torch.uint8, device=self.dev)
        self._summarised = False
        self.chunk_states = self.ygate = self.h_in = None

    def _state(self):
        Bsz, L, Dch, N = self.shape
        return torch.empty((Bsz, Dch, N), dtype=torch.float32, device=self.dev)

    def summary(self):
        Bsz, L, Dch, N = self.shape
        pack = torch.empty((2, Bsz, Dch, N), dtype=torch.float32, device=self.dev)   # what exchange_summaries sends
        decay, hend = pack[0], pack[1]
        with torch.cuda.device(self.dev):
            rc = nat.lib().ssm_scan_fwd_summary(Bsz, L, Dch, N, nat.METHODS[self.method], nat.view3(self.x),
                                                nat.view3(self.delta), nat.ptr(self.A), nat.view3(self.Bm),
                                                nat.ptr(decay), nat.ptr(hend), self.ws.data_ptr(), self.wsb,
                                                nat.stream_of(self.dev))
        nat.check(rc, "ssm_scan_fwd_summary")
        self._summarised = True
        return decay, hend

    def finish(self, h_in, save=False):
        if not self._summarised:
            raise RuntimeError("SequenceShard.finish needs summary() to have run first")
        Bsz, L, Dch, N = self.shape
        h_in = h_in.to(torch.float32).contiguous()
        y = torch.empty((Bsz, L, Dch), dtype=self.x.dtype, device=self.dev)
        last = self._state()
        if save:
            self.h_in = h_in
            self.chunk_states = torch.empty((Bsz, -(-L // CHUNK), Dch, N), dtype=torch.float32, device=self.dev)
            self.ygate = torch.empty_like(y) if self.z is not None else None
        with torch.cuda.device(self.dev):
            rc = nat.lib().ssm_scan_fwd_finish(Bsz, L, Dch, N, nat.METHODS[self.method], nat.view3(self.x),
                                               nat.view3(self.delta), nat.ptr(self.A), nat.view3(self.Bm),
                                               nat.view3(self.Cm), nat.ptr(self.D), nat.view3(self.z),
                                               nat.ptr(h_in), nat.view3(y), nat.view3(self.ygate if save else None),
                                               nat.ptr(last), nat.ptr(self.chunk_states if save else None),
                                               self.ws.data_ptr(), self.wsb, nat.stream_of(self.dev))
        nat.check(rc, "ssm_scan_fwd_finish")
        return y.to(self.in_dtype), last

    def adjoint_summary(self, dy):
        Bsz, L, Dch, N = self.shape
        dy = _act(dy, self.x.dtype)
        decay, dstart = self._state(), self._state()
        with torch.cuda.device(self.dev):
            rc = nat.lib().ssm_scan_bwd_summary(Bsz, L, Dch, N, nat.METHODS[self.method], nat.view3(self.delta),
                                                nat.ptr(self.A), nat.view3(self.Cm), nat.view3(self.z),
                                                nat.view3(dy), nat.ptr(decay), nat.ptr(dstart), self.ws.data_ptr(),
                                                self.wsb, nat.stream_of(self.dev))
        nat.check(rc, "ssm_scan_bwd_summary")
        return decay, dstart

    def backward(self, dy, dlast):
        """ssm_scan_bwd over the shard from its saved forward, with ``dlast`` the adjoint entering
        from the right.  Returns (du, ddelta, dA, dB, dC, dh_in, dD, dz): dh_in is the gradient
        w.r.t. the shard's carried-in state; dA, dD are this shard's part of the sums over time."""
        if self.chunk_states is None:
            raise RuntimeError("SequenceShard.backward needs finish(..., save=True) first")
        return scan_backward(self.x, self.delta, self.A, self.Bm, self.Cm, self.h_in, self.D, self.z,
                             self.chunk_states, self.ygate, dy, dlast, self.method)[:8]


def compose_suffix(decays, dstarts, dlast=None):
    """Adjoint entering every shard from the right, and the gradient w.r.t. the first shard's
    initial state (h0 of the whole sequence).

    decays, dstarts: (W, B, D, N) adjoint summaries of shards 0..W-1 in sequence order;
    dlast: (B, D, N) gradient of the whole sequence's final state, or None.
    dl_in[W-1] = dlast, dl_in[r] = dstarts[r+1] + decays[r+1] * dl_in[r+1];
    dh0 = dstarts[0] + decays[0] * dl_in[0].  CUDA tensors: one ssm_compose_shards launch (reverse)."""
    if decays.is_cuda:
        return _compose_on_device(decays, dstarts, dlast, True)
    W = decays.shape[0]
    g = torch.zeros_like(dstarts[0]) if dlast is None else dlast.to(torch.float32)
    dl_in = torch.empty_like(dstarts)
    for r in range(W - 1, -1, -1):
        dl_in[r] = g
        g = torch.addcmul(dstarts[r], decays[r], g)
    return dl_in, g


# ------------------------------------------------------------------------------------------------
# failure detection between the steps of a sharded scan (host side)
# ------------------------------------------------------------------------------------------------
class PeerLost(RuntimeError):
    """A rank of the group did not reach a step of the sharded scan within the timeout."""

    def __init__(self, step, missing, timeout):
        super().__init__(f"rank(s) {missing} did not reach step {step} of the sharded scan within {timeout:.1f} s")
        self.step, self.missing = step, missing


class PeerCheck:
    """Host-side liveness check before every exchange of a sharded scan.

    Every rank announces step k in the process group's key-value store, then waits until all
    ranks have, for at most ``timeout`` seconds, polling the store (no GPU work and no collective).
    A rank that died, left, or hangs before step k makes the others raise ``PeerLost`` naming it
    before they enter the step's collective; a collective that a peer never joins would otherwise
    block until the process group's own timeout, with the caller's kernels already queued behind
    it.  A late rank (within the timeout) only delays the others.  Steps are numbered by the
    check itself, so every rank must call ``step()`` the same number of times, in the same order,
    as it does the collectives.  Keys of step k - 2 are deleted once step k is reached."""

    def __init__(self, store, rank, world, timeout=10.0, prefix="ssm_peer", poll=0.005):
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.prefix, self.poll = float(timeout), prefix, poll
        self.k = 0

    @classmethod
    def for_group(cls, timeout=10.0, group=None, prefix="ssm_peer"):
        """A check over the default process group's store (``group`` only sets rank and size)."""
        store = dist.distributed_c10d._get_default_store()
        return cls(store, _rank(group), _world(group), timeout, prefix)

    def _key(self, k, r):
        return f"{self.prefix}/{k}/{r}"

    def step(self):
        k = self.k
        self.k += 1
        self.store.set(self._key(k, self.rank), b"1")
        keys = [self._key(k, r) for r in range(self.world)]
        deadline = time.monotonic() + self.timeout
        while not self.store.check(keys):
            if time.monotonic() > deadline:
                missing = [r for r, key in enumerate(keys) if not self.store.check([key])]
                if missing:
                    raise PeerLost(k, missing, self.timeout)
                break
            time.sleep(self.poll)
        if k >= 2:
            self.store.delete_key(self._key(k - 2, self.rank))
        return k


def _rank(group):
    return dist.get_rank(group) if dist.is_initialized() else 0


def _world(group):
    return dist.get_world_size(group) if dist.is_initialized() else 1


class SequenceShardedScanFn(torch.autograd.Function):
    """Autograd over the sequence-sharded scan.  Forward: summary, all-gather, prefix, finish.
    Backward: adjoint summary, all-gather, suffix, full backward of the shard; dA, dD (sums over
    the whole sequence) are all-reduced, and dh0 comes out of the suffix composition on every rank."""

    @staticmethod
    def forward(ctx, x, delta, A, Bm, Cm, h0, D, z, method, group, peers):
        shard = SequenceShard(x, delta, A, Bm, Cm, method, D, z)
        decay, hend = shard.summary()
        if peers is not None:
            peers.step()
        decays, hends = exchange_summaries(decay, hend, group)
        h_in, last = compose_prefix(decays, hends, h0)
        need_bwd = any(ctx.needs_input_grad[:8])
        y, _ = shard.finish(h_in[_rank(group)], save=need_bwd)
        ctx.shard, ctx.group, ctx.has_h0, ctx.peers = (shard if need_bwd else None), group, h0 is not None, peers
        return y, last

    @staticmethod
    def backward(ctx, dy, dlast):
        shard, group = ctx.shard, ctx.group
        world, rank = _world(group), _rank(group)
        # the whole sequence's final state is replicated: its gradient is the sum of every rank's
        dl = torch.zeros(shard.shape[0], shard.shape[2], shard.shape[3], dtype=torch.float32, device=shard.dev)
        if dlast is not None:
            dl.copy_(dlast)
        if ctx.peers is not None:
            ctx.peers.step()
        if world > 1:
            dist.all_reduce(dl, group=group)
        decay, dstart = shard.adjoint_summary(dy)
        decays, dstarts = exchange_summaries(decay, dstart, group)
        dl_in, dh0 = compose_suffix(decays, dstarts, dl)
        du, ddelta, dA, dB, dC, _, dD, dz = shard.backward(dy, dl_in[rank])
        reduce_shared_grads([dA, dD], group)        # each rank holds its shard's share of the time sums
        return du, ddelta, dA, dB, dC, (dh0 if ctx.has_h0 else None), dD, dz, None, None, None


def sequence_sharded_scan(x, delta, A, Bm, Cm, h0=None, method="zoh", D=None, z=None, group=None, peers=None):
    """Selective scan of one sequence split over the ranks of ``group`` (differentiable).

    This rank holds shard ``rank``: x, delta, z: (B, L_shard, D); Bm, Cm: (B, L_shard, N); A, D,
    h0 are replicated.  Returns (y_shard, last) where last is the final state of the WHOLE
    sequence (on every rank).  Gradients: du, ddelta, dz, dBm, dCm for this shard's rows; dA, dD
    and dh0 for the whole sequence, identical on every rank.  ``peers`` (a ``PeerCheck``) makes every
    rank confirm that all others are alive before each exchange, raising ``PeerLost`` otherwise."""
    x2, delta2, A2, Bm2, Cm2, h02, D2, z2 = _prepare(x, delta, A, Bm, Cm, h0, D, z, method)
    y, last = SequenceShardedScanFn.apply(x2, delta2, A2, Bm2, Cm2, h02, D2, z2, method, group, peers)
    return y.to(x.dtype), last


__all__ = ["shard_range", "reduce_shared_grads", "exchange_summaries", "compose_prefix", "compose_suffix",
           "SequenceShard", "SequenceShardedScanFn", "sequence_sharded_scan"]
