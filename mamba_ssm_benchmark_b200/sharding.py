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
"""

import torch
import torch.distributed as dist

from . import _native as nat
from .scan import _prepare


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
    indexed by rank (= shard position along the sequence)."""
    pack = torch.stack((decay.to(torch.float32), hend.to(torch.float32))).contiguous()
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return pack[0:1], pack[1:2]
    world = dist.get_world_size(group)
    parts = [torch.empty_like(pack) for _ in range(world)]
    dist.all_gather(parts, pack, group=group)
    allp = torch.stack(parts)
    return allp[:, 0], allp[:, 1]


def compose_prefix(decays, hends, h0=None):
    """Carried-in state of every shard and the final state of the whole sequence.

    decays, hends: (W, B, D, N) summaries of shards 0..W-1 in sequence order; h0: (B, D, N) or None.
    h_in[0] = h0, h_in[r] = decays[r-1] * h_in[r-1] + hends[r-1]; last = the same step past shard W-1.
    (The combine of chunk ends in models/scan.py:160-164, written as a left-to-right walk because W
    is at most the number of GPUs.)"""
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
    """The two kernel phases over one contiguous shard of a sequence.

    ``summary()`` scans the shard from a zero state (``ssm_scan_fwd_summary``) and returns
    (decay, hend), each (B, D, N) float32: the product of the shard's per-step decays and its end
    state from zero.  ``finish(h_in)`` scans it again from the carried-in state
    (``ssm_scan_fwd_finish``) and returns (y, last) like ``selective_scan_fused`` with h0 = h_in.
    Both phases share one workspace, through which the kernels pass per-block summaries from the
    first phase to the second, so they must run in this order on the same stream."""

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

    def summary(self):
        Bsz, L, Dch, N = self.shape
        decay = torch.empty((Bsz, Dch, N), dtype=torch.float32, device=self.dev)
        hend = torch.empty((Bsz, Dch, N), dtype=torch.float32, device=self.dev)
        with torch.cuda.device(self.dev):
            rc = nat.lib().ssm_scan_fwd_summary(Bsz, L, Dch, N, nat.METHODS[self.method], nat.view3(self.x),
                                                nat.view3(self.delta), nat.ptr(self.A), nat.view3(self.Bm),
                                                nat.ptr(decay), nat.ptr(hend), self.ws.data_ptr(), self.wsb,
                                                nat.stream_of(self.dev))
        nat.check(rc, "ssm_scan_fwd_summary")
        self._summarised = True
        return decay, hend

    def finish(self, h_in):
        if not self._summarised:
            raise RuntimeError("SequenceShard.finish needs summary() to have run first")
        Bsz, L, Dch, N = self.shape
        h_in = h_in.to(torch.float32).contiguous()
        y = torch.empty((Bsz, L, Dch), dtype=self.x.dtype, device=self.dev)
        last = torch.empty((Bsz, Dch, N), dtype=torch.float32, device=self.dev)
        with torch.cuda.device(self.dev):
            rc = nat.lib().ssm_scan_fwd_finish(Bsz, L, Dch, N, nat.METHODS[self.method], nat.view3(self.x),
                                               nat.view3(self.delta), nat.ptr(self.A), nat.view3(self.Bm),
                                               nat.view3(self.Cm), nat.ptr(self.D), nat.view3(self.z),
                                               nat.ptr(h_in), nat.view3(y), nat.NULL_VIEW, nat.ptr(last), None,
                                               self.ws.data_ptr(), self.wsb, nat.stream_of(self.dev))
        nat.check(rc, "ssm_scan_fwd_finish")
        return y.to(self.in_dtype), last


def sequence_sharded_scan(x, delta, A, Bm, Cm, h0=None, method="zoh", D=None, z=None, group=None):
    """Forward of one sequence split over the ranks of ``group``: this rank holds shard ``rank``
    (x, delta, z: (B, L_shard, D); Bm, Cm: (B, L_shard, N)); A, D, h0 are replicated.
    Returns (y_shard, last) where last is the final state of the WHOLE sequence (on every rank)."""
    shard = SequenceShard(x, delta, A, Bm, Cm, method, D, z)
    decay, hend = shard.summary()
    decays, hends = exchange_summaries(decay, hend, group)
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    h_in, last = compose_prefix(decays, hends, h0)
    y, _ = shard.finish(h_in[rank])
    return y, last


__all__ = ["shard_range", "reduce_shared_grads", "exchange_summaries", "compose_prefix", "SequenceShard",
           "sequence_sharded_scan"]
