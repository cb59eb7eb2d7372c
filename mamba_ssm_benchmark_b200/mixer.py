"""A Mamba (S6) mixer and a byte-level Mamba LM whose scan path runs on the sm_100a kernels.

What has to match the reference is the parameter table: the names and shapes of
models/mamba.py:Mamba and of models/lm.py:LM built with layers "M" * n (embed, blocks.i.norm1,
blocks.i.mixer.{in_proj, conv, x_proj, dt_proj | dt_bias, B, C, A_log, D, out_proj}, norm_f, a head
tied to the embedding), so that state dicts load in either direction, and the computation those
parameters define (in_proj d -> 2 d_inner, causal depthwise conv k = 4 + SiLU,
x_proj -> dt_rank + 2N, dt_proj with softplus, the selective scan with D skip and SiLU(z) gate,
out_proj; pre-norm residual blocks with RMSNorm; tied embedding).  ``MIXER_PARAMS`` /
``mixer_param_shapes`` state that table; everything else here is this package's own code.

Per call the mixer runs one of three paths:
  * a sequence without state (training): ``causal_conv1d`` reading the x half of in_proj's output
    in place, then one ``selective_scan_fused`` that also applies softplus(dt_proj(dt)) (the
    projection goes in without its bias, the bias and softplus happen inside the scan kernels);
  * a sequence with a decode state (prefill): the same, with the conv state prepended and updated
    and the final SSM state written back;
  * one token with a state (decode): ``causal_conv1d`` on the conv state plus
    ``selective_state_update``, both updating the state in place.
The projections stay torch GEMMs.  ``GraphDecoder`` replays one decode step of a ``MambaLM`` as a
CUDA graph.
"""

import math
from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.nn as nn
import torch.nn.functional as F

from .conv import causal_conv1d
from .decode import selective_state_update
from .scan import selective_scan_fused


# ------------------------------------------------------------------------------------------------
# the parameter table (shared with the reference)
# ------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class MixerDims:
    d_model: int
    d_inner: int
    d_state: int
    d_conv: int
    dt_rank: int

    @classmethod
    def of(cls, d_model, d_state=16, expand=2, d_conv=4, dt_rank=None):
        return cls(d_model, expand * d_model, d_state, d_conv, dt_rank or -(-d_model // 16))


def mixer_param_shapes(dims, selective=True, a_mode="s4d"):
    """Parameter name -> shape of one mixer (the reference's names)."""
    di, n = dims.d_inner, dims.d_state
    shapes = {"in_proj.weight": (2 * di, dims.d_model),
              "conv.weight": (di, 1, dims.d_conv), "conv.bias": (di,)}
    if selective:
        shapes.update({"x_proj.weight": (dims.dt_rank + 2 * n, di),
                       "dt_proj.weight": (di, dims.dt_rank), "dt_proj.bias": (di,)})
    else:
        shapes.update({"dt_bias": (di,), "B": (n,), "C": (n,)})
    shapes.update({"A_log": (di, n if a_mode == "s4d" else 1), "D": (di,), "out_proj.weight": (dims.d_model, di)})
    return shapes


MIXER_PARAMS = tuple(mixer_param_shapes(MixerDims.of(256)))


class _Holder(nn.Module):
    """A bare container for a weight (and bias): the mixer applies its projections functionally."""

    def __init__(self, weight_shape, bias_shape=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(weight_shape))
        self.bias = nn.Parameter(torch.empty(bias_shape)) if bias_shape is not None else None


def _softplus_inverse(y):
    """x with softplus(x) = y, for y > 0: log(e^y - 1)."""
    return torch.log(torch.expm1(y))


# ------------------------------------------------------------------------------------------------
# the mixer
# ------------------------------------------------------------------------------------------------
class MambaMixer(nn.Module):
    """Selective-SSM mixer, constructor arguments as models/mamba.py:Mamba (scan, d_block and
    chunk_size are accepted and ignored: the fused kernels tile themselves)."""

    def __init__(self, d_model, d_state=16, expand=2, d_conv=4, dt_rank=None, selective=True,
                 discretization="zoh", scan="auto", d_block=None, chunk_size=None,
                 dt_min=1e-3, dt_max=0.1, a_mode="s4d"):
        super().__init__()
        del scan, d_block, chunk_size
        if a_mode not in ("s4d", "scalar"):
            raise ValueError(f"a_mode must be 's4d' or 'scalar', got {a_mode!r}")
        self.dims = dims = MixerDims.of(d_model, d_state, expand, d_conv, dt_rank)
        self.d_inner, self.d_state, self.d_conv, self.dt_rank = dims.d_inner, d_state, d_conv, dims.dt_rank
        self.selective, self.discretization, self.a_mode = selective, discretization, a_mode
        shapes = mixer_param_shapes(dims, selective, a_mode)
        for mod in ("in_proj", "conv", "x_proj", "dt_proj", "out_proj"):
            if mod + ".weight" in shapes:
                setattr(self, mod, _Holder(shapes[mod + ".weight"], shapes.get(mod + ".bias")))
        for name in ("dt_bias", "B", "C", "A_log", "D"):
            if name in shapes:
                self.register_parameter(name, nn.Parameter(torch.empty(shapes[name])))
        self.reset_parameters(dt_min, dt_max)

    @torch.no_grad()
    def reset_parameters(self, dt_min=1e-3, dt_max=0.1):
        """S4D-real decays A_n = -(n+1) (a_mode "scalar": one decay per channel in [1, 16]); step sizes
        log-uniform in [dt_min, dt_max] through softplus; D = 1; conv and projections uniform in
        +-1/sqrt(fan_in) (dt_proj: +-dt_rank^-1/2); B, C of the non-selective variant ~ N(0, 1/N)."""
        d = self.dims
        for holder in (self.in_proj, self.conv, self.out_proj) + ((self.x_proj,) if self.selective else ()):
            bound = 1.0 / math.sqrt(holder.weight[0].numel())
            holder.weight.uniform_(-bound, bound)
            if holder.bias is not None:
                holder.bias.uniform_(-bound, bound)
        log_lo, log_hi = math.log(dt_min), math.log(dt_max)
        dt = torch.empty(d.d_inner).uniform_(log_lo, log_hi).exp_().clamp_(min=1e-4)
        if self.selective:
            self.dt_proj.weight.uniform_(-d.dt_rank ** -0.5, d.dt_rank ** -0.5)
            self.dt_proj.bias.copy_(_softplus_inverse(dt))
        else:
            self.dt_bias.copy_(_softplus_inverse(dt))
            self.B.normal_(0.0, d.d_state ** -0.5)
            self.C.normal_(0.0, d.d_state ** -0.5)
        if self.a_mode == "s4d":
            self.A_log.copy_(torch.log(torch.arange(1.0, d.d_state + 1.0)).expand_as(self.A_log))
        else:
            self.A_log.uniform_(1.0, 16.0).log_()
        self.D.fill_(1.0)

    # -- pieces ---------------------------------------------------------------------------------
    def decay(self, dtype):
        """A = -exp(A_log) in the compute dtype, (d_inner, N)."""
        A = -torch.exp(self.A_log.to(torch.promote_types(dtype, torch.float32)))
        return A.expand(-1, self.d_state) if self.a_mode == "scalar" else A

    def _selective_inputs(self, x):
        """dt @ dt_proj.weight^T (before bias and softplus), Bm, Cm from x."""
        dt, Bm, Cm = F.linear(x, self.x_proj.weight).split([self.dt_rank, self.d_state, self.d_state], dim=-1)
        return F.linear(dt, self.dt_proj.weight), Bm, Cm

    def _constant_inputs(self, x):
        """Non-selective variant: delta, Bm, Cm broadcast over (batch, time)."""
        Bsz, L, _ = x.shape
        delta = F.softplus(self.dt_bias).expand(Bsz, L, -1)
        return delta, self.B.expand(Bsz, L, -1), self.C.expand(Bsz, L, -1)

    def init_state(self, batch, max_len, device, dtype=torch.float32):
        """Decode state: the last d_conv - 1 conv inputs and the (d_inner, N) SSM state; its size
        does not depend on max_len."""
        del max_len
        return SimpleNamespace(conv=torch.zeros(batch, self.d_inner, self.d_conv - 1, device=device, dtype=dtype),
                               ssm=torch.zeros(batch, self.d_inner, self.d_state, device=device,
                                               dtype=torch.promote_types(dtype, torch.float32)))

    @staticmethod
    def state_nbytes(state):
        return sum(t.numel() * t.element_size() for t in (state.conv, state.ssm))

    # -- forward --------------------------------------------------------------------------------
    def forward(self, u, state=None, pos=0, return_delta=False):
        del pos
        xz = F.linear(u, self.in_proj.weight)
        x, z = xz[..., :self.d_inner], xz[..., self.d_inner:]
        if state is not None and u.shape[1] == 1:
            y, delta = self._decode_step(x, z, state)
        else:
            y, delta = self._sequence(x, z, state, return_delta)
        out = F.linear(y, self.out_proj.weight)
        return (out, delta) if return_delta else out

    def _sequence(self, x, z, state, want_delta):
        conv_state = None if state is None else state.conv
        if conv_state is not None:
            x = x.to(conv_state.dtype)
        x = causal_conv1d(x, self.conv.weight, self.conv.bias, conv_state=conv_state,
                          update_state=conv_state is not None)
        A = self.decay(x.dtype)
        h0 = None if state is None else state.ssm
        delta = None
        if self.selective:
            dt_raw, Bm, Cm = self._selective_inputs(x)
            y, last = selective_scan_fused(x, dt_raw, A, Bm, Cm, h0=h0, method=self.discretization, D=self.D, z=z,
                                           delta_bias=self.dt_proj.bias, delta_softplus=True)
            if want_delta:
                delta = F.softplus(dt_raw.float() + self.dt_proj.bias)
        else:
            delta, Bm, Cm = self._constant_inputs(x)
            y, last = selective_scan_fused(x, delta, A, Bm, Cm, h0=h0, method=self.discretization, D=self.D, z=z)
        if state is not None:
            state.ssm.copy_(last)
        return y, delta

    def _decode_step(self, x, z, state):
        x = causal_conv1d(x.to(state.conv.dtype), self.conv.weight, self.conv.bias, conv_state=state.conv,
                          update_state=True)
        if self.selective:
            dt_raw, Bm, Cm = self._selective_inputs(x)
            delta = F.softplus(dt_raw.to(torch.promote_types(x.dtype, torch.float32)) + self.dt_proj.bias)
        else:
            delta, Bm, Cm = self._constant_inputs(x)
        y = selective_state_update(state.ssm, x[:, 0], delta[:, 0], self.decay(x.dtype), Bm[:, 0], Cm[:, 0], D=self.D,
                                   method=self.discretization, z=z[:, 0])
        return y.unsqueeze(1), delta


class RMSNorm(nn.Module):
    """Root-mean-square normalisation in float32, then a learned per-feature scale."""

    def __init__(self, d, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        return F.rms_norm(x.float(), (x.shape[-1],), eps=self.eps).to(x.dtype) * self.weight


class MambaBlock(nn.Module):
    """x + mixer(norm1(x)): a pre-norm residual block with a Mamba mixer and no MLP."""

    def __init__(self, d_model, **mixer_kw):
        super().__init__()
        self.kind = "M"
        self.norm1 = RMSNorm(d_model)
        self.mixer = MambaMixer(d_model, **mixer_kw)
        self.mlp = None

    def forward(self, x, state=None, pos=0):
        return x + self.mixer(self.norm1(x), state, pos)


# ------------------------------------------------------------------------------------------------
# the LM
# ------------------------------------------------------------------------------------------------
def _sample(logits, temperature, top_k):
    """One token per row from the last position's logits (temperature, optional top-k)."""
    scores = logits.float() / max(temperature, 1e-6)
    if top_k:
        kth = torch.topk(scores, top_k, dim=-1).values[..., -1:]
        scores = torch.where(scores < kth, torch.full_like(scores, float("-inf")), scores)
    return torch.multinomial(torch.softmax(scores, dim=-1), 1)


class MambaLM(nn.Module):
    """Byte-level LM: embedding, n_layers Mamba blocks, final RMSNorm, head tied to the embedding
    (the reference's "mamba" preset is 11 blocks at d_model 256)."""

    def __init__(self, n_layers=11, vocab_size=256, d_model=256, d_state=16, expand=2, d_conv=4,
                 discretization="zoh", selective=True, a_mode="s4d"):
        super().__init__()
        self.n_layers = n_layers
        self.embed = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList(MambaBlock(d_model, d_state=d_state, expand=expand, d_conv=d_conv,
                                               discretization=discretization, selective=selective, a_mode=a_mode)
                                    for _ in range(n_layers))
        self.norm_f = RMSNorm(d_model)
        self.head = nn.Linear(d_model, vocab_size, bias=False)
        self.head.weight = self.embed.weight
        self._init_projections()

    @torch.no_grad()
    def _init_projections(self):
        """GPT-2-style projections: N(0, 0.02) for the embedding and the input-side projections,
        N(0, 0.02 / sqrt(2 n_layers)) for the projections that write into the residual stream;
        the mixers keep their own dt_proj, conv, A and D initialisation."""
        self.embed.weight.normal_(0.0, 0.02)
        residual_std = 0.02 / math.sqrt(2 * self.n_layers)
        for block in self.blocks:
            m = block.mixer
            m.in_proj.weight.normal_(0.0, 0.02)
            if m.selective:
                m.x_proj.weight.normal_(0.0, 0.02)
            m.out_proj.weight.normal_(0.0, residual_std)

    def num_params(self, non_embedding=True):
        total = sum(p.numel() for p in self.parameters())
        return total - (self.embed.weight.numel() if non_embedding else 0)

    def init_state(self, batch, max_len, device, dtype=torch.float32):
        return [block.mixer.init_state(batch, max_len, device, dtype) for block in self.blocks]

    def forward(self, idx, states=None, pos=0):
        x = self.embed(idx)
        for i, block in enumerate(self.blocks):
            x = block(x, states[i] if states is not None else None, pos)
        return self.head(self.norm_f(x))

    @torch.no_grad()
    def generate(self, prompt, n_new, temperature=1.0, top_k=None, max_len=None, graph=False):
        """Samples n_new tokens after ``prompt`` (B, T): one prefill pass with decode states, then one
        decode step per token (a CUDA-graph replay each with ``graph=True``)."""
        Bsz, T = prompt.shape
        states = self.init_state(Bsz, max_len or T + n_new, prompt.device)
        logits = self(prompt, states, 0)
        if graph:
            replay = GraphDecoder(self, states)
            advance = lambda tok, pos: replay(tok)
        else:
            advance = lambda tok, pos: self(tok, states, pos)
        tokens = [prompt]
        for i in range(n_new):
            nxt = _sample(logits[:, -1], temperature, top_k)
            tokens.append(nxt)
            if i + 1 < n_new:
                logits = advance(nxt, T + i)
        return torch.cat(tokens, dim=1)


class GraphDecoder:
    """One decode step of a MambaLM (embedding, every block's conv-state and SSM-state update, head)
    captured once as a CUDA graph over static token / logits buffers; ``__call__(tok)`` copies the
    token in, replays, and returns the logits buffer (valid until the next call).  The states are
    updated in place exactly as the eager step does."""

    def __init__(self, model, states, warmup=2):
        self.model, self.states = model, states
        B = states[0].ssm.shape[0]
        dev = states[0].ssm.device
        self.tok = torch.zeros(B, 1, dtype=torch.long, device=dev)
        saved = [(s.conv.clone(), s.ssm.clone()) for s in states]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):
                model(self.tok, states, 0)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.logits = model(self.tok, states, 0)
        for s, (c, h) in zip(states, saved):          # warm-up and capture must not advance the state
            s.conv.copy_(c)
            s.ssm.copy_(h)

    def __call__(self, tok):
        self.tok.copy_(tok)
        self.graph.replay()
        return self.logits
