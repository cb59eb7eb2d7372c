"""The Mamba mixer and the byte-level Mamba LM of the reference, running their scan path on sm_100a.

``MambaMixer`` is a drop-in for models/mamba.py:Mamba: the same constructor arguments, parameter
names, shapes and initialisation (so state dicts load either way), the same forward contract
(``out = mixer(u, state=None, pos=0)``) and the same decode state.  What changes is the path
around the scan: the causal conv + SiLU is ``causal_conv1d`` (reads the x half of in_proj's
output in place), the scan with the D skip and the SiLU(z) gate is one ``selective_scan_fused``
call that also applies the step size's softplus(dt_proj(dt)) (the projection goes in without its
bias), and a decode step (L = 1 with a state) is ``causal_conv1d`` on the conv state plus
``selective_state_update``, both updating the state in place.  The projections stay torch GEMMs.

``MambaLM`` is models/lm.py:LM restricted to Mamba blocks ("M" * n_layers): embedding, pre-norm
residual blocks, final RMSNorm, tied head, with the reference's parameter names and init.
``GraphDecoder`` replays one decode step of a ``MambaLM`` as a CUDA graph.
"""

import math
from types import SimpleNamespace

import torch
import torch.nn as nn
import torch.nn.functional as F

from .conv import causal_conv1d
from .decode import selective_state_update
from .scan import selective_scan_fused


class MambaMixer(nn.Module):
    """models/mamba.py:Mamba with its conv, scan, gate and decode step on the sm_100a kernels."""

    def __init__(self, d_model, d_state=16, expand=2, d_conv=4, dt_rank=None, selective=True,
                 discretization="zoh", scan="auto", d_block=None, chunk_size=None,
                 dt_min=1e-3, dt_max=0.1, a_mode="s4d"):
        super().__init__()
        del scan, d_block, chunk_size           # the fused kernels tile themselves
        self.d_inner = d_inner = expand * d_model
        self.d_state, self.d_conv = d_state, d_conv
        self.dt_rank = dt_rank or math.ceil(d_model / 16)
        self.selective, self.discretization = selective, discretization
        self.in_proj = nn.Linear(d_model, 2 * d_inner, bias=False)
        self.conv = nn.Conv1d(d_inner, d_inner, d_conv, groups=d_inner, bias=True)
        # dt initialisation of models/mamba.py:39-41: log-uniform in [dt_min, dt_max], stored as
        # the softplus inverse in dt_proj's bias
        dt = torch.exp(torch.rand(d_inner) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
        dt = dt.clamp(min=1e-4)
        inv_softplus_dt = dt + torch.log(-torch.expm1(-dt))
        if selective:
            self.x_proj = nn.Linear(d_inner, self.dt_rank + 2 * d_state, bias=False)
            self.dt_proj = nn.Linear(self.dt_rank, d_inner, bias=True)
            self.dt_proj._no_reinit = True
            std = self.dt_rank ** -0.5
            with torch.no_grad():
                nn.init.uniform_(self.dt_proj.weight, -std, std)
                self.dt_proj.bias.copy_(inv_softplus_dt)
        else:
            self.dt_bias = nn.Parameter(inv_softplus_dt)
            self.B = nn.Parameter(torch.randn(d_state) / math.sqrt(d_state))
            self.C = nn.Parameter(torch.randn(d_state) / math.sqrt(d_state))
        if a_mode not in ("s4d", "scalar"):
            raise ValueError(f"a_mode must be 's4d' or 'scalar', got {a_mode!r}")
        self.a_mode = a_mode
        if a_mode == "s4d":
            A = torch.arange(1, d_state + 1, dtype=torch.float32).repeat(d_inner, 1)
        else:
            A = torch.empty(d_inner, 1).uniform_(1.0, 16.0)
        self.A_log = nn.Parameter(torch.log(A))
        self.D = nn.Parameter(torch.ones(d_inner))
        self.out_proj = nn.Linear(d_inner, d_model, bias=False)
        self.out_proj._residual_out = True

    def ssm_params(self, x):
        """x: (B, L, d_inner) -> delta (B, L, d_inner), A (d_inner, N), Bm, Cm (B, L, N)
        (models/mamba.py:70-84)."""
        Bsz, L, _ = x.shape
        ct = torch.promote_types(x.dtype, torch.float32)
        if self.selective:
            dt, Bm, Cm = self.x_proj(x).split([self.dt_rank, self.d_state, self.d_state], dim=-1)
            delta = F.softplus(self.dt_proj(dt).to(ct))
        else:
            delta = F.softplus(self.dt_bias).expand(Bsz, L, -1)
            Bm = self.B.expand(Bsz, L, -1)
            Cm = self.C.expand(Bsz, L, -1)
        A = -torch.exp(self.A_log.to(ct))
        if self.a_mode == "scalar":
            A = A.expand(-1, self.d_state)
        return delta, A, Bm, Cm

    def init_state(self, batch, max_len, device, dtype=torch.float32):
        """The reference's decode state (models/mamba.py:86-91): conv inputs and SSM state."""
        del max_len
        return SimpleNamespace(
            conv=torch.zeros(batch, self.d_inner, self.d_conv - 1, device=device, dtype=dtype),
            ssm=torch.zeros(batch, self.d_inner, self.d_state, device=device,
                            dtype=torch.promote_types(dtype, torch.float32)))

    @staticmethod
    def state_nbytes(state):
        return state.conv.numel() * state.conv.element_size() + state.ssm.numel() * state.ssm.element_size()

    def forward(self, u, state=None, pos=0, return_delta=False):
        del pos
        Bsz, L, _ = u.shape
        x, z = self.in_proj(u).chunk(2, dim=-1)
        if state is None:
            x = causal_conv1d(x, self.conv.weight, self.conv.bias)
        else:
            x = causal_conv1d(x.to(state.conv.dtype), self.conv.weight, self.conv.bias, conv_state=state.conv,
                              update_state=True)
        h0 = None if state is None else state.ssm
        if L == 1 and state is not None:                                  # recurrent decode step
            delta, A, Bm, Cm = self.ssm_params(x)
            y = selective_state_update(state.ssm, x[:, 0], delta[:, 0], A, Bm[:, 0], Cm[:, 0], D=self.D,
                                       method=self.discretization, z=z[:, 0]).unsqueeze(1)
        elif self.selective:
            # softplus(dt_proj(dt)) happens inside the scan: the projection without its bias goes in
            dt, Bm, Cm = self.x_proj(x).split([self.dt_rank, self.d_state, self.d_state], dim=-1)
            dt_raw = F.linear(dt, self.dt_proj.weight)
            A = -torch.exp(self.A_log.to(torch.promote_types(x.dtype, torch.float32)))
            if self.a_mode == "scalar":
                A = A.expand(-1, self.d_state)
            y, last = selective_scan_fused(x, dt_raw, A, Bm, Cm, h0=h0, method=self.discretization, D=self.D, z=z,
                                           delta_bias=self.dt_proj.bias, delta_softplus=True)
            delta = F.softplus(dt_raw.float() + self.dt_proj.bias) if return_delta else None
        else:
            delta, A, Bm, Cm = self.ssm_params(x)
            y, last = selective_scan_fused(x, delta, A, Bm, Cm, h0=h0, method=self.discretization, D=self.D, z=z)
        if state is not None and not (L == 1):
            state.ssm.copy_(last)
        out = self.out_proj(y)
        return (out, delta) if return_delta else out


class RMSNorm(nn.Module):
    """models/common.py:RMSNorm (normalise in float32, scale by a learned weight)."""

    def __init__(self, d, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight


class MambaBlock(nn.Module):
    """Pre-norm residual Mamba block (models/lm.py:Block with kind "M")."""

    def __init__(self, d_model, **mixer_kw):
        super().__init__()
        self.kind = "M"
        self.norm1 = RMSNorm(d_model)
        self.mixer = MambaMixer(d_model, **mixer_kw)
        self.mlp = None
        self.drop = nn.Dropout(0.0)

    def forward(self, x, state=None, pos=0):
        return x + self.drop(self.mixer(self.norm1(x), state, pos))


class MambaLM(nn.Module):
    """models/lm.py:LM with layers = "M" * n_layers (the reference's "mamba" preset has 11)."""

    def __init__(self, n_layers=11, vocab_size=256, d_model=256, d_state=16, expand=2, d_conv=4,
                 discretization="zoh", selective=True, a_mode="s4d"):
        super().__init__()
        self.n_layers = n_layers
        self.embed = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([MambaBlock(d_model, d_state=d_state, expand=expand, d_conv=d_conv,
                                                discretization=discretization, selective=selective, a_mode=a_mode)
                                     for _ in range(n_layers)])
        self.norm_f = RMSNorm(d_model)
        self.head = nn.Linear(d_model, vocab_size, bias=False)
        self.head.weight = self.embed.weight                        # tied embeddings
        self.apply(self._init)

    def _init(self, m):        # models/lm.py:LM._init
        if isinstance(m, nn.Linear) and not getattr(m, "_no_reinit", False):
            std = 0.02 / math.sqrt(2 * self.n_layers) if getattr(m, "_residual_out", False) else 0.02
            nn.init.normal_(m.weight, 0.0, std)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, 0.0, 0.02)

    def num_params(self, non_embedding=True):
        n = sum(p.numel() for p in self.parameters())
        return n - self.embed.weight.numel() if non_embedding else n

    def init_state(self, batch, max_len, device, dtype=torch.float32):
        return [b.mixer.init_state(batch, max_len, device, dtype) for b in self.blocks]

    def forward(self, idx, states=None, pos=0):
        x = self.embed(idx)
        for i, block in enumerate(self.blocks):
            x = block(x, None if states is None else states[i], pos)
        return self.head(self.norm_f(x))

    @torch.no_grad()
    def generate(self, prompt, n_new, temperature=1.0, top_k=None, max_len=None, graph=False):
        """Autoregressive sampling with the decode states (models/lm.py:130-146).  With
        ``graph=True`` every step after the prefill is one CUDA-graph replay."""
        B, T = prompt.shape
        states = self.init_state(B, max_len or T + n_new, prompt.device)
        logits = self(prompt, states, 0)[:, -1]
        step = GraphDecoder(self, states) if graph else None
        out = [prompt]
        for t in range(n_new):
            logits = logits.float() / max(temperature, 1e-6)
            if top_k:
                v, _ = torch.topk(logits, top_k)
                logits[logits < v[:, [-1]]] = float("-inf")
            nxt = torch.multinomial(F.softmax(logits, -1), 1)
            out.append(nxt)
            if t < n_new - 1:
                logits = (step(nxt) if step is not None else self(nxt, states, T + t))[:, -1]
        return torch.cat(out, 1)


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
