"""The Mamba mixer / LM built on the sm_100a ops against the reference's own LM (models/lm.py with
layers "MM"), recorded in tests/golden/lm_small.npz by tests/golden/make_golden.py."""

import pytest
import torch

from conftest import load_golden
from mamba_ssm_benchmark_b200 import _native as nat
from mamba_ssm_benchmark_b200.mixer import GraphDecoder, MambaLM
from mamba_ssm_benchmark_b200.workloads import markov_bytes
from oracle import scan_oracle as O

DEV = "cuda"


def _golden_model(device):
    gold = load_golden("lm_small.npz")
    model = MambaLM(n_layers=2, d_model=32, d_state=16, expand=2, d_conv=4)
    model.load_state_dict({k[2:]: v for k, v in gold.items() if k.startswith("p.")}, strict=True)
    return model.to(device), gold


def test_parameters_match_reference_layout():
    """Same parameter names and shapes as the reference LM (state dicts load either way)."""
    model, gold = _golden_model("cpu")
    ref = {k[2:]: tuple(v.shape) for k, v in gold.items() if k.startswith("p.")}
    assert {k: tuple(v.shape) for k, v in model.state_dict().items()} == ref
    fresh = MambaLM(n_layers=2, d_model=32)
    assert {k: tuple(v.shape) for k, v in fresh.state_dict().items()} == ref


def test_markov_bytes_is_seeded():
    a, b = markov_bytes(4, 64, seed=3), markov_bytes(4, 64, seed=3)
    assert torch.equal(a, b) and a.dtype == torch.long and int(a.min()) >= 0 and int(a.max()) < 256
    assert not torch.equal(a, markov_bytes(4, 64, seed=4))


@pytest.mark.gpu
def test_logits_loss_and_gradients_match_reference():
    model, gold = _golden_model(DEV)
    idx = gold["idx"].to(DEV)
    logits = model(idx)
    assert O.normwise_error(logits.detach().cpu(), gold["logits"]) < 1e-4
    loss = torch.nn.functional.cross_entropy(logits.view(-1, 256), idx.view(-1))
    assert abs(loss.item() - gold["loss"].item()) < 1e-4 * abs(gold["loss"].item())
    names = [n for n, _ in model.named_parameters()]
    grads = torch.autograd.grad(loss, [p for _, p in model.named_parameters()])
    for n, g in zip(names, grads):
        assert O.normwise_error(g.cpu(), gold["g." + n]) < 1e-3, n
    assert nat.read_device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("graph", [False, True])
def test_decode_steps_match_reference(graph):
    """Prefill 16 tokens with states, then 4 single-token steps (eager or CUDA-graph replays)."""
    model, gold = _golden_model(DEV)
    idx = gold["idx"].to(DEV)
    with torch.no_grad():
        states = model.init_state(2, 40, DEV)
        pre = model(idx[:, :16], states, 0)
        assert O.normwise_error(pre.cpu(), gold["prefill_logits"]) < 1e-4
        step = GraphDecoder(model, states) if graph else None
        for i in range(4):
            tok = idx[:, 16 + i:17 + i]
            out = step(tok) if graph else model(tok, states, 16 + i)
            assert O.normwise_error(out.cpu(), gold[f"step{i}_logits"]) < 1e-4, i
    assert nat.read_device_error() == 0


@pytest.mark.gpu
def test_generate_with_graph_equals_eager():
    model, _ = _golden_model(DEV)
    prompt = torch.randint(0, 256, (3, 8), device=DEV, generator=torch.Generator(device=DEV).manual_seed(0))
    torch.manual_seed(5)
    a = model.generate(prompt, 12, top_k=1)
    torch.manual_seed(5)
    b = model.generate(prompt, 12, top_k=1, graph=True)
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_training_step_decreases_loss():
    """Config-4 style step (AdamW) on Markov bytes: runs on the sm_100a ops and learns."""
    torch.manual_seed(0)
    model = MambaLM(n_layers=2, d_model=64).to(DEV)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    data = markov_bytes(8, 129, seed=1).to(DEV)
    losses = []
    for _ in range(30):
        logits = model(data[:, :-1])
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 256), data[:, 1:].reshape(-1))
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(loss.item())
    assert losses[-1] < losses[0] - 0.5
