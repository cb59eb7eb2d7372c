"""Failure detection of the sharded scan's exchanges, on CPU ranks over gloo (world size 3).

The failures are made on the host, as the GPU rules of this project require: a rank that leaves
between steps, a rank that arrives late, a rank that never joins a collective.  What is under
test is ``sharding.PeerCheck`` (the liveness check every rank runs through the process group's
store before an exchange) and the bounded process-group timeout around the exchange itself: the
surviving ranks must raise within the stated time instead of hanging, and a late rank must only
delay them.
"""

import datetime
import json
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mamba_ssm_benchmark_b200 import sharding

WORLD = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, port, pg_timeout):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=pg_timeout))


def _report(out_dir, rank, **kw):
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(kw, f)


def _summaries(rank):
    g = torch.Generator().manual_seed(rank)
    return torch.rand(2, 4, 4, generator=g), torch.randn(2, 4, 4, generator=g)


def _worker(rank, port, out_dir, scenario):
    _init(rank, port, pg_timeout=4)
    peers = sharding.PeerCheck.for_group(timeout=1.5)
    t0 = time.monotonic()
    try:
        for step in range(3):
            if scenario == "late" and rank == 2 and step == 1:
                time.sleep(0.7)                       # arrives late, within the check's timeout
            if scenario == "leaves" and rank == 2 and step == 1:
                _report(out_dir, rank, left_at=step)  # stops taking part between steps, nothing in
                time.sleep(3.0)                       # flight; its process ends after the others'
                return                                # check has run out (an exit in the middle can
                                                      # also surface as a reset gloo connection)
            if scenario == "skips_collective" and rank == 2 and step == 1:
                peers.step()                          # passes the check, then never joins the exchange
                time.sleep(8.0)
                _report(out_dir, rank, slept=True)
                return
            peers.step()
            decays, hends = sharding.exchange_summaries(*_summaries(rank))
            assert decays.shape[0] == WORLD
            h_in, _ = sharding.compose_prefix(decays, hends)
        _report(out_dir, rank, ok=True, elapsed=time.monotonic() - t0)
    except sharding.PeerLost as e:
        _report(out_dir, rank, peer_lost=e.missing, step=e.step, elapsed=time.monotonic() - t0)
    except RuntimeError as e:                          # the bounded collective timed out
        _report(out_dir, rank, collective_error=str(e)[:200], elapsed=time.monotonic() - t0)
    finally:
        if not (scenario in ("leaves", "skips_collective") and rank == 2):
            # rank 0's process hosts the store the others may still be polling: every rank waits
            # (bounded) until all have reported, then ends without teardown handshakes
            deadline = time.monotonic() + 15.0
            while time.monotonic() < deadline and not all(
                    os.path.exists(os.path.join(out_dir, f"rank{r}.json")) for r in range(WORLD)):
                time.sleep(0.05)
            os._exit(0)


def _run(scenario, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path), scenario)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        assert not p.is_alive(), "a rank hung"
    out = {}
    for r in range(WORLD):
        path = tmp_path / f"rank{r}.json"
        assert path.exists(), f"rank {r} reported nothing"
        out[r] = json.loads(path.read_text())
    return out


def test_healthy_ranks_pass_every_check(tmp_path):
    out = _run("healthy", tmp_path)
    assert all(out[r].get("ok") for r in range(WORLD))


def test_late_rank_only_delays_the_others(tmp_path):
    out = _run("late", tmp_path)
    assert all(out[r].get("ok") for r in range(WORLD))
    assert min(out[r]["elapsed"] for r in range(WORLD)) >= 0.6


def test_departed_rank_is_named_within_the_timeout(tmp_path):
    """Rank 2 leaves after step 0: ranks 0 and 1 raise PeerLost([2]) at step 1 within the check's
    1.5 s timeout (plus start-up) instead of entering an exchange that would wait for it."""
    out = _run("leaves", tmp_path)
    assert out[2] == {"left_at": 1}
    for r in (0, 1):
        assert out[r].get("peer_lost") == [2] and out[r]["step"] == 1, out[r]
        assert out[r]["elapsed"] < 1.5 + 3.0


def test_collective_without_a_peer_ends_with_an_error(tmp_path):
    """Rank 2 passes the liveness check and then never joins the all-gather: the others' exchange
    fails on the process group's 4 s timeout instead of hanging."""
    out = _run("skips_collective", tmp_path)
    for r in (0, 1):
        assert "collective_error" in out[r], out[r]
        assert out[r]["elapsed"] < 4.0 + 4.0
