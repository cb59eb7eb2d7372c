"""Rank program for tests/test_sharding_gpu.py: run under torchrun with one process per GPU.

Checks, against a single-GPU computation of the whole problem on every rank:
* sequence shards: ``sequence_sharded_scan`` over NCCL gives this rank's slice of y and the
  final state of the whole sequence;
* channel shards: each rank's backward over its channel range, then ``reduce_shared_grads``,
  gives the full-width dBm, dCm.
Exit status 0 on success.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from mamba_ssm_benchmark_b200 import selective_scan_fused, sharding  # noqa: E402
from mamba_ssm_benchmark_b200.workloads import make_inputs  # noqa: E402


def err(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


def main():
    rank, world, local = (int(os.environ[k]) for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = True
    try:
        # sequence shards
        B, L, D, N = 2, 4096, 128, 16
        ins = make_inputs(B, L, D, N, seed=21, dist="config", h0=True, device=dev)
        u, dl, A, Bm, Cm, Dk, z, h0 = (ins[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "h0"))
        y_full, last_full = selective_scan_fused(u, dl, A, Bm, Cm, h0=h0, D=Dk, z=z)
        lo, hi = sharding.shard_range(L, world, rank)          # contiguous split of the sequence
        y, last = sharding.sequence_sharded_scan(u[:, lo:hi], dl[:, lo:hi], A, Bm[:, lo:hi], Cm[:, lo:hi],
                                                 h0=h0, D=Dk, z=z[:, lo:hi])
        e_y, e_l = err(y, y_full[:, lo:hi]), err(last, last_full)
        print(f"rank {rank}: sequence shard [{lo},{hi}) y err {e_y:.2e} last err {e_l:.2e}", flush=True)
        ok &= e_y < 1e-5 and e_l < 1e-5

        # sequence shards, backward: shard gradients and the replicated dA, dD, dh0
        keys = ("u", "delta", "A", "Bm", "Cm", "Dskip", "z", "h0")
        full = {k: ins[k].clone().requires_grad_() for k in keys}
        yf, lf = selective_scan_fused(full["u"], full["delta"], full["A"], full["Bm"], full["Cm"], h0=full["h0"],
                                      D=full["Dskip"], z=full["z"])
        dy = torch.randn(yf.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(5))
        gf = dict(zip(keys, torch.autograd.grad(yf, [full[k] for k in keys], dy)))
        sh = {k: (ins[k][:, lo:hi] if k in ("u", "delta", "Bm", "Cm", "z") else ins[k]).clone().requires_grad_()
              for k in keys}
        ys, _ = sharding.sequence_sharded_scan(sh["u"], sh["delta"], sh["A"], sh["Bm"], sh["Cm"], h0=sh["h0"],
                                               D=sh["Dskip"], z=sh["z"])
        gs = dict(zip(keys, torch.autograd.grad(ys, [sh[k] for k in keys], dy[:, lo:hi])))
        for k in keys:
            want = gf[k][:, lo:hi] if k in ("u", "delta", "Bm", "Cm", "z") else gf[k]
            e = err(gs[k], want)
            ok &= e < 1e-4
            print(f"rank {rank}: sequence shard grad {k} err {e:.2e}", flush=True)

        # channel shards
        B, L, D, N = 4, 512, 256, 16
        ins = make_inputs(B, L, D, N, seed=22, dist="config", device=dev)
        keys = ("u", "delta", "A", "Bm", "Cm", "Dskip", "z")
        lo, hi = sharding.shard_range(D, world, rank)

        def grads(lo, hi):
            lv = {k: ins[k].clone() for k in keys}
            for k in ("u", "delta", "z"):
                lv[k] = lv[k][:, :, lo:hi]
            lv["A"], lv["Dskip"] = lv["A"][lo:hi], lv["Dskip"][lo:hi]
            lv = {k: v.requires_grad_() for k, v in lv.items()}
            y, _ = selective_scan_fused(lv["u"], lv["delta"], lv["A"], lv["Bm"], lv["Cm"], D=lv["Dskip"], z=lv["z"])
            return torch.autograd.grad(y, (lv["Bm"], lv["Cm"]), ins["dy"][:, :, lo:hi])

        full_b, full_c = grads(0, D)
        gb, gc = grads(lo, hi)
        sharding.reduce_shared_grads([gb, gc])
        e_b, e_c = err(gb, full_b), err(gc, full_c)
        print(f"rank {rank}: channel shard [{lo},{hi}) dB err {e_b:.2e} dC err {e_c:.2e}", flush=True)
        ok &= e_b < 1e-5 and e_c < 1e-5
        torch.cuda.synchronize()
        flag = torch.tensor([0 if ok else 1], device=dev)
        dist.all_reduce(flag)
        ok = flag.item() == 0
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
