"""Run a seeded case with FSDP2-style DTensor Shard(0) parameters on every rank.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P tests/sharded_worker.py --case NAME --out FILE.npz

Rank 0 writes the full (gathered) parameters and optimizer state after step 1
and after the last step, in the layout of the GPU parity tests.
"""
import argparse
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

import cases as C  # noqa: E402


def full(t):
    from torch.distributed.tensor import DTensor
    t = t.full_tensor() if isinstance(t, DTensor) else t
    return t.detach().float().cpu().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--pipeline-exchange", action="store_true")
    ap.add_argument("--exchange", default="rounds", choices=["rounds", "all_to_all", "peer"])
    ap.add_argument("--replicas", type=int, default=0,
                    help="HSDP: a (replicas, world / replicas) mesh with (Replicate(), Shard(0)) placements")
    args = ap.parse_args()
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local_rank))
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor

    from thorn_b200 import THORN

    world = dist.get_world_size()
    if args.replicas:
        # every replica row holds the whole parameter set, sharded over its ranks; the
        # gradients that reach the optimizer are the same on every replica (FSDP has
        # reduced them across replicas)
        mesh = init_device_mesh("cuda", (args.replicas, world // args.replicas),
                                mesh_dim_names=("replicate", "shard"))
        place = [Replicate(), Shard(0)]
    else:
        mesh = init_device_mesh("cuda", (world,))
        place = [Shard(0)]
    case = C.CASES[args.case]
    params = C.build_params(case)
    tp = [[torch.nn.Parameter(distribute_tensor(t.cuda(), mesh, place)) for t in ps] for ps in params]
    opt = THORN(C.group_dicts(case, tp))
    opt._update_rate = case.get("update_rate", 1)  # what setup_gradient_release(update_rate=...) sets
    opt.pipeline_exchange = args.pipeline_exchange
    opt.exchange = args.exchange
    out = {}
    for s in range(case["steps"]):
        for ps, gs in zip(tp, C.build_grads(case, s)):
            for p, g in zip(ps, gs):
                p.grad = distribute_tensor(g.cuda(), mesh, place)
        opt.step()
        if s == 0 or s == case["steps"] - 1:
            tag = "step1" if s == 0 else "final"
            for gi, ps in enumerate(tp):
                for pi, p in enumerate(ps):
                    out[f"{tag}/g{gi}/p{pi}/param"] = full(p)
                    for k, v in opt.state[p].items():
                        out[f"{tag}/g{gi}/p{pi}/{k}"] = full(v) if isinstance(v, torch.Tensor) else np.asarray(v)
    torch.cuda.synchronize()
    assert not opt.device_error()
    if args.replicas > 1:  # the replicas of every shard must hold bitwise-equal parameters and state
        rg = mesh.get_group(mesh_dim=0)
        same = True
        for ps in tp:
            for p in ps:
                for t in [p] + [v for v in opt.state[p].values() if isinstance(v, torch.Tensor)]:
                    loc = (t.to_local() if hasattr(t, "to_local") else t).detach().contiguous()
                    bufs = [torch.empty_like(loc) for _ in range(args.replicas)]
                    dist.all_gather(bufs, loc, group=rg)
                    same &= all(torch.equal(b, bufs[0]) for b in bufs)
        out["replicas_equal"] = np.asarray(same)
    if dist.get_rank() == 0:
        np.savez(args.out, **out)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
