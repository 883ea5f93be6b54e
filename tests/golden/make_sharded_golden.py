"""Generate golden vectors by running the reference THORN's FSDP2 (DTensor Shard(0)) path.

Usage (in a container where the reference checkout is available):

    python tests/golden/make_sharded_golden.py --ref /path/to/THORN [case ...]

Each case of ``SHARDED_CASES`` is stepped by ``world`` gloo ranks on CPU with the
reference's own ``thorn.THORN`` (its ``_sharded_ortho_step``, thorn.py:1459-1581):
every orthogonalized parameter and its gradient is a DTensor sharded ``Shard(0)``
over a 1-D CPU mesh.  Row counts divide evenly by ``world`` (the reference gathers
equal-size shards, thorn.py:1108).  Rank 0 stores the full (gathered) parameters
and state after step 1 and after the last step, in the layout of
``make_golden.py``.  The reference's decouple_md path does not run sharded on
this torch version, and neither does its sharded Magma masking (it all-reduces a DTensor,
thorn.py:820-826), so these cases leave both off.
"""
from __future__ import annotations

import argparse
import os
import socket
import sys

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import cases as C  # noqa: E402
from make_golden import _store  # noqa: E402

SHARDED_CASES = ("rate_shard",)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, ref, name, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sys.path.insert(0, ref)
        import thorn.thorn as mod  # the reference implementation
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import DTensor, Shard, distribute_tensor

        mesh = init_device_mesh("cpu", (world,))
        case = C.CASES[name]
        params = C.build_params(case)  # same seed on every rank
        tp = [[torch.nn.Parameter(distribute_tensor(t.clone(), mesh, [Shard(0)])) for t in ps] for ps in params]
        opt = mod.THORN(C.group_dicts(case, tp), backend=torch.cpu)
        opt._update_rate = case.get("update_rate", 1)  # what setup_gradient_release(update_rate=...) sets
        out = {}

        def full(t):
            return t.full_tensor() if isinstance(t, DTensor) else t

        for s in range(case["steps"]):
            for ps, gs in zip(tp, C.build_grads(case, s)):
                for p, g in zip(ps, gs):
                    p.grad = distribute_tensor(g.clone(), mesh, [Shard(0)])
            opt.step()
            if s == 0 or s == case["steps"] - 1:
                tag = "step1" if s == 0 else "final"
                for gi, ps in enumerate(tp):
                    for pi, p in enumerate(ps):
                        base = f"{tag}/g{gi}/p{pi}"
                        _store(out, base + "/param", full(p.data))
                        for k, v in opt.state[p].items():
                            if isinstance(v, torch.Tensor):
                                _store(out, f"{base}/{k}", full(v))
                            elif isinstance(v, int) and v >= 1 << 63:
                                out[f"{base}/{k}"] = np.asarray(v, dtype=np.uint64)
                            else:
                                out[f"{base}/{k}"] = np.asarray(v)
        if rank == 0:
            g0 = C.build_grads(case, 0)
            out["input/grad0_sum"] = np.array([C.checksum(t.float().numpy()) for ps in g0 for t in ps])
            out["input/param_sum"] = np.array([C.checksum(t.float().numpy()) for ps in params for t in ps])
            out["meta/world"] = np.asarray(world)
            np.savez_compressed(out_path, **out)
    finally:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference THORN checkout")
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("cases", nargs="*")
    args = ap.parse_args()
    for name in args.cases or SHARDED_CASES:
        path = os.path.join(HERE, f"{name}.npz")
        mp.start_processes(_worker, args=(args.world, _free_port(), args.ref, name, path), nprocs=args.world,
                           join=True, start_method="spawn")
        print(name, "written")


if __name__ == "__main__":
    main()
