"""The FSDP2 / DTensor Shard(0) path.

CPU (gloo, 2-4 ranks): owner assignment and the slab exchange plans move every
row slab to its owner and every result slab back.  GPU: the full sharded step
(world 1 on any box, world 2 when two GPUs are visible) against the CPU oracle
on the full tensors -- the reference's own MD + FSDP2 path does not run on
torch 2.11, so the single-device algorithm on full tensors is the oracle.
"""
import math
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases as C
import parity as P
from thorn_b200.sharded import assign_owners, ns_flops, plan_gather, plan_scatter, shard_rows
from thorn_b200.sharded import exchange as _exchange

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_assign_owners_balanced_and_deterministic():
    # the Llama-3-8B matrix set over 8 ranks: every rank gets the same NS work
    shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096),
              (4096, 14336)] * 32
    flops = [ns_flops(r, c, 5) for r, c in shapes]
    owners = assign_owners(flops, 8)
    load = [0] * 8
    for f, o in zip(flops, owners):
        load[o] += f
    assert max(load) == min(load)
    assert owners == assign_owners(flops, 8)
    assert assign_owners([5, 3, 3, 1], 2) == [0, 1, 1, 0]
    assert assign_owners([7], 4) == [0]
    # a rotating start: one matrix per call goes round the ranks; a balanced set stays balanced
    assert [assign_owners([7], 4, start)[0] for start in range(6)] == [0, 1, 2, 3, 0, 1]
    for start in range(8):
        rot = assign_owners(flops, 8, start)
        load = [sum(f for f, o in zip(flops, rot) if o == r) for r in range(8)]
        assert max(load) == min(load)


def _exchange_worker(rank, world, port, result, impl="rounds"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from thorn_b200.sharded import exchange_all_to_all
        exchange = _exchange if impl == "rounds" else exchange_all_to_all
        ranks = list(range(world))
        # even and uneven Shard(0) splits (torch.chunk sizes: the last shard is shorter)
        shapes = [(24, 3), (13, 5), (36, 2), (25, 7), (49, 4), (12, 3)]
        full = [torch.arange(r * c, dtype=torch.float32).reshape(r, c) + 100 * j for j, (r, c) in enumerate(shapes)]
        owners = assign_owners([r * c for r, c in shapes], world)
        parts = [shard_rows(r, world) for r, _ in shapes]

        def sl(j, s):
            r0, n = parts[j][s]
            return slice(r0, r0 + n)

        mine = [f[sl(j, rank)].clone() for j, f in enumerate(full)]
        owned = {j: torch.full_like(full[j], -1.0) for j in range(len(shapes)) if owners[j] == rank}
        for j in owned:  # own slab goes in directly
            owned[j][sl(j, rank)] = mine[j]
        sends, recvs = plan_gather(owners, rank, world, lambda j: mine[j], lambda j, s: owned[j][sl(j, s)])
        exchange(sends, recvs, ranks, None)
        ok = all(torch.equal(owned[j], full[j]) for j in owned)
        # owners return 2x the matrix, with a per-row factor
        res = {j: 2 * owned[j] for j in owned}
        fac = {j: torch.arange(full[j].shape[0], dtype=torch.float32) for j in owned}
        back = {j: torch.zeros(parts[j][rank][1], shapes[j][1]) for j in range(len(shapes)) if owners[j] != rank}
        bfac = {j: torch.zeros(parts[j][rank][1]) for j in back}
        sends, recvs = plan_scatter(owners, rank, world, lambda j, s: [res[j][sl(j, s)], fac[j][sl(j, s)]],
                                    lambda j: [back[j], bfac[j]])
        exchange(sends, recvs, ranks, None)
        for j in back:
            ok &= torch.equal(back[j], 2 * mine[j])
            r0, n = parts[j][rank]
            ok &= torch.equal(bfac[j], torch.arange(r0, r0 + n, dtype=torch.float32))
        # the same gather in two waves (even / odd matrices), both queued before either is waited on
        for j in owned:
            owned[j].fill_(-1.0)
            owned[j][sl(j, rank)] = mine[j]
        handles = []
        for js in ([j for j in range(len(shapes)) if j % 2 == 0], [j for j in range(len(shapes)) if j % 2 == 1]):
            sends, recvs = plan_gather(owners, rank, world, lambda j: mine[j], lambda j, s: owned[j][sl(j, s)],
                                       subset=js)
            handles.append(exchange(sends, recvs, ranks, None, wait=False))
        for h in handles:
            h.wait()
        ok &= all(torch.equal(owned[j], full[j]) for j in owned)
        # slabs back to back in one buffer travel as a view; mixed dtypes pack as bytes
        packed = torch.arange(12, dtype=torch.float32)
        views = [packed[0:4], packed[4:10], packed[10:12]]
        from thorn_b200.sharded import _bytes_of, _span
        ok &= _span(views) is not None and _span(views).data_ptr() == packed.data_ptr()
        ok &= _span([packed[0:4], packed[5:7]]) is None
        mixed = _bytes_of([torch.ones(3, dtype=torch.float16), torch.full((2,), 2.0)])
        ok &= mixed.numel() == 3 * 2 + 2 * 4
        result[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,impl", [(2, "rounds"), (3, "rounds"), (4, "rounds"), (3, "all_to_all")])
def test_slab_exchange_gloo(world, impl):
    """Gather and scatter plans through the shifted pairwise rounds (odd world sizes
    included) and through the all_to_all_single alternative."""
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    mp.start_processes(_exchange_worker, args=(world, _free_port(), result, impl), nprocs=world, join=True,
                       start_method="spawn")
    assert dict(result) == {r: True for r in range(world)}


def test_exchange_rounds_pair_every_message():
    """Llama-3-8B matrix set at 8 shards: in every round the messages i sends to i + d are, in
    order and by shape, the messages i + d receives from i (the condition NCCL matches on)."""
    world = 8
    shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096),
              (4096, 14336)] * 32
    owners = assign_owners([ns_flops(r, c, 5) for r, c in shapes], world)
    plans = {}
    for me in range(world):
        g = plan_gather(owners, me, world, lambda j, me=me: ("x", j, me, shapes[j][0] // world, shapes[j][1]),
                        lambda j, s: ("x", j, s, shapes[j][0] // world, shapes[j][1]))
        sc = plan_scatter(owners, me, world,
                          lambda j, s: [("u", j, s)] + ([("f", j, s)] if shapes[j][0] > shapes[j][1] else []),
                          lambda j, me=me: [("u", j, me)] + ([("f", j, me)] if shapes[j][0] > shapes[j][1] else []))
        plans[me] = (g, sc)
    for k in range(2):
        for d in range(1, world):
            for i in range(world):
                to = (i + d) % world
                sent = [s.tensor for s in plans[i][k][0] if s.peer == to]
                got = [r.tensor for r in plans[to][k][1] if r.peer == i]
                assert sent == got
        total_sent = sum(len(plans[i][k][0]) for i in range(world))
        total_recv = sum(len(plans[i][k][1]) for i in range(world))
        assert total_sent == total_recv > 0


def _mesh_error_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Shard, distribute_tensor

        from thorn_b200 import THORN
        m1 = init_device_mesh("cpu", (world,))
        m2 = init_device_mesh("cpu", (world,), mesh_dim_names=("other",))
        a = torch.nn.Parameter(distribute_tensor(torch.randn(8, 8), m1, [Shard(0)]))
        b = torch.nn.Parameter(distribute_tensor(torch.randn(8, 8), m2, [Shard(0)]))
        c = torch.nn.Parameter(distribute_tensor(torch.randn(1, 8), m1, [Shard(0)]))  # second shard empty
        d = torch.nn.Parameter(distribute_tensor(torch.randn(9, 8), m1, [Shard(0)]))  # uneven: 5 + 4 rows
        msgs = []
        for ps in ([a, b], [c], [d]):
            opt = THORN([{"orthogonalize": True, "params": ps, "lr": 1e-3}], backend=torch.cpu)
            for p in ps:
                p.grad = distribute_tensor(torch.randn(p.shape), p.device_mesh, [Shard(0)])
            try:
                opt.step()
                msgs.append("no error")
            except (ValueError, NotImplementedError, RuntimeError) as e:
                msgs.append(type(e).__name__ + ": " + str(e))
        result[rank] = msgs
    finally:
        dist.destroy_process_group()


def test_mesh_and_split_checks_gloo():
    """Host-side checks fire before any kernel: mixed meshes (thorn.py:1358-1359) and
    parameters that are not on a CUDA device (uneven splits, also with an empty shard, are
    accepted)."""
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_mesh_error_worker, args=(2, _free_port(), result), nprocs=2, join=True, start_method="spawn")
    for r in (0, 1):
        assert "same mesh" in result[r][0]
        assert "CUDA devices only" in result[r][1]  # an empty shard is accepted, and then the device check fires
        assert "CUDA devices only" in result[r][2]


def test_shard_rows_follow_torch_chunk():
    for rows in (1, 7, 8, 9, 13, 128256, 151936):
        for world in (1, 2, 3, 4, 8):
            want = [t.shape[0] for t in torch.arange(rows).chunk(world)]
            got = [n for _, n in shard_rows(rows, world)]
            assert got[:len(want)] == want and all(n == 0 for n in got[len(want):])
            assert sum(got) == rows and shard_rows(rows, world)[0][0] == 0


def _run_workers(n, name, tmp_path, extra=()):
    out = str(tmp_path / f"{name}_{n}.npz")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", str(n), "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(HERE, "sharded_worker.py"), "--case", name, "--out", out,
           *extra]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    with np.load(out) as z:
        return {k: z[k] for k in z.files}


def _sharded_compare(got, orc, name, init):
    """Per (tag, group, param, key) errors above tolerance of a sharded run against the oracle."""
    bad = {}
    for tag, (params, states) in orc.items():
        for gi, ps in enumerate(params):
            grp = C.CASES[name]["groups"][gi]
            for pi, p in enumerate(ps):
                g = got[f"{tag}/g{gi}/p{pi}/param"]
                tol = 2e-2 if grp["orthogonalize"] else 1e-5
                e = C.rel_fro(g - init[gi][pi], p - init[gi][pi])
                if not e <= tol:
                    bad[(tag, gi, pi, "param")] = e
                for k, v in states[gi][pi].items():
                    if k in ("step", "random_state"):  # integers: exact
                        assert int(got[f"{tag}/g{gi}/p{pi}/{k}"]) == int(v), (tag, gi, pi, k)
                        continue
                    ref = np.asarray(v, dtype=np.float32)
                    mine = got[f"{tag}/g{gi}/p{pi}/{k}"].reshape(ref.shape)
                    tol_k = 1e-3 if "gain" in k else 1e-5
                    e = C.rel_fro(mine, ref)
                    if not e <= tol_k:
                        bad[(tag, gi, pi, k)] = e
    return bad


PIPE = ("--pipeline-exchange",)
A2A = ("--exchange", "all_to_all")
PEER = ("--exchange", "peer")


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("name,extra", [("tiny", ()), ("md_shard", ()), ("shard_uneven", ()),
                                        ("shard_uneven", PIPE), ("md_shard", PIPE),
                                        ("magma_shard", ()), ("magma_shard", PIPE), ("rate_shard", ()),
                                        ("shard_odd_cols", ()), ("shard_odd_cols", PIPE),
                                        ("shard_tiny_rows", ()), ("shard_uneven", A2A), ("md_shard", A2A + PIPE),
                                        ("tiny", PEER), ("md_shard", PEER), ("shard_uneven", PEER),
                                        ("magma_shard", PEER), ("shard_odd_cols", PEER), ("shard_tiny_rows", PEER)])
def test_sharded_step_matches_oracle(world, name, extra, tmp_path):
    """The Shard(0) path (rounds or waves of the exchange, Magma masking whole matrices)
    against the oracle's sharded semantics; the oracle replays the run's Magma seeds."""
    from oracle.thorn_oracle import MASK64, W1_C

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if world == 1 and extra:
        pytest.skip("the exchange variants only differ with 2 or more ranks")
    got = _run_workers(world, name, tmp_path, extra)
    seeds = []
    for gi, grp in enumerate(C.CASES[name]["groups"]):
        if grp["opts"].get("momentum_align"):
            for pi in range(len(grp["shapes"])):
                seeds.append((int(got[f"step1/g{gi}/p{pi}/random_state"]) - W1_C) & MASK64)
    _, orc = P.run_oracle(name, seeds=seeds or None, sharded=True)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad = _sharded_compare(got, orc, name, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}


@pytest.mark.gpu
@pytest.mark.parametrize("replicas", [1, 2])
@pytest.mark.parametrize("name", ["tiny", "md_shard", "shard_uneven", "magma_shard"])
def test_hsdp_step_matches_oracle(replicas, name, tmp_path):
    """HSDP meshes on two GPUs: (Replicate(), Shard(0)) placements over a 1 x 2 mesh (one
    replica, its matrices sharded over both ranks) and a 2 x 1 mesh (two replicas, each
    holding whole matrices), against the oracle's sharded semantics (thorn.py:1015-1019).
    Each rank's optimizer works inside its own shard group only, and the two replicas of
    the 2 x 1 mesh end with bitwise-equal parameters and state."""
    from oracle.thorn_oracle import MASK64, W1_C

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    got = _run_workers(2, name, tmp_path, ("--replicas", str(replicas), "--exchange", "all_to_all"))
    if replicas > 1:
        assert bool(got["replicas_equal"])
    seeds = []
    for gi, grp in enumerate(C.CASES[name]["groups"]):
        if grp["opts"].get("momentum_align"):
            for pi in range(len(grp["shapes"])):
                seeds.append((int(got[f"step1/g{gi}/p{pi}/random_state"]) - W1_C) & MASK64)
    _, orc = P.run_oracle(name, seeds=seeds or None, sharded=True)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad = _sharded_compare(got, orc, name, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}


def _hsdp_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Replicate, Shard, distribute_tensor

        from thorn_b200.sharded import shard_group
        mesh = init_device_mesh("cpu", (2, 2), mesh_dim_names=("replicate", "shard"))
        full = torch.arange(9 * 4, dtype=torch.float32).reshape(9, 4)
        p = distribute_tensor(full, mesh, [Replicate(), Shard(0)])
        ranks, group = shard_group(p, rank)
        # the shard group is this rank's row of the mesh; an uneven split (5 + 4 rows)
        parts = shard_rows(9, len(ranks))
        me = ranks.index(rank)
        local = p.to_local()
        ok = ranks == [r for r in mesh.mesh.tolist() if rank in r][0]
        ok &= local.shape[0] == parts[me][1] and torch.equal(local, full[parts[me][0]:parts[me][0] + parts[me][1]])
        # a collective on the shard group reaches exactly the row's ranks
        t = torch.tensor([float(rank)])
        dist.all_reduce(t, group=group)
        ok &= float(t) == float(sum(ranks))
        result[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_hsdp_shard_groups_gloo():
    """(Replicate, Shard(0)) meshes: each replica row is a shard group of its own (thorn.py:1015-1019)."""
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_hsdp_worker, args=(4, _free_port(), result), nprocs=4, join=True, start_method="spawn")
    assert dict(result) == {r: True for r in range(4)}


class _StubLib:
    def thorn_ns_ld(self, n):
        return (n + 7) // 8 * 8

    def __getattr__(self, name):
        if name.endswith("_bytes"):
            return lambda *a: 256
        return lambda *a: 0


def _sharded_flow_worker(rank, world, port, result, exchange_impl, pipeline):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Shard, distribute_tensor

        from thorn_b200 import THORN, _native as N
        from thorn_b200 import sharded as S
        from thorn_b200.optimizer import GroupConfig, _Arena, _local

        N.load = lambda build_if_missing=False: _StubLib()
        N.stream_of = lambda dev: 0
        mesh = init_device_mesh("cpu", (world,))
        torch.manual_seed(0)
        shapes = [(24, 16), (13, 8), (40, 24), (33, 16), (12, 32), (17, 13), (2, 16)]
        ps = [torch.nn.Parameter(distribute_tensor(torch.randn(s) * 0.02, mesh, [Shard(0)])) for s in shapes]
        opt = THORN([{"orthogonalize": True, "params": ps, "lr": 1e-3, "decouple_md": True,
                      "momentum_align": True}])
        opt.exchange, opt.pipeline_exchange, opt.polar_decomp_batch_size = exchange_impl, pipeline, 300
        cfg = GroupConfig.from_kwargs(**opt.param_groups[0])
        ranks, group = S.shard_group(ps[0], rank)
        for step in range(2):
            for p, s in zip(ps, shapes):
                p.grad = distribute_tensor(torch.randn(s) * 1e-3, mesh, [Shard(0)])
            for p in ps:
                if "step" not in opt.state[p]:
                    opt._init_state(p, opt.state[p], cfg, opt.param_groups[0])
            from thorn_b200.optimizer import _Item
            recs = []
            for p in ps:
                it = _Item()
                it.g, it.state, it.split, it.apply = _local(p.grad), opt.state[p], True, True
                recs.append(it)
            opt._magma(recs, cfg, recovered=True, group=group)
            S._step_matrices(opt, ps, cfg, ranks, group, world, ranks.index(rank), torch.device("cpu"), _Arena,
                             _local, [it.scale for it in recs])
        # every rank drew or received the same generator state for each matrix
        states = [int(opt.state[p]["random_state"]) for p in ps]
        box = [None] * world
        dist.all_gather_object(box, states)
        result[rank] = all(b == states for b in box) and all(opt.state[p]["step"] == 3 for p in ps)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,impl,pipeline", [(2, "rounds", False), (3, "rounds", True), (3, "all_to_all", True)])
def test_sharded_host_flow_gloo(world, impl, pipeline):
    """The sharded step's host flow on gloo with a stub C ABI: owner planning, uneven
    splits, real slab exchanges (pairwise rounds or all-to-all, one wave or pipelined
    waves), Magma statistics all-reduced over the shard group with a shared seed."""
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_sharded_flow_worker, args=(world, _free_port(), result, impl, pipeline), nprocs=world,
                       join=True, start_method="spawn")
    assert dict(result) == {r: True for r in range(world)}


def _rank_loss_worker(rank, world, port, result):
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    from thorn_b200 import THORN, _native as N
    from thorn_b200 import sharded as S
    from thorn_b200.optimizer import GroupConfig, _Arena, _local

    N.load = lambda build_if_missing=False: _StubLib()
    N.stream_of = lambda dev: 0
    mesh = init_device_mesh("cpu", (world,))
    torch.manual_seed(0)
    shapes = [(24, 16), (13, 8), (40, 24)]
    ps = [torch.nn.Parameter(distribute_tensor(torch.randn(s) * 0.02, mesh, [Shard(0)])) for s in shapes]
    opt = THORN([{"orthogonalize": True, "params": ps, "lr": 1e-3}])
    cfg = GroupConfig.from_kwargs(**opt.param_groups[0])
    ranks, group = S.shard_group(ps[0], rank)

    def step():
        for p, s in zip(ps, shapes):
            p.grad = distribute_tensor(torch.randn(s) * 1e-3, mesh, [Shard(0)])
            if "step" not in opt.state[p]:
                opt._init_state(p, opt.state[p], cfg, opt.param_groups[0])
        S._step_matrices(opt, ps, cfg, ranks, group, world, ranks.index(rank), torch.device("cpu"), _Arena, _local,
                         [1.0] * len(ps))

    step()
    if rank == world - 1:  # leaves between steps, with nothing in flight
        result[rank] = "left"
        os._exit(0)
    t0 = time.time()
    try:
        step()
        result[rank] = "no error"
    except Exception as exc:  # the lost peer surfaces as an error, not a hang
        result[rank] = (type(exc).__name__, round(time.time() - t0, 1))
    os._exit(0)


def test_lost_rank_fails_the_next_step_gloo():
    """Failure detection on the host: a rank that leaves between steps makes the remaining
    rank's next sharded step raise (its first collective on the shard group fails) within the
    process group's timeout, instead of waiting for good."""
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_rank_loss_worker, args=(2, _free_port(), result), nprocs=2, join=True,
                       start_method="spawn")
    assert result[1] == "left"
    assert isinstance(result[0], tuple), result[0]
    assert result[0][1] < 30, result[0]


def _due_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Shard, distribute_tensor

        from thorn_b200 import THORN
        from thorn_b200 import sharded as S
        from thorn_b200.optimizer import GroupConfig

        mesh = init_device_mesh("cpu", (world,))
        torch.manual_seed(0)
        shapes = [(8, 4), (6, 4), (10, 4), (4, 4)]
        ps = [torch.nn.Parameter(distribute_tensor(torch.randn(s), mesh, [Shard(0)])) for s in shapes]
        opt = THORN([{"orthogonalize": True, "params": ps, "lr": 1e-3, "momentum_align": True}])
        opt._magma_stats = P.magma_stats_cpu  # the statistics kernel needs a GPU
        opt._update_rate = 2
        cfg = GroupConfig.from_kwargs(**opt.param_groups[0])
        ranks, group = S.shard_group(ps[0], rank)
        log = []
        for step in range(3):
            for p, s in zip(ps, shapes):
                p.grad = distribute_tensor(torch.randn(s), mesh, [Shard(0)])
                if "step" not in opt.state[p]:
                    opt._init_state(p, opt.state[p], cfg, opt.param_groups[0])
                opt.state[p]["moment"] = opt.state[p]["moment"] + 0.1  # a nonzero moment for Magma
            due, scales = S.due_matrices(opt, list(ps), cfg, group)
            sel = [any(d is p for d in due) for p in ps]
            assert all((p.grad is None) != s for p, s in zip(ps, sel))
            assert len(scales) == len(due) and all(sc > 0 for sc in scales)
            for p in due:  # what the step's finish does for an updated matrix
                opt.state[p]["step"] += 1
                p.grad = None
            log.append(sel)
        box = [None] * world
        dist.all_gather_object(box, log)
        steps = [opt.state[p]["step"] for p in ps]
        # every rank selects the same matrices; step 1 is due for every unmasked matrix, and a
        # matrix that updated (step 2) is never due again under update_rate 2
        result[rank] = (all(b == log for b in box), log, steps)
    finally:
        dist.destroy_process_group()


def test_sharded_due_matrices_gloo():
    """The sharded step's selection of the matrices it updates (Magma on, update_rate 2), on
    gloo ranks: the same on every rank, a masked or not-due matrix left out with its gradient
    dropped and its step count kept (thorn.py:1485-1490, 1564)."""
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_due_worker, args=(2, _free_port(), result), nprocs=2, join=True, start_method="spawn")
    same, log, steps = result[0]
    assert same and result[1][0]
    for j in range(4):
        col = [sel[j] for sel in log]
        assert sum(col) <= 1  # updates at most once
        assert steps[j] == 1 + sum(col)
    assert any(any(sel) for sel in log)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_peer_layout_disjoint_and_aligned(world):
    """The peer exchange's arena layout (the same computation on every rank): for every owner,
    the NS inputs of its chunks and the result slots of its shards of the other owners'
    matrices are disjoint, 256-byte aligned, past the flag slots, and sized for the rows
    that land there; the Llama-3-8B set and an uneven split with empty shards."""
    from thorn_b200.sharded import PEER_FLAG_BYTES, peer_layout

    for shapes in ([(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096),
                    (4096, 14336)] * 2, [(66, 64), (5, 37), (2, 48), (130, 8)]):
        rows = [r for r, _ in shapes]
        cols = [c for _, c in shapes]
        ld = [(c + 7) // 8 * 8 for c in cols]
        parts = [shard_rows(r, world) for r in rows]
        owners = assign_owners([ns_flops(r, c, 5) for r, c in shapes], world)
        for r in range(world):
            mine = [j for j in range(len(shapes)) if owners[j] == r]
            chunks = [(rows[j], cols[j], "bf16", "f32", [j]) for j in mine]
            x_off, u_off, f_off, total = peer_layout(r, owners, chunks, parts, cols, ld, 2, lambda j: rows[j] > cols[j])
            spans = [(x_off[ci], rows[js[0]] * ld[js[0]] * 2) for ci, (_, _, _, _, js) in enumerate(chunks)]
            for j, off in u_off.items():
                assert owners[j] != r and parts[j][r][1] > 0
                spans.append((off, parts[j][r][1] * cols[j] * 2))
            for j, off in f_off.items():
                spans.append((off, parts[j][r][1] * 4))
            assert set(u_off) == {j for j in range(len(shapes)) if owners[j] != r and parts[j][r][1] > 0}
            spans.sort()
            assert all(o % 256 == 0 and o >= PEER_FLAG_BYTES for o, _ in spans)
            assert all(a + n <= b for (a, n), (b, _) in zip(spans, spans[1:]))
            assert spans[-1][0] + spans[-1][1] <= total


def _stepper_worker(rank, world, port, result):
    import contextlib

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Shard, distribute_tensor

        import thorn_b200.host_stepper as HS

        class FakeEvent:
            def record(self, stream=None):
                pass

            def synchronize(self):
                pass

        class FakeStream:
            def wait_event(self, ev):
                pass

            def wait_stream(self, s):
                pass

            def synchronize(self):
                pass

        compute = FakeStream()
        HS.torch.cuda.Stream = lambda dev=None: FakeStream()
        HS.torch.cuda.Event = lambda *a, **k: FakeEvent()
        HS.torch.cuda.current_stream = lambda dev=None: compute
        HS.torch.cuda.stream = lambda s: contextlib.nullcontext()
        torch.Tensor.is_pinned = lambda self: True

        mesh = init_device_mesh("cpu", (world,))
        shapes = [(5, 4), (8, 3), (1, 6)]  # uneven splits; rank 1 holds no row of the last
        ps = [torch.nn.Parameter(distribute_tensor(torch.zeros(s), mesh, [Shard(0)])) for s in shapes]

        class AddGrad:  # stands in for THORN: p -= grad on the local shards
            def step(self):
                for p in ps:
                    p._local_tensor.sub_(p.grad.to_local())
                    p.grad = None

        local = [p.to_local().shape for p in ps]
        offs, n = HS._block_layout(local, torch.float32)
        fg, fp = torch.zeros(n), torch.zeros(n)
        hg = [fg[o:o + math.prod(s)].view(s) for o, s in zip(offs, local)]
        hp = [fp[o:o + math.prod(s)].view(s) for o, s in zip(offs, local)]
        st = HS.PinnedStepper(AddGrad(), ps, hg, hp)
        ok = st.grads_flat is None and st.snapshot_flat is not None  # DTensor grads stay per tensor
        for k in range(3):
            st.wait_host_grads()
            for h in hg:
                h.fill_(k + 1.0)
            st.step()
        st.synchronize()
        ok &= all(torch.equal(h, torch.full(h.shape, -6.0)) for h in hp)
        ok &= all(torch.equal(p.to_local(), torch.full(p.to_local().shape, -6.0)) for p in ps)
        result[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_pinned_stepper_dtensor_shards_gloo():
    """PinnedStepper on Shard(0) DTensor parameters (the bench's end-to-end run at N > 1):
    gradients are copied per local shard into DTensor gradients, the parameter snapshot is
    one block mirroring pinned_block's layout of the local shards (an empty shard included),
    and after three steps the host buffers hold every rank's updated local rows."""
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_stepper_worker, args=(2, _free_port(), result), nprocs=2, join=True, start_method="spawn")
    assert dict(result) == {0: True, 1: True}
