"""FSDP2 / DTensor ``Shard(0)`` path of the orthogonalized group.

Replaces the reference's ``_DistributedTHORNState`` (thorn.py:979-1186),
``_assign_params`` (thorn.py:1333-1374) and ``_sharded_ortho_step``
(thorn.py:1459-1581).  The reference gathers each matrix's fp32 momentum rows
to an owner rank with one ``dist.gather`` per matrix, runs Newton-Schulz there
and scatters fp32 results back.  Here, per step:

1. every rank runs the momentum pass on its own rows (one multi-tensor launch)
   and the per-matrix partial sums of u^2 (plus the decouple_md column-gain
   partials) are added with a single all-reduce;
2. every rank normalises its rows by the global norm and casts them to the NS
   operand type, writing straight into the owner's NS input buffer when it is
   the owner, else into a send slab;
3. one NCCL exchange moves all slabs to their owners (half the bytes of the
   reference's fp32 gather): by default one ``all_to_all_single`` whose send
   buffer is the owner-ordered slabs themselves; with ``exchange = "rounds"``
   world - 1 shifted pairwise point-to-point rounds, one packed message per
   direction per round;
4. owners run batched Newton-Schulz (+ per-neuron-norm statistics with the
   row scale folded into one factor per row);
5. one exchange of the same form returns the 16-bit result rows and the fp32
   row factors;
6. every rank applies the update to its own rows (and, with decouple_md,
   all-reduces ||p||^2 for the renorm).

Shards follow DTensor's ``torch.chunk`` split, so rows need not divide evenly,
and a matrix with fewer rows than ranks leaves some shards empty.  With ``pipeline_exchange``
steps 3-5 run in waves of NS batches so transfers overlap the owners' NS.  Magma
masking all-reduces its three sums over the shard group first; a masked matrix,
or one whose step is not due under ``update_rate``, is left out of the step.

Owners are chosen by longest-processing-time over the reference's NS FLOP
estimate (thorn.py:1001-1007), deterministically on every rank.  Parameters of
rank > 2 (conv kernels) split along their batch dimension hold whole matrices
on each rank and take the local path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch.distributed.tensor import DTensor, Replicate, Shard

from . import _native as N


def shard_group(p: DTensor, rank: int):
    """Ranks (in shard order) and process group of a sharded parameter (thorn.py:1009-1021)."""
    if p.placements == (Shard(dim=0),):
        return [int(r) for r in p.device_mesh.mesh.tolist()], p.device_mesh.get_group(mesh_dim=0)
    if p.placements == (Replicate(), Shard(dim=0)):
        for row in p.device_mesh.mesh:
            if rank in row.tolist():
                return [int(r) for r in row.tolist()], p.device_mesh.get_group(mesh_dim=1)
        raise ValueError("rank not found in the shard mesh")
    raise ValueError(f"Unsupported placements {p.placements}")


def shard_rows(rows: int, world: int) -> list[tuple[int, int]]:
    """(first row, row count) of every shard of a ``Shard(0)`` split: DTensor's
    ``torch.chunk`` rule, ceil(rows / world) rows per shard and a shorter (or
    empty) tail."""
    c = -(-rows // world)
    return [(min(i * c, rows), max(0, min(c, rows - i * c))) for i in range(world)]


def ns_flops(rows: int, cols: int, iters: int) -> int:
    """The reference's per-matrix NS cost estimate (thorn.py:1001-1007)."""
    m, n = min(rows, cols), max(rows, cols)
    return iters * ((m ** 3) * 2 + (m ** 2 * n) * 4 + m * n * 2 + m ** 2 * 3)


def assign_owners(flops: list[int], world: int, start: int = 0) -> list[int]:
    """Longest-processing-time assignment: heaviest matrix first, to the least-loaded rank.

    Ties go to the lower matrix index and to the first rank counting from ``start``, so
    every rank computes the same assignment.  (The reference deals sorted matrices
    round-robin, thorn.py:1348-1372; both balance the Llama sets exactly.)  ``start``
    rotates from call to call: steps of one matrix at a time (gradient release) then
    spread their Newton-Schulz work over the ranks instead of all landing on rank 0.
    """
    order = sorted(range(len(flops)), key=lambda j: (-flops[j], j))
    load = [0] * world
    owner = [0] * len(flops)
    for j in order:
        r = min(range(world), key=lambda k: (load[k], (k - start) % world))
        owner[j] = r
        load[r] += flops[j]
    return owner


@dataclass
class Slab:
    """One point-to-point message: ``tensor`` goes to / comes from shard index ``peer``."""

    tensor: torch.Tensor
    peer: int


def _span(ts: list[torch.Tensor]):
    """A flat uint8 view covering the given tensors in order when they are contiguous
    and back to back in one allocation, else None."""
    if not all(t.is_contiguous() for t in ts):
        return None
    if len(ts) == 1:
        return ts[0].reshape(-1).view(torch.uint8)
    st = ts[0].untyped_storage()
    if not all(a.data_ptr() + a.nbytes == b.data_ptr() and b.untyped_storage().data_ptr() == st.data_ptr()
               for a, b in zip(ts, ts[1:])):
        return None
    span = torch.empty(0, dtype=torch.uint8, device=ts[0].device)
    return span.set_(st, ts[0].data_ptr() - st.data_ptr(), (sum(t.nbytes for t in ts),), (1,))


def _bytes_of(ts: list[torch.Tensor]) -> torch.Tensor:
    """The tensors' bytes in order, as one flat uint8 tensor: a view when possible,
    else a packed copy."""
    span = _span(ts)
    if span is not None:
        return span
    return torch.cat([t.contiguous().reshape(-1).view(torch.uint8) for t in ts])


class Exchange:
    """Handle of a queued exchange: ``wait()`` makes the current stream wait for it
    and unpacks received messages that did not land in place (the host never blocks)."""

    def __init__(self):
        self.works = []
        self.unpack = []  # (received bytes, destination tensors)

    def wait(self):
        for w in self.works:
            w.wait()
        for buf, dsts in self.unpack:
            # one multi-tensor copy for all slabs of a message
            views = [t.reshape(-1).view(torch.uint8) for t in dsts]
            torch._foreach_copy_(views, list(buf.split([v.numel() for v in views])))
        self.works, self.unpack = [], []


def exchange(sends: list[Slab], recvs: list[Slab], ranks: list[int], group, wait: bool = True) -> Exchange:
    """All messages of one exchange, as world - 1 shifted pairwise rounds.

    In round d every shard index i sends only to i + d and receives only from
    i - d (mod world).  Each round is one batched P2P call with one message per
    direction, that peer's slabs packed in canonical order (matrix index
    ascending, then peer ascending) -- so NCCL sets up at most two new peer
    connections per call, the pattern is a permutation that NVSwitch serves at
    full bandwidth, and the host posts two operations per round, not one per
    slab.  Slabs that are back to back in memory travel without a packing copy.
    Empty slabs are left out on both sides.  With ``wait`` the current stream
    waits for the exchange now; otherwise the caller calls ``wait()`` on the
    returned handle.
    """
    world = len(ranks)
    me = ranks.index(dist.get_rank())
    ex = Exchange()
    for d in range(1, world):
        to, frm = (me + d) % world, (me - d) % world
        out = [s.tensor for s in sends if s.peer == to and s.tensor.numel()]
        inc = [r.tensor for r in recvs if r.peer == frm and r.tensor.numel()]
        ops = []
        if out:
            ops.append(dist.P2POp(dist.isend, _bytes_of(out), ranks[to], group))
        if inc:
            if not all(t.is_contiguous() for t in inc):
                raise ValueError("receive slabs must be contiguous")
            buf = _span(inc)  # received in place when the destinations are back to back
            if buf is None:
                buf = torch.empty(sum(t.nbytes for t in inc), dtype=torch.uint8, device=inc[0].device)
                ex.unpack.append((buf, inc))
            ops.append(dist.P2POp(dist.irecv, buf, ranks[frm], group))
        if ops:
            ex.works += dist.batch_isend_irecv(ops)
    if wait:
        ex.wait()
    return ex


def exchange_all_to_all(sends: list[Slab], recvs: list[Slab], ranks: list[int], group,
                        wait: bool = True) -> Exchange:
    """The same exchange as one ``all_to_all_single`` collective: each peer's slabs
    packed back to back (canonical order) in one send buffer, the received bytes
    unpacked per source.  Every rank of the group takes part, also with nothing to
    send.  This is the default exchange (``THORN.exchange = "all_to_all"``): NCCL moves
    all peers' messages at once, where the rounds move one peer's per call."""
    world = len(ranks)
    if sends or recvs:
        dev = (sends[0] if sends else recvs[0]).tensor.device
    else:
        dev = torch.device("cuda", torch.cuda.current_device())
    out_parts, in_parts = [[] for _ in range(world)], [[] for _ in range(world)]
    for s_ in sends:
        if s_.tensor.numel():
            out_parts[s_.peer].append(s_.tensor)
    for r in recvs:
        if r.tensor.numel():
            if not r.tensor.is_contiguous():
                raise ValueError("receive slabs must be contiguous")
            in_parts[r.peer].append(r.tensor)
    out_sizes = [sum(t.nbytes for t in ts) for ts in out_parts]
    in_sizes = [sum(t.nbytes for t in ts) for ts in in_parts]
    flat = [t for ts in out_parts for t in ts]
    # the gather's slabs are laid out by owner, so its send buffer is a view (no packing copy)
    send_buf = _bytes_of(flat) if flat else torch.empty(0, dtype=torch.uint8, device=dev)
    recv_buf = torch.empty(sum(in_sizes), dtype=torch.uint8, device=dev)
    ex = Exchange()
    ex.works.append(dist.all_to_all_single(recv_buf, send_buf, in_sizes, out_sizes, group=group, async_op=True))
    off = 0
    for peer in range(world):
        if in_sizes[peer]:
            ex.unpack.append((recv_buf[off:off + in_sizes[peer]], in_parts[peer]))
        off += in_sizes[peer]
    if wait:
        ex.wait()
    return ex


def plan_gather(owners: list[int], me: int, world: int, my_rows, owner_rows, subset=None):
    """Messages that bring every matrix's row slabs to its owner.

    ``my_rows(j)``: this rank's slab of matrix j (a send buffer, for j it does
    not own); ``owner_rows(j, s)``: where slab s of an owned matrix j lands.
    ``subset``: ascending matrix indices to plan for (default: all).
    """
    js = range(len(owners)) if subset is None else subset
    sends = [Slab(my_rows(j), owners[j]) for j in js if owners[j] != me]
    recvs = [Slab(owner_rows(j, s), s) for j in js if owners[j] == me for s in range(world) if s != me]
    return sends, recvs


def plan_scatter(owners: list[int], me: int, world: int, owner_parts, my_parts, subset=None):
    """Messages that return result slabs from owners.

    ``owner_parts(j, s)``: list of tensors of owned matrix j destined for shard
    s; ``my_parts(j)``: matching receive buffers for a matrix this rank does
    not own.  ``subset``: ascending matrix indices to plan for (default: all).
    """
    js = range(len(owners)) if subset is None else subset
    sends = [Slab(t, s) for j in js if owners[j] == me for s in range(world) if s != me for t in owner_parts(j, s)]
    recvs = [Slab(t, owners[j]) for j in js if owners[j] != me for t in my_parts(j)]
    return sends, recvs


def sharded_ortho_step(opt, params, cfg) -> None:
    """One step of the orthogonalized group for DTensor ``Shard(0)`` parameters."""
    from .optimizer import _Arena, _local

    rank = dist.get_rank()
    ranks, group = shard_group(params[0], rank)
    mesh0 = params[0].device_mesh
    for p in params:
        if p.device_mesh != mesh0:
            raise ValueError("All parameters must be on the same mesh.")
        shard_group(p, rank)
    world, me = len(ranks), ranks.index(rank)
    mats, batched = [], []
    for p in params:
        if p.ndim == 2:
            parts = shard_rows(p.shape[0], world)
            if _local(p).shape[0] != parts[me][1]:
                raise ValueError(f"local shard of {_local(p).shape[0]} rows does not follow the Shard(0) split of "
                                 f"{p.shape[0]} rows over {world} ranks")
            mats.append(p)
        else:
            batched.append(p)  # whole (in, k) matrices on every rank
    dev_type = _local(params[0]).device.type
    if dev_type != "cuda":
        raise RuntimeError(f"thorn_b200 runs its step on CUDA devices only; got a sharded parameter on {dev_type}")
    if batched:
        with torch.cuda.device(_local(batched[0]).device):
            opt._ortho_local(batched, cfg)
    if not mats:
        return
    dev = _local(mats[0]).device
    with torch.cuda.device(dev):
        mats, scales = due_matrices(opt, mats, cfg, group)
        if mats:
            _step_matrices(opt, mats, cfg, ranks, group, world, me, dev, _Arena, _local, scales)


def due_matrices(opt, mats, cfg, group):
    """The sharded matrices this step updates, and their Magma LR scales.

    Magma scores every matrix first, its three sums all-reduced over the shard group
    (thorn.py:1483-1490).  A masked matrix, or one whose step is not due under
    ``update_rate``, is then left out of the step entirely: its gradient is dropped, its
    momentum and step count stay (thorn.py:1485-1490, 1564).  So with update_rate > 1 a
    sharded matrix updates once and is never due again; the reference's sharded path
    behaves so, and it is kept for drop-in parity."""
    from .optimizer import _Item, _local

    scales = [1.0] * len(mats)
    if cfg.momentum_align:
        recs = []
        for p in mats:
            it = _Item()
            it.g, it.state = _local(p.grad), opt.state[p]
            it.split, it.apply = "row_gain" in it.state, True
            recs.append(it)
        opt._magma(recs, cfg, recovered=True, group=group)
        scales = [it.scale for it in recs]
    due = [sc != 0.0 and (opt.state[p]["step"] + 1) % opt._update_rate == 0 for p, sc in zip(mats, scales)]
    for p, d in zip(mats, due):
        if not d:
            p.grad = None
    return [p for p, d in zip(mats, due) if d], [sc for sc, d in zip(scales, due) if d]


PEER_FLAG_BYTES = 4096  # gather slots at 0, scatter slots at 512: 64 x 8 bytes each
PEER_WAIT_LIMIT_NS = 10 * 1000 ** 3


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def peer_layout(r, owners, chunks_r, parts, cols, ld, esz, pnn_rows):
    """Byte offsets in owner r's arena (the same on every rank): the NS input of each of r's
    chunks, then the result rows (and pnn row factors) of r's shard of every matrix another
    rank owns.  ``cols[j]``, ``ld[j]``: columns and NS leading dimension of matrix j;
    ``pnn_rows(j)``: whether matrix j's results carry per-row factors.  Returns
    (x_off by chunk, u_off by matrix, f_off by matrix, total bytes)."""
    off = PEER_FLAG_BYTES
    x_off, u_off, f_off = {}, {}, {}
    for ci, (R, C, _pdt, _sdt, js) in enumerate(chunks_r):
        x_off[ci] = off
        off += _align(len(js) * R * ld[js[0]] * esz)
    for j in range(len(owners)):
        n = parts[j][r][1]
        if owners[j] != r and n > 0:
            u_off[j] = off
            off += _align(n * cols[j] * esz)
            if pnn_rows(j):
                f_off[j] = off
                off += _align(n * 4)
    return x_off, u_off, f_off, off


class PeerArenas:
    """This rank's exported device arena and its shard-group peers' arenas mapped by CUDA
    IPC (``THORN.exchange = "peer"``).  Every rank computes the same size from the same
    plan, so all ranks of the group re-export together when it grows."""

    def __init__(self):
        self.base = None
        self.bytes = 0
        self.ranks = None
        self.group = None
        self.ptrs = []  # arena of shard index s, as mapped into this process

    def ensure(self, lib, need, ranks, me, group, dev):
        need = _align(need, 1 << 20)
        if self.base is not None and self.bytes >= need and self.ranks == ranks:
            return
        torch.cuda.synchronize(dev)  # nothing still reads or writes the old mappings
        self.close(lib)
        ptr = N.ctypes.c_void_p()
        N.check(lib.thorn_peer_alloc(need, N.ctypes.byref(ptr)), "peer_alloc")
        self.base, self.bytes, self.ranks, self.group = ptr.value, need, list(ranks), group
        h = (N.ctypes.c_char * 64)()
        N.check(lib.thorn_ipc_handle(self.base, h), "ipc_handle")
        handles = [None] * len(ranks)
        dist.all_gather_object(handles, bytes(h), group=group)
        self.ptrs = []
        for s, hb in enumerate(handles):
            if s == me:
                self.ptrs.append(self.base)
                continue
            q = N.ctypes.c_void_p()
            N.check(lib.thorn_ipc_open(hb, N.ctypes.byref(q)), "ipc_open")
            self.ptrs.append(q.value)
        dist.barrier(group=group)  # every rank has mapped every arena before any store

    def release(self, lib, dev):
        """Unmap the peers' arenas and free this rank's, once no rank touches them any more:
        every rank of the group must call this together (it synchronises and barriers)."""
        if self.base is None:
            return
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)
        self.close(lib)

    def close(self, lib):
        for s, q in enumerate(self.ptrs):
            if q is not None and q != self.base:
                lib.thorn_ipc_close(q)
        if self.base is not None:
            lib.thorn_peer_free(self.base)
        self.base, self.bytes, self.ptrs = None, 0, []


def _signal_and_wait(lib, pa, world, me, slot0, value, err, stream, limit_ns):
    """Release this rank's slot ``slot0 + me`` in every arena of the group (its own
    included), then wait until all ``world`` slots of its own arena hold ``value``."""
    slots = (N.ctypes.c_void_p * world)(*[pa.ptrs[s] + 8 * (slot0 + me) for s in range(world)])
    N.check(lib.thorn_peer_signal(slots, world, value, stream), "peer_signal")
    N.check(lib.thorn_peer_wait(pa.base + 8 * slot0, world, value, limit_ns, err.data_ptr(), stream), "peer_wait")


def peer_exchange_and_ns(opt, lib, items, chunks, owner_chunks, owners, parts, rows_g, ld, world, me, ranks, group,
                         dev, stream, arena, cfg, err, pnn_h, b1, write_grad, mark):
    """Steps 2-5 of the sharded step over NVLink peer memory.

    2+3. The NS input pass stores this rank's normalised rows straight into each owner's
         arena (the gather is fused into that kernel); a flag release per owner and a
         bounded wait on this rank's own slots order the stores before the owners' NS.
    4.   Owners run batched NS (+ pnn factors) on their arena-resident inputs.
    5.   Result rows and row factors go back to every shard by copy-engine peer copies
         (cudaMemcpyAsync: no SMs taken from the GEMMs), ordered the same way.
    Every rank passes every flag every step, so a rank with nothing to send still signals.
    A flag that does not arrive within ``PEER_WAIT_LIMIT_NS`` sets the error flag
    (``THORN.device_error()``) instead of hanging the GPU.
    Returns (U, factors, slot, u_ptr, f_ptr) like the NCCL path."""
    md = cfg.decouple_md
    ns_dt = opt.ns_dtype
    ns_code = N.dtype_code(ns_dt)
    esz = torch.empty(0, dtype=ns_dt).element_size()
    cols = [it.C for it in items]

    def pnn_rows(j):
        return cfg.needs_pnn(rows_g[j], cols[j])

    chunks_of = [chunks if r == me else owner_chunks(r) for r in range(world)]
    lay = [peer_layout(r, owners, chunks_of[r], parts, cols, ld, esz, pnn_rows) for r in range(world)]
    arenas = opt.__dict__.setdefault("_peer_arenas", {})
    pa = arenas.setdefault(dev, PeerArenas())
    pa.ensure(lib, max(l[3] for l in lay), ranks, me, group, dev)
    epoch = opt.__dict__.get("_peer_epoch", 0) + 1
    opt._peer_epoch = epoch
    limit = int(getattr(opt, "peer_wait_limit_ns", PEER_WAIT_LIMIT_NS))
    where = {}  # j -> (chunk index, position) in its owner's chunk list
    for r in range(world):
        for ci, ch in enumerate(chunks_of[r]):
            for k, j in enumerate(ch[4]):
                where[j] = (ci, k)

    # 2+3. normalised rows straight into the owners' NS inputs
    casts: dict = {}
    for j, it in enumerate(items):
        r = owners[j]
        ci, k = where[j]
        r0, _n = parts[j][me]
        dst = pa.ptrs[r] + lay[r][0][ci] + (k * rows_g[j] + r0) * ld[j] * esz
        casts.setdefault((it.pdt, it.sdt), []).append(N.NsCastTensor(
            it.g.data_ptr(), _local_of(it.state["moment"]).data_ptr(), arena.ptr(it.normsq), dst,
            it.B, it.R, it.C, arena.ptr(it.rs) if md else None, arena.ptr(it.cs) if md else None,
            1 if (md and not it.split) else 0, 1 if (md and not write_grad) else 0))
    for (pdt, sdt), ts in casts.items():
        udt = pdt if pdt == sdt else torch.float32
        N.check(lib.thorn_ns_cast_multi(N.array(N.NsCastTensor, ts), len(ts), N.dtype_code(pdt), N.dtype_code(sdt),
                                        N.dtype_code(udt), ns_code, b1, stream), "ns_cast_multi")
    mark("gains_and_cast" if md else "cast")
    _signal_and_wait(lib, pa, world, me, 0, 2 * epoch, err, stream, limit)
    mark("exchange_out")

    # 4. Newton-Schulz (+ pnn factors) on the owned, arena-resident inputs
    coeffs = (N.ctypes.c_double * (3 * max(1, cfg.iters)))(*[x for abc in cfg.coeffs[:cfg.iters] for x in abc])
    rs_ = list(cfg.restarts)
    restarts = (N.ctypes.c_int32 * max(1, len(rs_)))(*rs_)
    U, factors, slot = {}, {}, {}
    for ci, (R, C, pdt, sdt, js) in enumerate(chunks):
        nb = len(js)
        for k, j in enumerate(js):
            slot[j] = (ci, k)
        U[ci] = torch.empty((nb, R, C), dtype=ns_dt, device=dev)
        wsb = int(lib.thorn_ns_workspace_bytes(nb, R, C))
        ws = torch.empty(max(256, wsb), dtype=torch.uint8, device=dev)
        if opt.profile_ns is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev0.record()
            f0 = N.gemm_flops()
        N.check(lib.thorn_ns_batched(pa.base + lay[me][0][ci], U[ci].data_ptr(), ws.data_ptr(), wsb, nb, R, C,
                                     ns_code, coeffs, cfg.iters, restarts, len(rs_), err.data_ptr(), stream),
                "ns_batched")
        if opt.profile_ns is not None:
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record()
            f1 = N.gemm_flops()
            opt.profile_ns.append((ev0, ev1, f1[0] - f0[0], f1[1] - f0[1], (nb, R, C)))
        del ws
        if ci in pnn_h:
            rsh, msh = pnn_h[ci]
            (sp,) = opt._scratch(dev, [lib.thorn_pnn_scratch_bytes(nb, R)])
            # the sharded reference runs pnn on fp32 u (thorn.py:1079-1081): no rounding, fp32 eps
            pt = N.PnnTensor(U[ci].data_ptr(), arena.ptr(rsh), arena.ptr(msh), nb, R, C, sp, 1)
            N.check(lib.thorn_pnn_stats_multi(N.array(N.PnnTensor, [pt]), 1, ns_code, N.F32, stream), "pnn_stats")
            factors[ci] = arena.get(rsh).view(nb, R)
    mark("newton_schulz")

    # 5. result rows (+ row factors) to every other shard of each owned matrix
    for ci, (R, C, pdt, sdt, js) in enumerate(chunks):
        for k, j in enumerate(js):
            for s in range(world):
                r0, n = parts[j][s]
                if s == me or n == 0:
                    continue
                src = U[ci].data_ptr() + (k * R + r0) * C * esz
                N.check(lib.thorn_copy_async(pa.ptrs[s] + lay[s][1][j], src, n * C * esz, stream), "copy_async")
                if ci in factors:
                    fsrc = factors[ci].data_ptr() + (k * R + r0) * 4
                    N.check(lib.thorn_copy_async(pa.ptrs[s] + lay[s][2][j], fsrc, n * 4, stream), "copy_async")
    _signal_and_wait(lib, pa, world, me, 64, 2 * epoch + 1, err, stream, limit)
    mark("exchange_back")
    u_ptr = {j: pa.base + off for j, off in lay[me][1].items()}
    f_ptr = {j: pa.base + off for j, off in lay[me][2].items()}
    return U, factors, slot, u_ptr, f_ptr


def _local_of(t):
    return t.to_local() if isinstance(t, DTensor) else t


def _stage_marks(opt):
    """A function that records a named CUDA event on the current stream into this step's
    stage list when ``opt.profile_stages`` is a list, else does nothing."""
    log = getattr(opt, "profile_stages", None)
    if log is None:
        return lambda name: None
    marks = []
    log.append(marks)

    def mark(name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))

    return mark


def _step_matrices(opt, mats, cfg, ranks, group, world, me, dev, Arena, _local, scales):
    from .optimizer import balanced_cap

    lib = N.load()
    stream = N.stream_of(dev)
    mark = _stage_marks(opt)
    mark("start")
    err = opt._err_flag(dev)
    md = cfg.decouple_md
    arena = Arena()
    items = opt._items(mats, cfg, arena, ortho=True, reduce_regions=True)
    b1 = float(cfg.betas[0])
    ns_dt = opt.ns_dtype
    ns_code = N.dtype_code(ns_dt)
    rows_g = [int(p.shape[0]) for p in mats]  # global rows
    parts = [shard_rows(r, world) for r in rows_g]  # (first row, count) of every shard
    # NS input rows (owner buffers and send slabs) use the padded leading dimension the
    # NS kernels need (16-byte TMA rows); results come back unpadded
    ld = [int(lib.thorn_ns_ld(it.C)) for it in items]
    start = getattr(opt, "_owner_start", 0) % world
    owners = assign_owners([ns_flops(rows_g[j], it.C, cfg.iters) for j, it in enumerate(items)], world, start)
    opt._owner_start = start + len(items)  # the same on every rank: every rank steps the same matrices

    def owner_chunks(r):
        """NS batches of owner r: its matrices by (global shape, dtypes), in batches of at
        most polar_decomp_batch_size elements.  Every rank computes every owner's list."""
        buckets: dict = {}
        for j, it in enumerate(items):
            if owners[j] == r:
                buckets.setdefault((rows_g[j], it.C, it.pdt, it.sdt), []).append(j)
        out = []
        for (R, C, pdt, sdt), js in buckets.items():
            cap = max(1, opt.polar_decomp_batch_size // max(1, R * C)) if opt.polar_decomp_batch_size > 0 else 1
            cap = balanced_cap(len(js), cap)
            for i in range(0, len(js), cap):
                out.append((R, C, pdt, sdt, js[i:i + cap]))
        return out

    chunks = owner_chunks(me)
    # Exchange waves.  One wave: every slab moves before any NS starts.  With
    # pipeline_exchange, wave w holds every owner's w-th NS batch: all gathers are
    # queued at once, so later waves' slabs move while the owners compute earlier ones,
    # and each wave's results go back while the next wave computes.
    wave_of = [0] * len(items)
    n_waves = 1
    if getattr(opt, "pipeline_exchange", False) and world > 1:
        for r in range(world):
            cs = chunks if r == me else owner_chunks(r)
            n_waves = max(n_waves, len(cs))
            for w, ch in enumerate(cs):
                for j in ch[4]:
                    wave_of[j] = w
    wave_js = [[j for j in range(len(items)) if wave_of[j] == w] for w in range(n_waves)]
    pnn_h = {}
    for ci, (R, C, pdt, sdt, js) in enumerate(chunks):
        if cfg.needs_pnn(R, C):
            pnn_h[ci] = (arena.empty(len(js) * R), arena.empty(2 * len(js)))
    # a rank whose shard of a matrix has no rows (fewer rows than ranks) launches no block for
    # it, so that matrix's entries of the all-reduced sums start at zero
    arena.materialize(dev, zero=("red1", "red2") if any(it.R == 0 for it in items) else ())

    # 1. momentum pass on local rows, then one all-reduce of the partial sums
    if md:
        opt._md_prep(items, arena, new=False, stream=stream)
    write_grad = 1 if (md and not cfg.none_grad) else 0
    scr = opt._scratch(dev, [lib.thorn_ortho_pre_scratch_bytes(it.B, it.R, it.C, 1 if md else 0) for it in items])
    by_dt: dict = {}
    for it, sp in zip(items, scr):
        by_dt.setdefault((it.pdt, it.sdt), []).append(N.OrthoPreTensor(
            it.p.data_ptr() if md else None, it.g.data_ptr(), _local(it.state["moment"]).data_ptr(),
            arena.ptr(it.normsq), it.B, it.R, it.C, arena.ptr(it.rs) if md else None,
            arena.ptr(it.cs) if md else None, 1 if (md and not it.split) else 0,
            arena.ptr(it.rgs) if md else None, arena.ptr(it.cgs) if md else None, sp))
    ev = opt._profile_start(opt.profile_momentum)
    for (pdt, sdt), ts in by_dt.items():
        udt = pdt if pdt == sdt else torch.float32
        N.check(lib.thorn_ortho_pre_multi(N.array(N.OrthoPreTensor, ts), len(ts), N.dtype_code(pdt),
                                          N.dtype_code(sdt), N.dtype_code(udt), b1, 1 if md else 0, write_grad,
                                          stream), "ortho_pre_multi")
    opt._profile_end(opt.profile_momentum, ev, opt._momentum_bytes(items, md))
    mark("momentum")
    dist.all_reduce(arena.region("red1"), group=group)
    mark("all_reduce")
    if md:
        opt._md_gains(items, cfg, arena, stream)

    def _nccl_exchange_and_ns():
        """Steps 2-5 with NCCL exchanges: (U, factors, slot, u_ptr, f_ptr) for the apply."""
        # 2. normalised rows -> owner buffers / send slabs
        X = {}
        U = {}
        slot = {}  # j -> (chunk index, position in chunk)
        for ci, (R, C, pdt, sdt, js) in enumerate(chunks):
            X[ci] = torch.empty((len(js), R, ld[js[0]]), dtype=ns_dt, device=dev)
            U[ci] = torch.empty((len(js), R, C), dtype=ns_dt, device=dev)
            for k, j in enumerate(js):
                slot[j] = (ci, k)
        # send slabs grouped by owner (matrix index ascending within an owner): each
        # round's message to one owner is then one contiguous range of this buffer
        send_rows = {}
        n_send = sum(it.R * ld[j] for j, it in enumerate(items) if owners[j] != me)
        send_buf = torch.empty(max(1, n_send), dtype=ns_dt, device=dev)
        off = 0
        for j in sorted((j for j in range(len(items)) if owners[j] != me), key=lambda j: (owners[j], j)):
            it = items[j]
            send_rows[j] = send_buf[off:off + it.R * ld[j]].view(it.R, ld[j])
            off += it.R * ld[j]

        def owner_rows(j, s):
            ci, k = slot[j]
            r0, n = parts[j][s]
            return X[ci][k, r0:r0 + n]

        casts: dict = {}
        for j, it in enumerate(items):
            dst = owner_rows(j, me) if owners[j] == me else send_rows[j]
            casts.setdefault((it.pdt, it.sdt), []).append(N.NsCastTensor(
                it.g.data_ptr(), _local(it.state["moment"]).data_ptr(), arena.ptr(it.normsq), dst.data_ptr(),
                it.B, it.R, it.C, arena.ptr(it.rs) if md else None, arena.ptr(it.cs) if md else None,
                1 if (md and not it.split) else 0, 1 if (md and not write_grad) else 0))
        for (pdt, sdt), ts in casts.items():
            udt = pdt if pdt == sdt else torch.float32
            N.check(lib.thorn_ns_cast_multi(N.array(N.NsCastTensor, ts), len(ts), N.dtype_code(pdt), N.dtype_code(sdt),
                                            N.dtype_code(udt), ns_code, b1, stream), "ns_cast_multi")
        mark("gains_and_cast" if md else "cast")

        xchg = exchange if getattr(opt, "exchange", "all_to_all") == "rounds" else exchange_all_to_all
        # 3. slabs to owners: every wave's exchange is queued now (the NCCL stream runs them
        # in order); each NS batch waits only for its own wave
        gathers = []
        for js in wave_js:
            sends, recvs = plan_gather(owners, me, world, lambda j: send_rows[j], owner_rows, subset=js)
            gathers.append(xchg(sends, recvs, ranks, group, wait=False))

        # 5. (buffers) result rows (+ row factors) come back to every shard
        u_loc, f_loc = {}, {}
        for j, it in enumerate(items):
            if owners[j] != me:
                u_loc[j] = torch.empty((it.R, it.C), dtype=ns_dt, device=dev)
                if cfg.needs_pnn(rows_g[j], it.C):
                    f_loc[j] = torch.empty(it.R, dtype=torch.float32, device=dev)
        factors = {}

        def owner_parts(j, s):
            ci, k = slot[j]
            r0, n = parts[j][s]
            out = [U[ci][k, r0:r0 + n]]
            if ci in factors:
                out.append(factors[ci][k, r0:r0 + n])
            return out

        def my_parts(j):
            return [u_loc[j]] + ([f_loc[j]] if j in f_loc else [])

        # 4. Newton-Schulz (+ pnn factors) on owned matrices, wave by wave, and 5. each
        # wave's results back to their shards
        coeffs = (N.ctypes.c_double * (3 * max(1, cfg.iters)))(*[x for abc in cfg.coeffs[:cfg.iters] for x in abc])
        rs_ = list(cfg.restarts)
        restarts = (N.ctypes.c_int32 * max(1, len(rs_)))(*rs_)
        scatters = []
        for w, js_w in enumerate(wave_js):
            gathers[w].wait()  # the current stream waits; the host does not
            if n_waves == 1:
                mark("exchange_out")
            for ci, (R, C, pdt, sdt, js) in enumerate(chunks):
                if wave_of[js[0]] != w:
                    continue
                nb = len(js)
                wsb = int(lib.thorn_ns_workspace_bytes(nb, R, C))
                ws = torch.empty(max(256, wsb), dtype=torch.uint8, device=dev)
                if opt.profile_ns is not None:
                    ev0 = torch.cuda.Event(enable_timing=True)
                    ev0.record()
                    f0 = N.gemm_flops()
                N.check(lib.thorn_ns_batched(X[ci].data_ptr(), U[ci].data_ptr(), ws.data_ptr(), wsb, nb, R, C, ns_code,
                                             coeffs, cfg.iters, restarts, len(rs_), err.data_ptr(), stream), "ns_batched")
                if opt.profile_ns is not None:
                    ev1 = torch.cuda.Event(enable_timing=True)
                    ev1.record()
                    f1 = N.gemm_flops()
                    opt.profile_ns.append((ev0, ev1, f1[0] - f0[0], f1[1] - f0[1], (nb, R, C)))
                del ws
                X[ci] = None
                if ci in pnn_h:
                    rsh, msh = pnn_h[ci]
                    (sp,) = opt._scratch(dev, [lib.thorn_pnn_scratch_bytes(nb, R)])
                    # the sharded reference runs pnn on fp32 u (thorn.py:1079-1081): no rounding, fp32 eps
                    pt = N.PnnTensor(U[ci].data_ptr(), arena.ptr(rsh), arena.ptr(msh), nb, R, C, sp, 1)
                    N.check(lib.thorn_pnn_stats_multi(N.array(N.PnnTensor, [pt]), 1, ns_code, N.F32, stream),
                            "pnn_stats")
                    factors[ci] = arena.get(rsh).view(nb, R)
            if n_waves == 1:
                mark("newton_schulz")
            sends, recvs = plan_scatter(owners, me, world, owner_parts, my_parts, subset=js_w)
            scatters.append(xchg(sends, recvs, ranks, group, wait=False))
        for ex in scatters:
            ex.wait()
        mark("exchange_back" if n_waves == 1 else "exchange_and_newton_schulz")
        del X, send_buf, send_rows
        keep.extend([u_loc, f_loc])
        return (U, factors, slot, {j: t.data_ptr() for j, t in u_loc.items()},
                {j: t.data_ptr() for j, t in f_loc.items()})

    keep = []  # the NCCL path's receive buffers live until the apply has been enqueued
    if getattr(opt, "exchange", "all_to_all") == "peer" and world > 1:
        # 2-5 over peer memory: rows stored into the owners' arenas, results copied back
        U, factors, slot, u_ptr, f_ptr = peer_exchange_and_ns(
            opt, lib, items, chunks, owner_chunks, owners, parts, rows_g, ld, world, me, ranks, group, dev, stream,
            arena, cfg, err, pnn_h, b1, write_grad, mark)
    else:
        U, factors, slot, u_ptr, f_ptr = _nccl_exchange_and_ns()

    # 6. apply on local rows
    scr = opt._scratch(dev, [lib.thorn_sumsq_scratch_bytes(it.B, it.R, it.C) if md else 0 for it in items])
    posts: dict = {}
    for j, (it, sp) in enumerate(zip(items, scr)):
        if owners[j] == me:
            ci, k = slot[j]
            r0, n = parts[j][me]
            uj = U[ci][k, r0:r0 + n].data_ptr()
            fj = factors[ci][k, r0:r0 + n].data_ptr() if ci in factors else None
        else:
            uj, fj = u_ptr.get(j), f_ptr.get(j)  # none when this rank's shard of j is empty
        lr_eff = float(cfg.lr) * cfg.lr_scale(rows_g[j], it.C) * scales[j]
        posts.setdefault(it.pdt, []).append(N.OrthoPostTensor(
            uj, it.p.data_ptr(), fj, None,
            arena.ptr(it.pnorm) if md else None, it.B, it.R, it.C, lr_eff, sp if md else None, 0))
    for pdt, ts in posts.items():
        N.check(lib.thorn_ortho_post_multi(N.array(N.OrthoPostTensor, ts), len(ts), ns_code, N.dtype_code(pdt),
                                           float(cfg.weight_decay), stream), "ortho_post_multi")
    mark("apply")
    if md:
        dist.all_reduce(arena.region("red2"), group=group)
        opt._md_prep(items, arena, new=True, stream=stream)
        opt._md_finalize(items, arena, lambda it: True, stream)
        mark("md_renorm")
    del U, keep
    opt._finish(mats, cfg)
