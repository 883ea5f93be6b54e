"""Comparison helpers shared by the oracle pin tests and the GPU parity tests."""
from __future__ import annotations

import math

import numpy as np

import cases as C


def magma_stats_cpu(items, cfg, recovered):
    """CPU stand-in for ``thorn_magma_stats_multi`` in host-logic tests (the kernel needs a
    GPU): ``THORN._magma_stats``'s [n, 3] fp64 sums (g*m, g^2, m^2) of each item, the
    gradient recovered as g * gain in its own dtype under decouple_md, as the kernel's
    contract states."""
    import torch
    import torch.nn.functional as F

    from thorn_b200.optimizer import _local

    rows = []
    for it in items:
        g, st = it.g, it.state
        m = getattr(it, "m_rows", None)
        m = _local(st["moment"]) if m is None else m
        if recovered and cfg.decouple_md:
            if it.split:
                gain = F.softplus(_local(st["row_gain"])) * F.softplus(_local(st["col_gain"]))
            else:
                gain = F.softplus(_local(st["gain"]))
            g = g * gain
        g, m = g.double().flatten(), m.double().flatten()
        rows.append(torch.stack([(g * m).sum(), (g * g).sum(), (m * m).sum()]))
    return torch.stack(rows)


def load_golden(path: str) -> dict:
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def run_oracle(name: str, steps: int | None = None, state_dtype: str | None = None, cpu_quirks: bool = False,
               seeds: list | None = None, sharded: bool = False):
    """Step the CPU oracle on a case; returns (oracle, snapshots{tag: (params, states)}).

    ``cpu_quirks`` models the reference's eager CPU path (used to pin the oracle
    against the golden vectors, which were produced on CPU); otherwise the
    oracle models the reference's CUDA path (fused fp32 Triton kernels).
    ``seeds``: the Magma seeds in initialisation order (default: drawn from
    torch's CPU generator exactly where the reference draws them).
    """
    from oracle import thorn_oracle as O
    from oracle.thorn_oracle import OracleTHORN

    O.CPU_EAGER = cpu_quirks

    case = C.CASES[name]
    params = C.build_params(case)
    groups = []
    for grp, ps in zip(case["groups"], params):
        d = {"orthogonalize": grp["orthogonalize"], "dtype": grp["dtype"], **grp["opts"]}
        if state_dtype:
            d["state_dtype"] = state_dtype
        d["params"] = [t.float().numpy() for t in ps]
        groups.append(d)
    seed_fn = C.magma_seed if seeds is None else iter(list(seeds)).__next__
    orc = OracleTHORN(groups, seed_fn=seed_fn, sharded=sharded)
    orc.update_rate = case.get("update_rate", 1)
    n = case["steps"] if steps is None else steps
    snaps = {}
    for s in range(n):
        grads = C.build_grads(case, s)
        orc.step([[oracle_grad(t) for t in gs] for gs in grads])
        if s == 0 or s == n - 1:
            tag = "step1" if s == 0 else "final"
            snaps[tag] = (
                [[p.copy() for p in g.params] for g in orc.groups],
                [[{**{k: (np.array(v, copy=True) if isinstance(v, np.ndarray) else v) for k, v in st.items()},
                   **({"grad_after": np.array(g.grad_after[i], copy=True)} if i in g.grad_after else {})}
                  for i, st in enumerate(g.state)] for g in orc.groups],
            )
    return orc, snaps


def oracle_grad(t):
    """A torch gradient as the oracle takes it: float32 array, or ``SparseRows``."""
    from oracle.thorn_oracle import SparseRows

    if t.is_sparse:
        return SparseRows(t._indices()[0].numpy(), t._values().float().numpy())
    return t.float().numpy()


def compare_tensor(mine: np.ndarray, gold: dict, key: str, base: np.ndarray | None = None):
    """Relative error of ``mine`` (minus ``base``) against a golden entry.

    Returns the worst of: relative Frobenius error over the stored values
    (full array or head), and the checksum bound |d proj| / (||d|| ||r||).
    """
    mine = np.asarray(mine)
    b = np.zeros(mine.shape, dtype=np.float32) if base is None else np.asarray(base)
    if key + "/full" in gold:
        mine, b = mine.astype(np.float64), b.astype(np.float64)
        ref = gold[key + "/full"].astype(np.float64).reshape(mine.shape)
        return C.rel_fro(mine - b, ref - b)
    # large tensors: the head in full, the rest through checksums (float64, accumulated
    # over blocks; no tensor-sized temporaries)
    head = gold[key + "/head"].astype(np.float64)
    n = head.size
    mh = mine.reshape(-1)[:n].astype(np.float64)
    bh = b.reshape(-1)[:n].astype(np.float64)
    e1 = C.rel_fro(mh - bh, head - bh)
    cs_ref = gold[key + "/sum"]
    cs_mine = C.checksum(mine)
    cs_base = C.checksum(b)
    scale = math.sqrt(C.sq_dist(mine, b)) * math.sqrt(C.probe_norm_sq(mine.size))
    e2 = abs((cs_mine[2] - cs_base[2]) - (cs_ref[2] - cs_base[2])) / max(scale, 1e-30)
    sq_scale = max(float(cs_mine[1]), 1e-30)
    e3 = abs(cs_mine[1] - cs_ref[1]) / sq_scale if base is None else 0.0
    return max(e1, e2, e3)


def compare_run(name: str, gold: dict, snaps: dict, init_params):
    """Per (tag, group, param, key) relative errors; params compared as cumulative updates."""
    errs = {}
    for tag, (params, states) in snaps.items():
        for gi, (ps, sts) in enumerate(zip(params, states)):
            for pi, (p, st) in enumerate(zip(ps, sts)):
                base = f"{tag}/g{gi}/p{pi}"
                errs[(tag, gi, pi, "param")] = compare_tensor(p, gold, base + "/param", init_params[gi][pi])
                for k, v in st.items():
                    if k in ("step", "random_state"):  # integers: exact (Magma's generator state too)
                        assert int(v) == int(gold[f"{base}/{k}"]), (base, k, int(v), int(gold[f"{base}/{k}"]))
                        continue
                    if isinstance(v, np.ndarray) or np.isscalar(v):
                        errs[(tag, gi, pi, k)] = compare_tensor(np.asarray(v, dtype=np.float32), gold, f"{base}/{k}")
    return errs
