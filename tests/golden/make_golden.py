"""Generate golden vectors by running the reference THORN optimizer on CPU.

Usage (in a container where the reference checkout is available):

    python tests/golden/make_golden.py --ref /path/to/THORN [case ...]

Each case in ``tests/cases.py`` is stepped with the reference's own
``thorn.THORN`` (its eager CPU path: Triton and torch.compile are off on CPU).
For every parameter the fixture stores, after step 1 and after the last step,
the parameter and each optimizer-state tensor: in full when small, otherwise a
checksum (sum, sum of squares, projection on ``cases.probe_vector``) and the
first 1024 values.  Inputs are not stored; they are rebuilt from seeds.

The reference's Polar-Express coefficients and Gram-NS restarts for a few
(lower_bound, iters, safety_factor, cushion) settings are stored too.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import cases as C  # noqa: E402

FULL_LIMIT = 20000
SLICE = 1024
# the many-matrix VAD case keeps checksums and short heads only
LIMITS = {"vad": (256, 256)}


def _np(t: torch.Tensor) -> np.ndarray:
    if t.is_sparse:
        t = t.to_dense()
    return t.detach().to(torch.float32).cpu().numpy().copy()


def _store(out: dict, key: str, t, limits=(FULL_LIMIT, SLICE)):
    a = _np(t) if isinstance(t, torch.Tensor) else np.asarray(t, dtype=np.float32)
    if a.size <= limits[0]:
        out[key + "/full"] = a
    else:
        out[key + "/sum"] = C.checksum(a)
        out[key + "/head"] = a.reshape(-1)[:limits[1]].copy()
    out[key + "/shape"] = np.asarray(a.shape, dtype=np.int64)


def run_case(THORN, name: str) -> dict:
    case = C.CASES[name]
    params = C.build_params(case)
    torch_params = [[torch.nn.Parameter(t.clone()) for t in ps] for ps in params]
    opt = THORN(C.group_dicts(case, torch_params))
    opt._update_rate = case.get("update_rate", 1)  # what setup_gradient_release(update_rate=...) sets
    out = {}
    lim = LIMITS.get(name, (FULL_LIMIT, SLICE))
    g0 = C.build_grads(case, 0)
    out["input/grad0_sum"] = np.array([C.checksum(_np(t)) for ps in g0 for t in ps])
    out["input/param_sum"] = np.array([C.checksum(_np(t)) for ps in params for t in ps])
    for s in range(case["steps"]):
        grads = C.build_grads(case, s)
        for ps, gs in zip(torch_params, grads):
            for p, g in zip(ps, gs):
                p.grad = g.clone()
        opt.step()
        if s == 0 or s == case["steps"] - 1:
            tag = "step1" if s == 0 else "final"
            for gi, ps in enumerate(torch_params):
                for pi, p in enumerate(ps):
                    base = f"{tag}/g{gi}/p{pi}"
                    _store(out, base + "/param", p.data, lim)
                    if p.grad is not None:  # groups with none_grad=False keep it (MD: recovered)
                        _store(out, base + "/grad_after", p.grad, lim)
                    for k, v in opt.state[p].items():
                        if isinstance(v, torch.Tensor):
                            _store(out, f"{base}/{k}", v, lim)
                        elif isinstance(v, int) and v >= 1 << 63:
                            out[f"{base}/{k}"] = np.asarray(v, dtype=np.uint64)  # Magma generator state
                        else:
                            out[f"{base}/{k}"] = np.asarray(v)
    return out


def coeff_table(mod) -> dict:
    out = {}
    settings = [(1e-3, 5, 0.03, 0.02), (1e-3, 8, 0.03, 0.02), (1e-2, 5, 0.0, 0.0), (1e-3, 6, 0.05, 0.1)]
    for i, (l, it, sf, cu) in enumerate(settings):
        co = mod._optimal_composition(l=l, num_iters=it, safety_factor_eps=sf, cushion=cu)
        out[f"coeffs/{i}/setting"] = np.array([l, it, sf, cu], dtype=np.float64)
        out[f"coeffs/{i}/values"] = np.array(co, dtype=np.float64)
        out[f"coeffs/{i}/restarts"] = np.array(mod._gram_ns_restarts(*co), dtype=np.int64)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference THORN checkout")
    ap.add_argument("cases", nargs="*")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import thorn.thorn as mod  # the reference implementation
    torch.set_num_threads(os.cpu_count() or 1)
    np.savez_compressed(os.path.join(HERE, "coeffs.npz"), **coeff_table(mod))
    names = args.cases or [n for n in C.CASES]
    for n in names:
        data = run_case(mod.THORN, n)
        np.savez_compressed(os.path.join(HERE, f"{n}.npz"), **data)
        print(n, len(data), "arrays")


if __name__ == "__main__":
    main()
