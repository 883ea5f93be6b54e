"""Pin the CPU port's speed to the reference's own CPU step (test infrastructure).

    python oracle/time_reference.py [--reference-path DIR] [--out FILE]

``bench.py``'s CPU baseline times the numpy port (``oracle/thorn_oracle.py``) on
a bounded sample of the Llama-3-8B step and extrapolates it, because the
reference is a Python package that does not exist on the GPU box.  This script
runs where the reference can be imported (it reads it from ``--reference-path``)
and times, on the same host cores and the same sample shapes, both the
reference's ``thorn.THORN.step`` (its eager CPU path: thorn.py:1583-1732) and the
port's step.  The ratio reference / port says how the port's figure relates to
the reference's own CPU step.  The result is one JSON line (and, with ``--out``,
a Markdown summary).

The sample is the one ``bench.py`` uses: one 4096x4096, one 1024x4096 and one
14336x4096 orthogonalized matrix with decouple_md, a 4096-row slice of the
128256x4096 embedding and one norm vector in the (R)AdamW group.  The reference
keeps its state in the parameter dtype (thorn.py:1596-1599), so both sides run
fp32 parameters and state here (the bf16 / fp32-state mix of the bench is an
option of this build only); each piece is timed over one step after its state
exists, like the bench.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

HIDDEN, KV, FFN, EMB_ROWS = 4096, 1024, 14336, 4096
PIECES = [("ortho", (HIDDEN, HIDDEN)), ("ortho", (KV, HIDDEN)), ("ortho", (FFN, HIDDEN)),
          ("adamw", (EMB_ROWS, HIDDEN)), ("adamw", (HIDDEN,))]


def _inputs(shape, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape, dtype=np.float32) * 0.02,
            rng.standard_normal(shape, dtype=np.float32) * 1e-4)


def time_reference(kind, shape, seed, md=True, lr=8e-3):
    """One step of the reference's THORN on one parameter (state created by a first step).
    ``md``: decouple_md on an orthogonalized parameter (else the default moonlight scaling)."""
    import torch
    from thorn import THORN

    p0, g0 = _inputs(shape, seed)
    p = torch.nn.Parameter(torch.from_numpy(p0.copy()))
    group = {"orthogonalize": kind == "ortho", "params": [p], "lr": lr}
    if kind == "ortho" and md:
        group["decouple_md"] = True
    opt = THORN([group], backend=torch.cpu)
    p.grad = torch.from_numpy(g0.copy())
    opt.step()  # state creation and first-call costs outside the timed step
    p.grad = torch.from_numpy(g0.copy())
    t0 = time.perf_counter()
    opt.step()
    return time.perf_counter() - t0


def time_port(kind, shape, seed):
    """The same step of the numpy port (oracle/thorn_oracle.py)."""
    from oracle.thorn_oracle import OracleTHORN

    p0, g0 = _inputs(shape, seed)
    group = {"orthogonalize": kind == "ortho", "lr": 8e-3, "dtype": "f32", "params": [p0.copy()]}
    if kind == "ortho":
        group["decouple_md"] = True
    orc = OracleTHORN([group])
    orc.step([[g0.copy()]])
    t0 = time.perf_counter()
    orc.step([[g0.copy()]])
    return time.perf_counter() - t0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-path", default=os.environ.get("THORN_REFERENCE_PATH", ""),
                    help="directory that holds the reference's `thorn` package")
    ap.add_argument("--out", default=None,
                    help="write a Markdown summary here, and the JSON line beside it (same name, .json)")
    args = ap.parse_args()
    if not args.reference_path or not os.path.isdir(os.path.join(args.reference_path, "thorn")):
        raise SystemExit("--reference-path must name the directory holding the reference's thorn package")
    sys.path.insert(0, args.reference_path)
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    rows = []
    for i, (kind, shape) in enumerate(PIECES):
        tr = time_reference(kind, shape, i)
        tp = time_port(kind, shape, i)
        rows.append({"piece": f"{kind} {'x'.join(map(str, shape))}", "reference_s": round(tr, 3),
                     "port_s": round(tp, 3), "reference_over_port": round(tr / tp, 3)})
        print(json.dumps(rows[-1]), flush=True)
    tot_r = sum(r["reference_s"] for r in rows)
    tot_p = sum(r["port_s"] for r in rows)
    cpu = ""
    try:
        with open("/proc/cpuinfo") as f:
            cpu = next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), "")
    except OSError:
        pass
    summary = {"threads": torch.get_num_threads(), "cpu": cpu, "torch": torch.__version__,
               "sample_reference_s": round(tot_r, 3), "sample_port_s": round(tot_p, 3),
               "reference_over_port": round(tot_r / tot_p, 3), "pieces": rows}
    print(json.dumps(summary), flush=True)
    if args.out:
        with open(os.path.splitext(args.out)[0] + ".json", "w") as f:
            f.write(json.dumps(summary) + "\n")
        with open(args.out, "w") as f:
            f.write("# CPU step: the reference's thorn.THORN against the numpy port\n\n")
            f.write("Command: `python oracle/time_reference.py --reference-path <dir holding thorn/> "
                    f"--out {args.out}`\n\n")
            f.write(f"Host: {cpu}, {summary['threads']} torch threads, torch {torch.__version__}. fp32 "
                    "parameters and state (the reference keeps state in the parameter dtype); one step per "
                    "piece after its state exists; decouple_md on the orthogonalized matrices, lr 8e-3.\n\n")
            f.write("| piece | reference s | port s | reference / port |\n|---|---:|---:|---:|\n")
            for r in rows:
                f.write(f"| {r['piece']} | {r['reference_s']} | {r['port_s']} | {r['reference_over_port']} |\n")
            f.write(f"| **sample total** | **{summary['sample_reference_s']}** | **{summary['sample_port_s']}** "
                    f"| **{summary['reference_over_port']}** |\n")


if __name__ == "__main__":
    main()
