#!/usr/bin/env python
"""THORN.step benchmark on the Llama-3-8B-shaped parameter set.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl thorn_b200|reference|reference_gpu]

For N > 1 launch one process per GPU with torch.distributed.run; parameters
are then DTensors sharded Shard(0) over the ranks (FSDP2 layout) and the
orthogonalized group takes the sharded path.  ``--model llama70b`` runs
BASELINE configs[4] instead (80 layers, hidden 8192, moonlight scaling; 8 GPUs).

Workload: 32 layers, hidden 4096; per layer q/o
4096x4096, k/v 1024x4096, gate/up 14336x4096, down 4096x14336 in the
orthogonalized group (decouple_md=True, lr=8e-3); embedding and lm_head
128256x4096 plus 65 RMSNorm weights of 4096 in the (R)AdamW group.  bf16
params ~N(0, 0.02), bf16 grads ~N(0, 1e-4), fp32 optimizer state.  Synthetic
data; every input is far larger than L2, so no L2 flush is needed.

One line of JSON on rank 0:
* value / ms_per_step: device time of one full optimizer step (CUDA events,
  max over ranks), inputs resident in HBM;
* e2e: the same step through the public API with every step's grads copied in
  from pinned host memory and its updated params copied back out, inside the
  timed region; by default through thorn_b200.PinnedStepper, which overlaps the
  copies of one step with the compute of its neighbours on two copy streams
  (``--e2e-mode serial``: copy in, step, copy out, one after the other);
* roofline: Newton-Schulz GEMM phase, dense-equivalent FLOPs / event time,
  against the measured sustained bf16 peak;
* cpu_baseline: the reference's own CPU step (thorn.THORN from its install
  under baseline/_ref, made by oracle/install_reference.sh; the numpy port of
  the oracle when it is not installed) on a bounded sample (one q, k and gate
  matrix, an embedding slice and a norm vector), extrapolated to the full set.
``--impl reference`` times that CPU step alone (rank 0; other ranks exit).
``--impl reference_gpu`` times the reference's own GPU step (its Triton kernels
and torch.compile Newton-Schulz) on cuda:0 on the same parameter set.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, HIDDEN, KV, FFN, VOCAB = 32, 4096, 1024, 14336, 128256
LAYER_SHAPES = [(HIDDEN, HIDDEN), (KV, HIDDEN), (KV, HIDDEN), (HIDDEN, HIDDEN), (FFN, HIDDEN), (FFN, HIDDEN),
                (HIDDEN, FFN)]
ORTHO_LR, ADAM_LR = 8e-3, 8e-3
MD = True  # decouple_md on the orthogonalized group
METRIC = "THORN.step ms, Llama-3-8B shapes"
WORKLOAD = "llama3-8b-fsdp2 (BASELINE configs[3])"


def use_llama70b():
    """80 layers, hidden 8192, gate/up 28672; scaling_mode moonlight
    without decouple_md.  Fits 8 GPUs (about 72 GB of params, grads and state per rank)."""
    global LAYERS, HIDDEN, KV, FFN, LAYER_SHAPES, ORTHO_LR, ADAM_LR, MD, METRIC, WORKLOAD
    LAYERS, HIDDEN, KV, FFN = 80, 8192, 1024, 28672
    LAYER_SHAPES = [(HIDDEN, HIDDEN), (KV, HIDDEN), (KV, HIDDEN), (HIDDEN, HIDDEN), (FFN, HIDDEN), (FFN, HIDDEN),
                    (HIDDEN, FFN)]
    ORTHO_LR, ADAM_LR, MD = 1e-3, 1e-3, False
    METRIC = "THORN.step ms, Llama-3-70B shapes"
    WORKLOAD = "llama3-70b-fsdp2 (BASELINE configs[4])"


# DRAM bytes (read + write) of one ns_gemm2_kernel launch from an ncu capture of
# X X^T on two 4096x4096 matrices (K = 4096), whose compulsory traffic is 67 MB
# read + 67 MB written.
NS_GEMM_TRAFFIC = 101.5e6
NS_GEMM_TRAFFIC_CASE = "one X X^T launch on 2 x 4096x4096 (K=4096); compulsory 67 MB read + 67 MB write"


def shapes(layers=None):
    layers = LAYERS if layers is None else layers
    ortho = [s for _ in range(layers) for s in LAYER_SHAPES]
    adamw = [(VOCAB, HIDDEN), (VOCAB, HIDDEN)] + [(HIDDEN,)] * (2 * layers + 1)
    return ortho, adamw


def dense_ns_flops(r, c, iters=5):
    m, n = min(r, c), max(r, c)
    if m == n:
        return iters * (4 * m * m * n + 2 * m ** 3)
    return 28 * m ** 3 + 8 * m * m * n


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return pk["hbm_gbs"], pk["bf16_tflops"], pk["bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, ids):
        self.ids = ids
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.ids:
            cmd += ["-i", ",".join(self.ids)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------- CPU baseline
def cpu_oracle_sample(warm_only: bool = False):
    """Time the CPU oracle on a bounded sample and extrapolate to one full step (ms).

    ``warm_only``: run the two smallest pieces only (thread pools and allocator
    warm-up for the reference arm's warm-up steps); returns None."""
    import numpy as np

    from oracle.thorn_oracle import OracleTHORN

    rng = np.random.default_rng(0)
    ortho_lr, adam_lr = ORTHO_LR, ADAM_LR

    def timed(group, shapes_):
        params = [(rng.standard_normal(s, dtype=np.float32) * 0.02) for s in shapes_]
        grads = [(rng.standard_normal(s, dtype=np.float32) * 1e-4) for s in shapes_]
        g = dict(group)
        g["params"] = params
        orc = OracleTHORN([g])
        for i in range(len(params)):  # state creation outside the timed region
            orc._init_state(orc.groups[0], i)
        t0 = time.perf_counter()
        orc.step([grads])
        return time.perf_counter() - t0

    og = {"orthogonalize": True, "lr": ortho_lr, "decouple_md": MD, "dtype": "bf16", "state_dtype": "f32"}
    ag = {"orthogonalize": False, "lr": adam_lr, "dtype": "bf16", "state_dtype": "f32"}
    if warm_only:
        timed(og, [(KV, HIDDEN)])
        timed(ag, [(HIDDEN,)])
        return None
    t_sq = timed(og, [(HIDDEN, HIDDEN)])
    t_kv = timed(og, [(KV, HIDDEN)])
    t_ffn = timed(og, [(FFN, HIDDEN)])
    emb_rows = 4096
    t_emb = timed(ag, [(emb_rows, HIDDEN)])
    t_norm = timed(ag, [(HIDDEN,)])
    total = (LAYERS * (2 * t_sq + 2 * t_kv + 3 * t_ffn) + 2 * (VOCAB / emb_rows) * t_emb
             + (2 * LAYERS + 1) * t_norm)
    sample = (f"one {HIDDEN}x{HIDDEN}, one {KV}x{HIDDEN} and one {FFN}x{HIDDEN} orthogonalized matrix "
              f"({'decouple_md' if MD else 'moonlight'}), a {emb_rows}x{HIDDEN} embedding slice and one norm "
              f"vector; sum scaled to {LAYERS} layers + 2 x {VOCAB}-row embeddings + {2 * LAYERS + 1} norms "
              "(extrapolated)")
    return total * 1e3, sample, (t_sq + t_kv + t_ffn + t_emb + t_norm)


def cpu_reference_sample(warm_only: bool = False):
    """The reference's own CPU step (thorn.THORN with backend=torch.cpu, its eager
    path: thorn.py:1583-1732) on the same bounded sample as ``cpu_oracle_sample``,
    extrapolated to one full step (ms); None when the reference is not installed
    under baseline/_ref.  fp32 parameters: the reference keeps state in the
    parameter dtype, so this is its fp32-state configuration."""
    if import_reference() is None:
        return None
    import torch

    from oracle.time_reference import time_reference

    torch.set_num_threads(os.cpu_count() or 1)
    if warm_only:
        time_reference("ortho", (KV, HIDDEN), 0, md=MD, lr=ORTHO_LR)
        time_reference("adamw", (HIDDEN,), 0, lr=ADAM_LR)
        return None
    t_sq = time_reference("ortho", (HIDDEN, HIDDEN), 1, md=MD, lr=ORTHO_LR)
    t_kv = time_reference("ortho", (KV, HIDDEN), 2, md=MD, lr=ORTHO_LR)
    t_ffn = time_reference("ortho", (FFN, HIDDEN), 3, md=MD, lr=ORTHO_LR)
    emb_rows = 4096
    t_emb = time_reference("adamw", (emb_rows, HIDDEN), 4, lr=ADAM_LR)
    t_norm = time_reference("adamw", (HIDDEN,), 5, lr=ADAM_LR)
    total = (LAYERS * (2 * t_sq + 2 * t_kv + 3 * t_ffn) + 2 * (VOCAB / emb_rows) * t_emb
             + (2 * LAYERS + 1) * t_norm)
    sample = (f"the reference's thorn.THORN.step (CPU, fp32 params and state) on one {HIDDEN}x{HIDDEN}, one "
              f"{KV}x{HIDDEN} and one {FFN}x{HIDDEN} orthogonalized matrix "
              f"({'decouple_md' if MD else 'moonlight'}), a {emb_rows}x{HIDDEN} embedding slice and one norm "
              f"vector; sum scaled to {LAYERS} layers + 2 x {VOCAB}-row embeddings + {2 * LAYERS + 1} norms "
              "(extrapolated)")
    return total * 1e3, sample, (t_sq + t_kv + t_ffn + t_emb + t_norm), torch.get_num_threads()


def cpu_sample(warm_only: bool = False):
    """One bounded CPU sample of the step: the reference's own thorn.THORN when it is
    installed under baseline/_ref (kind "reference"), else the numpy port (kind "port").
    Returns (ms per full step, sample description, seconds spent, threads, kind)."""
    r = cpu_reference_sample(warm_only)
    if warm_only:
        if import_reference() is None:
            cpu_oracle_sample(warm_only=True)
        return None
    if r is not None:
        v, sample, secs, threads = r
        return v, sample, secs, threads, "reference"
    v, sample, secs = cpu_oracle_sample()
    return v, sample, secs, os.cpu_count() or 1, "port"


def port_calibration():
    """The reference's own CPU step time over the port's on the same sample, measured where the
    reference can be imported (oracle/time_reference.py; committed under profiles/), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "cpu_reference_vs_port.json")) as f:
            cal = json.load(f)
        return float(cal["reference_over_port"]), f"{cal.get('threads')} threads of {cal.get('cpu', '?')}"
    except (OSError, ValueError, KeyError):
        return None


def cpu_baseline_entry(v, sample, cores, kind="port", extra=None) -> dict:
    """The cpu_baseline object.  For the port, the reference-equivalent figure is added
    when the port has been timed against the reference itself."""
    d = {"value": round(v, 3), "unit": "ms", "cores": cores, "kind": kind, "sample": sample}
    cal = port_calibration() if kind == "port" else None
    if cal is not None:
        d["reference_over_port"] = cal[0]
        d["reference_equivalent_ms"] = round(v * cal[0], 3)
        d["calibration"] = (f"the reference's thorn.THORN.step / the port's step on the same sample, timed on "
                            f"{cal[1]} (profiles/cpu_reference_vs_port.md)")
    d.update(extra or {})
    return d


def reference_arm(args, rank):
    if rank != 0:
        return
    if args.model != "llama8b":
        print(json.dumps({"impl": "reference", "unavailable": "the CPU sample covers the llama8b set only (one "
                          "28672x8192 Newton-Schulz takes hours on the host cores)"}), flush=True)
        return
    vals = []
    sample, cores, kind = "", os.cpu_count() or 1, "port"
    for _ in range(args.warmup):  # warm-up steps: the sample's small pieces only
        cpu_sample(warm_only=True)
    for _ in range(args.steps):
        v, sample, _, cores, kind = cpu_sample()
        vals.append(v)
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "ms", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 3), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": bench_config(args, int(os.environ.get("WORLD_SIZE", "1"))),
            "cpu_baseline": cpu_baseline_entry(v, sample, cores, kind),
            "e2e": {"value": round(v, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def import_reference():
    """The reference's ``thorn`` package from its install under baseline/_ref
    (``oracle/install_reference.sh``), or None when it is not installed."""
    if not os.path.isfile(os.path.join(REF_DIR, "thorn", "thorn.py")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import thorn

    return thorn


def reference_gpu_arm(args, rank):
    """The reference's own GPU step (Triton kernels and torch.compile Newton-Schulz,
    thorn.py:53-377, 387-423, 1427-1457) on cuda:0, same parameter set and groups
    as the GPU arm.  The reference keeps optimizer state in the parameter dtype
    (thorn.py:1596-1599), so its state is bf16 here where this build's is fp32."""
    if rank != 0:
        return
    ref = import_reference()
    if ref is None:
        print(json.dumps({"impl": "reference_gpu", "unavailable": "no reference install under baseline/_ref"}),
              flush=True)
        return
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ortho, adamw, g_ortho, g_adam = build_params(torch, dev, 0, 1, None, args.layers)
    params, grads = ortho + adamw, g_ortho + g_adam
    opt = ref.THORN([
        {"orthogonalize": True, "params": ortho, "lr": ORTHO_LR, "decouple_md": MD},
        {"orthogonalize": False, "params": adamw, "lr": ADAM_LR},
    ])

    def feed():
        for p, g in zip(params, grads):
            p.grad = g.clone() if MD else g  # the reference scales the gradient in place under decouple_md

    t0 = time.perf_counter()
    for i in range(args.warmup):
        feed()
        opt.step()
        torch.cuda.synchronize()
        progress(rank, f"reference warm-up step {i + 1} done")
    warm_s = time.perf_counter() - t0
    sampler = ClockSampler(None)
    sampler.start()
    ms = []
    for _ in range(args.steps):
        feed()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        opt.step()
        e1.record()
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    clocks = sampler.stop()
    v = statistics.median(ms)
    line = {"impl": "reference_gpu", "metric": METRIC, "value": round(v, 3), "unit": "ms", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 3), "higher_is_better": False,
            "dtype": "f16", "data": "synthetic", "config": bench_config(args, 1),
            "reference": "thorn 3.1.1 from baseline/_ref, unmodified",
            "state_dtype": "bf16 (the reference keeps state in the parameter dtype)",
            "ms_all_steps": [round(x, 3) for x in ms], "warmup_s_incl_compile": round(warm_s, 1),
            "clocks": clocks}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU arm
def build_params(torch, dev, rank, world, mesh, layers=None):
    """Llama-shaped params (bf16 ~N(0, 0.02)) and grads (bf16 ~N(0, 1e-4)) on `dev`."""
    ortho_s, adam_s = shapes(layers)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def make(shape, std):
        if world == 1:
            t = torch.randn(shape, device=dev, dtype=torch.bfloat16, generator=gen) * std
            return t
        from torch.distributed.tensor import DTensor, Shard

        from thorn_b200.sharded import shard_rows
        local = (shard_rows(shape[0], world)[rank][1],) + tuple(shape[1:])  # DTensor's torch.chunk split
        t = torch.randn(local, device=dev, dtype=torch.bfloat16, generator=gen) * std
        return DTensor.from_local(t, mesh, [Shard(0)], run_check=False, shape=shape,
                                  stride=torch.empty(shape, device="meta").stride())

    ortho = [torch.nn.Parameter(make(s, 0.02)) for s in ortho_s]
    adamw = [torch.nn.Parameter(make(s, 0.02)) for s in adam_s]
    g_ortho = [make(s, 1e-4) for s in ortho_s]
    g_adam = [make(s, 1e-4) for s in adam_s]
    return ortho, adamw, g_ortho, g_adam


_T0 = time.time()
_LAST = [time.time(), "start"]


def progress(rank, msg):
    """One line of progress on stderr (stdout carries only the result line)."""
    _LAST[0], _LAST[1] = time.time(), msg
    print(f"[bench rank {rank} +{time.time() - _T0:.1f}s] {msg}", file=sys.stderr, flush=True)


def stall_watchdog(rank, limit_s):
    """Multi-rank runs: end the process if no stage completes for `limit_s` seconds.

    A rank blocked on the host inside a collective call is invisible to the
    process group's own timeout; this turns such a stall into an exit with the
    last completed stage in the log instead of a run that waits for its caller's
    time limit.
    """
    import threading

    def run():
        while True:
            time.sleep(5)
            if time.time() - _LAST[0] > limit_s:
                print(f"[bench rank {rank}] no progress for {limit_s}s after '{_LAST[1]}'; exiting",
                      file=sys.stderr, flush=True)
                os._exit(3)

    threading.Thread(target=run, daemon=True).start()


def bench_config(args, world) -> dict:
    """The workload description of the line, the same on both arms."""
    layers = getattr(args, "layers", None) or LAYERS
    ortho_s, adam_s = shapes(layers)
    return {"workload": WORKLOAD + (" sharded Shard(0)" if world > 1 else "")
            + ("" if layers == LAYERS else f" REDUCED to {layers} layers (profiling only)"),
            "ortho_matrices": len(ortho_s), "adamw_tensors": len(adam_s),
            "params": sum(math.prod(s) for s in ortho_s + adam_s), "param_dtype": "bf16",
            "state_dtype": "f32", "ns_dtype": "f16", "decouple_md": MD, "lr": ORTHO_LR,
            "parallelism": f"fsdp{world}" if world > 1 else "single",
            "l2": "no flush: every step reads params, grads and state (~70 GB) >> 126 MB L2"}


def result_line(args, world, ms, ns_launch_ms, ns_dense_all, ns_exec_all, mom_ms, mom_bytes, cpu, e2e, host_ms,
                host_enqueue_ms, launches, clocks) -> dict:
    """The JSON line of a GPU run (rank 0) from its measurements: device time per step, the
    NS phase (ms per step, dense-equivalent and executed FLOPs of all ranks), the momentum
    pass (ms and compulsory bytes per step), the CPU baseline, the end-to-end figure, host
    times, launch count and clock record."""
    hbm, peak_burst, peak_sus, peak_src = load_peaks()
    peak_job = peak_sus * world  # whole-job peak: the NS work is spread over all ranks
    achieved = ns_dense_all / (ns_launch_ms * 1e-3) / 1e12 if ns_launch_ms > 0 else None
    achieved_exec = ns_exec_all / (ns_launch_ms * 1e-3) / 1e12 if ns_launch_ms > 0 else None
    line = {
        "metric": METRIC, "value": round(ms, 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": bench_config(args, world),
        "roofline": {"bound": "tensor", "kernel": "ns_gemm2_kernel (Newton-Schulz phase)",
                     "achieved": round(achieved, 1) if achieved else None, "peak": round(peak_job, 1),
                     "unit": "TFLOP/s", "frac": round(achieved / peak_job, 3) if achieved else None,
                     "traffic": NS_GEMM_TRAFFIC,
                     "traffic_case": NS_GEMM_TRAFFIC_CASE,
                     "flops": "dense-equivalent (2MNK per reference GEMM)",
                     "achieved_executed": round(achieved_exec, 1) if achieved_exec else None,
                     "peak_source": f"{peak_src} sustained bf16 (MEASURED_PEAKS.json) x {world} GPU(s); "
                                    f"burst {peak_burst} per GPU",
                     "ns_ms_per_step": round(ns_launch_ms, 3),
                     "ns_dense_tflop_per_step": round(ns_dense_all / 1e12, 2)},
        "roofline_elementwise": {
            "bound": "hbm", "kernel": "ortho_pre_kernel + pre_reduce_kernel (momentum pass)",
            "achieved": round(mom_bytes / (mom_ms * 1e-3) / 1e9, 1) if mom_ms > 0 else None,
            "peak": round(hbm * world, 1), "unit": "GB/s",
            "frac": round(mom_bytes / (mom_ms * 1e-3) / 1e9 / (hbm * world), 3) if mom_ms > 0 else None,
            "bytes": ("g read + m read/write + p read/write (decouple_md), compulsory" if MD
                      else "g read + m read/write, compulsory"),
            "ms_per_step": round(mom_ms, 3), "gb_per_step": round(mom_bytes / 1e9, 2)},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "host_ms_per_step": round(host_ms, 2),
        "host_enqueue_ms_idle_gpu": round(host_enqueue_ms, 2),
        "gpu_launches": int(launches),
        "gpu_launches_per_step": round(launches / args.steps, 1),
        "clocks": clocks,
    }
    return line


def gpu_arm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from thorn_b200 import THORN, _native

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    mesh = None
    if world > 1:
        from torch.distributed.device_mesh import init_device_mesh
        mesh = init_device_mesh("cuda", (world,))
        progress(rank, "device mesh ready")
    ortho, adamw, g_ortho, g_adam = build_params(torch, dev, rank, world, mesh, args.layers)
    params = ortho + adamw
    grads = g_ortho + g_adam
    opt = THORN([
        {"orthogonalize": True, "params": ortho, "lr": ORTHO_LR, "decouple_md": MD, "state_dtype": torch.float32},
        {"orthogonalize": False, "params": adamw, "lr": ADAM_LR, "state_dtype": torch.float32},
    ])
    opt.pipeline_exchange = bool(args.pipeline_exchange)
    opt.exchange = args.exchange
    if args.ns_batch_elems:
        opt.polar_decomp_batch_size = int(args.ns_batch_elems)
    apply_switches(args)

    def local(t):
        return t.to_local() if hasattr(t, "to_local") else t

    def feed():
        for p, g in zip(params, grads):
            p.grad = g

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def host_buffers(ts):
        """Pinned host copies of ``ts``' shapes: one block (one copy per direction and step)
        when they share a dtype, else one allocation each."""
        if len({t.dtype for t in ts}) == 1:
            from thorn_b200.host_stepper import pinned_block
            return pinned_block([tuple(t.shape) for t in ts], ts[0].dtype)
        return [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in ts]

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    progress(rank, "params built")
    for i in range(args.warmup):
        feed()
        opt.step()
        torch.cuda.synchronize()
        progress(rank, f"warm-up step {i + 1} done")

    # ---------------- device-timed steps (inputs resident in HBM)
    clocks = None
    sampler = None
    if rank == 0:
        # the GPUs of this job: local ranks 0..world-1 (one node)
        ids = []
        try:
            for i in range(min(world, torch.cuda.device_count())):
                u = str(torch.cuda.get_device_properties(i).uuid)
                ids.append(u if u.startswith("GPU-") else "GPU-" + u)
        except Exception:
            ids = [str(i) for i in range(world)]
        sampler = ClockSampler(ids)
        sampler.start()
        time.sleep(0.3)
    opt.profile_ns = []
    opt.profile_momentum = []
    opt.profile_stages = [] if world > 1 else None
    launches0 = _native.launch_count()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    h0 = time.perf_counter()
    for _ in range(args.steps):
        feed()
        opt.step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # host time to enqueue one step
    e1.record()
    torch.cuda.synchronize()
    barrier()
    launches = _native.launch_count() - launches0
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    progress(rank, "timed steps done")
    prof = opt.profile_ns
    opt.profile_ns = None
    prof_m = opt.profile_momentum
    opt.profile_momentum = None
    stages = stage_times(torch, dist, dev, opt.profile_stages, args.steps) if world > 1 else None
    opt.profile_stages = None
    mom_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b, _ in prof_m) / args.steps)
    mom_bytes = sum(nb for _, _, nb in prof_m) / args.steps
    if world > 1:
        t = torch.tensor([mom_bytes], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        mom_bytes = float(t[0])
    # host cost of one step on an idle GPU (nothing blocks on a full launch queue)
    feed()
    torch.cuda.synchronize()
    barrier()
    h1 = time.perf_counter()
    opt.step()
    host_enqueue_ms = max_over_ranks((time.perf_counter() - h1) * 1e3)
    torch.cuda.synchronize()
    ns_ms = sum(a.elapsed_time(b) for a, b, *_ in prof) / args.steps
    ns_dense = sum(d for _, _, d, _, _ in prof) / args.steps
    ns_exec = sum(x for _, _, _, x, _ in prof) / args.steps
    ns_launch_ms = max_over_ranks(ns_ms)
    # whole-job NS throughput: FLOPs of all ranks / the slowest rank's NS time
    if world > 1:
        t = torch.tensor([ns_dense, ns_exec], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        ns_dense_all, ns_exec_all = float(t[0]), float(t[1])
    else:
        ns_dense_all, ns_exec_all = ns_dense, ns_exec
    if sampler is not None:
        time.sleep(0.2)
        clocks = sampler.stop()

    # ---------------- end to end: grads in from pinned host memory, params back out
    e2e = None
    if not args.no_e2e:
        h_grads = host_buffers([local(g) for g in grads])
        for h, g in zip(h_grads, grads):
            h.copy_(local(g))
        h_params = host_buffers([local(p) for p in params])
        bi = sum(h.numel() * h.element_size() for h in h_grads)
        bo = sum(h.numel() * h.element_size() for h in h_params)
        # the device-resident grads of the timed loop are not needed any more
        for lst in (grads, g_ortho, g_adam):
            lst.clear()
        torch.cuda.synchronize()
    e2e_note = None
    if not args.no_e2e and args.e2e_mode == "pipelined":
        from thorn_b200.host_stepper import PinnedStepper

        ok = 1.0
        stepper = None
        try:  # the stepper's device buffers: two gradient sets and a parameter snapshot
            stepper = PinnedStepper(opt, params, h_grads, h_params)
        except (RuntimeError, ValueError, TypeError) as exc:  # e.g. out of device memory
            ok = 0.0
            e2e_note = f"pipelined mode unavailable ({type(exc).__name__}: {str(exc)[:120]}); serial mode"
        if world > 1:  # every rank takes the same branch before any step runs
            t = torch.tensor([ok], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            if float(t.item()) == 0.0:
                e2e_note = e2e_note or "pipelined mode unavailable on another rank; serial mode"
        if e2e_note is not None:
            stepper = None
            torch.cuda.empty_cache()
    if not args.no_e2e and args.e2e_mode == "pipelined" and e2e_note is None:
        try:
            for _ in range(2):
                stepper.wait_host_grads()
                stepper.step()
            stepper.synchronize()
            barrier()
            torch.cuda.synchronize()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            stepper.h2d.wait_stream(torch.cuda.current_stream())  # no copy starts before t0
            marks = []  # end of each step's work on the compute stream
            for _ in range(args.steps):
                # the documented loop: the host may rewrite its gradient buffers only after
                # the previous step's copy has read them (the buffers stay as they are here)
                stepper.wait_host_grads()
                stepper.step()
                marks.append(torch.cuda.Event(enable_timing=True))
                marks[-1].record()
            stepper.wait_on()
            t1.record()
            torch.cuda.synchronize()
            barrier()
            e2e_ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
            # once the pipeline is full: the first gradient copy (before step 1 can start)
            # and the last parameter copy (after the last step) fall outside this period
            steady_ms = max_over_ranks(marks[0].elapsed_time(marks[-1]) / (len(marks) - 1)) \
                if len(marks) > 1 else None
            if world > 1:
                t = torch.tensor([bi, bo], device=dev, dtype=torch.float64)
                dist.all_reduce(t)
                bi, bo = int(t[0]), int(t[1])
            e2e = {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                   "mode": "pipelined: both copies overlap the steps on two copy streams (thorn_b200.PinnedStepper)",
                   "steady_ms_per_step": None if steady_ms is None else round(steady_ms, 3),
                   "steady_note": "period between consecutive steps with the copy pipeline full; value also "
                                  "holds the first gradient copy and the last parameter copy, once per run"}
            progress(rank, "end-to-end steps done")
            del stepper, h_grads, h_params
        except Exception as exc:  # one GPU: keep the device-timed line and measure serially
            if world > 1:
                raise
            e2e_note = f"pipelined mode failed ({type(exc).__name__}: {str(exc)[:120]}); serial mode"
            stepper = None
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
    if not args.no_e2e and e2e is None:
        d_grads = [torch.empty_like(p) for p in params]

        def e2e_step():
            for dg, h in zip(d_grads, h_grads):
                local(dg).copy_(h, non_blocking=True)
            for p, dg in zip(params, d_grads):
                p.grad = dg
            opt.step()
            for h, p in zip(h_params, params):
                h.copy_(local(p).detach(), non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            e2e_step()
        t1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
        if world > 1:
            t = torch.tensor([bi, bo], device=dev, dtype=torch.float64)
            dist.all_reduce(t)
            bi, bo = int(t[0]), int(t[1])
        e2e = {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
               "mode": e2e_note or "serial: copy in, step, copy out on one stream"}
        progress(rank, "end-to-end steps done")
        del h_grads, h_params, d_grads

    if rank != 0:
        return
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        v, sample, secs, cores, kind = cpu_sample()
        cpu = cpu_baseline_entry(v, sample, cores, kind, {"sample_cpu_seconds": round(secs, 2)})
    line = result_line(args, world, ms, ns_launch_ms, ns_dense_all, ns_exec_all, mom_ms, mom_bytes, cpu, e2e,
                       host_ms, host_enqueue_ms, launches, clocks)
    if stages:
        line["sharded_stages_ms"] = stages
    print(json.dumps(line), flush=True)


def stage_times(torch, dist, dev, logs, steps):
    """Per-stage device time of the sharded step (ms per step, max over ranks): each entry of
    ``logs`` is one sharded step's list of (stage, event) marks on the launching stream."""
    slots = 8  # every rank all-reduces the same fixed-size tensor, whatever it recorded
    names = [n for n, _ in logs[0][1:]][:slots] if logs else []
    tot = [0.0] * slots
    ok = 1.0 if names else 0.0
    for marks in logs or []:
        if [n for n, _ in marks[1:]][:slots] != names:
            ok = 0.0
            break
        for i in range(1, min(len(marks), slots + 1)):
            tot[i - 1] += marks[i - 1][1].elapsed_time(marks[i][1])
    t = torch.tensor([x / steps for x in tot] + [-ok], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the last slot: -1 only if every rank recorded alike
    if t[-1].item() != -1.0:
        return None
    return {n: round(float(v), 3) for n, v in zip(names, t[:len(names)].tolist())}


def apply_switches(args):
    """Kernel options of the library (all off by default)."""
    from thorn_b200 import _native

    lib = _native.load()
    if args.gemm_pdl:
        lib.thorn_set_gemm_pdl(1)
    if args.gemm_l2_hints:
        lib.thorn_set_gemm_l2_hints(1)


def ns_only(args):
    """Time thorn_ns_batched alone on one batch shape (profiling entry point)."""
    import ctypes

    import torch

    from thorn_b200 import _native as N
    from thorn_b200.coeffs import gram_ns_restarts, optimal_composition

    B, R, C = (int(x) for x in args.ns_only.lower().split("x"))
    lib = N.load()
    apply_switches(args)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    co = optimal_composition(1e-3, 5, 0.03, 0.02)
    rs = gram_ns_restarts(*co)
    cc = (ctypes.c_double * 15)(*[v for t in co for v in t])
    rr = (ctypes.c_int32 * max(1, len(rs)))(*rs)
    ldc = int(lib.thorn_ns_ld(C))
    X = (torch.randn(B, R, ldc, device=dev) / math.sqrt(R * C)).half()
    U = torch.empty(B, R, C, dtype=torch.float16, device=dev)
    wsb = int(lib.thorn_ns_workspace_bytes(B, R, C))
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = N.stream_of(dev)

    def run():
        N.check(lib.thorn_ns_batched(X.data_ptr(), U.data_ptr(), ws.data_ptr(), wsb, B, R, C, N.F16, cc, 5, rr,
                                     len(rs), err.data_ptr(), st), "ns_batched")

    if args.ns_library:
        # the same recurrences with every product a dense cuBLAS GEMM (torch.bmm / baddbmm),
        # for a library baseline on the same box: no symmetry, no fused epilogues
        Xw = X[:, :, :C] if R <= C else X[:, :, :C].mT  # wide orientation, m = min(R, C)
        Xw = Xw.contiguous()
        lib_out = {}

        def run():  # noqa: F811  (replaces the thorn_b200 call)
            lib_out["U"] = ns_library(Xw, co, rs)

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    d0, x0 = N.gemm_flops()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    d1, x1 = N.gemm_flops()
    ms = e0.elapsed_time(e1) / args.steps
    dense = B * dense_ns_flops(R, C)
    line = {"ns_only": f"{B}x{R}x{C}", "ms": round(ms, 4), "dense_tflops": round(dense / ms / 1e9, 1),
            "executed_tflops": round((x1 - x0) / args.steps / ms / 1e9, 1), "err_flag": int(err.item()),
            "finite": bool(torch.isfinite(U).all())}
    if args.ns_library:
        Ul = lib_out["U"] if R <= C else lib_out["U"].mT
        N.check(lib.thorn_ns_batched(X.data_ptr(), U.data_ptr(), ws.data_ptr(), wsb, B, R, C, N.F16, cc, 5, rr,
                                     len(rs), err.data_ptr(), st), "ns_batched")
        line.update(impl="torch.bmm/baddbmm (cuBLAS), dense", executed_tflops=line["dense_tflops"],
                    finite=bool(torch.isfinite(Ul).all()),
                    rel_fro_vs_thorn_b200=round(float((Ul.float() - U.float()).norm() / U.float().norm()), 6))
    print(json.dumps(line), flush=True)


def ns_library(X, coeffs, restarts):
    """Newton-Schulz of a batch of wide (m <= n) fp16 matrices with the recurrences of
    thorn_ns_batched (thorn.py:626-662), every product a torch GEMM."""
    import torch

    B_, m, n = X.shape
    if m == n:
        for a, b, c in coeffs:
            A = torch.bmm(X, X.mT)
            Bm = torch.baddbmm(A, A, A, beta=b, alpha=c)
            X = torch.baddbmm(X, Bm, X, beta=a)
        return X
    eye = torch.eye(m, dtype=X.dtype, device=X.device)
    R = torch.bmm(X, X.mT)
    Q = None
    iters = len(coeffs)
    for i, (a, b, c) in enumerate(coeffs):
        rs = i in restarts
        if rs and i != 0:
            X = torch.bmm(Q, X)
            R = torch.bmm(X, X.mT)
        Z = torch.baddbmm(R, R, R, beta=b, alpha=c)
        Q = Z + a * eye if (Q is None or rs) else torch.baddbmm(Q, Q, Z, beta=a)
        if i < iters - 1 and (i + 1) not in restarts:
            RZ = torch.baddbmm(R, R, Z, beta=a)
            R = torch.baddbmm(RZ, Z, RZ, beta=a)
    return torch.bmm(Q, X)


def ortho_only(args):
    """Time THORN steps of one orthogonalized group of B x (R x C) bf16 matrices with
    decouple_md and fp32 state (profiling entry point for the elementwise passes)."""
    import torch

    from thorn_b200 import THORN

    B, R, C = (int(x) for x in args.ortho_only.lower().split("x"))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    apply_switches(args)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(R, C, device=dev, dtype=torch.bfloat16, generator=gen) * 0.02)
          for _ in range(B)]
    gs = [torch.randn(R, C, device=dev, dtype=torch.bfloat16, generator=gen) * 1e-4 for _ in range(B)]
    opt = THORN([{"orthogonalize": True, "params": ps, "lr": ORTHO_LR, "decouple_md": True,
                  "state_dtype": torch.float32}])

    def step():
        for p, g in zip(ps, gs):
            p.grad = g
        opt.step()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"ortho_only": args.ortho_only, "ms": round(ms, 4), "err_flag": int(opt.device_error()),
                      "finite": bool(all(torch.isfinite(p).all() for p in ps))}), flush=True)


def copy_rate(args):
    """Host<->device copy rate of this box, the bound of the end-to-end figure (which moves
    16 GB each way per Llama-3-8B step): 8 GiB of bf16 from pinned host memory to the
    device, back, and both directions at once on two streams (CUDA events, best of 3)."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = 4 * 1024 ** 3  # 4 Gi bf16 elements: 8 GiB per direction (the rate, not the size, is reported)
    h_in = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)
    h_out = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)
    d_in = torch.empty(n, dtype=torch.bfloat16, device=dev)
    d_out = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    nbytes = n * 2

    def timed(h2d, d2h):
        best = None
        for _ in range(3):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            s1.wait_stream(torch.cuda.current_stream())
            s2.wait_stream(torch.cuda.current_stream())
            if h2d:
                with torch.cuda.stream(s1):
                    d_in.copy_(h_in, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s2):
                    h_out.copy_(d_out, non_blocking=True)
            torch.cuda.current_stream().wait_stream(s1)
            torch.cuda.current_stream().wait_stream(s2)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        return round(nbytes / (best * 1e-3) / 1e9, 1)

    print(json.dumps({"copy_rate_gbs": {"h2d": timed(True, False), "d2h": timed(False, True),
                                        "both_each_direction": timed(True, True)},
                      "bytes_per_direction": nbytes, "pinned": True}), flush=True)


def small_config_groups(name):
    """(groups, param dtype, state dtype, grad std) of BASELINE configs[0]-[2]: lists of
    (orthogonalize, shapes, init std or None for ones, group options)."""
    if name == "tiny":  # configs[0]
        return [(True, [(512, 512)] * 4 + [(1024, 512)] * 2 + [(512, 1024)] * 2, 0.02,
                 dict(lr=1e-3, weight_decay=0.1, scaling_mode="moonlight")),
                (False, [(512,)] * 8, None, dict(lr=1e-3, weight_decay=0.0, scaling_mode="moonlight"))], \
            "f32", "f32", 1e-3
    if name == "vad":  # configs[1]: 24 Conv1d kernels flattened to out x (in*k), 4 + 2 Linear weights
        convs = [[(64, 32, 3), (64, 64, 3), (128, 64, 5), (128, 128, 3)][i % 4] for i in range(24)]
        mats = [(o, i * k) for o, i, k in convs] + [(128, 128)] * 4 + [(2, 128)] * 2
        vecs = [(o,) for o, _, _ in convs for _ in range(3)] + [(128,)] * 4 + [(2,)] * 2
        return [(True, mats, 0.05, dict(lr=1e-3, weight_decay=0.1)),
                (False, vecs, 0.05, dict(lr=1e-3, weight_decay=0.0))], "f32", "f32", 1e-3
    if name == "qwen300m":  # configs[2]: 20 layers, hidden 1024, tied embedding
        layer = [(2048, 1024), (1024, 1024), (1024, 1024), (1024, 2048), (3072, 1024), (3072, 1024), (1024, 3072)]
        norms = [(1024,), (1024,), (128,), (128,)] * 20 + [(1024,)]
        return [(True, layer * 20, 0.02, dict(lr=1e-3, weight_decay=0.1)),
                (False, [(151936, 1024)], 0.02, dict(lr=1e-3, weight_decay=0.1)),
                (False, norms, None, dict(lr=1e-3, weight_decay=0.0))], "bf16", "f32", 1e-4
    raise ValueError(name)


def small_config(args):
    """Time THORN steps on BASELINE configs[0]-[2] (one GPU): device time per step, the NS phase
    and the host time to enqueue a step (these configs are launch- and host-bound)."""
    import torch

    from thorn_b200 import THORN

    groups, pdt, sdt, gstd = small_config_groups(args.model)
    dtypes = {"f32": torch.float32, "bf16": torch.bfloat16}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    apply_switches(args)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    params, grads, tg = [], [], []
    for ortho, shapes_, std, opts in groups:
        ps = [torch.nn.Parameter(torch.ones(s, device=dev, dtype=dtypes[pdt]) if std is None else
                                 torch.randn(s, device=dev, dtype=dtypes[pdt], generator=gen) * std) for s in shapes_]
        grads += [torch.randn(s, device=dev, dtype=dtypes[pdt], generator=gen) * gstd for s in shapes_]
        params += ps
        tg.append({"orthogonalize": ortho, "params": ps, "state_dtype": dtypes[sdt], **opts})
    opt = THORN(tg)
    opt.profile_ns = []

    def step():
        for p, g in zip(params, grads):
            p.grad = g
        opt.step()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    opt.profile_ns = []
    from thorn_b200 import _native

    launches0 = _native.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    launches = (_native.launch_count() - launches0) / args.steps
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    prof, opt.profile_ns = opt.profile_ns, None
    ns_ms = sum(a.elapsed_time(b) for a, b, *_ in prof) / args.steps
    ns_dense = sum(d for _, _, d, _, _ in prof) / args.steps
    print(json.dumps({"model": args.model, "ms_per_step": round(ms, 4), "host_ms_per_step": round(host_ms, 3),
                      "gpu_launches_per_step": launches,
                      "ns_ms_per_step": round(ns_ms, 4),
                      "ns_dense_tflops": round(ns_dense / (ns_ms * 1e-3) / 1e12, 1) if ns_ms > 0 else None,
                      "params": sum(p.numel() for p in params), "param_dtype": pdt, "state_dtype": sdt,
                      "err_flag": int(opt.device_error()),
                      "finite": bool(all(torch.isfinite(p).all() for p in params))}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="thorn_b200", choices=["thorn_b200", "reference", "reference_gpu"],
                    help="reference: the reference's CPU step (rank 0); reference_gpu: the reference's own GPU "
                         "step (Triton + torch.compile) on cuda:0, from its install under baseline/_ref")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gemm-pdl", action="store_true",
                    help="NS GEMMs with programmatic dependent launch (thorn_set_gemm_pdl)")
    ap.add_argument("--gemm-l2-hints", action="store_true",
                    help="L2 cache policies on the 2-CTA NS GEMM's loads and stores (thorn_set_gemm_l2_hints)")
    ap.add_argument("--exchange", default="all_to_all", choices=["rounds", "all_to_all", "peer"],
                    help="N > 1: slab exchange as one all_to_all_single (default), pairwise P2P rounds, or "
                         "peer: stores into the owners' IPC-mapped arenas and copy-engine peer copies")
    ap.add_argument("--pipeline-exchange", action="store_true",
                    help="N > 1: exchange row slabs in waves that overlap the owners' Newton-Schulz work")
    ap.add_argument("--e2e-mode", default="pipelined", choices=["serial", "pipelined"],
                    help="pipelined (default): thorn_b200.PinnedStepper overlaps both copies with the steps, "
                         "falling back to serial if it cannot run; serial: copy in, step, copy out on one stream")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ns-batch-elems", type=int, default=None,
                    help="THORN.polar_decomp_batch_size: elements per Newton-Schulz batch (default: the optimizer's)")
    ap.add_argument("--ns-only", default=None, help="BxRxC: time thorn_ns_batched alone on this batch (profiling)")
    ap.add_argument("--ns-library", action="store_true",
                    help="with --ns-only: time the same recurrences on torch/cuBLAS GEMMs instead (library baseline)")
    ap.add_argument("--layers", type=int, default=None, help="transformer layers (profiling runs use fewer)")
    ap.add_argument("--model", default="llama8b", choices=["llama8b", "llama70b", "tiny", "vad", "qwen300m"],
                    help="parameter set: llama8b (BASELINE configs[3], the headline), llama70b (configs[4], 8 "
                         "GPUs), or tiny / vad / qwen300m (configs[0]-[2], one GPU, step timing only)")
    ap.add_argument("--copy-rate", action="store_true",
                    help="measure the host<->device copy rate (pinned, one direction and both at once)")
    ap.add_argument("--ortho-only", default=None,
                    help="BxRxC: time steps of one decouple_md group of B bf16 RxC matrices (profiling)")
    args = ap.parse_args()
    if args.copy_rate:
        copy_rate(args)
        return
    if args.model in ("tiny", "vad", "qwen300m"):
        small_config(args)
        return
    if args.model == "llama70b":
        use_llama70b()
    if args.layers is None:
        args.layers = LAYERS
    if args.ns_only:
        ns_only(args)
        return
    if args.ortho_only:
        ortho_only(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    if args.impl == "reference_gpu":
        reference_gpu_arm(args, rank)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if world > 1:
        import datetime

        # the exchanges are point-to-point and the all-reduces a few KB: NVLink
        # SHARP buys nothing here, so NCCL skips setting up its NVLS buffers
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        stall_watchdog(rank, 420)
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        gpu_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
