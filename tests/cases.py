"""Seeded parameter/gradient sets shared by the golden generator and the tests.

Inputs are rebuilt from seeds everywhere (``torch.manual_seed(0)`` before the
params in group order; ``torch.manual_seed(1000 + s)`` before step ``s``'s
grads in param order), so fixtures only need to hold outputs.
"""
from __future__ import annotations

import functools
import math

import numpy as np
import torch

TORCH_DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _fro(p) -> float:
    """Frobenius norm of a torch tensor or a numpy array, as a Python float (float64 sum)."""
    a = p.detach().double().cpu().numpy() if isinstance(p, torch.Tensor) else np.asarray(p, dtype=np.float64)
    return float(np.sqrt((a * a).sum()))


def _conv_flat(shape):
    o, i, k = shape
    return (o, i * k)


def _vad_groups(flatten=True, grad_dtype="f32"):
    convs = []
    for i in range(24):
        convs.append([(64, 32, 3), (64, 64, 3), (128, 64, 5), (128, 128, 3)][i % 4])
    mats = [(_conv_flat(c) if flatten else c) for c in convs] + [(128, 128)] * 4 + [(2, 128)] * 2
    vecs = []
    for c in convs:
        vecs += [(c[0],)] * 3          # conv bias, BN weight, BN bias
    vecs += [(128,)] * 4 + [(2,)] * 2  # Linear biases
    return [
        dict(orthogonalize=True, shapes=mats, init=("normal", 0.05), dtype="f32",
             opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)),
        dict(orthogonalize=False, shapes=vecs, init=("normal", 0.05), dtype="f32",
             opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.0)),
    ]


CASES = {
    # BASELINE config 1 ("CPU-runnable tiny step"), exact shapes.
    "tiny": dict(steps=10, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(512, 512)] * 4 + [(1024, 512)] * 2 + [(512, 1024)] * 2,
             init=("normal", 0.02), dtype="f32",
             opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, scaling_mode="moonlight")),
        dict(orthogonalize=False, shapes=[(512,)] * 8, init=("const", 1.0), dtype="f32",
             opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.0, scaling_mode="moonlight")),
    ]),
    # Same structure at reduced shapes, stored in full.
    "tiny_small": dict(steps=10, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64)] * 4 + [(128, 64)] * 2 + [(64, 128)] * 2,
             init=("normal", 0.02), dtype="f32",
             opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, scaling_mode="moonlight")),
        dict(orthogonalize=False, shapes=[(64,)] * 8, init=("const", 1.0), dtype="f32",
             opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.0, scaling_mode="moonlight")),
    ]),
    # Magnitude-direction decoupling on both groups (split row/col gains, scalar gains).
    "md_small": dict(steps=4, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (96, 64), (64, 160), (128, 128)],
             init=("normal", 0.02), dtype="f32", opts=dict(lr=8e-3, decouple_md=True)),
        dict(orthogonalize=False, shapes=[(64,), (32,), (48, 16)], init=("normal", 0.5), dtype="f32",
             opts=dict(lr=1e-3, decouple_md=True, weight_decay=0.05)),
    ]),
    # bf16 params with state in the param dtype (the reference's own layout).
    "bf16_small": dict(steps=4, grad_std=1e-4, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (192, 64), (64, 192), (128, 64)],
             init=("normal", 0.02), dtype="bf16", opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)),
        dict(orthogonalize=False, shapes=[(64,), (128, 32)], init=("normal", 0.02), dtype="bf16",
             opts=dict(lr=1e-3, weight_decay=0.1)),
    ]),
    # 3-D conv kernels are batches of (in, k) matrices (thorn.py:628-633).
    "conv_small": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(8, 4, 3), (16, 8, 5), (4, 6, 6)], init=("normal", 0.05),
             dtype="f32", opts=dict(lr=1e-3, weight_decay=0.1, scaling_mode="jordan")),
        dict(orthogonalize=False, shapes=[(16,)], init=("const", 1.0), dtype="f32", opts=dict(lr=1e-3)),
    ]),
    # Option variants: jordan scaling + forced per-neuron norm; RAdam rectification with eps>0.
    "variants_small": dict(steps=8, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (64, 96), (96, 32)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, betas=(0.95, 0.9), weight_decay=0.2, scaling_mode="jordan",
                       force_per_neuron_norm=True)),
        dict(orthogonalize=True, shapes=[(80, 48)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, betas=(0.9, 0.0), weight_decay=0.0, scaling_mode="md")),
        dict(orthogonalize=False, shapes=[(64,), (40, 24)], init=("normal", 0.1), dtype="f32",
             opts=dict(lr=1e-3, rectify=True, eps=1e-8, weight_decay=0.1, betas=(0.9, 0.95))),
    ]),
    # decouple_md on the orthogonalized group with 2-D matrices whose rows split over 2 ranks
    # (the FSDP2 tests), next to a plain (R)AdamW vector group.
    "md_shard": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (96, 64), (64, 160), (128, 128)],
             init=("normal", 0.02), dtype="f32", opts=dict(lr=8e-3, decouple_md=True)),
        dict(orthogonalize=False, shapes=[(64,), (32,)], init=("normal", 0.5), dtype="f32",
             opts=dict(lr=1e-3, weight_decay=0.05)),
    ]),
    # BASELINE config 2 shapes (flattened conv kernels) -- the many-tiny-matrices case.
    "vad": dict(steps=3, grad_std=1e-3, groups=_vad_groups(flatten=True)),
    # Row counts that split unevenly over 2 (and 4) shards, with and without MD, next to AdamW
    # vectors whose shards are uneven too (the FSDP2 tests at world 1 and 2).
    "shard_uneven": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(66, 64), (97, 64), (64, 160)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, weight_decay=0.1)),
        dict(orthogonalize=True, shapes=[(75, 64), (33, 96)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True)),
        dict(orthogonalize=False, shapes=[(65,), (33,)], init=("normal", 0.5), dtype="f32",
             opts=dict(lr=1e-3, weight_decay=0.05)),
    ]),
    # Magma momentum-aligned masking (thorn.py:800-836) on both group kinds, with and without MD.
    "magma_small": dict(steps=6, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (96, 64), (64, 160)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, weight_decay=0.1, momentum_align=True)),
        dict(orthogonalize=True, shapes=[(64, 96)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True, momentum_align=True)),
        dict(orthogonalize=False, shapes=[(64,), (40, 24)], init=("normal", 0.1), dtype="f32",
             opts=dict(lr=1e-3, weight_decay=0.1, momentum_align=True)),
        dict(orthogonalize=False, shapes=[(48, 16)], init=("normal", 0.5), dtype="f32",
             opts=dict(lr=1e-3, decouple_md=True, momentum_align=True)),
    ]),
    # Edge inputs: all-zero gradients on tall matrices (zero Frobenius norm, so the NS input is
    # 0 / (0 + 1e-8), and per-neuron norm of a zero update; zero AdamW moments), a one-row
    # matrix, a tall matrix with an odd column count, MD on a matrix whose gradient is zero.
    "edge_small": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(96, 64), (1, 64), (130, 37), (40, 40)], init=("normal", 0.02),
             dtype="f32", opts=dict(lr=2e-3, weight_decay=0.1), zero=[0]),
        dict(orthogonalize=True, shapes=[(72, 24), (80, 48)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True), zero=[1]),
        dict(orthogonalize=False, shapes=[(64,), (33,)], init=("normal", 0.5), dtype="f32",
             opts=dict(lr=1e-3, weight_decay=0.1), zero=[0]),
    ]),
    # One decoder layer of BASELINE config 3 (Qwen3-style, hidden 1024) at full size, with its
    # tied 151936 x 1024 embedding: bf16 params and state in the param dtype (the reference's
    # own layout), q/k RMSNorm weights of 128 and layer norms of 1024 without weight decay.
    # The orthogonalized lr makes each step's update ~10 bf16 ulps of the parameter, so that
    # rounding flips do not dominate the compared update.
    "qwen_layer": dict(steps=2, grad_std=1e-4, groups=[
        dict(orthogonalize=True, shapes=[(2048, 1024), (1024, 1024), (1024, 1024), (1024, 2048), (3072, 1024),
                                         (3072, 1024), (1024, 3072)], init=("normal", 0.02), dtype="bf16",
             opts=dict(lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)),
        dict(orthogonalize=False, shapes=[(151936, 1024)], init=("normal", 0.02), dtype="bf16",
             opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)),
        dict(orthogonalize=False, shapes=[(1024,), (1024,), (128,), (128,), (1024,)], init=("const", 1.0),
             dtype="bf16", opts=dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.0)),
    ]),
    # Magma on the FSDP2 path (world 1 and 2): orthogonalized matrices, even and uneven splits,
    # with and without MD, next to a Magma (R)AdamW vector group.
    "magma_shard": dict(steps=6, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (97, 64)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, weight_decay=0.1, momentum_align=True)),
        dict(orthogonalize=True, shapes=[(64, 96)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True, momentum_align=True)),
        dict(orthogonalize=False, shapes=[(64,), (40,)], init=("normal", 0.1), dtype="f32",
             opts=dict(lr=1e-3, momentum_align=True)),
    ]),
    # decouple_md with norm_axis=-1 (thorn.py:594-595, 605, 1717): the (R)AdamW group's "init"
    # target norms and renorm run per row (per last-dim slice, also of a 3-D tensor); the
    # orthogonalized group renorms whole matrices whatever norm_axis says (thorn.py:1417).
    "md_axis_small": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (96, 64)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True, norm_axis=-1)),
        dict(orthogonalize=False, shapes=[(48, 16), (32, 8), (4, 6, 8), (64,)], init=("normal", 0.5),
             dtype="f32", opts=dict(lr=1e-3, decouple_md=True, norm_axis=-1, weight_decay=0.05)),
    ]),
    # Column counts that are not multiples of 8 on the FSDP2 path: the NS input rows travel with
    # the padded leading dimension of the NS kernels (world 1 and 2, uneven splits included).
    "shard_odd_cols": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(66, 37), (40, 20), (97, 64), (30, 90)], init=("normal", 0.02),
             dtype="f32", opts=dict(lr=2e-3, weight_decay=0.1)),
        dict(orthogonalize=False, shapes=[(21,)], init=("normal", 0.5), dtype="f32", opts=dict(lr=1e-3)),
    ]),
    # MD options: scalar gains on matrices (split_gain=False), gain_lr and gain_betas, "min" and
    # "max" target norms, and none_grad=False, which leaves the gradient in p.grad (under MD the
    # direction-recovered one, thorn.py:890-908).
    "md_options_small": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (96, 64)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True, split_gain=False, gain_lr=3e-3, gain_betas=(0.8, 0.99),
                       target_norm="min", none_grad=False)),
        dict(orthogonalize=True, shapes=[(64, 96)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, none_grad=False)),
        dict(orthogonalize=False, shapes=[(48, 16), (20, 12)], init=("normal", 0.5), dtype="f32",
             opts=dict(lr=1e-3, decouple_md=True, split_gain=False, target_norm="max", none_grad=False)),
    ]),
    # MD on conv kernels (batches of matrices: row and column gains per batch entry) with the
    # "init" target norm on an orthogonalized group (one target per matrix of the batch).
    "md_conv_small": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(8, 4, 3), (16, 8, 5), (4, 6, 6)], init=("normal", 0.05), dtype="f32",
             opts=dict(lr=4e-3, decouple_md=True, target_norm="init")),
        dict(orthogonalize=True, shapes=[(6, 8, 8)], init=("normal", 0.05), dtype="f32",
             opts=dict(lr=4e-3, decouple_md=True)),
    ]),
    # Matrices with fewer rows than ranks on the FSDP2 path: at world 2 the one-row matrices leave
    # the second shard empty (with and without MD).
    "shard_tiny_rows": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(1, 64), (3, 32), (66, 37)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, weight_decay=0.1)),
        dict(orthogonalize=True, shapes=[(1, 48), (5, 40)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True)),
    ]),
    # A callable target norm (thorn.py:601-602) on both group kinds with decouple_md: half the
    # initial Frobenius norm, as a Python float.
    "md_target_fn_small": dict(steps=3, grad_std=1e-3, groups=[
        dict(orthogonalize=True, shapes=[(64, 48), (32, 96)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True, target_norm=lambda p: 0.5 * _fro(p))),
        dict(orthogonalize=False, shapes=[(40, 12)], init=("normal", 0.5), dtype="f32",
             opts=dict(lr=1e-3, decouple_md=True, target_norm=lambda p: 0.5 * _fro(p))),
    ]),
    # update_rate 2 on one device (what setup_gradient_release(update_rate=2) sets): the moments
    # and the step count advance every step, the parameters every second step (thorn.py:1395,
    # 1681, 1707).
    "rate_small": dict(steps=4, grad_std=1e-3, update_rate=2, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (96, 64)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, weight_decay=0.1)),
        dict(orthogonalize=True, shapes=[(64, 96)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=8e-3, decouple_md=True)),
        dict(orthogonalize=False, shapes=[(64,), (40, 24)], init=("normal", 0.1), dtype="f32",
             opts=dict(lr=1e-3, weight_decay=0.1)),
    ]),
    # The reference's own FSDP2 path (its goldens come from 2 gloo ranks, make_sharded_golden.py):
    # even splits, no decouple_md (which the reference cannot run sharded on this torch).
    # update_rate 2 (what setup_gradient_release(update_rate=2) sets): the sharded reference
    # leaves a matrix whose step is not due out of the step entirely, step count included
    # (thorn.py:1485-1490, 1564), so after its first update no later step is ever due.
    "rate_shard": dict(steps=4, grad_std=1e-3, update_rate=2, groups=[
        dict(orthogonalize=True, shapes=[(64, 64), (96, 64), (64, 160)], init=("normal", 0.02), dtype="f32",
             opts=dict(lr=2e-3, weight_decay=0.1)),
    ]),
    # Row-sparse gradients on (R)AdamW parameters (thorn.py:1667-1698): duplicate rows, a 1-D
    # embedding, a step whose sparse gradient has no rows, Magma on sparse rows.
    "sparse_small": dict(steps=4, grad_std=1e-3, groups=[
        dict(orthogonalize=False, shapes=[(100, 16), (32,), (60, 8), (40,)], init=("normal", 0.1), dtype="f32",
             opts=dict(lr=1e-3, weight_decay=0.1), sparse={0: 24, 2: 10, 3: 6}, sparse_empty={2: [2]}),
        dict(orthogonalize=False, shapes=[(50, 12)], init=("normal", 0.1), dtype="f32",
             opts=dict(lr=1e-3, momentum_align=True, rectify=True, eps=1e-8), sparse={0: 16}),
    ]),
}


def build_params(case: dict):
    """Per group, a list of CPU tensors in the group's dtype."""
    torch.manual_seed(0)
    out = []
    for grp in case["groups"]:
        dt = TORCH_DTYPES[grp["dtype"]]
        ps = []
        for shp in grp["shapes"]:
            kind, val = grp["init"]
            if kind == "normal":
                t = torch.randn(shp) * val
            else:
                t = torch.full(shp, float(val))
            ps.append(t.to(dt))
        out.append(ps)
    return out


def build_grads(case: dict, s: int):
    """Grads for step ``s`` (0-based), per group, in the group's dtype.

    Parameters listed in a group's ``sparse`` map get a torch sparse COO
    gradient with one sparse dimension: ``nnz`` row indices drawn with
    replacement (so rows repeat) and one value row each; ``sparse_empty`` lists
    steps at which such a gradient has no rows at all.  Parameters listed in
    ``zero`` get an all-zero gradient at every step."""
    torch.manual_seed(1000 + s)
    out = []
    for grp in case["groups"]:
        dt = TORCH_DTYPES[grp["dtype"]]
        sparse, empty = grp.get("sparse", {}), grp.get("sparse_empty", {})
        gs = []
        for pi, shp in enumerate(grp["shapes"]):
            if pi in grp.get("zero", ()):
                gs.append(torch.zeros(shp, dtype=dt))
            elif pi in sparse:
                nnz = 0 if s in empty.get(pi, ()) else sparse[pi]
                idx = torch.randint(0, shp[0], (nnz,))
                vals = (torch.randn((nnz, *shp[1:])) * case["grad_std"]).to(dt)
                gs.append(torch.sparse_coo_tensor(idx[None], vals, shp))
            else:
                gs.append((torch.randn(shp) * case["grad_std"]).to(dt))
        out.append(gs)
    return out


def magma_seed() -> int:
    """The reference's Magma seed draw at state initialisation (thorn.py:1616-1620)."""
    return int(torch.randint(0, (1 << 63) - 1, (), dtype=torch.uint64).item())


def group_dicts(case: dict, params):
    """Reference-style param-group dicts (without the dtype bookkeeping)."""
    gs = []
    for grp, ps in zip(case["groups"], params):
        gs.append({"orthogonalize": grp["orthogonalize"], "params": ps, **grp["opts"]})
    return gs


@functools.lru_cache(maxsize=16)
def probe_vector(n: int) -> np.ndarray:
    """Deterministic projection vector for checksums (no RNG involved); cached and
    read-only, since a large tensor's checksums ask for the same length many times."""
    i = np.arange(n, dtype=np.float64)
    v = np.cos(0.37 * i + 0.11)
    v.setflags(write=False)
    return v


_SUM_BLOCK = 1 << 20


@functools.lru_cache(maxsize=16)
def probe_norm_sq(n: int) -> float:
    """Squared norm of ``probe_vector(n)``."""
    v = probe_vector(n)
    return float(sum(float((v[i:i + _SUM_BLOCK] ** 2).sum()) for i in range(0, n, _SUM_BLOCK)))


def checksum(a: np.ndarray) -> np.ndarray:
    """(sum, sum of squares, projection on ``probe_vector``) in float64, accumulated over
    blocks so that a large tensor needs no tensor-sized float64 temporaries."""
    flat = np.asarray(a).reshape(-1)
    pv = probe_vector(flat.size)
    out = np.zeros(3, dtype=np.float64)
    for i in range(0, flat.size, _SUM_BLOCK):
        x = flat[i:i + _SUM_BLOCK].astype(np.float64)
        out += (x.sum(), (x * x).sum(), (x * pv[i:i + _SUM_BLOCK]).sum())
    return out


def sq_dist(a: np.ndarray, b) -> float:
    """Sum of (a - b)^2 (of a^2 when b is None) in float64, over blocks."""
    fa = np.asarray(a).reshape(-1)
    fb = None if b is None else np.asarray(b).reshape(-1)
    s = 0.0
    for i in range(0, fa.size, _SUM_BLOCK):
        d = fa[i:i + _SUM_BLOCK].astype(np.float64)
        if fb is not None:
            d -= fb[i:i + _SUM_BLOCK]
        s += float((d * d).sum())
    return s


def rel_fro(a, b) -> float:
    """||a - b|| / ||b|| in float64 (||a - b|| when b is zero), accumulated over blocks."""
    a, b = np.broadcast_arrays(np.asarray(a), np.asarray(b))
    den = math.sqrt(sq_dist(b, None))
    num = math.sqrt(sq_dist(a, b))
    return num / den if den > 0 else num
