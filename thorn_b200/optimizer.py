"""Drop-in ``THORN`` optimizer whose step runs on the sm_100a kernels.

Public surface follows the reference ``thorn.THORN`` (thorn/thorn.py of
pykeio/THORN v3.1.1): the constructor (thorn.py:1271-1300), the group keys and
defaults of ``_THORNParameterGroup`` (thorn.py:535-612), ``step(closure=None, *,
param=None)`` (thorn.py:1738-1753), ``setup_gradient_release``
(thorn.py:1755-1776), ``polar_decomp_batch_size`` (thorn.py:1237) and the
optimizer-state layout (thorn.py:1591-1634), so ``state_dict`` /
``load_state_dict`` round-trip between the two.

Every pass over parameters, gradients and state (momentum, Newton-Schulz,
per-neuron norm, weight decay and apply, (R)AdamW, magnitude-direction
decoupling) is a kernel of ``libthorn_b200.so`` called through its C ABI.  Host
code plans launches and allocates scratch from the torch caching allocator.  Two
optional features use torch ops on the device the way the reference does: Magma's
three sums and score (thorn.py:806-836) and the row gather/scatter of sparse
gradients (thorn.py:1669-1698).  Parameters must live on a CUDA device; there is
no CPU path.

Extensions (all optional, off by default):
* group key ``state_dtype``: dtype of the optimizer state (the reference keeps
  it in the parameter dtype);
* attribute ``ns_dtype``: operand type of the Newton-Schulz GEMMs,
  ``torch.float16`` (the reference's choice, thorn.py:634-635) or
  ``torch.bfloat16``.
"""
from __future__ import annotations

import ctypes
from dataclasses import MISSING, dataclass, field, fields
from functools import partial
from math import prod
from typing import Any, Callable, Literal, Optional, Union

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.distributed.tensor import DTensor, Replicate
from torch.optim import Optimizer

from . import _native as N
from .coeffs import gram_ns_restarts, optimal_composition

__all__ = ["THORN", "THORNOrthoGroup", "THORNNonOrthoGroup", "THORNGroup"]

_TargetNorm = Union[Literal["init", "min", "max"], Callable[[torch.Tensor], Union[torch.Tensor, float]]]
LN_E_SUB_1 = 0.5413248546  # softplus(LN_E_SUB_1) == 1 (thorn.py:1602)

# Magma momentum-aligned masking (thorn.py:806-836): score temperature and EMA
# weight, and the 64-bit generator that decides which steps are masked.
MAGMA_TAU = 2.0
MAGMA_EMA = 0.9
_W1_C = 0xD07EBC63274654C7
_U64 = (1 << 64) - 1


def _w1rand(state: int) -> tuple[int, int]:
    """One generator step (thorn.py:800-804): state += C; t = state * (state ^ C)
    as a 128-bit product; output = high half ^ low half.  Returns (state, output)."""
    state = (state + _W1_C) & _U64
    t = state * (state ^ _W1_C)
    return state, ((t >> 64) ^ t) & _U64


@dataclass
class GroupConfig:
    """Per-group settings; same fields and defaults as thorn.py:535-561."""

    orthogonalize: bool
    params: list
    lr: float
    base_lr: float = field(init=False)
    none_grad: bool = field(default=True)
    weight_decay: float = field(default=0.1)
    betas: tuple = field(default_factory=lambda: (0.9, 0.95))
    scaling_mode: Optional[str] = field(default=None)
    target_rms: float = field(default=0.2)
    target_norm: Optional[_TargetNorm] = field(default=None)
    iters: int = field(default=5)
    rectify: bool = field(default=False)
    eps: float = field(default=0)
    lower_bound: float = field(default=1e-3)
    safety_factor: float = field(default=0.03)
    cushion: float = field(default=0.02)
    momentum_align: bool = field(default=False)
    coeffs: list = field(init=False)
    restarts: list = field(init=False)
    decouple_md: bool = field(default=False)
    gain_lr: float = field(default=1e-3)
    gain_betas: tuple = field(default_factory=lambda: (0.9, 0.95))
    norm_axis: Optional[Any] = field(default=None)
    split_gain: bool = field(default=True)
    force_per_neuron_norm: bool = field(default=False)

    @classmethod
    def from_kwargs(cls, **kw) -> "GroupConfig":
        return cls(**{k: kw[k] for k in kw if k in cls.__dataclass_fields__})

    def __post_init__(self):
        # validation messages as in thorn.py:567-573
        if self.lr < 0.0:
            raise ValueError(f"Invalid learning rate `{self.lr}`; should be >= 0")
        if not (0.0 <= self.betas[0] < 1.0):
            raise ValueError(f"Invalid beta1 `{self.betas[0]}`; should be in [0, 1)")
        if not (0.0 <= self.betas[1] < 1.0):
            raise ValueError(f"Invalid beta2 `{self.betas[1]}`; should be in [0, 1)")
        self.base_lr = self.lr
        self.coeffs = optimal_composition(self.lower_bound, self.iters, self.safety_factor, self.cushion)
        self.restarts = gram_ns_restarts(*self.coeffs)

    @property
    def scaling_mode_(self) -> str:
        if self.scaling_mode is None:
            return "md" if self.decouple_md else "moonlight"
        return self.scaling_mode

    @property
    def gain_lr_(self) -> float:
        return self.gain_lr * (float(self.lr) / self.base_lr) if self.base_lr else self.gain_lr

    def norm_axis_(self, p) -> Any:
        return self.norm_axis if self.norm_axis is not None else ((-2, -1) if p.ndim > 1 else -1)

    def needs_pnn(self, rows: int, cols: int) -> bool:
        """Per-neuron norm only for tall matrices unless forced (thorn.py:704-707)."""
        return self.betas[1] > 0 and (rows > cols or self.force_per_neuron_norm)

    def lr_scale(self, rows: int, cols: int) -> float:
        """thorn.py:768-780."""
        mode = self.scaling_mode_
        if mode == "md":
            return max(rows / cols, cols / rows) ** 0.5
        if mode == "moonlight":
            assert self.target_rms > 0
            return self.target_rms * (max(1, rows, cols) ** 0.5)
        if mode == "jordan":
            return max(1, rows / cols) ** 0.5
        raise ValueError(f"unknown scaling_mode {mode!r}")

    def rect(self, step) -> float:
        """RAdam rectification (thorn.py:782-798)."""
        beta2 = self.betas[1]
        if beta2 > 0.0:
            rho_inf = 2 / (1 - beta2) - 1
            rho = rho_inf - 2 * step * (beta2 ** step) / (1 - beta2 ** step)
            r = ((rho - 4) * (rho - 2) * rho_inf / ((rho_inf - 4) * (rho_inf - 2) * rho)) ** 0.5 if rho > 4.0 else 0.0
            return r ** float(self.rectify)
        return 1.0

    def target_norm_(self, p: torch.Tensor) -> torch.Tensor:
        """thorn.py:597-612 (run once, at state creation)."""
        tn = self.target_norm
        if tn is None:
            tn = "max" if self.orthogonalize else "init"
        if callable(tn):
            tn = tn(p)
        elif tn == "init":
            tn = p.norm(dim=self.norm_axis_(p), keepdim=True)
        elif tn == "min":
            tn = min(p.size(-2), p.size(-1)) ** 0.5
        elif tn == "max":
            tn = max(p.size(-2), p.size(-1)) ** 0.5
        if isinstance(tn, (float, int)):
            return torch.full((), tn, dtype=p.dtype, device=p.device)
        return tn.to(dtype=p.dtype, device=p.device)


THORNOrthoGroup = dict
THORNNonOrthoGroup = dict
THORNGroup = dict


def balanced_cap(total: int, cap: int) -> int:
    """Batch size that splits ``total`` matrices into the fewest batches of at most ``cap``
    with sizes as equal as possible (64 with cap 18: four batches of 16, not 18+18+18+10):
    the last batch's GEMM waves are then as full as the others'."""
    if total <= 0 or cap <= 0:
        return max(1, cap)
    k = -(-total // cap)
    return -(-total // k)


def _local(t):
    return t.to_local() if isinstance(t, DTensor) else t


def _sharded_gains(p: DTensor):
    """Magnitude gains of a Shard(0) parameter as DTensors."""
    mesh, pl = p.device_mesh, p.placements
    loc = p.to_local()
    row_shape = (*p.shape[:-1], 1)
    rg = torch.full((*loc.shape[:-1], 1), LN_E_SUB_1, dtype=p.dtype, device=loc.device)
    row = DTensor.from_local(rg, mesh, pl, run_check=False, shape=row_shape,
                             stride=torch.empty(row_shape, device="meta").stride())
    col_shape = (*p.shape[:-2], 1, p.shape[-1])
    if p.ndim == 2:
        cg = torch.full(col_shape, LN_E_SUB_1, dtype=p.dtype, device=loc.device)
        col = DTensor.from_local(cg, mesh, [Replicate()] * mesh.ndim, run_check=False)
    else:  # batch dimension split: each rank holds whole matrices and their column gains
        cg = torch.full((*loc.shape[:-2], 1, p.shape[-1]), LN_E_SUB_1, dtype=p.dtype, device=loc.device)
        col = DTensor.from_local(cg, mesh, pl, run_check=False, shape=col_shape,
                                 stride=torch.empty(col_shape, device="meta").stride())
    return row, col


def _mat_view(shape) -> tuple[int, int, int]:
    """(batch, rows, cols) view of a tensor: leading dims are a batch (thorn.py:628-633)."""
    if len(shape) >= 2:
        return int(prod(shape[:-2])), int(shape[-2]), int(shape[-1])
    if len(shape) == 1:
        return 1, 1, int(shape[0])
    return 1, 1, 1


def _row_norm_axis(cfg, p) -> bool:
    """Whether the (R)AdamW decouple_md renorm of ``p`` runs per last-dim slice.

    norm_axis (thorn.py:594-595) defaults to the last two dims of a matrix (one norm per
    matrix of the batch) and to the last dim of a vector; a norm_axis naming only the last
    dim of a tensor of rank >= 2 renorms every row (thorn.py:605, 1717).  Other axes are not
    implemented here and raise."""
    ax = cfg.norm_axis_(p)
    axes = tuple(ax) if isinstance(ax, (tuple, list)) else (ax,)
    nd = max(p.ndim, 1)
    axes = tuple(sorted(a % nd for a in axes))
    if p.ndim <= 1:
        if axes == (0,):
            return False
    elif axes == (nd - 2, nd - 1):
        return False
    elif axes == (nd - 1,):
        return True
    raise NotImplementedError(f"decouple_md with norm_axis={ax!r} on a {p.ndim}-D parameter is not implemented by "
                              "thorn_b200 (the last dim, or the default, is)")


def _renorm_view(it) -> tuple[int, int, int]:
    """(batch, rows, cols) over which the renorm's norms are taken: per matrix, or per row."""
    return (it.B * it.R, 1, it.C) if getattr(it, "row_norm", False) else (it.B, it.R, it.C)


class _Arena:
    """Carves fp32 scratch views out of a few buffers ("regions").

    Region "z" is zero-filled; every other region is uninitialised.  Values
    that are all-reduced together are allocated from one region so a single
    collective covers them.
    """

    def __init__(self):
        self.sizes: dict = {}
        self.bufs: dict = {}

    def alloc(self, n, region="r"):
        off = self.sizes.get(region, 0)
        self.sizes[region] = off + (n + 3) // 4 * 4
        return (region, off, n)

    def empty(self, n):
        return self.alloc(n, "r")

    def zeros(self, n):
        return self.alloc(n, "z")

    def materialize(self, device, zero=()):
        """Allocate the regions; "z" and the regions named in ``zero`` start at zero."""
        for reg, n in self.sizes.items():
            make = torch.zeros if (reg == "z" or reg in zero) else torch.empty
            self.bufs[reg] = make(max(4, n), dtype=torch.float32, device=device)

    def region(self, name):
        return self.bufs[name][:self.sizes[name]]

    def get(self, h):
        if h is None:
            return None
        reg, off, n = h
        return self.bufs[reg][off:off + n]

    def ptr(self, h):
        t = self.get(h)
        return None if t is None else t.data_ptr()


class _Item:
    __slots__ = ("p", "g", "state", "B", "R", "C", "apply", "pdt", "sdt", "normsq", "rs", "cs", "sig_r", "sig_c",
                 "rgs", "cgs", "rs_new", "cs_new", "pnorm", "scalar", "ggrad_r", "ggrad_c", "split", "scale",
                 "m_rows", "v_rows", "row_norm")


class THORN(Optimizer):
    """THORN optimizer (see module docstring)."""

    # elements per Newton-Schulz batch (thorn.py:1237; 0 disables batching).  The
    # reference defaults to 32 Mi; with 180 GB of HBM and 148 SMs the B200 path
    # defaults to 512 Mi, so the 14336x4096 matrices of an 8B model batch by 8 and the
    # symmetric 4096x4096 products of their Gram iteration fill 15 waves of the 74
    # SM pairs instead of 7.4 (the Llama-3-8B step's NS phase: 289.6 vs 295.7 ms).
    polar_decomp_batch_size: int = 512 * 1024 * 1024
    ns_dtype: torch.dtype = torch.float16
    # when a list: each Newton-Schulz call appends (start event, end event, dense-equivalent
    # FLOPs, executed FLOPs, (batch, rows, cols)); events are recorded on the launching stream
    profile_ns: Optional[list] = None
    # when a list: each momentum pass of an orthogonalized group appends (start event, end
    # event, algorithmic bytes: g read, m read + write, p read + write with decouple_md)
    profile_momentum: Optional[list] = None
    # when a list: each sharded step appends a list of (stage name, event) pairs recorded on
    # the launching stream at the end of each stage (the first is the step's start); with
    # pipeline_exchange the exchange and NS stages overlap and are timed as one
    profile_stages: Optional[list] = None
    # sharded path: exchange row slabs in waves of NS batches so that transfers overlap
    # the owners' Newton-Schulz work (False: every slab moves before any NS starts)
    pipeline_exchange: bool = False
    # sharded path: "all_to_all" (one all_to_all_single collective per exchange),
    # "rounds" (world - 1 pairwise point-to-point rounds) or "peer" (ranks of one node:
    # the NS input pass stores rows into the owners' CUDA-IPC-mapped arenas, results come
    # back by copy-engine peer copies, flags order both; see sharded.peer_exchange_and_ns).
    # On 8 B200s the Llama-3-8B step takes 58.9 ms with all_to_all and 95.8 ms with rounds
    exchange: str = "all_to_all"

    def __init__(self, params, *, backend=torch.cuda, **conf):
        self._update_rate = 1
        self.backend = backend
        param_groups = THORN._auto_assign(params, **conf) if isinstance(params, nn.Module) else list(params)
        for group in param_groups:
            assert "orthogonalize" in group
            if group["orthogonalize"]:
                assert all(map(lambda x: x.ndim >= 2, group["params"])), \
                    "Only parameters with ndim >= 2 can be orthogonalized"
        self.is_distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank() if self.is_distributed else None
        self.comm_stream = None
        self.compute_stream = None
        defaults = dict()
        for f in fields(GroupConfig):
            if f.default is not MISSING:
                defaults[f.name] = f.default
            elif f.default_factory is not MISSING:
                defaults[f.name] = f.default_factory()
        super().__init__(param_groups, defaults)
        self._param_to_group: dict[int, dict[str, Any]] = {}
        for group in self.param_groups:
            for p in group["params"]:
                self._param_to_group[id(p)] = group
        self._err = {}
        self._scratch_bufs = {}
        self._targets = {}
        self._ones_cache = {}
        if isinstance(params, nn.Module) and conf.get("gradient_release", False):
            self.setup_gradient_release(params)

    # ------------------------------------------------------------------ API
    @staticmethod
    def _auto_assign(module: nn.Module, **keys) -> list:
        """thorn.py:1302-1331: ndim>=2 params outside embeddings and lm_head are orthogonalized."""
        emb = set()
        module.apply(lambda m: emb.add(id(m.weight)) if isinstance(m, nn.Embedding) else None)
        ortho, regular = [], []
        for name, param in module.named_parameters():
            if param.ndim >= 2 and "lm_head" not in name and id(param) not in emb:
                ortho.append(param)
            else:
                regular.append(param)
        return [{"orthogonalize": True, "params": ortho, **keys}, {"orthogonalize": False, "params": regular, **keys}]

    @torch.no_grad()
    def step(self, closure=None, *, param=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if param is None:
            for group in self.param_groups:
                self._step_params(group["params"], GroupConfig.from_kwargs(**group), group)
        else:
            group = self._param_to_group[id(param)]
            self._step_params([param], GroupConfig.from_kwargs(**group), group)
        return loss

    def setup_gradient_release(self, model: nn.Module, update_rate: int = 1, ignore_existing_hooks: bool = False):
        """thorn.py:1755-1776: step each parameter from its post-accumulate-grad hook."""
        def hook(param, optimizer):
            optimizer.step(param=param)
            param.grad = None

        hooks = []
        for p in model.parameters():
            if p.requires_grad:
                if p._post_accumulate_grad_hooks and not ignore_existing_hooks:
                    for h in hooks:
                        h.remove()
                    raise ValueError("Model already has post_accumulate_grad_hooks. If this is expected, pass "
                                     "`ignore_existing_hooks=True`.")
                hooks.append(p.register_post_accumulate_grad_hook(partial(hook, optimizer=self)))
        model._gradient_release_hooks = hooks
        self._update_rate = update_rate

    def release_peer_memory(self) -> None:
        """Free the device arenas of the peer-memory exchange (``exchange = "peer"``) and
        unmap the peers' ones.  Collective: every rank of the shard group calls it at the
        same point, between steps.  A later peer-exchange step allocates them again."""
        arenas = self.__dict__.get("_peer_arenas", {})
        if arenas:
            lib = N.load()
            for dev, pa in arenas.items():
                pa.release(lib, dev)
            arenas.clear()

    def device_error(self) -> bool:
        """True if a bounded device-side wait of a kernel gave up (reads a device flag; syncs)."""
        return any(int(t.item()) != 0 for t in self._err.values())

    # ------------------------------------------------------------- routing
    def _init_state(self, p, state, cfg: GroupConfig, gdict):
        state["step"] = 1
        sdt = gdict.get("state_dtype") or p.dtype
        state["moment"] = torch.zeros_like(p, dtype=sdt)
        if not cfg.orthogonalize:
            state["variance"] = torch.zeros_like(p, dtype=sdt)
        if cfg.decouple_md:
            if p.ndim > 1 and cfg.split_gain:
                if isinstance(p, DTensor) and not all(isinstance(pl, Replicate) for pl in p.placements):
                    # Shard(0): row gains are split like the rows; column gains of a 2-D matrix are
                    # replicated (the reference creates them at the global shape, thorn.py:1604-1605)
                    state["row_gain"], state["col_gain"] = _sharded_gains(p)
                else:
                    state["row_gain"] = torch.full((*p.shape[:-1], 1), LN_E_SUB_1, dtype=p.dtype, device=p.device)
                    state["col_gain"] = torch.full((*p.shape[:-2], 1, *p.shape[-1:]), LN_E_SUB_1, dtype=p.dtype,
                                                   device=p.device)
                for k in ("row_gain", "col_gain"):
                    state[f"{k}_moment"] = torch.zeros_like(state[k])
                    state[f"{k}_variance"] = torch.zeros_like(state[k])
            else:
                state["gain"] = torch.full((), LN_E_SUB_1, dtype=p.dtype, device=p.device)
                state["gain_moment"] = torch.zeros((), dtype=p.dtype, device=p.device)
                state["gain_variance"] = torch.zeros((), dtype=p.dtype, device=p.device)
            state["target_norm"] = cfg.target_norm_(p)
        if cfg.momentum_align:
            # drawn from torch's generator of the gradient's device, so torch.manual_seed
            # reproduces it (thorn.py:1616-1633): a value in [0, 2^63 - 1).  The reference
            # asks for uint64; int64 draws the same value from the same generator state and
            # every device type implements it.
            g = p.grad
            seed = int(torch.randint(0, (1 << 63) - 1, (), device=_local(g).device, dtype=torch.int64).item())
            if isinstance(p, DTensor) and cfg.orthogonalize and \
                    not all(isinstance(pl, Replicate) for pl in p.placements):
                # every shard of a matrix must mask the same steps: take the first shard's seed
                from .sharded import shard_group
                ranks, group = shard_group(p, self.rank)
                box = [seed]
                dist.broadcast_object_list(box, src=ranks[0], group=group)
                seed = int(box[0])
            state["random_state"] = seed
            state["s"] = torch.ones((), dtype=p.dtype, device=_local(p).device)

    def _magma(self, items, cfg, recovered: bool, group=None) -> None:
        """Magma masking (thorn.py:806-836) for a list of launch records.

        Sets ``it.scale``, the LR multiplier, on every item, and clears ``it.apply``
        where the generator masks the step.  The score compares the gradient
        (direction-recovered under decouple_md when ``recovered``) with the moment
        before this step's update (``it.m_rows`` when set: the gathered moment
        rows of a sparse update).  The three sums of every item come from one
        ``thorn_magma_stats_multi`` launch per dtype pair (:meth:`_magma_stats`);
        the cosine, the sigmoid and the smoothed score of all items are formed from
        them with a few vectorised ops.  ``group``: shard process group: the sums
        are all-reduced in one call and the cosine is formed in fp32
        (thorn.py:820-829).  The smoothed scores of all items are read back to the
        host once per call (the reference reads each with ``.item()``).
        """
        for it in items:
            it.scale = 1.0
        if not cfg.momentum_align or not items:
            return
        stats = self._magma_stats(items, cfg, recovered)
        scores = self._magma_scores(items, stats, group)
        for it, v in zip(items, scores):
            st = it.state
            st["random_state"], out = _w1rand(int(st["random_state"]))
            if out % 2:
                it.scale, it.apply = 0.0, False
            else:
                it.scale = v

    def _magma_stats(self, items, cfg, recovered: bool) -> torch.Tensor:
        """``[len(items), 3]`` fp64 device tensor: sum g*m, sum g^2, sum m^2 of every item
        (thorn.py:818-826), the gradient recovered as ``g * gain`` under decouple_md
        (thorn.py:896-905) inside the kernel.  Items with no elements keep zeros."""
        lib = N.load()
        dev = items[0].g.device
        stream = N.stream_of(dev)
        stats = torch.zeros((len(items), 3), dtype=torch.float64, device=dev)
        recs, keep = [], []
        for it in items:
            st = it.state
            g = it.g if it.g.is_contiguous() else it.g.contiguous()
            m = getattr(it, "m_rows", None)
            if m is None:
                m = _local(st["moment"])
            if not m.is_contiguous():
                m = m.contiguous()
            if m.shape != g.shape:
                raise ValueError(f"Magma: moment shape {tuple(m.shape)} differs from gradient {tuple(g.shape)}")
            rg = cg = None
            scalar = 0
            if recovered and cfg.decouple_md:
                if it.split:
                    rg, cg = _local(st["row_gain"]), _local(st["col_gain"])
                else:
                    rg, scalar = _local(st["gain"]), 1
            keep.append((g, m))
            recs.append((g, m, rg, cg, scalar) + _mat_view(g.shape))
        scr = self._scratch(dev, [lib.thorn_magma_scratch_bytes(B, R, C) for *_, B, R, C in recs])
        by_dt: dict = {}
        base = stats.data_ptr()
        for i, ((g, m, rg, cg, scalar, B, R, C), sp) in enumerate(zip(recs, scr)):
            if rg is not None and rg.dtype != g.dtype:
                raise TypeError("Magma: the gains must have the gradient dtype")
            by_dt.setdefault((N.dtype_code(g.dtype), N.dtype_code(m.dtype)), []).append(N.MagmaTensor(
                g.data_ptr(), m.data_ptr(), None if rg is None else rg.data_ptr(),
                None if cg is None else cg.data_ptr(), scalar, B, R, C, base + 24 * i, sp))
        for (gc, mc), ts in by_dt.items():
            N.check(lib.thorn_magma_stats_multi(N.array(N.MagmaTensor, ts), len(ts), gc, mc, stream),
                    "magma_stats_multi")
        del keep  # contiguous copies: freed in stream order after the launch
        return stats

    @staticmethod
    def _magma_scores(items, stats: torch.Tensor, group=None) -> list:
        """Smoothed scores ``s`` of the items from their three sums (thorn.py:818-833), stored
        in ``it.state["s"]``; returns them as host floats.

        Single device: the cosine of ``F.cosine_similarity`` (each norm clamped at 1e-8)
        from the fp64 sums, in the promoted dtype of gradient and moment.  Sharded: the sums
        rounded to fp32, all-reduced over ``group``, dot / (|g| |m|) clamped at 1e-12 in fp32.
        Then ``s = 0.9 s + 0.1 sigmoid(cos / 2)`` with torch's dtype promotion, as the
        reference's 0-d tensor ops, for all items of one dtype pair at once."""
        n = len(items)
        if group is not None:
            st32 = stats.float()
            dist.all_reduce(st32, group=group)
            cos = st32[:, 0] / (st32[:, 1].sqrt() * st32[:, 2].sqrt()).clamp_min(1e-12)
            cdts = [torch.float32] * n
        else:
            cos = (stats[:, 0] / (stats[:, 1].sqrt().clamp_min(1e-8) * stats[:, 2].sqrt().clamp_min(1e-8))).float()
            cdts = [torch.promote_types(it.g.dtype, (it.m_rows if getattr(it, "m_rows", None) is not None
                                                     else _local(it.state["moment"])).dtype) for it in items]
        keys: dict = {}
        for j, it in enumerate(items):
            keys.setdefault((cdts[j], it.state["s"].dtype), []).append(j)
        order, parts = [], []
        for (cdt, _sdt), js in keys.items():
            c = (cos if len(js) == n else torch.stack([cos[j] for j in js])).to(cdt)
            s_old = torch.stack([items[j].state["s"] for j in js])
            s_new = MAGMA_EMA * s_old + (1 - MAGMA_EMA) * torch.sigmoid(c / MAGMA_TAU)
            for t, j in enumerate(js):
                items[j].state["s"] = s_new[t]
            order += js
            parts.append(s_new.float())
        vals = torch.cat(parts).tolist()
        out = [0.0] * n
        for j, v in zip(order, vals):
            out[j] = v
        return out

    def _step_params(self, params, cfg: GroupConfig, gdict):
        sharded, local = [], []
        for p in params:
            if p is None or p.grad is None:
                continue
            if p.grad.is_sparse:
                if cfg.orthogonalize or isinstance(p.data, DTensor):
                    raise NotImplementedError("sparse gradients are implemented for (R)AdamW parameters on one "
                                              "device only")
                if cfg.decouple_md or p.grad.sparse_dim() != 1:
                    p.grad = p.grad.to_dense()  # thorn.py:1667-1668
            state = self.state[p]
            if "step" not in state:
                self._init_state(p, state, cfg, gdict)
            is_sharded = isinstance(p.data, DTensor) and not all(isinstance(pl, Replicate) for pl in p.placements)
            if is_sharded and cfg.orthogonalize:
                sharded.append(p)
            elif is_sharded and cfg.decouple_md:
                raise NotImplementedError("decouple_md on sharded (R)AdamW parameters is not implemented by "
                                          "thorn_b200")
            else:
                local.append(p)
        if sharded:
            from .sharded import sharded_ortho_step
            sharded_ortho_step(self, sharded, cfg)
        by_dev: dict = {}
        for p in local:
            by_dev.setdefault(_local(p).device, []).append(p)
        for dev, ps in by_dev.items():
            if dev.type != "cuda":
                raise RuntimeError(f"thorn_b200 runs its step on CUDA devices only; got a parameter on {dev}")
            with torch.cuda.device(dev):
                if cfg.orthogonalize:
                    self._ortho_local(ps, cfg)
                else:
                    self._adam_local(ps, cfg)

    @staticmethod
    def _profile_start(log):
        if log is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    @staticmethod
    def _profile_end(log, ev0, nbytes):
        if log is not None:
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record()
            log.append((ev0, ev1, nbytes))

    @staticmethod
    def _momentum_bytes(items, md: bool) -> int:
        """Compulsory bytes of the momentum pass: g read, m read and written, p read and
        written when directions are recovered (decouple_md)."""
        tot = 0
        for it in items:
            n = it.B * it.R * it.C
            tot += n * (it.g.element_size() + 2 * _local(it.state["moment"]).element_size()
                        + (2 * it.p.element_size() if md else 0))
        return tot

    def _scratch(self, dev, sizes):
        """Pointers to disjoint regions of a per-device scratch buffer (zeroed once).

        The kernels leave the counters of their scratch at zero, so the buffer is
        reused by every call without clearing; calls on one stream run in order.
        """
        offs, total = [], 0
        for sz in sizes:
            offs.append(total)
            total += (int(sz) + 255) // 256 * 256
        buf = self._scratch_bufs.get(dev)
        if buf is None or buf.numel() < total:
            buf = torch.zeros(max(total, 1 << 20), dtype=torch.uint8, device=dev)
            self._scratch_bufs[dev] = buf
        base = buf.data_ptr()
        return [base + o for o in offs]

    def _err_flag(self, dev):
        t = self._err.get(dev)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=dev)
            self._err[dev] = t
        return t

    # ------------------------------------------------------ shared helpers
    def _items(self, params, cfg, arena: _Arena, ortho: bool, reduce_regions: bool = False):
        """Per-parameter launch records.  With ``reduce_regions`` the values the
        sharded path all-reduces (sums of squares, column-gain and scalar-gain
        gradients) are laid out contiguously in regions "red1" / "red2"."""
        red1 = "red1" if reduce_regions else "r"
        red2 = "red2" if reduce_regions else "r"
        items = []
        for p in params:
            st = self.state[p]
            it = _Item()
            it.p = _local(p)
            g = _local(p.grad)
            if not g.is_contiguous():
                g = g.contiguous()
            it.g = g
            if not it.p.is_contiguous():
                raise ValueError("thorn_b200 needs contiguous parameters")
            it.state = st
            it.B, it.R, it.C = _mat_view(it.p.shape)
            it.apply = (st["step"] + 1) % self._update_rate == 0
            it.pdt = it.p.dtype
            it.sdt = _local(st["moment"]).dtype
            N.dtype_code(it.pdt), N.dtype_code(it.sdt)
            if g.dtype != it.pdt:
                raise TypeError(f"gradient dtype {g.dtype} differs from parameter dtype {it.pdt}")
            it.normsq = arena.alloc(it.B, red1) if ortho else None
            it.split = "row_gain" in st
            it.scalar = "gain" in st
            if cfg.decouple_md:
                nr, nc = (it.B * it.R, it.B * it.C) if it.split else (1, 1)
                it.rs, it.sig_r, it.rs_new = arena.empty(nr), arena.empty(nr), arena.empty(nr)
                # row-gain gradients are local to the rows a rank holds; a scalar gain sums everything
                it.rgs = arena.empty(nr) if it.split else arena.alloc(1, red1)
                if it.split:
                    it.cs, it.sig_c, it.cs_new = arena.empty(nc), arena.empty(nc), arena.empty(nc)
                    it.cgs = arena.alloc(nc, red1)
                else:
                    it.cs = it.sig_c = it.cs_new = it.cgs = None
                # per-slice norms when norm_axis names the last dim of a matrix ((R)AdamW renorm)
                it.row_norm = not ortho and _row_norm_axis(cfg, it.p)
                it.pnorm = arena.alloc(it.B * it.R if it.row_norm else it.B, red2)
            items.append(it)
        return items

    def _md_prep(self, items, arena, new: bool, stream):
        """softplus (and sigmoid) of the gains as fp32, one launch per dtype."""
        lib = N.load()
        by_dt: dict = {}
        for it in items:
            st = it.state
            if it.split:
                pairs = [(st["row_gain"], it.rs_new if new else it.rs, None if new else it.sig_r),
                         (st["col_gain"], it.cs_new if new else it.cs, None if new else it.sig_c)]
            else:
                pairs = [(st["gain"], it.rs_new if new else it.rs, None if new else it.sig_r)]
            for gain, sp, sig in pairs:
                gl = _local(gain)
                by_dt.setdefault(N.dtype_code(it.pdt), []).append(
                    N.MdPrepTensor(gl.data_ptr(), arena.ptr(sp), arena.ptr(sig), gl.numel()))
        for pc, ts in by_dt.items():
            N.check(lib.thorn_md_prep_multi(N.array(N.MdPrepTensor, ts), len(ts), pc, stream), "md_prep_multi")

    def _md_gains(self, items, cfg, arena, stream):
        """Gradient of the gains and their Adam step (thorn.py:910-967)."""
        lib = N.load()
        grads_by_dt: dict = {}
        adam_by_dt: dict = {}
        keep = []
        for it in items:
            if not it.apply:
                continue
            st = it.state
            pc = N.dtype_code(it.pdt)
            keys = [("row_gain", it.rgs, it.sig_r), ("col_gain", it.cgs, it.sig_c)] if it.split else \
                [("gain", it.rgs, it.sig_r)]
            step = st["step"]
            bc1 = 1 / (1 - cfg.gain_betas[0] ** step)
            bc2 = 1 / (1 - cfg.gain_betas[1] ** step)
            for key, gsum, sig in keys:
                gain = _local(st[key])
                keep.append((gain, gsum, sig, pc, key, st, bc1, bc2))
        # gain gradients: one buffer per dtype for all gains of the group
        sizes: dict = {}
        for gain, *_rest in keep:
            sizes[gain.dtype] = sizes.get(gain.dtype, 0) + (gain.numel() + 7) // 8 * 8
        bufs = {dt: torch.empty(max(8, n), dtype=dt, device=keep[0][0].device) for dt, n in sizes.items()} \
            if keep else {}
        offs = {dt: 0 for dt in bufs}
        for gain, gsum, sig, pc, key, st, bc1, bc2 in keep:
            n = gain.numel()
            grad = bufs[gain.dtype][offs[gain.dtype]:offs[gain.dtype] + n]
            offs[gain.dtype] += (n + 7) // 8 * 8
            grads_by_dt.setdefault(pc, []).append(
                N.MdGradTensor(arena.ptr(gsum), arena.ptr(sig), grad.data_ptr(), n))
            mom, var = _local(st[key + "_moment"]), _local(st[key + "_variance"])
            adam_by_dt.setdefault((pc, N.dtype_code(mom.dtype)), []).append(
                N.AdamTensor(gain.data_ptr(), grad.data_ptr(), mom.data_ptr(), var.data_ptr(), n,
                             cfg.gain_lr_, bc1, bc2, 0))
        for pc, ts in grads_by_dt.items():
            N.check(lib.thorn_md_gain_grad_multi(N.array(N.MdGradTensor, ts), len(ts), pc, stream),
                    "md_gain_grad_multi")
        for (pc, sc), ts in adam_by_dt.items():
            N.check(lib.thorn_adamw_multi(N.array(N.AdamTensor, ts), len(ts), pc, sc, cfg.gain_betas[0],
                                          cfg.gain_betas[1], 0.0, float(cfg.eps), stream), "adamw_multi(gains)")
        keep.append(bufs)
        del keep

    def _target_f32(self, st):
        """fp32 copy of a parameter's target norm, cached while the state tensor is unchanged
        (same object, same in-place version counter)."""
        t = st["target_norm"]
        loc = _local(t)
        hit = self._targets.get(id(t))
        if hit is not None and hit[0] is t and hit[1] == loc._version:
            return hit[2]
        f = loc.reshape(-1).float().contiguous()
        self._targets[id(t)] = (t, loc._version, f)
        return f

    def _md_finalize(self, items, arena, renorm_of, stream):
        lib = N.load()
        by_dt: dict = {}
        keep = []
        rows_first: dict = {}  # per-row renorms, launched before the gains are applied
        for it in items:
            st = it.state
            normsq = arena.ptr(it.pnorm) if (it.apply and renorm_of(it)) else None
            tgt = self._target_f32(st)
            keep.append(tgt)
            stride = 0 if tgt.numel() == 1 else 1
            vb, vr, vc = _renorm_view(it)
            if stride and tgt.numel() != vb:
                raise NotImplementedError("target_norm must be a scalar or one value per renormed slice")
            if getattr(it, "row_norm", False) and normsq is not None:
                # p *= target / (||row|| + 1e-8) on the (B*R, 1, C) view, gains of one, then the
                # gains on the natural view: the same roundings as one fused pass
                ones = self._ones(it.p.device)
                rows_first.setdefault(N.dtype_code(it.pdt), []).append(N.MdFinalTensor(
                    it.p.data_ptr(), normsq, tgt.data_ptr(), stride, ones.data_ptr(), None, 1, vb, vr, vc))
                normsq = None
            t = N.MdFinalTensor(it.p.data_ptr(), normsq, tgt.data_ptr(), stride, arena.ptr(it.rs_new),
                                arena.ptr(it.cs_new), 0 if it.split else 1, it.B, it.R, it.C)
            by_dt.setdefault(N.dtype_code(it.pdt), []).append(t)
        for pc, ts in rows_first.items():
            N.check(lib.thorn_md_finalize_multi(N.array(N.MdFinalTensor, ts), len(ts), pc, stream), "md_finalize")
        for pc, ts in by_dt.items():
            N.check(lib.thorn_md_finalize_multi(N.array(N.MdFinalTensor, ts), len(ts), pc, stream), "md_finalize")
        return keep

    def _ones(self, dev):
        """A device float 1.0 (the unit gain of a renorm-only pass)."""
        t = self._ones_cache.get(dev)
        if t is None:
            t = torch.ones(1, dtype=torch.float32, device=dev)
            self._ones_cache[dev] = t
        return t

    def _finish(self, params, cfg):
        for p in params:
            if cfg.none_grad:
                p.grad = None
            self.state[p]["step"] += 1

    # ------------------------------------------- orthogonalized group (1 GPU)
    def _ortho_local(self, params, cfg: GroupConfig):
        """thorn.py:1376-1457 on the kernels: momentum -> NS input -> NS -> pnn -> apply (-> md)."""
        lib = N.load()
        dev = _local(params[0]).device
        stream = N.stream_of(dev)
        err = self._err_flag(dev)
        md = cfg.decouple_md
        arena = _Arena()
        items = self._items(params, cfg, arena, ortho=True)
        # Magma looks at the direction-recovered gradient and the moment before this step (thorn.py:1389-1392)
        self._magma(items, cfg, recovered=True)
        b1 = float(cfg.betas[0])
        ns_code = N.dtype_code(self.ns_dtype)
        # NS batches: bucket by (rows, cols, p dtype, state dtype)
        buckets: dict = {}
        for it in items:
            if it.apply:
                buckets.setdefault((it.R, it.C, it.pdt, it.sdt), []).append(it)
        chunks = []
        for (R, C, pdt, sdt), its in buckets.items():
            cap = max(1, self.polar_decomp_batch_size // max(1, R * C)) if self.polar_decomp_batch_size > 0 else 1
            cap = balanced_cap(sum(it.B for it in its), cap)
            cur, n = [], 0
            for it in its:
                if cur and n + it.B > cap:
                    chunks.append((R, C, pdt, sdt, cur))
                    cur, n = [], 0
                cur.append(it)
                n += it.B
            if cur:
                chunks.append((R, C, pdt, sdt, cur))
        pnn_h = {}
        for ci, (R, C, pdt, sdt, its) in enumerate(chunks):
            if cfg.needs_pnn(R, C):
                nb = sum(it.B for it in its)
                pnn_h[ci] = (arena.empty(nb * R), arena.empty(2 * nb))
        arena.materialize(dev)

        if md:
            self._md_prep(items, arena, new=False, stream=stream)
        write_grad = 1 if (md and not cfg.none_grad) else 0
        by_dt: dict = {}
        scr = self._scratch(dev, [lib.thorn_ortho_pre_scratch_bytes(it.B, it.R, it.C, 1 if md else 0) for it in items])
        for it, sp in zip(items, scr):
            t = N.OrthoPreTensor(it.p.data_ptr() if md else None, it.g.data_ptr(), _local(it.state["moment"]).data_ptr(),
                                 arena.ptr(it.normsq), it.B, it.R, it.C,
                                 arena.ptr(it.rs) if md else None, arena.ptr(it.cs) if md else None,
                                 1 if (md and not it.split) else 0,
                                 arena.ptr(it.rgs) if md else None, arena.ptr(it.cgs) if md else None, sp)
            by_dt.setdefault((it.pdt, it.sdt), []).append(t)
        ev = self._profile_start(self.profile_momentum)
        for (pdt, sdt), ts in by_dt.items():
            udt = pdt if pdt == sdt else torch.float32
            N.check(lib.thorn_ortho_pre_multi(N.array(N.OrthoPreTensor, ts), len(ts), N.dtype_code(pdt),
                                              N.dtype_code(sdt), N.dtype_code(udt), b1, 1 if md else 0, write_grad,
                                              stream), "ortho_pre_multi")
        self._profile_end(self.profile_momentum, ev, self._momentum_bytes(items, md))
        if md:
            self._md_gains(items, cfg, arena, stream)

        coeffs = (ctypes.c_double * (3 * max(1, cfg.iters)))(*[x for abc in cfg.coeffs[:cfg.iters] for x in abc])
        rs = list(cfg.restarts)
        restarts = (ctypes.c_int32 * max(1, len(rs)))(*rs)
        for ci, (R, C, pdt, sdt, its) in enumerate(chunks):
            nb = sum(it.B for it in its)
            ldc = int(lib.thorn_ns_ld(C))
            X = torch.empty((nb, R, ldc), dtype=self.ns_dtype, device=dev)
            U = torch.empty((nb, R, C), dtype=self.ns_dtype, device=dev)
            casts, off = [], 0
            esz = X.element_size()
            for it in its:
                casts.append(N.NsCastTensor(it.g.data_ptr(), _local(it.state["moment"]).data_ptr(), arena.ptr(it.normsq),
                                            X.data_ptr() + off * R * ldc * esz, it.B, it.R, it.C,
                                            arena.ptr(it.rs) if md else None, arena.ptr(it.cs) if md else None,
                                            1 if (md and not it.split) else 0, 1 if (md and not write_grad) else 0))
                off += it.B
            udt = pdt if pdt == sdt else torch.float32
            N.check(lib.thorn_ns_cast_multi(N.array(N.NsCastTensor, casts), len(casts), N.dtype_code(pdt),
                                            N.dtype_code(sdt), N.dtype_code(udt), ns_code, b1, stream), "ns_cast_multi")
            wsb = int(lib.thorn_ns_workspace_bytes(nb, R, C))
            ws = torch.empty(max(256, wsb), dtype=torch.uint8, device=dev)
            if self.profile_ns is not None:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev0.record()
                f0 = N.gemm_flops()
            N.check(lib.thorn_ns_batched(X.data_ptr(), U.data_ptr(), ws.data_ptr(), wsb, nb, R, C, ns_code, coeffs,
                                         cfg.iters, restarts, len(rs), err.data_ptr(), stream), "ns_batched")
            if self.profile_ns is not None:
                ev1 = torch.cuda.Event(enable_timing=True)
                ev1.record()
                f1 = N.gemm_flops()
                self.profile_ns.append((ev0, ev1, f1[0] - f0[0], f1[1] - f0[1], (nb, R, C)))
            del X, ws
            row_scale = mat_stats = None
            if ci in pnn_h:
                rsh, msh = pnn_h[ci]
                row_scale, mat_stats = arena.get(rsh), arena.get(msh)
                (sp,) = self._scratch(dev, [lib.thorn_pnn_scratch_bytes(nb, R)])
                pt = N.PnnTensor(U.data_ptr(), row_scale.data_ptr(), mat_stats.data_ptr(), nb, R, C, sp, 0)
                N.check(lib.thorn_pnn_stats_multi(N.array(N.PnnTensor, [pt]), 1, ns_code, N.dtype_code(pdt), stream),
                        "pnn_stats_multi")
            posts, off = [], 0
            usz = U.element_size()
            lr_eff = float(cfg.lr) * cfg.lr_scale(R, C)
            scr = self._scratch(dev, [lib.thorn_sumsq_scratch_bytes(it.B, R, C) if md else 0 for it in its])
            for it, sp in zip(its, scr):
                posts.append(N.OrthoPostTensor(
                    U.data_ptr() + off * R * C * usz, it.p.data_ptr(),
                    None if row_scale is None else row_scale.data_ptr() + off * R * 4,
                    None if mat_stats is None else mat_stats.data_ptr() + off * 2 * 4,
                    arena.ptr(it.pnorm) if md else None, it.B, it.R, it.C, lr_eff * it.scale, sp if md else None, 1))
                off += it.B
            N.check(lib.thorn_ortho_post_multi(N.array(N.OrthoPostTensor, posts), len(posts), ns_code,
                                               N.dtype_code(pdt), float(cfg.weight_decay), stream), "ortho_post_multi")
            del U
        keep = None
        if md:
            self._md_prep(items, arena, new=True, stream=stream)
            keep = self._md_finalize(items, arena, lambda it: True, stream)
        self._finish(params, cfg)
        del keep

    # ------------------------------------------------------- (R)AdamW group
    def _sparse_rows(self, params, cfg):
        """Launch records of row-sparse gradients (thorn.py:1669-1698): the moment,
        variance (and, when applied, parameter) rows a gradient touches are gathered
        into contiguous buffers, updated by the AdamW kernel and copied back by
        ``_scatter_rows``.  Parameters whose gradient has no rows are left out: the
        reference then keeps their step count and gradient."""
        recs = []
        for p in params:
            g = p.grad.coalesce()
            idx = g.indices()[0]
            if idx.numel() == 0:
                continue
            st = self.state[p]
            it = _Item()
            it.g = g.values().contiguous()
            it.state = st
            it.apply = (st["step"] + 1) % self._update_rate == 0
            it.pdt, it.sdt = p.dtype, st["moment"].dtype
            it.m_rows = st["moment"].index_select(0, idx)
            it.v_rows = st["variance"].index_select(0, idx)
            recs.append((p, idx, it))
        self._magma([it for _, _, it in recs], cfg, recovered=False)
        for p, idx, it in recs:
            it.p = p.index_select(0, idx) if it.apply else None
        return recs

    def _scatter_rows(self, recs):
        for p, idx, it in recs:
            st = it.state
            st["moment"].index_copy_(0, idx, it.m_rows)
            st["variance"].index_copy_(0, idx, it.v_rows)
            if it.p is not None:
                p.data.index_copy_(0, idx, it.p)

    def _adam_local(self, params, cfg: GroupConfig):
        """thorn.py:1659-1727 on the multi-tensor kernel."""
        lib = N.load()
        dev = _local(params[0]).device
        stream = N.stream_of(dev)
        md = cfg.decouple_md
        sparse = [p for p in params if p.grad.is_sparse]
        if sparse:
            params = [p for p in params if not p.grad.is_sparse]
            recs = self._sparse_rows(sparse, cfg)
            by_dt: dict = {}
            for _, _, it in recs:
                step = it.state["step"]
                rect = cfg.rect(step)
                b1, b2 = cfg.betas
                by_dt.setdefault((it.pdt, it.sdt), []).append(N.AdamTensor(
                    None if it.p is None else it.p.data_ptr(), it.g.data_ptr(), it.m_rows.data_ptr(),
                    it.v_rows.data_ptr(), it.g.numel(), float(cfg.lr) * rect * it.scale, 1 / (1 - b1 ** step),
                    1 / (1 - b2 ** step), 1 if rect == 0.0 else 0))
            for (pdt, sdt), ts in by_dt.items():
                N.check(lib.thorn_adamw_multi(N.array(N.AdamTensor, ts), len(ts), N.dtype_code(pdt),
                                              N.dtype_code(sdt), float(cfg.betas[0]), float(cfg.betas[1]),
                                              float(cfg.weight_decay), float(cfg.eps), stream), "adamw_multi(rows)")
            self._scatter_rows(recs)
            self._finish([p for p, _, _ in recs], cfg)
            if not params:
                return
        arena = _Arena()
        items = self._items(params, cfg, arena, ortho=False)
        # Magma on the raw gradient, before direction recovery (thorn.py:1702); a sharded
        # parameter scores its whole tensor (sums all-reduced over its shard group)
        plain, by_group = [], {}
        for p, it in zip(params, items):
            if isinstance(p, DTensor) and not all(isinstance(pl, Replicate) for pl in p.placements):
                from .sharded import shard_group
                by_group.setdefault(shard_group(p, self.rank)[1], []).append(it)
            else:
                plain.append(it)
        self._magma(plain, cfg, recovered=False)
        for grp, its in by_group.items():
            self._magma(its, cfg, recovered=False, group=grp)
        if md:
            for it in items:
                _row_norm_axis(cfg, it.p)  # raises for a norm_axis other than the default or the last dim
        arena.materialize(dev)
        b1, b2 = cfg.betas
        if md:
            self._md_prep(items, arena, new=False, stream=stream)
            by_dt: dict = {}
            scr = self._scratch(dev, [lib.thorn_ortho_pre_scratch_bytes(it.B, it.R, it.C, 1) for it in items])
            for it, sp in zip(items, scr):
                t = N.OrthoPreTensor(it.p.data_ptr(), it.g.data_ptr(), None, None, it.B, it.R, it.C,
                                     arena.ptr(it.rs), arena.ptr(it.cs), 0 if it.split else 1,
                                     arena.ptr(it.rgs), arena.ptr(it.cgs), sp)
                by_dt.setdefault((it.pdt, it.sdt), []).append(t)
            for (pdt, sdt), ts in by_dt.items():
                N.check(lib.thorn_ortho_pre_multi(N.array(N.OrthoPreTensor, ts), len(ts), N.dtype_code(pdt),
                                                  N.dtype_code(sdt), N.dtype_code(pdt), float(b1), 1, 1, stream),
                        "md recover_direction")
        by_dt = {}
        for it in items:
            step = it.state["step"]
            rect = cfg.rect(step)
            bc1 = 1 / (1 - b1 ** step)
            bc2 = 1 / (1 - b2 ** step)
            t = N.AdamTensor(it.p.data_ptr() if it.apply else None, it.g.data_ptr(),
                             _local(it.state["moment"]).data_ptr(), _local(it.state["variance"]).data_ptr(),
                             it.p.numel(), float(cfg.lr) * rect * it.scale, bc1, bc2, 1 if rect == 0.0 else 0)
            by_dt.setdefault((it.pdt, it.sdt), []).append(t)
        for (pdt, sdt), ts in by_dt.items():
            N.check(lib.thorn_adamw_multi(N.array(N.AdamTensor, ts), len(ts), N.dtype_code(pdt), N.dtype_code(sdt),
                                          float(b1), float(b2), float(cfg.weight_decay), float(cfg.eps), stream),
                    "adamw_multi")
        keep = None
        if md:
            self._md_gains(items, cfg, arena, stream)
            app = [it for it in items if it.apply]
            if app:
                scr = self._scratch(dev, [lib.thorn_sumsq_scratch_bytes(*_renorm_view(it)) for it in app])
                for pdt in {it.pdt for it in app}:
                    ts = [N.SumsqTensor(it.p.data_ptr(), arena.ptr(it.pnorm), *_renorm_view(it), sp)
                          for it, sp in zip(app, scr) if it.pdt == pdt]
                    N.check(lib.thorn_sumsq_multi(N.array(N.SumsqTensor, ts), len(ts), N.dtype_code(pdt), stream),
                            "sumsq_multi")
            self._md_prep(items, arena, new=True, stream=stream)
            keep = self._md_finalize(items, arena, lambda it: True, stream)
        self._finish(params, cfg)
        del keep
