"""CPU oracle for the THORN optimizer step (test infrastructure only).

This module is a numpy restatement of the reference optimizer's step in
``thorn/thorn.py`` (pykeio/THORN v3.1.1).  It is the *checker* used by the
parity tests, by ``__graft_entry__.smoke()`` and by ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` arm.  Nothing in the product package
(``thorn_b200``) imports it, and the product never falls back to it.

Numerics follow the reference's eager CPU path (the path the golden vectors
under ``tests/golden`` were produced with):

* every torch op on a tensor of storage dtype D computes in fp32 and rounds
  once to D -- emulated with :func:`rnd`;
* Newton-Schulz runs on fp16 operands with fp32 accumulation and one rounding
  per GEMM (torch CPU ``bmm``/``baddbmm`` on half tensors behave this way);
* host-side scalars (bias corrections, LR scales) are float64 like the
  reference's Python floats.

Parity is pinned by ``tests/test_oracle_golden.py`` against vectors produced
by running the reference itself (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

from itertools import combinations

import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------
# dtype emulation
# ---------------------------------------------------------------------------

DTYPES = ("f32", "bf16", "f16")
EPS = {"f32": float(np.finfo(np.float32).eps), "bf16": 0.0078125, "f16": float(np.finfo(np.float16).eps)}


_CHUNK = 1 << 18  # elements per block of the rounding loops (working set stays in cache)


def to_bf16(x) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even); returns float32.

    uint32 arithmetic: only NaN bit patterns can wrap, and those are restored.
    Large arrays are rounded in cache-sized blocks with reused temporaries.
    """
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    b = x.reshape(-1).view(np.uint32)
    out = np.empty_like(x)
    o = out.reshape(-1).view(np.uint32)
    r = np.empty(min(b.size, _CHUNK), dtype=np.uint32)
    for i in range(0, b.size, _CHUNK):
        bb = b[i:i + _CHUNK]
        rr = r[:bb.size]
        np.right_shift(bb, 16, out=rr)
        rr &= np.uint32(1)
        rr += np.uint32(0x7FFF)
        rr += bb
        rr &= np.uint32(0xFFFF0000)
        o[i:i + _CHUNK] = rr
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def to_f16(x) -> np.ndarray:
    """Round float32 values to float16 (round-to-nearest-even); returns float32.

    Same result as ``x.astype(float16).astype(float32)`` without numpy's slow
    per-element path for fp16 subnormals: the 10-bit mantissa rounding is done
    on the float32 bits, subnormals are rounded to multiples of 2**-24 and
    overflow goes to +-inf.
    """
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    b = x.view(np.uint32)
    r = (b >> 13) & np.uint32(1)
    r += np.uint32(0xFFF)
    r += b
    r &= np.uint32(0xFFFFE000)
    out = r.view(F32)
    sub = np.rint(x * F32(2.0 ** 24))
    sub *= F32(2.0 ** -24)
    out = np.where(np.abs(x) < F32(2.0 ** -14), sub, out)
    big = np.abs(out) >= F32(65520.0)
    if big.any():
        out[big] = np.copysign(np.inf, x[big]).astype(F32)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def rnd(x, dt: str) -> np.ndarray:
    """Round to storage dtype ``dt`` and return the value as float32."""
    x = np.asarray(x, dtype=F32)
    if dt == "f32":
        return x
    if dt == "f16":
        return to_f16(x)
    if dt == "bf16":
        return to_bf16(x)
    raise ValueError(dt)


def h16(x) -> np.ndarray:
    return rnd(x, "f16")


# Which of the reference's two execution paths the oracle models.
#
# CPU_EAGER = True: the reference on CPU (how the golden vectors were made):
#   every torch op rounds to the tensor dtype, and torch's CPU kernels for
#   ``add(..., alpha=a)`` / ``sub_(..., alpha=a)`` round the scalar ``a`` to
#   the tensor's dtype first (bf16: 0.9 -> 0.8984375).
# CPU_EAGER = False: the reference on CUDA: scalars stay fp32, and the Adam
#   update (thorn.py:147-185), the cautious-WD apply (thorn.py:187-203) and
#   per-neuron norm (thorn.py:205-280) are fused Triton kernels that compute
#   in fp32 and round once per stored value.  The GPU parity tests use this.
CPU_EAGER = False


def alpha(a: float, dt: str) -> np.float32:
    return F32(rnd(F32(a), dt)) if CPU_EAGER else F32(a)


# ---------------------------------------------------------------------------
# Polar-Express coefficients and Gram-NS restarts (thorn.py:425-514)
# ---------------------------------------------------------------------------

def optimal_composition(l: float, num_iters: int, safety_factor_eps: float = 0.0, cushion: float = 0.0):
    """Polar Express minimax quintic composition (thorn.py:425-480).

    For each iteration, solve the 4x4 equioscillation system for the optimal
    odd quintic on [max(l, cushion*u), u] (Remez exchange on the two interior
    extrema), rescale when the cushion is active, divide by the safety factor
    (except on the last iteration) and map the interval forward.  All in f64.
    """
    assert 0 <= l <= 1

    def optimal_quintic(lo: float, hi: float):
        assert 0 <= lo <= hi
        eps_d = 1e-15
        if lo / hi >= 1.0 - eps_d:
            return (15.0 / 8.0) / hi, (-10.0 / 8.0) / (hi ** 3.0), (3.0 / 8.0) / (hi ** 5.0)
        q = (3.0 * lo + hi) / 4.0
        r = (lo + 3.0 * hi) / 4.0
        E, old_E = float("inf"), None
        a = b = c = 1.0
        while not old_E or abs(old_E - E) > eps_d:
            old_E = E
            lhs = np.array([
                [lo, lo ** 3.0, lo ** 5.0, 1.0],
                [q, q ** 3.0, q ** 5.0, -1.0],
                [r, r ** 3.0, r ** 5.0, 1.0],
                [hi, hi ** 3.0, hi ** 5.0, -1.0],
            ], dtype=np.float64)
            a, b, c, E = np.linalg.solve(lhs, np.ones(4, dtype=np.float64))
            disc = (9.0 * b ** 2.0 - 20.0 * a * c) ** 0.5
            q, r = np.sqrt((-3.0 * b + np.array([-1.0, 1.0]) * disc) / (10.0 * c))
        return float(a), float(b), float(c)

    u = 1.0
    sf = 1.0 + safety_factor_eps
    coeffs = []
    for it in range(num_iters):
        a, b, c = optimal_quintic(max(l, cushion * u), u)
        if cushion * u > l:
            pl = a * l + b * l ** 3.0 + c * l ** 5.0
            pu = a * u + b * u ** 3.0 + c * u ** 5.0
            rescale = 2.0 / (pl + pu)
            a, b, c = a * rescale, b * rescale, c * rescale
        if it < num_iters - 1:
            a /= sf
            b /= sf ** 3.0
            c /= sf ** 5.0
        coeffs.append((a, b, c))
        l = a * l + b * l ** 3.0 + c * l ** 5.0
        u = 2.0 - l
    return coeffs


def gram_ns_restarts(coeffs):
    """Stability-driven restart positions for Gram NS (thorn.py:482-514)."""
    E = np.logspace(0, -10, 10000, dtype=np.float64)
    K = -4e-4

    def cond(t):
        return float(t.max() / t.min())

    for nres in range(1, len(coeffs)):
        q_max = float("inf")
        best = []
        for combo in combinations(range(1, len(coeffs)), nres):
            qv = []
            e = E.copy()
            q = None
            r = None
            for j, (a, b, c) in enumerate(coeffs):
                if j == 0 or j in combo:
                    if j != 0:
                        e *= q
                    r = e ** 2 + K
                    q = np.ones(len(e), dtype=np.float64)
                z = a + r * (b + r * c)
                # in place, as the reference does: entries appended earlier alias q
                q *= z
                r *= z ** 2
                qv.append(q)
            qm = max(cond(t) for t in qv)
            if qm < q_max:
                q_max = qm
                best = list(combo)
        if q_max < 1e8:
            return best
    raise ValueError("No stable restarts with these parameters")


# ---------------------------------------------------------------------------
# Newton-Schulz polar factor (thorn.py:614-667)
# ---------------------------------------------------------------------------

# Operand type of the NS GEMMs: "f16" as in the reference (thorn.py:634-635);
# "bf16" models the optional bf16 mode of the B200 kernels.
NS_DTYPE = "f16"


def _mm16(a, b, c=None, alpha=1.0, beta=1.0):
    """16-bit GEMM with fp32 accumulation, one rounding: out = alpha*a@b + beta*c."""
    acc = np.matmul(a, b)
    if alpha != 1.0:
        acc *= F32(alpha)
    if c is not None:
        acc += F32(beta) * c
    return rnd(acc, NS_DTYPE)


def polar_decomp_2d(X: np.ndarray, coeffs, restarts, src_dtype: str) -> np.ndarray:
    """One matrix of ``_polar_decomp_impl`` (thorn.py:626-662); returns dtype ``src_dtype``."""
    m0, n0 = X.shape
    gram = max(m0, n0) > min(m0, n0)
    tall = m0 > n0
    if tall:
        X = X.T
    X = np.ascontiguousarray(X, dtype=F32)
    nrm = F32(np.sqrt(np.sum(X.astype(np.float64) ** 2)))
    X = rnd(X / (nrm + F32(1e-8)), NS_DTYPE)
    if gram:
        R = _mm16(X, X.T)
        Q = None
        last = len(coeffs) - 1
        for i, (a, b, c) in enumerate(coeffs):
            if i in restarts and i != 0:
                X = _mm16(Q, X)
                R = _mm16(X, X.T)
            Z = _mm16(R, R, R, alpha=c, beta=b)
            if i != 0 and i not in restarts:
                Q = _mm16(Q, Z, Q, beta=a)
            else:
                # Z + a*I (thorn.py:648); on CPU a*I first rounds a to fp16
                Q = Z.copy()
                d = np.arange(Q.shape[0])
                a16 = rnd(F32(a), NS_DTYPE) if CPU_EAGER else F32(a)
                Q[d, d] = rnd(Q[d, d] + a16, NS_DTYPE)
            if i < last and (i + 1) not in restarts:
                RZ = _mm16(R, Z, R, beta=a)
                R = _mm16(Z, RZ, RZ, beta=a)
        # the reference multiplies X.mT @ Q for tall inputs (thorn.py:653); Q is not
        # exactly symmetric on the eager path, so keep the same operand order
        X = _mm16(X.T, Q) if tall else _mm16(Q, X)
    else:
        for (a, b, c) in coeffs:
            A = _mm16(X, X.T)
            B = _mm16(A, A, A, alpha=c, beta=b)
            X = _mm16(B, X, X, beta=a)
        if tall:
            X = X.T
    return rnd(np.ascontiguousarray(X), src_dtype)


def polar_decomp(u: np.ndarray, coeffs, restarts, src_dtype: str) -> np.ndarray:
    """Batched over leading dims: NS works on ``shape[-2:]`` (thorn.py:628-633)."""
    if u.ndim == 2:
        return polar_decomp_2d(u, coeffs, restarts, src_dtype)
    lead = u.shape[:-2]
    flat = u.reshape(-1, *u.shape[-2:])
    out = np.stack([polar_decomp_2d(x, coeffs, restarts, src_dtype) for x in flat])
    return out.reshape(*lead, *u.shape[-2:])


# ---------------------------------------------------------------------------
# Elementwise pieces
# ---------------------------------------------------------------------------

def softplus(x, dt):
    """F.softplus(beta=1, threshold=20) in storage dtype ``dt``."""
    x = np.asarray(x, dtype=F32)
    y = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    return rnd(y, dt)


def sigmoid(x, dt):
    x = np.asarray(x, dtype=F32)
    return rnd(1.0 / (1.0 + np.exp(-x.astype(np.float64))), dt)


def weight_decay_update(p, u, wd: float, lr: float, dt: str, udt: str | None = None):
    """Cautious weight decay + apply, eager path (thorn.py:669-702).

    mask = (u*p >= 0); u += p*(mask*wd); p -= lr*u.  ``dt`` is p's dtype,
    ``udt`` the update's dtype (defaults to ``dt``).
    """
    udt = udt or dt
    if not CPU_EAGER:
        # Triton _wd_update_helper: fp32 throughout, one rounding of p
        u = np.asarray(u, F32)
        if wd > 0.0:
            u = np.where(u * p >= 0, u + F32(wd) * p, u).astype(F32)
        return rnd(p - F32(lr) * u, dt), u
    if wd > 0.0:
        mdt = _promote(dt, udt)
        mask = (rnd(u * p, mdt) >= 0).astype(F32)
        u = rnd(u + p * rnd(mask * F32(wd), dt), udt)
    return rnd(p - alpha(lr, dt) * u, dt), u


def per_neuron_norm(u, dt: str):
    """Per-row normalisation (thorn.py:709-762). u: (..., M, N).

    CUDA path: the Triton kernels (thorn.py:205-280) in fp32 -- row sums of
    squares, s = rsqrt(max(sumsq/N, eps)), gscale = sqrt(sum sumsq) /
    max(sqrt(sum s^2 sumsq), eps) per matrix, u * s * gscale (left in fp32 for
    the fused apply).  CPU path: eager torch ops rounding to ``dt``.
    """
    eps = F32(EPS[dt])
    if not CPU_EAGER:
        u = np.asarray(u, F32)
        sumsq = np.sum(u.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(F32)
        s = (1.0 / np.sqrt(np.maximum(sumsq * F32(1.0 / u.shape[-1]), eps))).astype(F32)
        tot = np.sum(sumsq.astype(np.float64), axis=(-2, -1), keepdims=True)
        new = np.sum((s.astype(np.float64) ** 2) * sumsq, axis=(-2, -1), keepdims=True)
        gscale = (np.sqrt(tot) / np.maximum(np.sqrt(new), eps)).astype(F32)
        return (u * (s * gscale)).astype(F32)
    v_norm = rnd(np.sqrt(np.sum(u.astype(np.float64) ** 2, axis=(-2, -1), keepdims=True)), dt)
    v_mean = rnd(np.mean(rnd(u * u, dt), axis=-1, keepdims=True, dtype=np.float64), dt)
    s = rnd(1.0 / np.sqrt(np.maximum(v_mean, eps)), dt)
    u = rnd(u * s, dt)
    v_norm_new = rnd(np.sqrt(np.sum(u.astype(np.float64) ** 2, axis=(-2, -1), keepdims=True)), dt)
    scale = rnd(v_norm / np.maximum(v_norm_new, eps), dt)
    return rnd(u * scale, dt)


def lr_scale_ortho(shape, scaling_mode: str, target_rms: float) -> float:
    """thorn.py:768-780."""
    d_out, d_in = shape[-2], shape[-1]
    if scaling_mode == "md":
        return max(d_out / d_in, d_in / d_out) ** 0.5
    if scaling_mode == "moonlight":
        return target_rms * (max(1, d_out, d_in) ** 0.5)
    if scaling_mode == "jordan":
        return max(1, d_out / d_in) ** 0.5
    raise ValueError(scaling_mode)


def compute_rect(betas, rectify: bool, step) -> float:
    """RAdam rectification term (thorn.py:782-798)."""
    beta2 = betas[1]
    if beta2 > 0.0:
        rho_inf = 2 / (1 - beta2) - 1
        rho = rho_inf - 2 * step * (beta2 ** step) / (1 - beta2 ** step)
        r = (((rho - 4) * (rho - 2) * rho_inf / ((rho_inf - 4) * (rho_inf - 2) * rho)) ** 0.5 if rho > 4.0 else 0.0)
        return r ** float(rectify)
    return 1.0


def adam_update(p, g, m, v, step, beta1, beta2, lr, wd, eps, dt, degenerate=False, sdt=None):
    """(R)Adam(-atan2)W, eager path (thorn.py:838-888). Returns (p, m, v); p may be None.

    ``dt``: param/grad dtype; ``sdt``: moment/variance dtype (defaults to ``dt``).
    """
    sdt = sdt or dt
    bc1 = 1 / (1 - beta1 ** step)
    bc2 = 1 / (1 - beta2 ** step)
    w = F32(1 - beta1)
    if not CPU_EAGER:
        # Triton _adam_update_kernel: fp32 math on the loaded values; m and v
        # round only when stored; u and the apply use the fp32 values
        # (g - m) * w + m contracts to one fma on the GPU; float64 emulates it
        mf = (m.astype(np.float64) + (g - m).astype(np.float64) * np.float64(w)).astype(F32)
        vf = v * F32(beta2) + (g * g) * F32(1 - beta2)
        m_out, v_out = rnd(mf, sdt), rnd(vf, sdt)
        if p is None:
            return None, m_out, v_out
        if degenerate:
            u = mf
        elif eps == 0.0:
            u = np.arctan2(mf * F32(bc1), np.sqrt(vf * F32(bc2))).astype(F32)
        else:
            u = ((mf * F32(bc1)) / (np.sqrt(vf * F32(bc2)) + F32(eps))).astype(F32)
        if wd > 0.0:
            u = np.where(u * p >= 0, u + F32(wd) * p, u).astype(F32)
        return rnd(p - F32(lr) * u, dt), m_out, v_out
    # torch lerp: weight < 0.5 -> self + w*(end-self), else end - (end-self)*(1-w)
    if (1 - beta1) < 0.5:
        m = rnd(m + w * (g - m), sdt)
    else:
        m = rnd(g - (g - m) * F32(1 - (1 - beta1)), sdt)
    v = rnd(v * F32(beta2), sdt)
    v = rnd(v + F32(1 - beta2) * g * g, sdt)
    if p is None:
        return None, m, v
    if not degenerate:
        den = rnd(np.sqrt(rnd(v * F32(bc2), sdt)), sdt)
        num = rnd(m * F32(bc1), sdt)
        if eps == 0.0:
            u = rnd(np.arctan2(num, den), sdt)
        else:
            u = rnd(num / rnd(den + F32(eps), sdt), sdt)
    else:
        u = m.copy()
    p, _ = weight_decay_update(p, u, wd, lr, dt, sdt)
    return p, m, v


_BLOCK = 1 << 18  # elements per block of a large tensor's AdamW update


def adam_update_blocked(p, g, m, v, *args, **kw):
    """:func:`adam_update` over 256 Ki-element blocks of the flattened tensors: every
    operation of the update is elementwise, so the result is the same, without the
    tensor-sized temporaries (a 151936 x 1024 embedding otherwise allocates dozens)."""
    n = g.size
    if n <= _BLOCK:
        return adam_update(p, g, m, v, *args, **kw)
    shape = g.shape
    flat = [None if t is None else np.ascontiguousarray(t).reshape(-1) for t in (p, g, m, v)]
    outs = [None if p is None else np.empty(n, F32), np.empty(n, F32), np.empty(n, F32)]
    for i in range(0, n, _BLOCK):
        sl = slice(i, i + _BLOCK)
        res = adam_update(*[None if t is None else t[sl] for t in flat], *args, **kw)
        for o, r in zip(outs, res):
            if o is not None:
                o[sl] = r
    return tuple(None if o is None else o.reshape(shape) for o in outs)


# ---------------------------------------------------------------------------
# Group config (thorn.py:535-612)
# ---------------------------------------------------------------------------

GROUP_DEFAULTS = dict(
    none_grad=True, weight_decay=0.1, betas=(0.9, 0.95), scaling_mode=None, target_rms=0.2,
    target_norm=None, iters=5, rectify=False, eps=0.0, lower_bound=1e-3, safety_factor=0.03,
    cushion=0.02, momentum_align=False, decouple_md=False, gain_lr=1e-3, gain_betas=(0.9, 0.95),
    norm_axis=None, split_gain=True, force_per_neuron_norm=False,
)

LN_E_SUB_1 = 0.5413248546  # softplus(x) == 1 (thorn.py:1602)


class Group:
    def __init__(self, d: dict):
        cfg = dict(GROUP_DEFAULTS)
        cfg.update({k: v for k, v in d.items() if k != "params"})
        self.__dict__.update(cfg)
        self.orthogonalize = bool(d["orthogonalize"])
        self.lr = float(d["lr"])
        self.coeffs = optimal_composition(self.lower_bound, self.iters, self.safety_factor, self.cushion)
        self.restarts = gram_ns_restarts(self.coeffs)

    @property
    def scaling_mode_(self):
        if self.scaling_mode is None:
            return "md" if self.decouple_md else "moonlight"
        return self.scaling_mode

    def needs_pnn(self, shape) -> bool:
        """thorn.py:704-707."""
        return self.betas[1] > 0 and (shape[-2] > shape[-1] or self.force_per_neuron_norm)

    def norm_axes(self, p):
        """thorn.py:594-595: the group's norm_axis, else the last two dims (the last of a vector)."""
        if self.norm_axis is not None:
            ax = self.norm_axis
            return tuple(ax) if isinstance(ax, (tuple, list)) else (ax,)
        return (-2, -1) if p.ndim > 1 else (-1,)

    def target_norm_(self, p, dt):
        """thorn.py:597-612.  A callable target gets the parameter as a float32 numpy array
        (the reference passes the torch tensor); its float or array result is rounded to
        the parameter dtype, like the reference's ``torch.full`` / ``.to(dtype)``."""
        tn = self.target_norm
        if tn is None:
            tn = "max" if self.orthogonalize else "init"
        if callable(tn):
            return rnd(np.asarray(tn(p), dtype=F32), dt)
        if tn == "init":
            val = np.sqrt(np.sum(p.astype(np.float64) ** 2, axis=self.norm_axes(p), keepdims=True))
            return rnd(val, dt)
        if tn == "min":
            return rnd(F32(min(p.shape[-2], p.shape[-1]) ** 0.5), dt)
        if tn == "max":
            return rnd(F32(max(p.shape[-2], p.shape[-1]) ** 0.5), dt)
        raise NotImplementedError(tn)


# ---------------------------------------------------------------------------
# Magma: momentum-aligned gradient masking (thorn.py:800-836)
# ---------------------------------------------------------------------------
W1_C = 0xD07EBC63274654C7
MASK64 = (1 << 64) - 1


def w1rand(s: int) -> tuple[int, int]:
    """The reference's 64-bit generator step (thorn.py:800-804): (new state, output)."""
    s = (s + W1_C) & MASK64
    t = s * (s ^ W1_C)
    return s, ((t >> 64) ^ t) & MASK64


def cosine_similarity(a, b) -> float:
    """torch.nn.functional.cosine_similarity of two flat vectors (eps 1e-8), in float64."""
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    na = max(float(np.sqrt(np.sum(a * a))), 1e-8)
    nb = max(float(np.sqrt(np.sum(b * b))), 1e-8)
    return float(np.sum((a / na) * (b / nb)))


def magma_scale(g, m, st, dt: str, tau: float = 2.0, p: float = 0.9, sharded: bool = False) -> float:
    """LR multiplier of one Magma step (thorn.py:806-836); 0.0 means "skip this update".

    ``g``: the (direction-recovered) gradient, ``m``: the moment before this
    step's update.  ``sharded``: the statistics path of the sharded step
    (fp32 dot / (|g| |m|) clamped at 1e-12, thorn.py:820-829).
    """
    if sharded:
        g64, m64 = np.asarray(g, np.float64).reshape(-1), np.asarray(m, np.float64).reshape(-1)
        dot = F32(np.sum(g64 * m64))
        gsq, msq = F32(np.sum(g64 * g64)), F32(np.sum(m64 * m64))
        cos = F32(dot / F32(max(F32(np.sqrt(gsq)) * F32(np.sqrt(msq)), F32(1e-12))))
        s_t = F32(1.0 / (1.0 + np.exp(-np.float64(F32(cos / F32(tau))))))
        sdt = "f32"  # a 0-d bf16 tensor plus a 0-d fp32 tensor promotes to fp32
    else:
        cos = rnd(F32(cosine_similarity(g, m)), dt)
        s_t = rnd(1.0 / (1.0 + np.exp(-np.float64(rnd(cos / F32(tau), dt)))), dt)
        sdt = dt
    st["s"] = rnd(rnd(F32(p) * st["s"], dt) + rnd(F32(1 - p) * s_t, sdt), sdt)
    st["random_state"], out = w1rand(int(st["random_state"]))
    if out % 2 != 0:
        return 0.0
    return float(st["s"])


# ---------------------------------------------------------------------------
# Magnitude-direction decoupling (thorn.py:890-977)
# ---------------------------------------------------------------------------

def recover_direction(p, g, st, dt):
    if "row_gain" in st:
        rs = softplus(st["row_gain"], dt)
        cs = softplus(st["col_gain"], dt)
        gain = rnd(rs * cs, dt)
        gains = (rs, cs)
    else:
        gain = softplus(st["gain"], dt)
        gains = None
    p = rnd(p / gain, dt)
    p_g = rnd(p * g, dt)
    g = rnd(g * gain, dt)
    return p, g, p_g, gains


def _sum_keep(x, axis):
    return np.sum(x.astype(np.float64), axis=axis, keepdims=True)


def update_magnitude(p_g, key, gain2, axis, st, grp: Group, dt):
    gain = st[key]
    d_gain = sigmoid(gain, dt)
    if gain2 is not None:
        p_g = rnd(p_g * gain2, dt)
    if axis is None:
        grad = rnd(np.sum(p_g.astype(np.float64)), dt)
        grad = rnd(grad * d_gain, dt)
    else:
        grad = rnd(_sum_keep(p_g, axis), dt)
        grad = rnd(grad * d_gain, dt)
    gain_lr = grp.gain_lr  # gain_lr_ == gain_lr because base_lr is refreshed every step (thorn.py:575, 590-592)
    newg, m, v = adam_update(gain, grad, st[key + "_moment"], st[key + "_variance"], st["step"],
                             grp.gain_betas[0], grp.gain_betas[1], gain_lr, 0.0, grp.eps, dt)
    st[key] = newg
    st[key + "_moment"] = m
    st[key + "_variance"] = v


def update_magnitudes(p_g, gains, st, grp, dt):
    if "row_gain" in st:
        update_magnitude(p_g, "row_gain", gains[1], -1, st, grp, dt)
        update_magnitude(p_g, "col_gain", gains[0], -2, st, grp, dt)
    else:
        update_magnitude(p_g, "gain", None, None, st, grp, dt)


def reassemble_md(p, st, dt):
    if "row_gain" in st:
        p = rnd(p * softplus(st["row_gain"], dt), dt)
        p = rnd(p * softplus(st["col_gain"], dt), dt)
    else:
        p = rnd(p * softplus(st["gain"], dt), dt)
    return p


def renorm(p, target, axes, dt):
    nrm = rnd(np.sqrt(np.sum(p.astype(np.float64) ** 2, axis=axes, keepdims=True)), dt)
    return rnd(p * rnd(target / rnd(nrm + F32(1e-8), dt), dt), dt)


# ---------------------------------------------------------------------------
# The optimizer (thorn.py:1229-1753, single device)
# ---------------------------------------------------------------------------

class OracleTHORN:
    """Single-device THORN step over numpy parameters.

    ``groups``: list of dicts with the reference's group keys plus ``params``
    (list of float32 arrays holding values of storage dtype ``dtype``) and
    ``dtype`` ('f32' | 'bf16' | 'f16').  ``state_dtype`` (optional) keeps the
    optimizer state in another dtype (the reference keeps it in the param
    dtype, thorn.py:1596-1599).
    """

    def __init__(self, groups, seed_fn=None, sharded: bool = False):
        """``seed_fn()``: the next Magma seed, called once per momentum_align
        parameter at state initialisation in group and parameter order -- where
        the reference draws ``torch.randint`` (thorn.py:1616-1633).
        ``sharded``: orthogonalized groups follow the reference's FSDP2 step
        (thorn.py:1459-1581): Magma statistics in fp32 from summed shard
        partials, and a masked matrix skips the whole step (no momentum update,
        no step count)."""
        self.seed_fn = seed_fn
        self.sharded = sharded
        self.groups = []
        for d in groups:
            g = Group(d)
            g.params = [np.array(p, dtype=F32) for p in d["params"]]
            g.dtype = d.get("dtype", "f32")
            g.state_dtype = d.get("state_dtype") or g.dtype
            if g.orthogonalize:
                assert all(p.ndim >= 2 for p in g.params)
            g.state = [dict() for _ in g.params]
            g.grad_after = {}  # none_grad=False: the gradient each parameter keeps after the step
            self.groups.append(g)
        self.update_rate = 1

    def _init_state(self, grp: Group, i):
        p, st, dt = grp.params[i], grp.state[i], grp.dtype
        if "step" in st:
            return
        st["step"] = 1
        st["moment"] = np.zeros_like(p)
        if not grp.orthogonalize:
            st["variance"] = np.zeros_like(p)
        if grp.decouple_md:
            if p.ndim > 1 and grp.split_gain:
                st["row_gain"] = rnd(np.full((*p.shape[:-1], 1), LN_E_SUB_1, F32), dt)
                st["col_gain"] = rnd(np.full((*p.shape[:-2], 1, p.shape[-1]), LN_E_SUB_1, F32), dt)
                for k in ("row_gain", "col_gain"):
                    st[k + "_moment"] = np.zeros_like(st[k])
                    st[k + "_variance"] = np.zeros_like(st[k])
            else:
                st["gain"] = rnd(np.full((), LN_E_SUB_1, F32), dt)
                st["gain_moment"] = np.zeros((), F32)
                st["gain_variance"] = np.zeros((), F32)
            st["target_norm"] = grp.target_norm_(p, dt)
        if grp.momentum_align:
            st["random_state"] = int(self.seed_fn())
            st["s"] = rnd(np.ones((), F32), dt)

    def step(self, grads):
        """``grads``: per group, a list of float32 arrays, ``SparseRows`` (AdamW
        groups) or None (no grad)."""
        for grp, gl in zip(self.groups, grads):
            idx = [i for i, g in enumerate(gl) if g is not None]
            for i in idx:
                self._init_state(grp, i)
            if grp.orthogonalize:
                self._ortho_step(grp, idx, gl)
            else:
                self._adam_step(grp, idx, gl)

    # -- orthogonalized group (thorn.py:1376-1457) ---------------------------
    def _ortho_step(self, grp: Group, idx, gl):
        dt, sdt = grp.dtype, grp.state_dtype
        b1 = F32(grp.betas[0])
        for i in idx:
            st = grp.state[i]
            p = grp.params[i]
            g = rnd(gl[i], dt)
            p_g = gains = None
            if grp.decouple_md:
                p, g, p_g, gains = recover_direction(p, g, st, dt)
            # Magma on the recovered gradient and the moment before this step (thorn.py:1392)
            scale = magma_scale(g, st["moment"], st, dt, sharded=self.sharded) if grp.momentum_align else 1.0
            if self.sharded and (scale == 0.0 or (st["step"] + 1) % self.update_rate != 0):
                # thorn.py:1485-1490: a masked matrix, or one whose step is not due, is left out
                # of the step entirely (no momentum update, no step count: thorn.py:1564)
                continue
            # momentum (thorn.py:1376-1381): m = m*b1 + g ; u = g + b1*m
            m = rnd(st["moment"] * b1, sdt)
            m = rnd(m + g, sdt)
            st["moment"] = m
            udt = _promote(dt, sdt)
            u = rnd(g + alpha(grp.betas[0], udt) * m, udt)
            apply = scale != 0.0 and (st["step"] + 1) % self.update_rate == 0
            if apply:
                U = polar_decomp(u, grp.coeffs[: grp.iters], grp.restarts, udt)
                U = rnd(U, dt)
                lr = grp.lr * lr_scale_ortho(U.shape, grp.scaling_mode_, grp.target_rms) * scale
                if grp.needs_pnn(p.shape):
                    U = per_neuron_norm(U, dt)
                p, _ = weight_decay_update(p, U, grp.weight_decay, lr, dt)
                if grp.decouple_md:
                    p = renorm(p, st["target_norm"], (-2, -1), dt)
                    update_magnitudes(p_g, gains, st, grp, dt)
            if grp.decouple_md:
                p = reassemble_md(p, st, dt)
            grp.params[i] = p
            st["step"] += 1
            if not grp.none_grad:
                grp.grad_after[i] = g  # what p.grad holds after the step (MD: the recovered gradient)

    # -- AdamW group (thorn.py:1659-1727) ------------------------------------
    def _adam_step(self, grp: Group, idx, gl):
        dt = grp.dtype
        b1, b2 = grp.betas
        for i in idx:
            st = grp.state[i]
            p = grp.params[i]
            step = st["step"]
            rect = compute_rect(grp.betas, grp.rectify, step)
            gi = gl[i]
            if isinstance(gi, SparseRows) and grp.decouple_md:
                gi = gi.dense(p.shape)  # thorn.py:1667-1668: sparse grads are densified under MD
            if isinstance(gi, SparseRows):
                if self._sparse_adam_step(grp, i, gi, rect):
                    st["step"] += 1
                continue
            g = rnd(gi, dt)
            # Magma on the raw gradient, before direction recovery (thorn.py:1702)
            scale = magma_scale(g, st["moment"], st, dt) if grp.momentum_align else 1.0
            p_g = gains = None
            if grp.decouple_md:
                p, g, p_g, gains = recover_direction(p, g, st, dt)
            apply = scale != 0.0 and (step + 1) % self.update_rate == 0
            newp, m, v = adam_update_blocked(p if apply else None, g, st["moment"], st["variance"], step, b1,
                                             b2, grp.lr * rect * scale, grp.weight_decay, grp.eps, dt,
                                             degenerate=(rect == 0.0), sdt=grp.state_dtype)
            st["moment"], st["variance"] = m, v
            if apply:
                p = rnd(newp, dt)
                if grp.decouple_md:
                    p = renorm(p, st["target_norm"], grp.norm_axes(p), dt)  # thorn.py:1717
                    update_magnitudes(p_g, gains, st, grp, dt)
            if grp.decouple_md:
                p = reassemble_md(p, st, dt)
            grp.params[i] = p
            st["step"] += 1
            if not grp.none_grad:
                grp.grad_after[i] = g


class SparseRows:
    """A row-sparse gradient (torch sparse COO with one sparse dimension):
    ``indices`` of rows (duplicates allowed) and one value row per index."""

    def __init__(self, indices, values):
        self.indices = np.asarray(indices, dtype=np.int64).reshape(-1)
        self.values = np.asarray(values, dtype=F32)

    def coalesce(self):
        """Sorted unique rows; duplicate rows summed (torch ``coalesce``)."""
        uniq, inv = np.unique(self.indices, return_inverse=True)
        vals = np.zeros((len(uniq),) + self.values.shape[1:], dtype=np.float64)
        np.add.at(vals, inv, self.values.astype(np.float64))
        return uniq, vals.astype(F32)

    def dense(self, shape):
        out = np.zeros(shape, dtype=np.float64)
        np.add.at(out, self.indices, self.values.astype(np.float64))
        return out.astype(F32)


def _sparse_adam_step(self, grp: Group, i, gs: SparseRows, rect) -> bool:
    """Row-sparse (R)AdamW (thorn.py:1669-1698); False when the gradient has no rows
    (the reference then leaves the step count unchanged)."""
    st, p, dt = grp.state[i], grp.params[i], grp.dtype
    idx, rows = gs.coalesce()
    if idx.size == 0:
        return False
    rows = rnd(rows, dt)
    m_rows, v_rows = st["moment"][idx], st["variance"][idx]
    scale = magma_scale(rows, m_rows, st, dt) if grp.momentum_align else 1.0
    step = st["step"]
    apply = scale != 0.0 and (step + 1) % self.update_rate == 0
    newp, m_rows, v_rows = adam_update(p[idx] if apply else None, rows, m_rows, v_rows, step, grp.betas[0],
                                       grp.betas[1], grp.lr * rect * scale, grp.weight_decay, grp.eps, dt,
                                       degenerate=(rect == 0.0), sdt=grp.state_dtype)
    st["moment"] = st["moment"].copy()
    st["variance"] = st["variance"].copy()
    st["moment"][idx], st["variance"][idx] = m_rows, v_rows
    if apply:
        p = p.copy()
        p[idx] = rnd(newp, dt)
        grp.params[i] = p
    return True


OracleTHORN._sparse_adam_step = _sparse_adam_step


def _promote(a: str, b: str) -> str:
    if a == b:
        return a
    return "f32"
