"""Newton-Schulz coefficients (host side, float64).

Polar Express (arXiv:2505.16932) optimal odd-quintic composition and the
stability-driven restart positions for Gram Newton-Schulz, computed exactly as
the reference does (thorn.py:425-514) so the coefficients are bit-identical:
float64 torch tensors on the CPU, the same solver and the same iteration
order.
"""
from __future__ import annotations

from functools import lru_cache
from itertools import combinations

import torch


@lru_cache(maxsize=None)
def optimal_composition(l: float, num_iters: int, safety_factor_eps: float = 0.0, cushion: float = 0.0):
    """(a, b, c) per iteration (thorn.py:425-480)."""
    assert 0 <= l <= 1
    f64 = torch.float64

    def quintic(lo: float, hi: float):
        assert 0 <= lo <= hi
        eps_d = 1e-15
        if lo / hi >= 1.0 - eps_d:
            return (15.0 / 8.0) / hi, (-10.0 / 8.0) / (hi ** 3.0), (3.0 / 8.0) / (hi ** 5.0)
        q = (3.0 * lo + hi) / 4.0
        r = (lo + 3.0 * hi) / 4.0
        err, prev = float("inf"), None
        a = b = c = 1.0
        while not prev or abs(prev - err) > eps_d:
            prev = err
            lhs = torch.tensor([
                [lo, lo ** 3.0, lo ** 5.0, 1.0],
                [q, q ** 3.0, q ** 5.0, -1.0],
                [r, r ** 3.0, r ** 5.0, 1.0],
                [hi, hi ** 3.0, hi ** 5.0, -1.0],
            ], dtype=f64)
            a, b, c, err = torch.linalg.solve(lhs, torch.ones(4, dtype=f64))
            q, r = torch.sqrt((-3.0 * b + torch.tensor([-1.0, 1.0], dtype=f64) * (9.0 * b ** 2.0 - 20.0 * a * c) ** 0.5)
                              / (10.0 * c))
        return float(a), float(b), float(c)

    u = 1.0
    sf = 1.0 + safety_factor_eps
    out = []
    for it in range(num_iters):
        a, b, c = quintic(max(l, cushion * u), u)
        if cushion * u > l:
            pl = a * l + b * l ** 3.0 + c * l ** 5.0
            pu = a * u + b * u ** 3.0 + c * u ** 5.0
            k = 2.0 / (pl + pu)
            a, b, c = a * k, b * k, c * k
        if it < num_iters - 1:
            a /= sf
            b /= sf ** 3.0
            c /= sf ** 5.0
        out.append((a, b, c))
        l = a * l + b * l ** 3.0 + c * l ** 5.0
        u = 2.0 - l
    return out


@lru_cache(maxsize=None)
def gram_ns_restarts(*coeffs):
    """Restart positions with the smallest worst-case conditioning (thorn.py:482-514)."""
    E = torch.logspace(0, -10, 10000, dtype=torch.float64)
    K = -4e-4

    def cond(t):
        lo, hi = t.aminmax()
        return (hi / lo).item()

    for n in range(1, len(coeffs)):
        best_q, best = float("inf"), []
        for combo in combinations(range(1, len(coeffs)), n):
            qs = []
            e = E.clone()
            q = r = None
            for j, (a, b, c) in enumerate(coeffs):
                if j == 0 or j in combo:
                    if j != 0:
                        e *= q
                    r = e ** 2 + K
                    q = torch.ones(len(e), dtype=torch.float64)
                z = a + r * (b + r * c)
                q *= z
                r *= z ** 2
                qs.append(q)
            worst = max(cond(t) for t in qs)
            if worst < best_q:
                best_q, best = worst, list(combo)
        if best_q < 1e8:
            return best
    raise ValueError("No stable restarts with these parameters")
