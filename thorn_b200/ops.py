"""PyTorch custom operators over the C ABI.

* ``torch.ops.thorn_b200.sym_addmm(A, B, C, alpha, beta)``: the contract of the
  reference's operator seam ``thorn::sym_addmm`` (thorn.py:298-368), i.e.
  ``beta * C + alpha * (A @ B)`` for products known to be symmetric, computed on
  the lower-triangle tiles of the tcgen05 GEMM and mirrored.  The same kernel is
  also registered under the reference's own name, ``torch.ops.thorn.sym_addmm``,
  unless the reference's module registered that name first (then its operator
  stays in place; importing the reference after this package would fail on the
  duplicate name, so code that imports both imports ``thorn`` first).
* ``torch.ops.thorn_b200.polar_decomp(X, coeffs, restarts)``: the Newton-Schulz
  polar factor of a stack of matrices (thorn.py:626-662): Frobenius-normalised in
  fp32 and cast to fp16 by the library's NS-input pass, iterated on fp16 operands,
  returned in X's dtype.

Both have fake (meta) implementations, so they trace under ``torch.compile`` and
``torch.export`` as opaque nodes.  They run on CUDA devices only; there is no CPU
path.
"""
from __future__ import annotations

from math import prod
from typing import List, Optional

import torch
import torch.nn.functional as F

from . import _native as N

_HALF = (torch.float16, torch.bfloat16)


def _err_flag(dev: torch.device) -> torch.Tensor:
    flags = _err_flag.cache
    t = flags.get(dev)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        flags[dev] = t
    return t


_err_flag.cache = {}


def _check_cuda(*ts):
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError(f"thorn_b200 operators run on CUDA devices only; got a tensor on {t.device}")


def _sym_addmm_cuda(A: torch.Tensor, B: torch.Tensor, C: Optional[torch.Tensor], alpha: float,
                    beta: float) -> torch.Tensor:
    """``beta * C + alpha * (A @ B)`` with ``A @ B`` and ``C`` symmetric.

    A: (..., M, K), B: (..., K, M), C: (..., M, M), (M, M) or None; fp16 or bf16.
    Returns (..., M, M), exactly symmetric.
    """
    _check_cuda(A, B, C)
    if A.dtype not in _HALF or B.dtype != A.dtype or (C is not None and C.dtype != A.dtype):
        raise TypeError("sym_addmm takes float16 or bfloat16 operands of one dtype")
    if A.ndim < 2 or B.ndim != A.ndim:
        raise ValueError("A and B must have the same number (>= 2) of dimensions")
    *batch, M, K = A.shape
    if tuple(B.shape) != (*batch, K, M):
        raise ValueError(f"B must be {(*batch, K, M)}, got {tuple(B.shape)}")
    if C is not None and not (tuple(C.shape) == (M, M) or tuple(C.shape) == (*batch, M, M)):
        raise ValueError(f"C must be {(*batch, M, M)} or {(M, M)}, got {tuple(C.shape)}")
    nn = prod(batch) if batch else 1
    a = A.reshape(nn, M, K).contiguous()
    b = B.reshape(nn, K, M).contiguous()
    c_batched = C is not None and C.ndim > 2
    c = None if C is None else (C.reshape(nn, M, M) if c_batched else C).contiguous()
    # the kernel's TMA rows need M and K in multiples of 8: zero rows and columns are
    # appended (zeros along K add nothing to A @ B; the extra output rows and columns
    # are dropped), which the reference's Triton kernel does not need
    Mp, Kp = -(-M // 8) * 8, -(-K // 8) * 8
    if (Mp, Kp) != (M, K):
        a = F.pad(a, (0, Kp - K, 0, Mp - M))
        b = F.pad(b, (0, Mp - M, 0, Kp - K))
        c = None if c is None else F.pad(c, (0, Mp - M, 0, Mp - M))
    out = torch.empty((nn, Mp, Mp), dtype=A.dtype, device=A.device)
    if nn and M:
        lib = N.load()
        with torch.cuda.device(A.device):
            N.check(lib.thorn_sym_addmm(a.data_ptr(), b.data_ptr(), None if c is None else c.data_ptr(),
                                        out.data_ptr(), nn, Mp, Kp, 1 if c_batched else 0, float(alpha),
                                        float(beta), N.dtype_code(A.dtype), _err_flag(A.device).data_ptr(),
                                        N.stream_of(A.device)), "sym_addmm")
    if Mp != M:
        out = out[:, :M, :M].contiguous()
    return out.reshape(*batch, M, M)


def _sym_addmm_fake(A, B, C, alpha, beta):
    *batch, M, _ = A.shape
    return A.new_empty((*batch, M, M))


sym_addmm = torch.library.custom_op("thorn_b200::sym_addmm", _sym_addmm_cuda, mutates_args=())
sym_addmm.register_fake(_sym_addmm_fake)


def _reference_op_registered() -> bool:
    """True when ``thorn::sym_addmm`` exists already (the reference's module was imported)."""
    try:
        torch.ops.thorn.sym_addmm
    except (AttributeError, RuntimeError):
        return False
    return True


# the reference's operator name (thorn.py:298): code written against the reference that calls
# torch.ops.thorn.sym_addmm reaches the same tcgen05 kernel
reference_sym_addmm = None
if not _reference_op_registered():
    reference_sym_addmm = torch.library.custom_op("thorn::sym_addmm", _sym_addmm_cuda, mutates_args=())
    reference_sym_addmm.register_fake(_sym_addmm_fake)


@torch.library.custom_op("thorn_b200::polar_decomp", mutates_args=())
def polar_decomp(X: torch.Tensor, coeffs: List[float], restarts: List[int]) -> torch.Tensor:
    """Polar factor of every matrix of X (..., R, C) by Newton-Schulz.

    ``coeffs``: the flat (a, b, c) triples of the iterations (3 x iters floats);
    ``restarts``: Gram-NS restart positions.  X is normalised to unit Frobenius
    norm in fp32, iterated on fp16 operands with fp32 accumulation, and the result
    is returned in X's dtype.
    """
    _check_cuda(X)
    if X.ndim < 2:
        raise ValueError("polar_decomp takes (..., R, C) stacks of matrices")
    if len(coeffs) % 3:
        raise ValueError("coeffs must hold whole (a, b, c) triples")
    *batch, R, C = X.shape
    nb = prod(batch) if batch else 1
    out = torch.empty((nb, R, C), dtype=torch.float16, device=X.device)
    if nb and R and C:
        lib = N.load()
        dev = X.device
        code = N.dtype_code(X.dtype)
        x = X.reshape(nb, R, C).contiguous()
        st = N.stream_of(dev)
        with torch.cuda.device(dev):
            # ||x||^2 per matrix (fixed-order sums), then x / (||x|| + 1e-8) cast to fp16 rows of
            # the padded leading dimension: the NS-input pass with u = x (beta1 = 0)
            normsq = torch.empty(nb, dtype=torch.float32, device=dev)
            scr = torch.zeros(max(16, int(lib.thorn_sumsq_scratch_bytes(nb, R, C))), dtype=torch.uint8, device=dev)
            N.check(lib.thorn_sumsq_multi(N.array(N.SumsqTensor, [N.SumsqTensor(
                x.data_ptr(), normsq.data_ptr(), nb, R, C, scr.data_ptr())]), 1, code, st), "polar_decomp norms")
            xin = torch.empty((nb, R, int(lib.thorn_ns_ld(C))), dtype=torch.float16, device=dev)
            N.check(lib.thorn_ns_cast_multi(N.array(N.NsCastTensor, [N.NsCastTensor(
                x.data_ptr(), x.data_ptr(), normsq.data_ptr(), xin.data_ptr(), nb, R, C, None, None, 0, 0)]), 1,
                code, code, code, N.F16, 0.0, st), "polar_decomp input")
            wsb = int(lib.thorn_ns_workspace_bytes(nb, R, C))
            ws = torch.empty(max(256, wsb), dtype=torch.uint8, device=dev)
            iters = len(coeffs) // 3
            cc = (N.ctypes.c_double * max(1, len(coeffs)))(*coeffs)
            rr = (N.ctypes.c_int32 * max(1, len(restarts)))(*restarts)
            N.check(lib.thorn_ns_batched(xin.data_ptr(), out.data_ptr(), ws.data_ptr(), wsb, nb, R, C, N.F16, cc,
                                         iters, rr, len(restarts), _err_flag(dev).data_ptr(), st), "polar_decomp")
        # the fp16 result converted to X's dtype (a dtype conversion, as in thorn.py:662)
    return out.reshape(*batch, R, C).to(X.dtype)


@polar_decomp.register_fake
def _polar_decomp_fake(X, coeffs, restarts):
    return torch.empty_like(X)
