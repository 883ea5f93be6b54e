"""ctypes bindings of ``libthorn_b200.so`` (declared in ``include/thorn_b200.h``).

The library is the only compute path: if it is missing or fails to load, every
call raises.  There is no CPU or eager-PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, Structure, c_char_p, c_double, c_float, c_int, c_int32, c_int64, c_uint64, c_void_p

import torch

from . import build as _build

F32, BF16, F16 = 0, 1, 2
DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}
STATUS = {0: "ok", 1: "invalid argument", 2: "misaligned pointer or leading dimension", 3: "CUDA error",
          4: "unsupported device or configuration", 5: "problem needs more than the 64 MiB static NS workspace"}
NS_STATIC_WORKSPACE_BYTES = 64 * 1024 * 1024


class AdamTensor(Structure):
    _fields_ = [("p", c_void_p), ("g", c_void_p), ("m", c_void_p), ("v", c_void_p), ("numel", c_int64),
                ("lr", c_float), ("bc1", c_float), ("bc2", c_float), ("degenerate", c_int32)]


class OrthoPreTensor(Structure):
    _fields_ = [("p", c_void_p), ("g", c_void_p), ("m", c_void_p), ("normsq", c_void_p),
                ("batch", c_int64), ("rows", c_int64), ("cols", c_int64),
                ("row_sp", c_void_p), ("col_sp", c_void_p), ("scalar_gain", c_int32),
                ("row_gsum", c_void_p), ("col_gsum", c_void_p), ("scratch", c_void_p)]


class NsCastTensor(Structure):
    _fields_ = [("g", c_void_p), ("m", c_void_p), ("normsq", c_void_p), ("x", c_void_p),
                ("batch", c_int64), ("rows", c_int64), ("cols", c_int64),
                ("row_sp", c_void_p), ("col_sp", c_void_p), ("scalar_gain", c_int32), ("md", c_int32)]


class PnnTensor(Structure):
    _fields_ = [("U", c_void_p), ("row_scale", c_void_p), ("mat_stats", c_void_p),
                ("batch", c_int64), ("rows", c_int64), ("cols", c_int64), ("scratch", c_void_p), ("fold", c_int32)]


class OrthoPostTensor(Structure):
    _fields_ = [("U", c_void_p), ("p", c_void_p), ("row_scale", c_void_p), ("mat_stats", c_void_p),
                ("p_normsq", c_void_p), ("batch", c_int64), ("rows", c_int64), ("cols", c_int64), ("lr", c_float),
                ("scratch", c_void_p), ("round_u", c_int32)]


class SumsqTensor(Structure):
    _fields_ = [("x", c_void_p), ("out", c_void_p), ("batch", c_int64), ("rows", c_int64), ("cols", c_int64),
                ("scratch", c_void_p)]


class MagmaTensor(Structure):
    _fields_ = [("g", c_void_p), ("m", c_void_p), ("row_gain", c_void_p), ("col_gain", c_void_p),
                ("scalar_gain", c_int32), ("batch", c_int64), ("rows", c_int64), ("cols", c_int64),
                ("out", c_void_p), ("scratch", c_void_p)]


class MdPrepTensor(Structure):
    _fields_ = [("gain", c_void_p), ("sp", c_void_p), ("sig", c_void_p), ("n", c_int64)]


class MdGradTensor(Structure):
    _fields_ = [("gsum", c_void_p), ("sig", c_void_p), ("grad", c_void_p), ("n", c_int64)]


class MdFinalTensor(Structure):
    _fields_ = [("p", c_void_p), ("normsq", c_void_p), ("target", c_void_p), ("target_stride", c_int64),
                ("row_sp", c_void_p), ("col_sp", c_void_p), ("scalar_gain", c_int32),
                ("batch", c_int64), ("rows", c_int64), ("cols", c_int64)]


# name -> (restype, argtypes)
_PROTOS = {
    "thorn_abi_version": (c_int, []),
    "thorn_status_string": (c_char_p, [c_int]),
    "thorn_launch_count": (c_uint64, []),
    "thorn_last_cuda_error": (c_int, []),
    "thorn_gemm_flops": (None, [POINTER(c_double), POINTER(c_double)]),
    "thorn_set_gemm_pair": (c_int, [c_int]),
    "thorn_set_gemm_staged_epilogue": (c_int, [c_int]),
    "thorn_set_gemm_pdl": (c_int, [c_int]),
    "thorn_set_gemm_l2_hints": (c_int, [c_int]),
    "thorn_set_wait_limit_ns": (c_uint64, [c_uint64]),
    "thorn_set_gemm_test_stall": (c_int, [c_int]),
    "thorn_set_ns_small": (c_int, [c_int]),
    "thorn_adamw_multi": (c_int, [POINTER(AdamTensor), c_int, c_int, c_int, c_double, c_double, c_float, c_float,
                                  c_void_p]),
    "thorn_ortho_pre_scratch_bytes": (c_int64, [c_int64, c_int64, c_int64, c_int]),
    "thorn_ortho_pre_multi": (c_int, [POINTER(OrthoPreTensor), c_int, c_int, c_int, c_int, c_float, c_int, c_int,
                                      c_void_p]),
    "thorn_ns_ld": (c_int64, [c_int64]),
    "thorn_ns_cast_multi": (c_int, [POINTER(NsCastTensor), c_int, c_int, c_int, c_int, c_int, c_float, c_void_p]),
    "thorn_ns_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "thorn_ns_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int,
                                 POINTER(c_double), c_int, POINTER(c_int32), c_int, c_void_p, c_void_p]),
    "thorn_sym_addmm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_float,
                                c_float, c_int, c_void_p, c_void_p]),
    "thorn_ns_batched_static": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, POINTER(c_double),
                                        c_int, POINTER(c_int32), c_int, c_void_p, c_void_p]),
    "thorn_pnn_scratch_bytes": (c_int64, [c_int64, c_int64]),
    "thorn_pnn_stats_multi": (c_int, [POINTER(PnnTensor), c_int, c_int, c_int, c_void_p]),
    "thorn_ortho_post_multi": (c_int, [POINTER(OrthoPostTensor), c_int, c_int, c_int, c_float, c_void_p]),
    "thorn_md_prep_multi": (c_int, [POINTER(MdPrepTensor), c_int, c_int, c_void_p]),
    "thorn_md_gain_grad_multi": (c_int, [POINTER(MdGradTensor), c_int, c_int, c_void_p]),
    "thorn_md_finalize_multi": (c_int, [POINTER(MdFinalTensor), c_int, c_int, c_void_p]),
    "thorn_sumsq_scratch_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "thorn_sumsq_multi": (c_int, [POINTER(SumsqTensor), c_int, c_int, c_void_p]),
    "thorn_magma_scratch_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "thorn_magma_stats_multi": (c_int, [POINTER(MagmaTensor), c_int, c_int, c_int, c_void_p]),
    "thorn_peer_alloc": (c_int, [c_int64, POINTER(c_void_p)]),
    "thorn_peer_free": (c_int, [c_void_p]),
    "thorn_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "thorn_ipc_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "thorn_ipc_close": (c_int, [c_void_p]),
    "thorn_copy_async": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "thorn_peer_signal": (c_int, [POINTER(c_void_p), c_int, c_uint64, c_void_p]),
    "thorn_peer_wait": (c_int, [c_void_p, c_int, c_uint64, c_uint64, c_void_p, c_void_p]),
}

_lock = threading.Lock()
_lib = None


def library_path() -> str:
    """The in-tree build, or the file named by THORN_B200_LIBRARY (a build kept elsewhere)."""
    return os.environ.get("THORN_B200_LIBRARY") or _build.LIB


def load(build_if_missing: bool = False):
    """Load the shared library (raises if it is not built)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not os.path.exists(path):
            if build_if_missing:
                _build.build()
            else:
                raise RuntimeError(
                    f"thorn_b200 CUDA library not found at {path}; build it with `python -m thorn_b200.build`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in _PROTOS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int, what: str):
    if status != 0:
        lib = load()
        cuda = lib.thorn_last_cuda_error()
        msg = STATUS.get(status, f"status {status}")
        raise RuntimeError(f"thorn_b200: {what} failed: {msg}" + (f" (cudaError {cuda})" if status == 3 else ""))


def dtype_code(dt: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"thorn_b200 supports float32, bfloat16 and float16 tensors, got {dt}") from None


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def array(struct_type, items):
    arr = (struct_type * max(1, len(items)))()
    for i, it in enumerate(items):
        arr[i] = it
    return arr


def gemm_flops() -> tuple[float, float]:
    d, e = c_double(), c_double()
    load().thorn_gemm_flops(ctypes.byref(d), ctypes.byref(e))
    return d.value, e.value


def launch_count() -> int:
    return int(load().thorn_launch_count())
