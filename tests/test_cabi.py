"""C-ABI checks that need no GPU: the library loads, exports every symbol that
``include/thorn_b200.h`` declares, the ctypes mirrors match the C layouts, and
the host-only entry points (sizes, status strings, argument validation) work."""
import ctypes
import os
import re
import subprocess

import pytest

from thorn_b200 import _native as N
from thorn_b200 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "thorn_b200.h")


@pytest.fixture(scope="module")
def lib():
    B.build()
    return N.load()


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"THORN_API\s+[\w\s\*]+?\b(thorn_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ["thorn_adamw_multi", "thorn_ortho_pre_multi", "thorn_ns_cast_multi", "thorn_ns_batched",
                 "thorn_sym_addmm", "thorn_pnn_stats_multi", "thorn_ortho_post_multi", "thorn_md_prep_multi",
                 "thorn_md_gain_grad_multi", "thorn_md_finalize_multi", "thorn_sumsq_multi"]:
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", N.library_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\b(thorn_\w+)$", out, flags=re.M))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    for n in declared_functions():
        assert hasattr(lib, n)
    # everything the ctypes layer binds is declared
    assert set(N._PROTOS) <= set(declared_functions())


STRUCTS = {
    "thorn_adam_tensor": (N.AdamTensor, ["p", "g", "m", "v", "numel", "lr", "bc1", "bc2", "degenerate"]),
    "thorn_ortho_pre_tensor": (N.OrthoPreTensor, ["p", "g", "m", "normsq", "batch", "rows", "cols", "row_sp",
                                                  "col_sp", "scalar_gain", "row_gsum", "col_gsum", "scratch"]),
    "thorn_ns_cast_tensor": (N.NsCastTensor, ["g", "m", "normsq", "x", "batch", "rows", "cols", "row_sp", "col_sp",
                                              "scalar_gain", "md"]),
    "thorn_pnn_tensor": (N.PnnTensor, ["U", "row_scale", "mat_stats", "batch", "rows", "cols", "scratch", "fold"]),
    "thorn_ortho_post_tensor": (N.OrthoPostTensor, ["U", "p", "row_scale", "mat_stats", "p_normsq", "batch",
                                                    "rows", "cols", "lr", "scratch", "round_u"]),
    "thorn_sumsq_tensor": (N.SumsqTensor, ["x", "out", "batch", "rows", "cols", "scratch"]),
    "thorn_magma_tensor": (N.MagmaTensor, ["g", "m", "row_gain", "col_gain", "scalar_gain", "batch", "rows",
                                           "cols", "out", "scratch"]),
    "thorn_md_prep_tensor": (N.MdPrepTensor, ["gain", "sp", "sig", "n"]),
    "thorn_md_grad_tensor": (N.MdGradTensor, ["gsum", "sig", "grad", "n"]),
    "thorn_md_final_tensor": (N.MdFinalTensor, ["p", "normsq", "target", "target_stride", "row_sp", "col_sp",
                                                "scalar_gain", "batch", "rows", "cols"]),
}


def test_struct_layouts_match_header(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "thorn_b200.h"', "int main(void) {"]
    for cname, (_, flds) in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f in flds:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("  return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    c = {}
    for line in out:
        if line:
            name, f, v = line.split()
            c[(name, f)] = int(v)
    for cname, (st, flds) in STRUCTS.items():
        assert ctypes.sizeof(st) == c[(cname, "size")], cname
        for f in flds:
            assert getattr(st, f).offset == c[(cname, f)], (cname, f)


def test_host_only_entry_points(lib):
    assert lib.thorn_abi_version() == 1
    assert lib.thorn_status_string(0) == b"ok"
    assert lib.thorn_status_string(2).startswith(b"misaligned")
    assert lib.thorn_ns_ld(1) == 8 and lib.thorn_ns_ld(8) == 8 and lib.thorn_ns_ld(4097) == 4104
    # gram: 2 x-buffers + 5 m x m buffers; square: 4 m x m buffers (bytes, 256-aligned)
    assert lib.thorn_ns_workspace_bytes(1, 1024, 4096) == 2 * 1024 * 4096 * 2 + 5 * 1024 * 1024 * 2
    assert lib.thorn_ns_workspace_bytes(3, 512, 512) == 4 * 3 * 512 * 512 * 2
    assert lib.thorn_ns_workspace_bytes(2, 96, 32) == lib.thorn_ns_workspace_bytes(2, 32, 96)
    assert lib.thorn_ns_workspace_bytes(0, 8, 8) == 0
    # scratch: counters + one partial per 64x256 tile (+ md row/col partials); the renorm sums
    # of squares keep fp64 partials
    assert lib.thorn_sumsq_scratch_bytes(1, 64, 256) == 4 * 4 + 1 * 8
    assert lib.thorn_sumsq_scratch_bytes(5, 130, 300) == 8 * 4 + 5 * 3 * 2 * 8
    assert lib.thorn_ortho_pre_scratch_bytes(2, 128, 512, 0) > 0
    assert lib.thorn_ortho_pre_scratch_bytes(2, 128, 512, 1) > lib.thorn_ortho_pre_scratch_bytes(2, 128, 512, 0)
    assert lib.thorn_pnn_scratch_bytes(3, 100) == (4 + 2 * 300) * 4
    # Magma sums: one counter (16 bytes), then three fp64 partials per 64x256 tile
    assert lib.thorn_magma_scratch_bytes(1, 64, 256) == 16 + 3 * 8
    assert lib.thorn_magma_scratch_bytes(2, 130, 300) == 16 + 3 * 2 * 3 * 2 * 8
    assert lib.thorn_magma_scratch_bytes(0, 8, 8) == 0


def test_argument_validation_without_gpu(lib):
    """Bad arguments are rejected before anything touches the device."""
    arr = N.array(N.AdamTensor, [])
    assert lib.thorn_adamw_multi(arr, -1, 0, 0, 0.9, 0.95, 0.0, 0.0, None) == 1
    assert lib.thorn_adamw_multi(arr, 0, 7, 0, 0.9, 0.95, 0.0, 0.0, None) == 1  # bad dtype
    bad = N.array(N.AdamTensor, [N.AdamTensor(None, None, None, None, 16, 1e-3, 1.0, 1.0, 0)])
    assert lib.thorn_adamw_multi(bad, 1, 0, 0, 0.9, 0.95, 0.0, 0.0, None) == 1  # null grad
    assert lib.thorn_adamw_multi(arr, 0, 0, 0, 0.9, 0.95, 0.0, 0.0, None) == 0  # nothing to do
    co = (ctypes.c_double * 3)(1.0, 0.0, 0.0)
    rs = (ctypes.c_int32 * 1)(0)
    assert lib.thorn_ns_batched(None, None, None, 0, 1, 8, 8, 2, co, 1, rs, 0, None, None) == 1
    assert lib.thorn_ns_batched(None, None, None, 0, 0, 8, 8, 2, co, 1, rs, 0, None, None) == 0
    assert lib.thorn_ns_batched(1024, 2048, 4096, 1 << 30, 1, 8, 8, 0, co, 1, rs, 0, None, None) == 1  # f32 NS
    # sizes whose workspace does not fit in int64 are rejected, not wrapped to a small or negative size
    big = (1 << 31) - 1
    assert lib.thorn_ns_workspace_bytes(big, big, big) == -1
    assert lib.thorn_ns_workspace_bytes(1, 1 << 62, 3) == -1
    assert lib.thorn_ns_batched(1024, 2048, 4096, 1 << 62, big, big, big, 2, co, 1, rs, 0, None, None) == 1
    assert lib.thorn_ns_batched_static(1024, 2048, big, big, big, 2, co, 1, rs, 0, None, None) == 5  # too large
    mg = N.array(N.MagmaTensor, [N.MagmaTensor(None, None, None, None, 0, 1, 4, 4, None, None)])
    assert lib.thorn_magma_stats_multi(mg, 1, 0, 0, None) == 1  # null operands
    assert lib.thorn_magma_stats_multi(mg, 1, 9, 0, None) == 1  # bad dtype
    split = N.array(N.MagmaTensor, [N.MagmaTensor(16, 16, 16, None, 0, 1, 4, 4, 16, 16)])
    assert lib.thorn_magma_stats_multi(split, 1, 0, 0, None) == 1  # split gain without column gains
    empty = N.array(N.MagmaTensor, [N.MagmaTensor(None, None, None, None, 0, 1, 0, 4, None, None)])
    assert lib.thorn_magma_stats_multi(empty, 1, 0, 0, None) == 0  # empty tensor: nothing to do
    # symmetric GEMM needs 8-element leading dimensions
    assert lib.thorn_sym_addmm(16, 16, None, 16, 1, 12, 16, 0, 1.0, 0.0, 2, None, None) == 2
    pre = N.array(N.OrthoPreTensor, [N.OrthoPreTensor(None, None, None, None, 1, 4, 4, None, None, 0, None, None,
                                                       None)])
    assert lib.thorn_ortho_pre_multi(pre, 1, 0, 0, 0, 0.9, 0, 0, None) == 1
    mp = N.array(N.MdPrepTensor, [N.MdPrepTensor(None, None, None, 4)])
    assert lib.thorn_md_prep_multi(mp, 1, 0, None) == 1


@pytest.mark.parametrize("name,default", [("thorn_set_gemm_pair", 1), ("thorn_set_gemm_staged_epilogue", 1),
                                          ("thorn_set_gemm_pdl", 0),
                                          ("thorn_set_gemm_l2_hints", 0), ("thorn_set_gemm_test_stall", 0),
                                          ("thorn_set_ns_small", 1)])
def test_kernel_switches(lib, name, default):
    """Each switch returns its previous setting; the defaults are the measured kernels."""
    fn = getattr(lib, name)
    prev = fn(default)
    assert prev == default
    assert fn(1 - default) == default
    assert fn(default) == 1 - default
    assert fn(7 if default else 0) == default  # any nonzero value means on
    fn(default)


def test_empty_shards_accepted_without_device_work(lib):
    """A Shard(0) shard with no rows (a matrix with fewer rows than ranks) arrives with null
    data pointers; every entry point accepts it and launches nothing, with and without
    decouple_md (so no GPU is needed here)."""
    pre = N.array(N.OrthoPreTensor, [N.OrthoPreTensor(None, None, None, None, 1, 0, 48, None, None, 0, None, None,
                                                       None)])
    for md in (0, 1):
        assert lib.thorn_ortho_pre_multi(pre, 1, 0, 0, 0, 0.9, md, 0, None) == 0
    cast = N.array(N.NsCastTensor, [N.NsCastTensor(None, None, None, None, 1, 0, 48, None, None, 0, 1)])
    assert lib.thorn_ns_cast_multi(cast, 1, 0, 0, 0, 2, 0.9, None) == 0
    post = N.array(N.OrthoPostTensor, [N.OrthoPostTensor(None, None, None, None, None, 1, 0, 48, 1e-3, None, 0)])
    assert lib.thorn_ortho_post_multi(post, 1, 2, 0, 0.1, None) == 0
    fin = N.array(N.MdFinalTensor, [N.MdFinalTensor(None, None, None, 0, None, None, 0, 1, 0, 48)])
    assert lib.thorn_md_finalize_multi(fin, 1, 0, None) == 0
    pnn = N.array(N.PnnTensor, [N.PnnTensor(None, None, None, 1, 0, 48, None, 1)])
    assert lib.thorn_pnn_stats_multi(pnn, 1, 2, 0, None) == 0
    # a non-empty tensor with the same null pointers is still rejected
    fin_bad = N.array(N.MdFinalTensor, [N.MdFinalTensor(None, None, None, 0, None, None, 0, 1, 2, 48)])
    assert lib.thorn_md_finalize_multi(fin_bad, 1, 0, None) == 1


def test_wait_limit_setter(lib):
    """The GEMM wait limit: returns the previous value; 0 restores the 10 s default."""
    default = 10 * 10 ** 9
    assert lib.thorn_set_wait_limit_ns(0) == default
    assert lib.thorn_set_wait_limit_ns(20 * 10 ** 6) == default
    assert lib.thorn_set_wait_limit_ns(0) == 20 * 10 ** 6
    assert lib.thorn_set_wait_limit_ns(0) == default


def _ctype_of(decl: str):
    """The ctypes type that binds one C parameter or return type of the header."""
    d = " ".join(re.sub(r"\bconst\b", " ", decl).split())
    d = re.sub(r"\s*\*\s*", "*", d)
    base = d.split()[0] if " " in d and "*" not in d.split()[0] else d
    if d in ("void", ""):
        return None
    if d.endswith("**"):  # an out-parameter or an array of device pointers
        return ctypes.POINTER(ctypes.c_void_p)
    if d.endswith("*"):
        t = d.rstrip("*").split()[0]
        if d == "char*":
            return ctypes.c_char_p
        return {"double": ctypes.POINTER(ctypes.c_double), "int32_t": ctypes.POINTER(ctypes.c_int32)}.get(
            t, "struct" if t.startswith("thorn_") else ctypes.c_void_p)
    return {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "uint64_t": ctypes.c_uint64, "float": ctypes.c_float,
            "double": ctypes.c_double}[base.split()[0]]


def test_ctypes_prototypes_match_header():
    """Every function the ctypes layer binds has, in _native._PROTOS, exactly the parameter
    count and C types (and return type) the header declares: a mismatch would hand a kernel
    shifted arguments."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    protos = {}
    for m in re.finditer(r"THORN_API\s+([\w\s\*]+?)\b(thorn_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, args = m.group(1).strip(), m.group(2), m.group(3).strip()
        params = [] if args in ("", "void") else [re.sub(r"\b\w+$", "", a.strip()).strip() for a in args.split(",")]
        protos[name] = (ret, params)
    for name, (res, argtypes) in N._PROTOS.items():
        ret, params = protos[name]
        assert len(params) == len(argtypes), (name, params, argtypes)
        want_ret = _ctype_of(ret)
        assert res == want_ret, (name, ret, res)
        for i, (cdecl, got) in enumerate(zip(params, argtypes)):
            want = _ctype_of(cdecl)
            if want == "struct":  # an array of launch records: POINTER(<matching Structure>)
                assert hasattr(got, "_type_") and issubclass(got._type_, ctypes.Structure), (name, i, cdecl, got)
                cname = cdecl.replace("const", "").replace("*", "").strip()
                assert got._type_ is STRUCTS[cname][0], (name, i, cname, got._type_)
            else:
                assert got == want, (name, i, cdecl, got, want)


def test_peer_exchange_entry_points_validate_without_gpu(lib):
    """The peer-exchange entry points reject bad arguments before touching a device."""
    vp = ctypes.c_void_p()
    assert lib.thorn_peer_alloc(0, ctypes.byref(vp)) == 1
    assert lib.thorn_ipc_handle(None, None) == 1
    assert lib.thorn_ipc_open(None, ctypes.byref(vp)) == 1
    assert lib.thorn_copy_async(None, None, -1, None) == 1
    assert lib.thorn_copy_async(None, None, 0, None) == 0  # nothing to copy
    slots = (ctypes.c_void_p * 65)()
    assert lib.thorn_peer_signal(slots, 65, 1, None) == 1  # at most 64 peers
    assert lib.thorn_peer_signal(slots, 1, 1, None) == 1  # a null slot
    slots[0] = 12  # not 8-byte aligned
    assert lib.thorn_peer_signal(slots, 1, 1, None) == 1
    assert lib.thorn_peer_wait(12, 1, 1, 1000, None, None) == 1
    assert lib.thorn_peer_wait(None, 0, 1, 1000, None, None) == 0  # no slots: no launch
