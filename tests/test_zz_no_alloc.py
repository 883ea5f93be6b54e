"""The allocation-free Newton-Schulz entry point, thorn_ns_batched_static.

It serves callers that cannot allocate device memory -- a custom call inside a
host framework that hands over only its operands, or code that must not call
cudaMalloc after start-up -- by using a fixed 64 MiB device workspace built
into the library.  This file is collected last so that, if it fails, a run that
stops at the first failure has already run every other test; it also passes
when run alone in a fresh process.
"""
import ctypes

import pytest
import torch

import cases as C

pytestmark = pytest.mark.gpu


def _coeffs():
    from thorn_b200.coeffs import gram_ns_restarts, optimal_composition

    co = optimal_composition(1e-3, 5, 0.03, 0.02)
    rs = gram_ns_restarts(*co)
    return (ctypes.c_double * 15)(*[v for t in co for v in t]), (ctypes.c_int32 * max(1, len(rs)))(*rs), len(rs)


def _normalised_input(u):
    from thorn_b200 import _native as N

    B, R, Cc = u.shape
    ld = int(N.load().thorn_ns_ld(Cc))
    x = u.float()
    x = x / (x.norm(dim=(-2, -1), keepdim=True) + 1e-8)
    X = torch.zeros((B, R, ld), dtype=torch.float16, device="cuda")
    X[:, :, :Cc] = x.half()  # original orientation, also for tall matrices
    return X


@pytest.mark.parametrize("shape", [(3, 1024, 512), (2, 768, 768)])
def test_static_workspace_matches_allocating_entry_point(shape):
    from thorn_b200 import _native as N

    lib = N.load()
    cc, rr, nr = _coeffs()
    st = N.stream_of(torch.device("cuda"))
    B, R, Cc = shape
    wsb = int(lib.thorn_ns_workspace_bytes(B, R, Cc))
    assert wsb <= N.NS_STATIC_WORKSPACE_BYTES
    for call in range(2):  # two calls in a row: the shared array keeps the previous call's contents
        torch.manual_seed(100 + call)
        X = _normalised_input(torch.randn(shape, device="cuda") * 1e-3)
        err = torch.zeros(2, dtype=torch.int32, device="cuda")
        got = torch.empty((B, R, Cc), dtype=torch.float16, device="cuda")
        N.check(lib.thorn_ns_batched_static(X.data_ptr(), got.data_ptr(), B, R, Cc, N.F16, cc, 5, rr, nr,
                                            err.data_ptr(), st), "ns_batched_static")
        want = torch.empty_like(got)
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        N.check(lib.thorn_ns_batched(X.data_ptr(), want.data_ptr(), ws.data_ptr(), wsb, B, R, Cc, N.F16, cc, 5, rr,
                                     nr, err[1:].data_ptr(), st), "ns_batched")
        torch.cuda.synchronize()
        assert int(err[0]) == 0 and int(err[1]) == 0
        rel = C.rel_fro(got.float().cpu().numpy(), want.float().cpu().numpy())
        assert rel <= 2e-2, rel  # the NS parity tolerance of the other tests
        assert torch.equal(got, want)  # same kernels, deterministic: identical


def test_static_workspace_rejects_oversized_problem():
    from thorn_b200 import _native as N

    lib = N.load()
    cc, rr, nr = _coeffs()
    assert int(lib.thorn_ns_workspace_bytes(1, 4096, 4096)) > N.NS_STATIC_WORKSPACE_BYTES
    st = lib.thorn_ns_batched_static(None, None, 1, 4096, 4096, N.F16, cc, 5, rr, nr, None,
                                     N.stream_of(torch.device("cuda")))
    assert st == 5  # THORN_ERR_TOO_LARGE, rejected before touching the device
