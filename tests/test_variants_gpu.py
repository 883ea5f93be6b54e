"""GPU parity beyond the core cases: full-size shapes, edge inputs, group options (update_rate,
norm_axis, MD options, conv kernels, callable target norms), Magma and row-sparse gradients,
and the torch custom operators; each against the CPU oracle or a property that holds at any
size.  Tolerances as in test_gpu_parity.py.  (Collected after test_sharded.py, before the
allocation-free test.)"""
import ctypes

import numpy as np
import pytest
import torch

import cases as C
import parity as P
from oracle import thorn_oracle as O
from test_gpu_parity import _ns_gpu, _ns_gpu_t, assert_block_symmetric, compare, run_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(1, 4096, 4096), (1, 14336, 4096)])
def test_ns_full_size_matches_oracle(shape):
    """One Llama-3-8B q/o (4096x4096) and one gate/up (14336x4096, tall: Gram NS on the
    original orientation, transposed final product) matrix against the CPU oracle at full
    size (the oracle needs ~10-35 s of host time for these)."""
    torch.manual_seed(8)
    u = sum(torch.randn(shape) * (0.9 ** k) for k in range(4)) * 1e-3
    got, co, rs = _ns_gpu(u.cuda())
    O.NS_DTYPE = "f16"
    want = O.polar_decomp_2d(u[0].numpy(), co, rs, "f32")
    err = C.rel_fro(got[0], want)
    assert err <= 2e-2, err


@pytest.mark.parametrize("shape,kind", [((1, 14336, 4096), "rand"), ((1, 4096, 14336), "rand"),
                                        ((2, 4096, 4096), "near_id"), ((4, 1024, 4096), "rand"),
                                        ((1, 28672, 8192), "rand"), ((1, 8192, 8192), "near_id")])
def test_ns_full_size_singular_values(shape, kind):
    """At the Llama-3-8B and 70B shapes (too large for the CPU oracle), a size-independent property:
    every singular value of the NS output lies in the band the Polar-Express composition
    maps [1e-3, 1] into (the oracle gives [0.848, 1.153] at smaller sizes), while the
    Frobenius-normalised inputs have singular values near 1/sqrt(min dim) ~ 0.016."""
    torch.manual_seed(17)
    if kind == "rand":  # rectangular Gaussian matrices are well conditioned
        u = torch.randn(shape, device="cuda")
    else:  # square: I + W/4 with W a scaled Gaussian keeps every singular value in [0.5, 1.5]
        n = shape[-1]
        u = torch.eye(n, device="cuda") + 0.25 * torch.randn(shape, device="cuda") / n ** 0.5
    out, _, _ = _ns_gpu_t(u)
    for U in out.float():
        G = U.T @ U if U.shape[0] >= U.shape[1] else U @ U.T
        ev = torch.linalg.eigvalsh(G.double())
        s_min, s_max = float(ev.min().clamp_min(0).sqrt()), float(ev.max().sqrt())
        assert 0.8 < s_min and s_max < 1.2, (shape, s_min, s_max)


def test_full_size_state_updates():
    """Full Llama-3-8B sizes, size-independent checks of the elementwise passes: the momentum
    of a 14336x4096 bf16 matrix with fp32 state is bit for bit torch's (m * beta1) + g, and
    the (R)AdamW moments of the 128256x4096 embedding match torch's formulas (fp32)."""
    from thorn_b200 import THORN

    torch.manual_seed(21)
    w = torch.nn.Parameter(torch.randn(14336, 4096, device="cuda", dtype=torch.bfloat16) * 0.02)
    e = torch.nn.Parameter(torch.randn(128256, 4096, device="cuda", dtype=torch.bfloat16) * 0.02)
    opt = THORN([{"orthogonalize": True, "params": [w], "lr": 1e-3, "state_dtype": torch.float32},
                 {"orthogonalize": False, "params": [e], "lr": 1e-3, "state_dtype": torch.float32}])
    b1, b2 = 0.9, 0.95
    m_w = torch.zeros(w.shape, device="cuda")
    m_e = torch.zeros(e.shape, device="cuda")
    v_e = torch.zeros(e.shape, device="cuda")
    for _ in range(2):
        gw = torch.randn_like(w) * 1e-4
        ge = torch.randn_like(e) * 1e-4
        w.grad, e.grad = gw, ge
        opt.step()
        m_w = m_w * b1 + gw.float()
        ge32 = ge.float()
        m_e = m_e + (ge32 - m_e) * (1 - b1)
        v_e = v_e * b2 + ge32 * ge32 * (1 - b2)
        torch.cuda.synchronize()
        assert torch.equal(opt.state[w]["moment"], m_w)
        assert C.rel_fro(opt.state[e]["moment"].cpu().numpy(), m_e.cpu().numpy()) <= 1e-6
        assert C.rel_fro(opt.state[e]["variance"].cpu().numpy(), v_e.cpu().numpy()) <= 1e-6


def test_edge_inputs_match_oracle():
    """All-zero gradients (tall ortho matrix, MD matrix, AdamW vector), a one-row matrix and a
    tall matrix with 37 columns, against the oracle (pinned to the reference's goldens)."""
    name = "edge_small"
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, worst = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}
    for tag in gpu:
        assert all(np.isfinite(p).all() for g in gpu[tag][0] for p in g)


def test_qwen_layer_matches_oracle():
    """One decoder layer of the Qwen3-style configuration at full size (q 2048x1024, k/v
    1024x1024, o 1024x2048, gate/up 3072x1024, down 1024x3072) with its 151936x1024 tied
    embedding and RMSNorm weights, bf16 params and state, two steps against the oracle (whose
    first step is pinned to the reference's goldens at these shapes)."""
    name = "qwen_layer"
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, worst = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}
    print(name, {k: f"{v:.2e}" for k, v in sorted(worst.items())})


def test_update_rate_matches_oracle():
    """update_rate 2 on one device (thorn.py:1395, 1681, 1707): moments and step counts advance
    every step, parameters (orthogonalized, MD and AdamW) every second step; against the
    oracle, which is pinned to the reference's goldens for this case."""
    name = "rate_small"
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, _ = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}


def test_md_norm_axis_matches_oracle():
    """decouple_md with norm_axis=-1: the (R)AdamW renorm per row (2-D and 3-D tensors, a
    vector), the orthogonalized renorm per matrix; against the oracle, which is pinned to the
    reference's goldens for this case."""
    name = "md_axis_small"
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, _ = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}


def test_md_options_match_oracle():
    """MD with scalar gains on matrices (split_gain=False), gain_lr / gain_betas, "min" and
    "max" target norms, and none_grad=False: the gradient each parameter keeps (the
    direction-recovered one under MD) is compared too; against the oracle, pinned to the
    reference's goldens for this case."""
    name = "md_options_small"
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, worst = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}
    assert any(k[2] == "grad_after" for k in worst)


@pytest.mark.parametrize("name", ["md_conv_small", "md_target_fn_small"])
def test_md_conv_kernels_and_target_fn_match_oracle(name):
    """decouple_md on 3-D conv kernels (batches of matrices with per-entry row and column gains)
    and the "init" target norm on an orthogonalized group; a callable target norm on both group
    kinds; against the oracle, pinned to the reference's goldens for these cases."""
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, _ = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}


def _magma_seeds(name, gpu):
    """The Magma seeds the GPU run drew, in initialisation order: each parameter's
    generator state after step 1 stepped back once (every Magma parameter of
    these cases runs the generator once in step 1)."""
    from oracle.thorn_oracle import MASK64, W1_C

    seeds = []
    _, states = gpu["step1"]
    for gi, grp in enumerate(C.CASES[name]["groups"]):
        if grp["opts"].get("momentum_align"):
            for st in states[gi]:
                seeds.append((int(st["random_state"]) - W1_C) & MASK64)
    return seeds


@pytest.mark.parametrize("name", ["magma_small", "sparse_small"])
def test_magma_and_sparse_rows_match_oracle(name):
    """Magma masking (both group kinds, with and without MD) and row-sparse (R)AdamW
    gradients (duplicate rows, 1-D rows, an empty gradient) against the oracle, which
    is pinned to the reference's own runs of these cases; the oracle replays the GPU
    run's Magma seeds."""
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name, seeds=_magma_seeds(name, gpu))
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, worst = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}
    print(name, {k: f"{v:.2e}" for k, v in sorted(worst.items())})


def test_magma_stats_kernel_matches_fp64_sums():
    """thorn_magma_stats_multi against torch's fp64 sums of the same gradients and moments on
    the device: plain (fp32; bf16 with fp32 moments; fp16 with bf16 moments), the split MD gain
    on a batch of matrices and the scalar MD gain, the gradient recovered as g * gain in its
    own dtype (thorn.py:896-905).  Shapes with ragged tiles and columns that are not a
    multiple of 8.  Each sum is within 1e-6 of the fp64 sum (relative; the cross sum
    relative to |g| |m|), and a second launch gives the same bits."""
    import torch.nn.functional as F

    from thorn_b200 import _native as N

    lib = N.load()
    torch.manual_seed(11)
    dev = torch.device("cuda")
    cases = [  # (shape, g dtype, m dtype, gain kind)
        ((130, 300), torch.float32, torch.float32, None),
        ((3, 97, 40), torch.bfloat16, torch.float32, "split"),
        ((64, 37), torch.float16, torch.bfloat16, None),
        ((256, 512), torch.float32, torch.float32, "scalar"),
        ((2, 1, 8), torch.float32, torch.float32, "split"),
        ((1000,), torch.bfloat16, torch.bfloat16, None),
    ]
    recs, want, keep = [], [], []
    for shape, gdt, mdt, gain in cases:
        g = (torch.randn(shape, device=dev) * 1e-3).to(gdt)
        m = (torch.randn(shape, device=dev) * 1e-3 + 0.3 * g.float()).to(mdt)
        rg = cg = None
        gr = g
        if gain == "split":
            rg = (torch.randn((*shape[:-1], 1), device=dev) * 0.5).to(gdt)
            cg = (torch.randn((*shape[:-2], 1, shape[-1]), device=dev) * 0.5).to(gdt)
            gr = g * (F.softplus(rg) * F.softplus(cg))
        elif gain == "scalar":
            rg = torch.tensor(0.7, device=dev).to(gdt)
            gr = g * F.softplus(rg)
        a, b = gr.double().flatten(), m.double().flatten()
        want.append(torch.stack([(a * b).sum(), (a * a).sum(), (b * b).sum()]).cpu())
        B = int(np.prod(shape[:-2])) if len(shape) > 2 else 1
        R, Cc = (shape[-2], shape[-1]) if len(shape) >= 2 else (1, shape[0])
        keep += [g, m, rg, cg]
        recs.append((g, m, rg, cg, 1 if gain == "scalar" else 0, B, R, Cc))
    out = torch.zeros((len(cases), 3), dtype=torch.float64, device=dev)
    sizes = [int(lib.thorn_magma_scratch_bytes(B, R, Cc)) for *_, B, R, Cc in recs]
    offs = np.cumsum([0] + [(s + 255) // 256 * 256 for s in sizes])
    scratch = torch.zeros(int(offs[-1]), dtype=torch.uint8, device=dev)
    stream = N.stream_of(dev)

    def launch():
        for i, (g, m, rg, cg, sc, B, R, Cc) in enumerate(recs):
            t = N.MagmaTensor(g.data_ptr(), m.data_ptr(), None if rg is None else rg.data_ptr(),
                              None if cg is None else cg.data_ptr(), sc, B, R, Cc, out.data_ptr() + 24 * i,
                              scratch.data_ptr() + int(offs[i]))
            N.check(lib.thorn_magma_stats_multi(N.array(N.MagmaTensor, [t]), 1, N.dtype_code(g.dtype),
                                                N.dtype_code(m.dtype), stream), "magma_stats_multi")
        torch.cuda.synchronize()
        return out.cpu().clone()

    got = launch()
    for i, (w, gt) in enumerate(zip(want, got)):
        scale = float(torch.sqrt(w[1] * w[2]))
        assert abs(float(gt[0] - w[0])) <= 1e-6 * scale, (i, gt, w)
        assert abs(float(gt[1] - w[1])) <= 1e-6 * float(w[1]), (i, gt, w)
        assert abs(float(gt[2] - w[2])) <= 1e-6 * float(w[2]), (i, gt, w)
    assert torch.equal(launch(), got)  # fixed-order sums; the scratch is left zero for the next call
    assert int(scratch.count_nonzero()) == 0


def test_custom_ops_match_c_abi():
    """torch.ops.thorn_b200.sym_addmm (the thorn::sym_addmm contract, thorn.py:298-368) against
    an fp32 product, and torch.ops.thorn_b200.polar_decomp against the C ABI it wraps."""
    import thorn_b200  # noqa: F401  (registers the operators)
    from thorn_b200.coeffs import gram_ns_restarts, optimal_composition

    torch.manual_seed(4)
    A = (torch.randn(3, 256, 128, device="cuda") / 16).half()
    Cs = torch.randn(256, 256, device="cuda").half()
    Cs = (Cs + Cs.T) / 2
    out = torch.ops.thorn_b200.sym_addmm(A, A.transpose(1, 2), Cs, 0.5, -1.0)
    want = 0.5 * (A.float() @ A.float().transpose(1, 2)) - Cs.float()
    assert (out.float() - want).abs().max() <= 2e-2 * want.abs().max()
    assert_block_symmetric(out)
    # the reference's operator name reaches the same kernel (bit for bit)
    assert torch.equal(torch.ops.thorn.sym_addmm(A, A.transpose(1, 2), Cs, 0.5, -1.0), out)
    # M and K that are not multiples of 8 (zero-padded inside the operator)
    A2 = (torch.randn(2, 37, 20, device="cuda") / 8).half()
    C2 = torch.randn(2, 37, 37, device="cuda").half()
    C2 = (C2 + C2.transpose(1, 2)) / 2
    out2 = torch.ops.thorn_b200.sym_addmm(A2, A2.transpose(1, 2), C2, 1.0, 0.5)
    want2 = A2.float() @ A2.float().transpose(1, 2) + 0.5 * C2.float()
    assert out2.shape == (2, 37, 37) and (out2.float() - want2).abs().max() <= 2e-2 * want2.abs().max()
    co = optimal_composition(1e-3, 5, 0.03, 0.02)
    rs = gram_ns_restarts(*co)
    for shape in [(2, 384, 128), (1, 100, 37)]:
        u = torch.randn(shape, device="cuda") * 1e-3
        got = torch.ops.thorn_b200.polar_decomp(u, [x for t in co for x in t], list(rs))
        # the same NS on an input normalised by torch instead of the library's passes
        ref, _, _ = _ns_gpu_t(u)
        assert got.dtype == u.dtype and got.shape == u.shape
        assert C.rel_fro(got.cpu().numpy(), ref.float().cpu().numpy()) <= 1e-2


@pytest.mark.parametrize("shape,small", [((2, 96, 64), True), ((2, 96, 64), False), ((1, 256, 512), False)])
def test_bounded_wait_runs_out_and_device_recovers(shape, small):
    """The failure path of the NS kernels' bounded waits, made to run without any fault.

    With the test stall switch on, the GEMMs' TMA producers issue no loads (the small-matrix
    kernel issues no MMA), so nothing is ever in flight and the first wait for one runs out
    after the (shortened) wait limit.  The call must return, the error flag must be set (also
    through THORN.device_error()), and the next normal call on the same device must be
    correct.  (96x64 runs the one-launch small-matrix kernel, or with it switched off the
    single-CTA GEMM; 256x512 the 2-CTA cluster GEMM.)"""
    import time

    from thorn_b200 import THORN
    from thorn_b200 import _native as N

    lib = N.load()
    torch.manual_seed(31)
    u = torch.randn(shape, device="cuda") * 1e-3
    prev_small = lib.thorn_set_ns_small(1 if small else 0)
    prev_limit = lib.thorn_set_wait_limit_ns(20 * 10 ** 6)
    prev_stall = lib.thorn_set_gemm_test_stall(1)
    try:
        ldc = int(lib.thorn_ns_ld(shape[2]))
        X = torch.zeros((shape[0], shape[1], ldc), dtype=torch.float16, device="cuda")
        out = torch.empty(shape, dtype=torch.float16, device="cuda")
        wsb = int(lib.thorn_ns_workspace_bytes(*shape))
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        co, rr = (ctypes.c_double * 3)(1.0, 0.0, 0.0), (ctypes.c_int32 * 1)(0)
        t0 = time.perf_counter()
        N.check(lib.thorn_ns_batched(X.data_ptr(), out.data_ptr(), ws.data_ptr(), wsb, *shape, N.F16, co, 1, rr, 0,
                                     err.data_ptr(), N.stream_of(torch.device("cuda"))), "ns_batched")
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 30.0
        assert int(err.item()) == 1
        # the optimizer sees it too: one step of a small orthogonalized group
        p = torch.nn.Parameter(torch.randn(shape[1], shape[2], device="cuda") * 0.02)
        opt = THORN([{"params": [p], "orthogonalize": True, "lr": 1e-3}])
        p.grad = torch.randn_like(p) * 1e-3
        opt.step()
        assert opt.device_error()
    finally:
        lib.thorn_set_gemm_test_stall(prev_stall)
        lib.thorn_set_wait_limit_ns(prev_limit)
        lib.thorn_set_ns_small(prev_small)
    # the context is usable: the same NS now matches the oracle
    got, co5, rs5 = _ns_gpu(u)
    O.NS_DTYPE = "f16"
    want = np.stack([O.polar_decomp_2d(x, co5, rs5, "f32") for x in u.cpu().numpy()])
    assert C.rel_fro(got, want) <= 2e-2
