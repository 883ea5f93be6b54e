"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

The oracle runs with fp32 scalars (the reference's CUDA/Triton semantics; the
golden-pinned CPU quirks are off).  Inputs are the seeded cases of
``tests/cases.py``.  Tolerances:

* orthogonalized params, cumulative update, relative Frobenius: 2e-2 for fp32
  params (north_star); 5e-2 for bf16 params, whose per-step update is only 1-2
  bf16 ulps so rounding flips dominate (the oracle itself sits at 2.7e-2 from
  the reference there);
* (R)AdamW / vector params and all fp32 optimizer state: 1e-5 (2e-3 when
  stored in bf16: one 1-ulp rounding flip in 4096 elements is 6e-5);
* MD gains (their gradients are sums over the orthogonalized update): 1e-3.
"""
import copy
import ctypes
import math

import numpy as np
import pytest
import torch

import cases as C
import parity as P
from oracle import thorn_oracle as O

pytestmark = pytest.mark.gpu

ORTHO_TOL = {"f32": 2e-2, "bf16": 5e-2}
VEC_TOL = 1e-5
# bf16-stored vectors: a single 1-ulp bf16 rounding flip (from fp32 fma ordering)
# in a 4096-element tensor is already 6e-5 relative
VEC_TOL_BF16 = 2e-3
GAIN_TOL = 1e-3


def _np(t):
    return t.detach().float().cpu().numpy()


def run_gpu(name, state_dtype=None, ns_dtype=None, steps=None):
    from thorn_b200 import THORN

    case = C.CASES[name]
    params = C.build_params(case)
    tp = [[torch.nn.Parameter(t.clone().cuda()) for t in ps] for ps in params]
    groups = C.group_dicts(case, tp)
    if state_dtype:
        for g in groups:
            g["state_dtype"] = C.TORCH_DTYPES[state_dtype]
    opt = THORN(groups)
    opt._update_rate = case.get("update_rate", 1)  # what setup_gradient_release(update_rate=...) sets
    if ns_dtype is not None:
        opt.ns_dtype = ns_dtype
    n = case["steps"] if steps is None else steps
    snaps = {}
    for s in range(n):
        grads = C.build_grads(case, s)
        for ps, gs in zip(tp, grads):
            for p, g in zip(ps, gs):
                p.grad = g.cuda()
        opt.step()
        if s == 0 or s == n - 1:
            tag = "step1" if s == 0 else "final"
            snaps[tag] = ([[_np(p) for p in ps] for ps in tp],
                          [[{**{k: (_np(v) if isinstance(v, torch.Tensor) else v) for k, v in opt.state[p].items()},
                             **({"grad_after": _np(p.grad)} if p.grad is not None else {})}
                            for p in ps] for ps in tp])
    torch.cuda.synchronize()
    assert not opt.device_error()
    for grp, ps in zip(case["groups"], tp):
        for p in ps:
            # none_grad (default True) drops the gradient; otherwise it stays (MD: recovered)
            assert (p.grad is None) == grp["opts"].get("none_grad", True)
    return opt, snaps


def _tol(name, gi, key):
    grp = C.CASES[name]["groups"][gi]
    if key == "param" and grp["orthogonalize"]:
        return ORTHO_TOL[grp["dtype"]]
    if "gain" in key and grp["orthogonalize"]:
        return GAIN_TOL
    if key == "param" and grp["opts"].get("decouple_md"):
        return 1e-4  # renorm/gain multiplies: a few fp32 roundings in another order
    if grp["dtype"] != "f32":
        return VEC_TOL_BF16
    return VEC_TOL


def compare(name, gpu, orc, init):
    bad = {}
    worst = {}
    for tag in gpu:
        gp, gs = gpu[tag]
        op, os_ = orc[tag]
        for gi in range(len(gp)):
            for pi in range(len(gp[gi])):
                e = C.rel_fro(gp[gi][pi] - init[gi][pi], op[gi][pi] - init[gi][pi])
                keyl = [("param", e)]
                for k, v in gs[gi][pi].items():
                    if k in ("step", "random_state"):  # integers: exact
                        assert int(v) == int(os_[gi][pi][k]), (tag, gi, pi, k)
                        continue
                    ref = np.asarray(os_[gi][pi][k], dtype=np.float32).reshape(np.shape(v))
                    keyl.append((k, C.rel_fro(v, ref)))
                for k, err in keyl:
                    worst[(tag, gi, k)] = max(worst.get((tag, gi, k), 0.0), err)
                    if not err <= _tol(name, gi, k):
                        bad[(tag, gi, pi, k)] = err
    return bad, worst


CASES = ["tiny_small", "md_small", "bf16_small", "conv_small", "variants_small", "vad", "tiny"]


@pytest.mark.parametrize("name", CASES)
def test_step_matches_oracle(name):
    _, gpu = run_gpu(name)
    _, orc = P.run_oracle(name)
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES[name])]
    bad, worst = compare(name, gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}
    print(name, {k: f"{v:.2e}" for k, v in sorted(worst.items())})


def test_bf16_params_with_fp32_state():
    _, gpu = run_gpu("bf16_small", state_dtype="f32")
    _, orc = P.run_oracle("bf16_small", state_dtype="f32")
    init = [[t.float().numpy() for t in g] for g in C.build_params(C.CASES["bf16_small"])]
    bad, _ = compare("bf16_small", gpu, orc, init)
    assert not bad, {k: f"{v:.3e}" for k, v in sorted(bad.items())[:10]}


# ---------------------------------------------------------------- NS / GEMM
def assert_block_symmetric(o: torch.Tensor, blk: int = 128):
    """A symmetric GEMM output (thorn::sym_addmm contract): outside the diagonal 128-blocks the
    output is an exact mirror image; inside them every element is stored as computed (as the
    reference's Triton kernel stores its diagonal tiles), which for a Gram product A A^T with a
    symmetric C is symmetric up to one rounding."""
    m = o.shape[-1]
    idx = torch.arange(m, device=o.device) // blk
    off = idx[:, None] != idx[None, :]
    ot = o.transpose(-2, -1)
    assert torch.equal(o[..., off], ot[..., off])
    gap = (o.float() - ot.float()).abs().max().item()
    assert gap <= 1e-3 * o.float().abs().max().item(), gap


def _ns_gpu(u: torch.Tensor, ns_dtype=torch.float16, iters=5):
    """Polar factor of each matrix of u (B, R, C) via thorn_ns_batched (as numpy on the host)."""
    out, co, rs = _ns_gpu_t(u, ns_dtype, iters)
    return out.float().cpu().numpy(), co, rs


def _ns_gpu_t(u: torch.Tensor, ns_dtype=torch.float16, iters=5):
    """Polar factor of each matrix of u (B, R, C) via thorn_ns_batched (device tensor)."""
    from thorn_b200 import _native as N
    from thorn_b200.coeffs import gram_ns_restarts, optimal_composition

    lib = N.load()
    Bn, R, Cc = u.shape
    ldc = int(lib.thorn_ns_ld(Cc))
    x = u.float()
    x = x / (x.norm(dim=(-2, -1), keepdim=True) + 1e-8)
    X = torch.zeros((Bn, R, ldc), dtype=ns_dtype, device="cuda")
    X[:, :, :Cc] = x.to(ns_dtype)  # original orientation, also for tall matrices
    out = torch.empty((Bn, R, Cc), dtype=ns_dtype, device="cuda")
    wsb = int(lib.thorn_ns_workspace_bytes(Bn, R, Cc))
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    co = optimal_composition(1e-3, iters, 0.03, 0.02)
    rs = gram_ns_restarts(*co)
    cc = (ctypes.c_double * (3 * iters))(*[v for t in co for v in t])
    rr = (ctypes.c_int32 * max(1, len(rs)))(*rs)
    N.check(lib.thorn_ns_batched(X.data_ptr(), out.data_ptr(), ws.data_ptr(), wsb, Bn, R, Cc,
                                 N.dtype_code(ns_dtype), cc, iters, rr, len(rs), err.data_ptr(),
                                 N.stream_of(torch.device("cuda"))), "ns_batched")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out, co, rs


@pytest.mark.parametrize("shape", [(1, 64, 64), (3, 128, 64), (2, 64, 128), (1, 512, 512), (1, 1024, 512),
                                   (1, 512, 1024), (4, 96, 32), (2, 2, 128), (6, 128, 384), (1, 300, 200),
                                   (1, 1024, 4096), (1, 2048, 2048), (1, 66, 64), (2, 64, 66), (1, 260, 256)])
def test_ns_matches_oracle(shape):
    torch.manual_seed(7)
    u = sum(torch.randn(shape) * (0.9 ** k) for k in range(4)) * 1e-3
    got, co, rs = _ns_gpu(u.cuda())
    O.NS_DTYPE = "f16"
    want = np.stack([O.polar_decomp_2d(x, co, rs, "f32") for x in u.numpy()])
    err = C.rel_fro(got, want)
    assert err <= 2e-2, err


@pytest.mark.parametrize("ns_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(6, 64, 96), (6, 128, 384), (4, 128, 128), (2, 2, 128), (3, 96, 64),
                                   (2, 100, 37), (1, 1, 64), (1, 512, 128), (2, 128, 512), (2, 40, 40)])
def test_ns_small_kernel_matches_gemm_sequence(shape, ns_dtype):
    """Matrices with min dim <= 128 and max dim <= 512 run the whole Newton-Schulz iteration in
    one launch (one CTA per matrix, operands resident in shared memory).  Against the same
    recurrences issued as separate GEMM launches on the same input: the same products, operand
    orders and roundings, so the two agree to accumulation order at most; and one launch."""
    from thorn_b200 import _native as N

    lib = N.load()
    torch.manual_seed(11)
    u = torch.randn(shape, device="cuda") * 1e-3
    prev = lib.thorn_set_ns_small(1)
    try:
        n0 = N.launch_count()
        small, co, rs = _ns_gpu_t(u, ns_dtype)
        assert N.launch_count() - n0 == 1
        lib.thorn_set_ns_small(0)
        n0 = N.launch_count()
        gemms, _, _ = _ns_gpu_t(u, ns_dtype)
        assert N.launch_count() - n0 > 1
    finally:
        lib.thorn_set_ns_small(prev)
    a, b = small.float().cpu().numpy(), gemms.float().cpu().numpy()
    assert np.isfinite(a).all()
    rel = C.rel_fro(a, b)
    print(shape, ns_dtype, "bitwise equal" if np.array_equal(a, b) else f"rel {rel:.2e}")
    assert rel <= 1e-3, rel


@pytest.mark.parametrize("transpose", [False, True])
def test_ns_ill_conditioned_near_square(transpose):
    """The 66 x 64 momentum of the shard_uneven case: its normalised smallest singular value
    (9.6e-4) is below the Polar-Express lower bound (1e-3), so Newton-Schulz amplifies every
    rounding difference in that direction, and a product stored with a different rounding
    (e.g. a mirrored instead of computed element) moves the result by ~2e-2.  Both orientations
    (Gram NS on the tall input read transposed, and on the wide input) against the oracle."""
    case = C.CASES["shard_uneven"]
    g = C.build_grads(case, 0)[0][0].float()
    u = (g + 0.9 * g)[None]  # step 1: m = g, u = g + beta1 m
    if transpose:
        u = u.mT.contiguous()
    got, co, rs = _ns_gpu(u.cuda())
    O.NS_DTYPE = "f16"
    want = O.polar_decomp_2d(u[0].numpy(), co, rs, "f32")
    err = C.rel_fro(got[0], want)
    assert err <= 2e-2, err


@pytest.mark.parametrize("shape", [(1, 256, 256), (2, 512, 256)])
def test_ns_bf16_option(shape):
    """bf16 NS (optional mode): close to the bf16-operand oracle and a valid polar factor."""
    torch.manual_seed(3)
    u = torch.randn(shape) * 1e-3
    got, co, rs = _ns_gpu(u.cuda(), ns_dtype=torch.bfloat16)
    O.NS_DTYPE = "bf16"
    try:
        want = np.stack([O.polar_decomp_2d(x, co, rs, "f32") for x in u.numpy()])
    finally:
        O.NS_DTYPE = "f16"
    assert C.rel_fro(got, want) <= 6e-2
    s = np.linalg.svd(got[0].astype(np.float64), compute_uv=False)
    assert s.max() < 1.3


@pytest.mark.parametrize("M,K,batch,c_mode", [(128, 64, 1, None), (256, 1000, 3, "batched"),
                                              (384, 512, 2, "broadcast"), (1024, 4096, 1, "batched")])
def test_sym_addmm_against_torch(M, K, batch, c_mode):
    """thorn::sym_addmm contract (thorn.py:298-363) against a torch fp32 reference."""
    from thorn_b200 import _native as N

    lib = N.load()
    torch.manual_seed(1)
    A = (torch.randn(batch, M, K, device="cuda") / math.sqrt(K)).half()
    Bm = A.mT.contiguous()
    Cm = None
    if c_mode == "batched":
        Cm = torch.randn(batch, M, M, device="cuda").half()
        Cm = ((Cm + Cm.mT) / 2).half()
    elif c_mode == "broadcast":
        Cm = torch.randn(M, M, device="cuda")
        Cm = ((Cm + Cm.T) / 2).half()
    O_ = torch.empty(batch, M, M, dtype=torch.float16, device="cuda")
    alpha, beta = 0.75, -1.25
    N.check(lib.thorn_sym_addmm(A.data_ptr(), Bm.data_ptr(), None if Cm is None else Cm.data_ptr(), O_.data_ptr(),
                                batch, M, K, 1 if c_mode == "batched" else 0, alpha, beta, N.F16, None,
                                N.stream_of(torch.device("cuda"))), "sym_addmm")
    ref = alpha * (A.float() @ Bm.float())
    if Cm is not None:
        ref = ref + beta * Cm.float()
    got = O_.float()
    assert_block_symmetric(O_)
    tol = 2e-3 * ref.abs().max().item() + 1e-3
    assert (got - ref).abs().max().item() <= tol


def test_adamw_known_answer():
    """First Adam-atan2 step with wd=0 moves every element by exactly lr*pi/4 (fp32)."""
    from thorn_b200 import THORN

    p = torch.nn.Parameter(torch.zeros(10000, device="cuda"))
    opt = THORN([{"orthogonalize": False, "params": [p], "lr": 1e-3, "weight_decay": 0.0}])
    g = torch.randn(10000, device="cuda")
    g[g == 0] = 1.0
    p.grad = g.clone()
    opt.step()
    torch.cuda.synchronize()
    want = -torch.sign(g) * 1e-3 * math.pi / 4
    assert torch.allclose(p.detach(), want, rtol=1e-6, atol=0)


def test_gradient_release_matches_step():
    """setup_gradient_release (thorn.py:1755-1776) gives the same update as a full step."""
    from thorn_b200 import THORN

    torch.manual_seed(0)

    def model():
        torch.manual_seed(0)
        return torch.nn.Sequential(torch.nn.Linear(64, 128), torch.nn.GELU(), torch.nn.Linear(128, 32)).cuda()

    x = torch.randn(16, 64, device="cuda")
    m1, m2 = model(), model()
    o1 = THORN(m1, lr=1e-2)
    o2 = THORN(m2, lr=1e-2)
    o2.setup_gradient_release(m2)
    for _ in range(3):
        m1(x).square().mean().backward()
        o1.step()
        m2(x).square().mean().backward()
    torch.cuda.synchronize()
    for a, b in zip(m1.parameters(), m2.parameters()):
        assert torch.equal(a, b)  # deterministic kernels: bitwise equal


@pytest.mark.parametrize("block", [True, False])
def test_pinned_stepper_matches_step(block):
    """Steps fed from pinned host memory (PinnedStepper) give bitwise the parameters of the
    same steps on device gradients, with the host buffers as one ``pinned_block`` (one copy
    per direction) or as separate allocations (one copy per tensor)."""
    from thorn_b200 import THORN, PinnedStepper, pinned_block

    shapes = [(96, 64), (64, 37), (37,), (128, 128), (5,)]

    def params():
        torch.manual_seed(1)
        return [torch.nn.Parameter(torch.randn(s, device="cuda").to(torch.bfloat16)) for s in shapes]

    def opt(ps):
        return THORN([{"params": [p for p in ps if p.ndim == 2], "orthogonalize": True, "decouple_md": True,
                       "lr": 1e-2},
                      {"params": [p for p in ps if p.ndim == 1], "orthogonalize": False, "lr": 1e-3}])

    gen = torch.Generator().manual_seed(2)
    grads = [[torch.randn(s, generator=gen).to(torch.bfloat16) for s in shapes] for _ in range(4)]
    ref = params()
    o_ref = opt(ref)
    for gs in grads:
        for p, g in zip(ref, gs):
            p.grad = g.cuda()
        o_ref.step()
    ps = params()
    if block:
        hg, hp = pinned_block(shapes, torch.bfloat16), pinned_block(shapes, torch.bfloat16)
    else:
        hg = [torch.empty(s, dtype=torch.bfloat16, pin_memory=True) for s in shapes]
        hp = [torch.empty(s, dtype=torch.bfloat16, pin_memory=True) for s in shapes]
    st = PinnedStepper(opt(ps), ps, hg, hp)
    assert (st.grads_flat is not None) == block
    for gs in grads:
        st.wait_host_grads()
        for h, g in zip(hg, gs):
            h.copy_(g)
        st.step()
    st.synchronize()
    for a, h, p in zip(ref, hp, ps):
        assert torch.equal(a.detach().cpu(), h) and torch.equal(a, p)


def test_step_is_deterministic():
    """Reductions are done in a fixed order: two runs give bitwise-equal results."""
    _, a = run_gpu("md_small")
    _, b = run_gpu("md_small")
    for (pa, sa), (pb, sb) in zip(a.values(), b.values()):
        for ga, gb in zip(pa, pb):
            for x, y in zip(ga, gb):
                assert np.array_equal(x, y)


def test_state_dict_roundtrip():
    from thorn_b200 import THORN

    case = C.CASES["md_small"]

    def make():
        params = C.build_params(case)
        tp = [[torch.nn.Parameter(t.clone().cuda()) for t in ps] for ps in params]
        return tp, THORN(C.group_dicts(case, tp))

    def feed(tp, s):
        for ps, gs in zip(tp, C.build_grads(case, s)):
            for p, g in zip(ps, gs):
                p.grad = g.cuda()

    tp1, o1 = make()
    for s in range(2):
        feed(tp1, s)
        o1.step()
    sd = copy.deepcopy(o1.state_dict())  # what a checkpoint on disk holds
    st0 = sd["state"][0]
    assert set(st0) == {"step", "moment", "row_gain", "col_gain", "row_gain_moment", "row_gain_variance",
                        "col_gain_moment", "col_gain_variance", "target_norm"}
    tp2, o2 = make()
    with torch.no_grad():
        for a, b in zip(sum(tp1, []), sum(tp2, [])):
            b.copy_(a)
    o2.load_state_dict(sd)
    feed(tp1, 2)
    feed(tp2, 2)
    o1.step()
    o2.step()
    torch.cuda.synchronize()
    for a, b in zip(sum(tp1, []), sum(tp2, [])):
        assert torch.equal(a, b)


def test_launch_counter_and_no_fallback():
    """Every step goes through the library's kernels (the launch counter moves)."""
    from thorn_b200 import THORN, _native as N

    p = torch.nn.Parameter(torch.randn(256, 128, device="cuda") * 0.02)
    v = torch.nn.Parameter(torch.ones(128, device="cuda"))
    opt = THORN([{"orthogonalize": True, "params": [p], "lr": 1e-3}, {"orthogonalize": False, "params": [v], "lr": 1e-3}])
    before = N.launch_count()
    p.grad = torch.randn_like(p) * 1e-3
    v.grad = torch.randn_like(v) * 1e-3
    opt.step()
    torch.cuda.synchronize()
    assert N.launch_count() - before >= 5


@pytest.mark.parametrize("shape", [(1, 512, 512), (2, 1024, 512), (1, 512, 1024), (1, 300, 700), (3, 640, 384)])
def test_pair_tiles_match_single_cta(shape):
    """2-CTA (cta_group::2) 256x256 tiles and single-CTA tiles give the same NS result."""
    from thorn_b200 import _native as N

    lib = N.load()
    torch.manual_seed(11)
    u = (torch.randn(shape) * 1e-3).cuda()
    prev = lib.thorn_set_gemm_pair(1)
    try:
        pair, co, rs = _ns_gpu(u)
        lib.thorn_set_gemm_pair(0)
        single, _, _ = _ns_gpu(u)
    finally:
        lib.thorn_set_gemm_pair(prev)
    assert np.isfinite(pair).all()
    assert C.rel_fro(pair, single) <= 1e-3, C.rel_fro(pair, single)
    want = np.stack([O.polar_decomp_2d(x, co, rs, "f32") for x in u.cpu().numpy()])
    assert C.rel_fro(pair, want) <= 2e-2


@pytest.mark.parametrize("shape,dt", [((2, 512, 512), torch.float16), ((1, 1024, 512), torch.float16),
                                      ((2, 512, 1024), torch.float16), ((1, 300, 700), torch.float16),
                                      ((1, 520, 1000), torch.float16), ((2, 1000, 520), torch.float16),
                                      ((1, 768, 768), torch.bfloat16), ((1, 1536, 512), torch.bfloat16)])
def test_staged_epilogue_bitwise(shape, dt):
    """The shared-memory/TMA-store epilogue of the 2-CTA tiles writes exactly what the
    register epilogue writes (mirrored symmetric blocks, D + aI, C operand, transposed output)."""
    from thorn_b200 import _native as N

    lib = N.load()
    torch.manual_seed(12)
    u = (torch.randn(shape) * 1e-3).cuda()
    prev = lib.thorn_set_gemm_staged_epilogue(1)
    try:
        staged, co, rs = _ns_gpu(u, ns_dtype=dt)
        lib.thorn_set_gemm_staged_epilogue(0)
        plain, _, _ = _ns_gpu(u, ns_dtype=dt)
    finally:
        lib.thorn_set_gemm_staged_epilogue(prev)
    assert np.isfinite(staged).all()
    assert np.array_equal(staged, plain)


@pytest.mark.parametrize("batch,m,k,c_batched", [(3, 512, 264, 1), (2, 520, 128, 0), (1, 768, 1024, 1)])
def test_staged_epilogue_sym_addmm(batch, m, k, c_batched):
    """sym_addmm with a per-matrix or a broadcast C: staged and register epilogues agree
    bit for bit, and both match torch within fp16 rounding."""
    from thorn_b200 import _native as N

    lib = N.load()
    torch.manual_seed(13)
    a = (torch.randn(batch, m, k, device="cuda") / k ** 0.5).half()
    bt = a.transpose(1, 2).contiguous()
    c = torch.randn(batch if c_batched else 1, m, m, device="cuda")
    c = ((c + c.transpose(1, 2)) / 2).half()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = N.stream_of(torch.device("cuda"))

    def run():
        o = torch.empty(batch, m, m, dtype=torch.float16, device="cuda")
        N.check(lib.thorn_sym_addmm(a.data_ptr(), bt.data_ptr(), c.data_ptr(), o.data_ptr(), batch, m, k, c_batched,
                                    0.75, -0.5, N.F16, err.data_ptr(), st), "sym_addmm")
        torch.cuda.synchronize()
        return o

    prev = lib.thorn_set_gemm_staged_epilogue(1)
    try:
        staged = run()
        lib.thorn_set_gemm_staged_epilogue(0)
        plain = run()
    finally:
        lib.thorn_set_gemm_staged_epilogue(prev)
    assert int(err.item()) == 0
    assert torch.equal(staged, plain)
    assert_block_symmetric(staged)
    want = 0.75 * (a.float() @ bt.float()) - 0.5 * c.float().expand(batch, m, m)
    assert (staged.float() - want).abs().max().item() <= 2e-2 * want.abs().max().item()
