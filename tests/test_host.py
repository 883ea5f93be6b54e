"""Host-side behaviour of the drop-in THORN class (no GPU needed)."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

import parity as P
from thorn_b200 import THORN
from thorn_b200.coeffs import gram_ns_restarts, optimal_composition
from thorn_b200.optimizer import GroupConfig, _mat_view

# defaults of the reference's _THORNParameterGroup (thorn.py:541-561)
REF_DEFAULTS = dict(none_grad=True, weight_decay=0.1, betas=(0.9, 0.95), scaling_mode=None, target_rms=0.2,
                    target_norm=None, iters=5, rectify=False, eps=0, lower_bound=1e-3, safety_factor=0.03,
                    cushion=0.02, momentum_align=False, decouple_md=False, gain_lr=1e-3, gain_betas=(0.9, 0.95),
                    norm_axis=None, split_gain=True, force_per_neuron_norm=False)


def test_group_defaults_match_reference():
    opt = THORN([{"orthogonalize": True, "params": [nn.Parameter(torch.zeros(4, 4))], "lr": 1.0}])
    assert opt.defaults == REF_DEFAULTS
    g = opt.param_groups[0]
    assert set(g) == set(REF_DEFAULTS) | {"orthogonalize", "params", "lr"}


def test_coefficients_bit_identical_to_reference(golden_dir):
    gold = P.load_golden(os.path.join(golden_dir, "coeffs.npz"))
    i = 0
    while f"coeffs/{i}/setting" in gold:
        l, it, sf, cu = gold[f"coeffs/{i}/setting"]
        co = optimal_composition(float(l), int(it), float(sf), float(cu))
        assert np.array_equal(np.array(co), gold[f"coeffs/{i}/values"])
        assert gram_ns_restarts(*co) == list(gold[f"coeffs/{i}/restarts"])
        i += 1


def test_validation_errors():
    with pytest.raises(ValueError, match="Invalid learning rate"):
        GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=-1.0)
    with pytest.raises(ValueError, match="Invalid beta1"):
        GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0, betas=(1.0, 0.9))
    with pytest.raises(ValueError, match="Invalid beta2"):
        GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0, betas=(0.9, -0.1))
    with pytest.raises(AssertionError, match="ndim >= 2"):
        THORN([{"orthogonalize": True, "params": [nn.Parameter(torch.zeros(4))], "lr": 1.0}])
    # the reference accepts bad hyper-parameters at construction and raises on step
    p = nn.Parameter(torch.zeros(4, 4))
    opt = THORN([{"orthogonalize": True, "params": [p], "lr": -1.0}])
    p.grad = torch.zeros(4, 4)
    with pytest.raises(ValueError):
        opt.step()


def test_scaling_modes_and_rect():
    g = GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0)
    assert g.scaling_mode_ == "moonlight"
    assert abs(g.lr_scale(512, 512) - 0.2 * 512 ** 0.5) < 1e-12
    g = GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0, decouple_md=True)
    assert g.scaling_mode_ == "md" and g.lr_scale(1024, 512) == 2 ** 0.5
    g = GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0, scaling_mode="jordan")
    assert g.lr_scale(512, 1024) == 1.0 and g.lr_scale(1024, 256) == 2.0
    g = GroupConfig.from_kwargs(orthogonalize=False, params=[], lr=1.0, rectify=True)
    assert g.rect(1) == 0.0 and 0 < g.rect(20) < 1
    assert GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0).needs_pnn(1024, 512)
    assert not GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0).needs_pnn(512, 1024)
    assert not GroupConfig.from_kwargs(orthogonalize=True, params=[], lr=1.0, betas=(0.9, 0.0)).needs_pnn(1024, 512)


def test_auto_assign_mirrors_reference():
    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(10, 8)
            self.proj = nn.Linear(8, 8)
            self.conv = nn.Conv1d(8, 8, 3)
            self.norm = nn.LayerNorm(8)
            self.lm_head = nn.Linear(8, 10, bias=False)

    m = M()
    opt = THORN(m, lr=1e-3)
    ortho = {id(p) for p in opt.param_groups[0]["params"]}
    assert ortho == {id(m.proj.weight), id(m.conv.weight)}
    assert opt.param_groups[0]["orthogonalize"] and not opt.param_groups[1]["orthogonalize"]


def test_state_layout_and_no_cpu_path():
    p = nn.Parameter(torch.randn(6, 4))
    q = nn.Parameter(torch.randn(5))
    opt = THORN([{"orthogonalize": True, "params": [p], "lr": 1e-3, "decouple_md": True},
                 {"orthogonalize": False, "params": [q], "lr": 1e-3, "decouple_md": True}])
    g0 = GroupConfig.from_kwargs(**opt.param_groups[0])
    g1 = GroupConfig.from_kwargs(**opt.param_groups[1])
    opt._init_state(p, opt.state[p], g0, opt.param_groups[0])
    opt._init_state(q, opt.state[q], g1, opt.param_groups[1])
    sp, sq = opt.state[p], opt.state[q]
    assert sp["step"] == 1 and sp["moment"].shape == p.shape
    assert sp["row_gain"].shape == (6, 1) and sp["col_gain"].shape == (1, 4)
    assert abs(float(torch.nn.functional.softplus(sp["row_gain"][0, 0])) - 1.0) < 1e-6
    assert float(sp["target_norm"]) == pytest.approx(6 ** 0.5)
    assert set(sq) == {"step", "moment", "variance", "gain", "gain_moment", "gain_variance", "target_norm"}
    assert float(sq["target_norm"]) == pytest.approx(float(q.norm()))
    # the step runs only on CUDA devices: no CPU fallback
    p.grad = torch.zeros_like(p)
    with pytest.raises(RuntimeError, match="CUDA"):
        opt.step()


def test_state_dtype_extension():
    p = nn.Parameter(torch.randn(8, 8, dtype=torch.bfloat16))
    opt = THORN([{"orthogonalize": True, "params": [p], "lr": 1e-3, "state_dtype": torch.float32}])
    g = GroupConfig.from_kwargs(**opt.param_groups[0])
    opt._init_state(p, opt.state[p], g, opt.param_groups[0])
    assert opt.state[p]["moment"].dtype == torch.float32


def test_mat_view():
    assert _mat_view((8, 4, 3)) == (8, 4, 3)
    assert _mat_view((2, 3, 4, 5)) == (6, 4, 5)
    assert _mat_view((7,)) == (1, 1, 7)


def test_pinned_stepper_checks_buffers():
    """PinnedStepper rejects host buffers of the wrong shape, dtype or memory kind before
    touching a device."""
    from thorn_b200 import PinnedStepper

    p = torch.nn.Parameter(torch.zeros(4, 3))
    with pytest.raises(ValueError, match="same length"):
        PinnedStepper(None, [p], [], [])
    with pytest.raises(ValueError, match="local shape"):
        PinnedStepper(None, [p], [torch.zeros(3, 4)], [torch.zeros(4, 3)])
    with pytest.raises(ValueError, match="pinned"):
        PinnedStepper(None, [p], [torch.zeros(4, 3)], [torch.zeros(4, 3)])


def test_magma_generator_matches_oracle():
    """The product's restatement of the reference's generator step (thorn.py:800-804)
    equals the oracle's, which reproduces the reference's own generator states."""
    from oracle import thorn_oracle as O
    from thorn_b200.optimizer import _w1rand

    rng = np.random.default_rng(5)
    for s in [0, 1, (1 << 64) - 1, O.W1_C, *map(int, rng.integers(0, 1 << 63, 50))]:
        assert _w1rand(s) == O.w1rand(s)


def test_magma_scores_keep_the_reference_dtype_rules():
    """THORN._magma_scores forms the smoothed scores of many parameters with a few vectorised
    ops; each must equal the reference's own 0-d tensor ops for that parameter alone
    (thorn.py:818-833): the cosine in the promoted dtype of gradient and moment, and
    s = 0.9 s + 0.1 sigmoid(cos / 2) with torch's promotion (so a bf16 score next to an
    fp32 cosine becomes fp32).  Mixed dtypes in one call, zero sums (an empty tensor)."""
    from thorn_b200.optimizer import MAGMA_EMA, MAGMA_TAU, _Item

    torch.manual_seed(5)
    combos = [(torch.float32, torch.float32, torch.float32), (torch.bfloat16, torch.float32, torch.bfloat16),
              (torch.bfloat16, torch.bfloat16, torch.bfloat16), (torch.float16, torch.float32, torch.float16),
              (torch.float32, torch.float32, torch.float32), (torch.bfloat16, torch.float32, torch.float32)]
    items, want = [], []
    for gdt, mdt, sdt in combos:
        it = _Item()
        it.g = torch.zeros(3, 4, dtype=gdt)
        it.state = {"moment": torch.zeros(3, 4, dtype=mdt), "s": torch.rand((), dtype=torch.float32).to(sdt)}
        items.append(it)
    stats = torch.rand(len(items), 3, dtype=torch.float64) * 1e-4
    stats[:, 0] -= 0.5e-4  # negative and positive cross sums
    stats[4] = 0.0  # no elements: the cosine is 0
    for j, it in enumerate(items):
        dot, gg, mm = stats[j]
        cos = (dot / (gg.sqrt().clamp_min(1e-8) * mm.sqrt().clamp_min(1e-8))).float()
        c = cos.to(torch.promote_types(it.g.dtype, it.state["moment"].dtype))
        want.append(MAGMA_EMA * it.state["s"] + (1 - MAGMA_EMA) * torch.sigmoid(c / MAGMA_TAU))
    got = THORN._magma_scores(items, stats)
    for it, w, v in zip(items, want, got):
        s_new = it.state["s"]
        assert s_new.dtype == w.dtype and s_new.ndim == 0
        assert float(s_new) == pytest.approx(float(w), rel=2 * torch.finfo(w.dtype).eps)
        assert v == float(s_new)
    assert items[1].state["s"].dtype == torch.float32 and items[2].state["s"].dtype == torch.bfloat16


@pytest.mark.parametrize("decouple_md", [False, True])
def test_magma_scores_and_masks_match_oracle(decouple_md, monkeypatch):
    """THORN._magma (the score, mask and state glue around the statistics kernel) on CPU
    tensors against the oracle's masking: same masked steps, same smoothed score, over
    several steps.  The three sums come from a CPU stand-in of the kernel."""
    from oracle import thorn_oracle as O
    from thorn_b200.optimizer import _Item

    torch.manual_seed(3)
    p = nn.Parameter(torch.randn(12, 8) * 0.1)
    opt = THORN([{"orthogonalize": True, "params": [p], "lr": 1e-3, "momentum_align": True,
                  "decouple_md": decouple_md}])
    monkeypatch.setattr(opt, "_magma_stats", P.magma_stats_cpu)
    cfg = GroupConfig.from_kwargs(**opt.param_groups[0])
    p.grad = torch.randn_like(p)
    st = opt.state[p]
    opt._init_state(p, st, cfg, opt.param_groups[0])
    ost = {"random_state": st["random_state"], "s": np.float32(1.0)}
    if decouple_md:  # non-trivial gains so the recovered gradient differs from the raw one
        st["row_gain"] = st["row_gain"] + torch.linspace(-0.5, 0.5, 12).reshape(12, 1)
        st["col_gain"] = st["col_gain"] + torch.linspace(0.3, -0.3, 8).reshape(1, 8)
    masked = 0
    for k in range(12):
        g = torch.randn(12, 8) * 1e-3
        st["moment"] = torch.randn(12, 8) * 1e-3 if k else torch.zeros(12, 8)
        it = _Item()
        it.g, it.state, it.split, it.apply = g, st, "row_gain" in st, True
        opt._magma([it], cfg, recovered=True)
        gd = g.numpy()
        if decouple_md:
            sp = lambda x: np.log1p(np.exp(x.numpy().astype(np.float64))).astype(np.float32)
            gd = (gd * (sp(st["row_gain"]) * sp(st["col_gain"]))).astype(np.float32)
        want = O.magma_scale(gd, st["moment"].numpy(), ost, "f32")
        assert st["random_state"] == ost["random_state"]
        assert float(st["s"]) == pytest.approx(float(ost["s"]), rel=1e-6)
        assert it.scale == pytest.approx(want, rel=1e-6)
        assert it.apply == (want != 0.0)
        masked += want == 0.0
    assert 0 < masked < 12


def test_sparse_row_gather_and_scatter():
    """The row bookkeeping around the AdamW kernel for row-sparse gradients: duplicate rows
    are summed (coalesce), only touched rows are gathered and written back, and a gradient
    without rows is left out (the reference keeps its step count)."""
    e = nn.Parameter(torch.randn(10, 3))
    f = nn.Parameter(torch.randn(6, 2))
    opt = THORN([{"orthogonalize": False, "params": [e, f], "lr": 1e-3}])
    cfg = GroupConfig.from_kwargs(**opt.param_groups[0])
    e.grad = torch.sparse_coo_tensor(torch.tensor([[7, 2, 7]]), torch.tensor([[1., 1, 1], [2, 2, 2], [3, 3, 3]]),
                                     (10, 3))
    f.grad = torch.sparse_coo_tensor(torch.zeros((1, 0), dtype=torch.long), torch.zeros((0, 2)), (6, 2))
    for p in (e, f):
        opt._init_state(p, opt.state[p], cfg, opt.param_groups[0])
    recs = opt._sparse_rows([e, f], cfg)
    assert len(recs) == 1
    p, idx, it = recs[0]
    assert p is e and idx.tolist() == [2, 7]
    assert torch.equal(it.g, torch.tensor([[2., 2, 2], [4, 4, 4]]))
    before = e.detach().clone()
    it.m_rows += 1.0
    it.v_rows += 2.0
    it.p += 3.0
    opt._scatter_rows(recs)
    st = opt.state[e]
    assert torch.equal(st["moment"][[2, 7]], torch.ones(2, 3)) and st["moment"][[0, 1, 3]].abs().sum() == 0
    assert torch.equal(st["variance"][[2, 7]], torch.full((2, 3), 2.0))
    assert torch.equal(e.detach()[[2, 7]], before[[2, 7]] + 3.0)
    assert torch.equal(e.detach()[[0, 1, 3, 4, 5, 6, 8, 9]], before[[0, 1, 3, 4, 5, 6, 8, 9]])


def test_custom_ops_registered_with_fake_impls():
    """torch.ops.thorn_b200.sym_addmm / polar_decomp exist and trace on meta tensors
    (shape and dtype from their fake implementations, no device work)."""
    import thorn_b200  # noqa: F401

    A = torch.empty(3, 64, 32, device="meta", dtype=torch.float16)
    B = torch.empty(3, 32, 64, device="meta", dtype=torch.float16)
    C = torch.empty(64, 64, device="meta", dtype=torch.float16)
    out = torch.ops.thorn_b200.sym_addmm(A, B, C, 1.0, 0.5)
    assert out.shape == (3, 64, 64) and out.dtype == torch.float16 and out.device.type == "meta"
    X = torch.empty(2, 5, 96, 40, device="meta", dtype=torch.bfloat16)
    U = torch.ops.thorn_b200.polar_decomp(X, [1.0, 0.0, 0.0], [])
    assert U.shape == X.shape and U.dtype == torch.bfloat16
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.thorn_b200.sym_addmm(torch.zeros(64, 32, dtype=torch.float16),
                                       torch.zeros(32, 64, dtype=torch.float16), None, 1.0, 0.0)
    # the reference's own operator name (thorn.py:298) is registered too, with the same schema
    out = torch.ops.thorn.sym_addmm(A, B, None, 1.0, 0.0)
    assert out.shape == (3, 64, 64) and out.device.type == "meta"
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.thorn.sym_addmm(torch.zeros(64, 32, dtype=torch.float16),
                                  torch.zeros(32, 64, dtype=torch.float16), None, 1.0, 0.0)


@pytest.mark.parametrize("block", [False, True])
def test_pinned_stepper_data_flow_with_fake_streams(monkeypatch, block):
    """Every line of PinnedStepper on CPU tensors, with CUDA streams and events replaced by
    recording fakes: each step sees that step's host gradients, and after synchronize the
    host parameter buffers hold the parameters of the last step.  ``block``: the host
    buffers are views of one allocation laid out like ``pinned_block``'s, so each direction
    is one copy of the whole block."""
    import contextlib

    import thorn_b200.host_stepper as HS

    log = []

    class FakeEvent:
        def record(self, stream=None):
            log.append(("record", id(self)))

        def synchronize(self):
            log.append(("event_sync", id(self)))

    class FakeStream:
        def wait_event(self, ev):
            log.append(("wait", id(ev)))

        def wait_stream(self, s):
            pass

        def synchronize(self):
            log.append(("sync",))

    compute = FakeStream()
    monkeypatch.setattr(HS.torch.cuda, "Stream", lambda dev=None: FakeStream())
    monkeypatch.setattr(HS.torch.cuda, "Event", lambda *a, **k: FakeEvent())
    monkeypatch.setattr(HS.torch.cuda, "current_stream", lambda dev=None: compute)
    monkeypatch.setattr(HS.torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(torch.Tensor, "is_pinned", lambda self: True)

    params = [nn.Parameter(torch.zeros(3, 2)), nn.Parameter(torch.zeros(5))]

    class AddGrad:  # stands in for THORN: p -= grad, grad consumed
        def __init__(self):
            self.seen = []

        def step(self):
            self.seen.append([p.grad.clone() for p in params])
            for p in params:
                p.data -= p.grad
                p.grad = None

    opt = AddGrad()
    if block:
        offs, n = HS._block_layout([(3, 2), (5,)], torch.float32)
        assert offs == [0, 64] and n == 128  # views start 256 bytes apart
        fg, fp = torch.zeros(n), torch.zeros(n)
        hg = [fg[0:6].view(3, 2), fg[64:69]]
        hp = [fp[0:6].view(3, 2), fp[64:69]]
    else:
        hg = [torch.zeros(3, 2), torch.zeros(5)]
        hp = [torch.zeros(3, 2), torch.zeros(5)]
    st = HS.PinnedStepper(opt, params, hg, hp)
    assert (st.grads_flat is not None) == block and (st.snapshot_flat is not None) == block
    if block:  # the device views mirror the host block's layout
        assert st.h_grads_flat.numel() == 69 and st.grads[0][1].data_ptr() == st.grads_flat[0][64:].data_ptr()
    for k in range(4):
        st.wait_host_grads()  # the previous step's gradient copy has read the host buffers
        for h in hg:
            h.fill_(k + 1.0)
        st.step()
    st.synchronize()
    assert [float(g[0].flatten()[0]) for g in opt.seen] == [1.0, 2.0, 3.0, 4.0]
    # wait_host_grads blocks on the event of the slot the last step loaded (none before step 1)
    assert [e[1] for e in log if e[0] == "event_sync"] == [id(st.loaded[0]), id(st.loaded[1]), id(st.loaded[0])]
    assert torch.equal(hp[0], torch.full((3, 2), -10.0)) and torch.equal(hp[1], torch.full((5,), -10.0))
    assert ("sync",) in log and any(e[0] == "wait" for e in log)


class _StubLib:
    """Entry points of the C ABI that succeed without doing anything (host-logic tests only)."""

    def thorn_ns_ld(self, n):
        return (n + 7) // 8 * 8

    def __getattr__(self, name):
        if name.endswith("_bytes"):
            return lambda *a: 256
        return lambda *a: 0


@pytest.mark.parametrize("magma", [False, True])
def test_local_paths_run_through_stub_library(monkeypatch, magma):
    """The Python control flow of the single-device paths (orthogonalized with and without MD,
    (R)AdamW dense and row-sparse, Magma on and off) runs end to end against a stub library:
    every launch record gets built and every entry point is called with an int status."""
    from thorn_b200 import _native as N

    monkeypatch.setattr(N, "load", lambda build_if_missing=False: _StubLib())
    monkeypatch.setattr(N, "stream_of", lambda dev: 0)

    class _Ev:  # the profiling hooks' events
        def __init__(self, **kw):
            pass

        def record(self, *a):
            pass

    monkeypatch.setattr(torch.cuda, "Event", _Ev)
    torch.manual_seed(0)
    w = nn.Parameter(torch.randn(24, 16) * 0.02)
    t = nn.Parameter(torch.randn(32, 16) * 0.02)
    v = nn.Parameter(torch.randn(16))
    e = nn.Parameter(torch.randn(10, 4))
    opt = THORN([{"orthogonalize": True, "params": [w], "lr": 1e-3, "momentum_align": magma},
                 {"orthogonalize": True, "params": [t], "lr": 1e-3, "decouple_md": True, "momentum_align": magma},
                 {"orthogonalize": False, "params": [v, e], "lr": 1e-3, "momentum_align": magma}])
    opt.profile_momentum = []
    for step in range(3):
        for p in (w, t, v):
            p.grad = torch.randn_like(p) * 1e-3
        e.grad = torch.sparse_coo_tensor(torch.tensor([[1, 4, 4]]), torch.randn(3, 4), (10, 4))
        for gi, grp in enumerate(opt.param_groups):
            cfg = GroupConfig.from_kwargs(**grp)
            ps = [p for p in grp["params"] if p.grad is not None]
            for p in ps:
                if "step" not in opt.state[p]:
                    opt._init_state(p, opt.state[p], cfg, grp)
            if cfg.orthogonalize:
                opt._ortho_local(ps, cfg)
            else:
                opt._adam_local(ps, cfg)
    # momentum-pass profile: one record per orthogonalized group and step, compulsory bytes
    # g + 2 m (+ 2 p under MD), all fp32 here
    assert [nb for _, _, nb in opt.profile_momentum] == [24 * 16 * 12, 32 * 16 * 20] * 3
    for p in (w, t, v, e):
        assert opt.state[p]["step"] == 4 and p.grad is None
        if magma:
            assert "random_state" in opt.state[p] and opt.state[p]["s"].ndim == 0


@pytest.mark.parametrize("name", ["tiny_small", "md_small", "bf16_small", "conv_small", "variants_small", "vad",
                                  "tiny", "edge_small", "magma_small", "sparse_small", "shard_uneven",
                                  "magma_shard", "md_axis_small", "rate_small", "md_options_small",
                                  "md_conv_small", "md_target_fn_small"])
def test_state_keys_and_shapes_match_reference_goldens(name, golden_dir):
    """Checkpoint compatibility: the state THORN initialises for every parameter of a case has
    exactly the keys, and the shapes, of the reference's own state after its first step (as the
    golden fixtures recorded it, thorn.py:1591-1633)."""
    import cases as C

    gold = P.load_golden(os.path.join(golden_dir, f"{name}.npz"))
    case = C.CASES[name]
    params = [[nn.Parameter(t.clone()) for t in ps] for ps in C.build_params(case)]
    opt = THORN(C.group_dicts(case, params))
    for gi, (grp, ps, gs) in enumerate(zip(opt.param_groups, params, C.build_grads(case, 0))):
        cfg = GroupConfig.from_kwargs(**grp)
        for pi, (p, g) in enumerate(zip(ps, gs)):
            p.grad = g
            opt._init_state(p, opt.state[p], cfg, grp)
            base = f"step1/g{gi}/p{pi}/"
            want = {k[len(base):].split("/")[0] for k in gold if k.startswith(base)} - {"param", "grad_after"}
            st = opt.state[p]
            assert set(st) == want, (gi, pi, sorted(set(st) ^ want))
            for k, v in st.items():
                if isinstance(v, torch.Tensor):
                    assert tuple(v.shape) == tuple(gold[f"{base}{k}/shape"]), (gi, pi, k)


@pytest.mark.parametrize("shape", [(2, 48, 48), (2, 40, 130)])
def test_ns_recurrences_equal_composed_polynomial(shape):
    """The Newton-Schulz recurrences that thorn_ns_batched runs (restated on torch GEMMs as
    bench.py's library baseline): square quintic and Gram NS with its restart, in float64,
    equal the composed Polar-Express polynomial applied to the singular values
    (thorn.py:626-662)."""
    from bench import ns_library

    co = optimal_composition(1e-3, 5, 0.03, 0.02)
    rs = gram_ns_restarts(*co)
    torch.manual_seed(1)
    X = torch.randn(*shape, dtype=torch.float64)
    X = X / X.norm(dim=(-2, -1), keepdim=True)
    u, s, vh = torch.linalg.svd(X, full_matrices=False)
    for a, b, c in co:
        s = a * s + b * s ** 3 + c * s ** 5
    want = u @ torch.diag_embed(s) @ vh
    got = ns_library(X, co, rs)
    assert float((got - want).norm() / want.norm()) < 1e-12


def test_bench_line_carries_the_contract_keys():
    """bench.py's JSON line (built by ``result_line`` from a run's measurements): every key the
    bench contract asks for, the whole-job roofline arithmetic, and the end-to-end object."""
    import argparse
    import json

    import bench

    args = argparse.Namespace(steps=5, warmup=3, layers=bench.LAYERS)
    e2e = {"value": 400.0, "unit": "ms", "h2d_bytes_per_step": 16 << 30, "d2h_bytes_per_step": 16 << 30,
           "mode": "pipelined"}
    cpu = {"value": 1.4e6, "unit": "ms", "cores": 16, "kind": "port", "sample": "s"}
    clocks = {"sm_mhz": 1400.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    line = bench.result_line(args, 2, 200.0, 150.0, 505.5e12, 321.5e12, 10.0, 49e9, cpu, e2e, 9.0, 18.0, 3485,
                             clocks)
    json.dumps(line)  # serialisable
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "roofline", "cpu_baseline", "e2e", "gpu_launches", "clocks"):
        assert k in line, k
    assert line["higher_is_better"] is False and line["n_gpus"] == 2 and line["value"] == 200.0
    assert "workload" in line["config"] and "model" not in line["config"]
    r = line["roofline"]
    for k in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert k in r, k
    _, _, peak_sus, _ = bench.load_peaks()
    assert r["peak"] == pytest.approx(2 * peak_sus, abs=0.1)  # whole-job peak at 2 GPUs
    assert r["achieved"] == pytest.approx(505.5e12 / 0.150 / 1e12, rel=1e-3)
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"], abs=1e-3)
    el = line["roofline_elementwise"]
    assert el["achieved"] == pytest.approx(49e9 / 0.010 / 1e9, rel=1e-3)
    assert set(line["e2e"]) >= {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"}
    assert line["gpu_launches"] == 3485 and line["cpu_baseline"]["kind"] == "port"


def test_bench_reference_arm_line(monkeypatch, capsys):
    """bench.py --impl reference: rank 0 prints one line with impl, cpu_baseline and an e2e of
    the line's own value with no host-device bytes; other ranks print nothing."""
    import argparse
    import json

    import bench

    # the reference installed under baseline/_ref: its own CPU step is the baseline
    monkeypatch.setattr(bench, "import_reference", lambda: object())
    monkeypatch.setattr(bench, "cpu_reference_sample",
                        lambda warm_only=False: None if warm_only else (1234.5, "s", 2.0, 8))
    args = argparse.Namespace(steps=2, warmup=1, gpus=1, model="llama8b")
    bench.reference_arm(args, 1)
    assert capsys.readouterr().out == ""
    bench.reference_arm(args, 0)
    line = json.loads(capsys.readouterr().out.strip())
    assert line["impl"] == "reference" and line["value"] == 1234.5 and line["higher_is_better"] is False
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] == 8
    # without the install: the numpy port
    monkeypatch.setattr(bench, "import_reference", lambda: None)
    monkeypatch.setattr(bench, "cpu_reference_sample", lambda warm_only=False: None)
    monkeypatch.setattr(bench, "cpu_oracle_sample", lambda warm_only=False: None if warm_only else (1234.5, "s", 2.0))
    bench.reference_arm(args, 0)
    line = json.loads(capsys.readouterr().out.strip())
    assert line["impl"] == "reference" and line["value"] == 1234.5 and line["higher_is_better"] is False
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == 1234.5
    assert line["e2e"] == {"value": 1234.5, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the same workload description as the GPU arm's line
    args.layers = None
    assert line["config"] == bench.bench_config(args, 1)


def test_bench_reference_gpu_arm_unavailable_without_install(monkeypatch, capsys):
    """bench.py --impl reference_gpu without the reference installed under baseline/_ref:
    rank 0 prints one line that says so and nothing runs; other ranks print nothing."""
    import argparse
    import json

    import bench

    monkeypatch.setattr(bench, "import_reference", lambda: None)
    args = argparse.Namespace(steps=2, warmup=1, gpus=1, model="llama8b", layers=None)
    bench.reference_gpu_arm(args, 1)
    assert capsys.readouterr().out == ""
    bench.reference_gpu_arm(args, 0)
    line = json.loads(capsys.readouterr().out.strip())
    assert line["impl"] == "reference_gpu" and "unavailable" in line


def test_sharded_exchange_defaults_to_all_to_all():
    """The sharded path's exchange default is one all_to_all_single per exchange (the
    faster form on 8 GPUs); the pairwise rounds stay selectable."""
    from thorn_b200 import THORN

    assert THORN.exchange == "all_to_all"
    assert THORN.pipeline_exchange is False


def test_block_of_accepts_only_ordered_views_of_one_storage():
    """The one-copy path of PinnedStepper needs the host tensors in parameter order inside one
    allocation; anything else keeps the per-tensor copies."""
    from thorn_b200.host_stepper import _block_of

    f = torch.zeros(256)
    flat, offs = _block_of([f[0:6].view(2, 3), f[64:69], f[128:128]])
    assert offs == [0, 64, 128] and flat.numel() == 128 and flat.data_ptr() == f.data_ptr()
    flat, offs = _block_of([f[8:16], f[16:20]])  # a block need not start at the storage's start
    assert offs == [0, 8] and flat.numel() == 12 and flat.data_ptr() == f[8:].data_ptr()
    assert _block_of([f[64:69], f[0:6]]) is None  # out of order
    assert _block_of([f[0:8], f[4:12]]) is None  # overlapping
    assert _block_of([f[0:8], torch.zeros(8)]) is None  # two allocations
    assert _block_of([f[0:8], f[8:16].to(torch.float64)]) is None  # two dtypes
    assert _block_of([f[0:16].view(4, 4).t()]) is None  # not contiguous
    assert _block_of([]) is None
