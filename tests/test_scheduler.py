"""The TorchDispatch scheduler (gpuos_b200.scheduler), the mirror of the
reference's pytorch_ext/scheduler.py.

CPU tests cover the dispatch tables; GPU tests run torch code inside
``scheduler_context`` and compare every scheduled result with the oracle
(the reference's formulas), including the chains whose results the reference
never writes to the returned tensor.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import gpuos_b200.scheduler as S

DEV = "cuda:0"


def test_dispatch_tables():
    assert S._scheduled_names(False) == {"aten::add.Tensor", "aten::sub.Tensor",
                                         "aten::mul.Tensor", "aten::div.Tensor"}
    jit = S._scheduled_names(True)
    for n in ("aten::maximum", "aten::pow.Tensor_Tensor", "aten::gelu", "aten::softplus",
              "aten::sum.dim_IntList", "aten::mean.dim"):
        assert n in jit
    assert S._param_expr("aten::hardtanh", (None, -0.5, 0.5), {}) == (
        "hardtanh|f32|-0.50000000|0.50000000", "fminf(fmaxf(A, -0.50000000f), 0.50000000f)")
    assert S._param_expr("aten::clamp", (None, -1.0, 1.0), {}) is None  # positional: torch


def test_expressions_are_precompiled():
    """Every expression the scheduler registers maps to a precompiled operator."""
    import gpuos_b200.cabi as C
    exprs = list(S._BINARY_EXPR.values()) + list(S._UNARY_EXPR.values())
    for name in S._PARAM_UNARY:
        ke = S._param_expr(name, (None, 0.25, 0.75), {"min": 0.25, "max": 0.75})
        exprs.append(ke[1])
    for e in exprs:
        arity = 2 if "B" in e else 1
        v, _, _ = C.match_expression(e, arity)
        assert v >= 0, e


def _exact(a, b, op, p0=0.0, p1=0.0):
    ref = torch.empty(a.shape, dtype=torch.float32)
    oracle.ew(op, a, b, ref, p0, p1)
    return ref


@pytest.mark.gpu
def test_default_mode_schedules_the_four_builtins(monkeypatch):
    from test_gpu_parity import compare
    monkeypatch.delenv("GPUOS_SCHEDULER_DISABLE_JIT", raising=False)
    g = torch.Generator().manual_seed(51)
    a = torch.randn(3000, generator=g)
    b = torch.randn(3000, generator=g)
    b = torch.sign(b) * (b.abs() + 0.1)
    ga, gb = a.to(DEV), b.to(DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None):
        c = ga + gb
        d = c * gb
        e = d - ga
        f = e / gb
        r = torch.relu(f)  # not scheduled in this mode: flushes first (reads f)
    C0 = _exact(a, b, "add")
    D0 = _exact(C0, b, "mul")
    E0 = _exact(D0, a, "sub")
    F0 = _exact(E0, b, "div0")
    for got, want in ((c, C0), (d, D0), (e, E0), (f, F0)):
        assert torch.equal(got.cpu(), want)
    assert torch.equal(r.cpu(), torch.relu(F0))
    compare("add", a, b, c.cpu())


@pytest.mark.gpu
def test_jit_mode_every_operator(monkeypatch):
    from test_gpu_parity import compare
    monkeypatch.setenv("GPUOS_SCHEDULER_DISABLE_JIT", "0")
    g = torch.Generator().manual_seed(52)
    x = torch.randn(2501, generator=g)
    y = torch.randn(2501, generator=g)
    xp = x.abs() + 1e-3
    yp = torch.rand(2501, generator=g) * 1.5 + 0.5
    gx, gy, gxp, gyp = (t.to(DEV) for t in (x, y, xp, yp))
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None):
        got = {
            "maximum": torch.maximum(gx, gy), "minimum": torch.minimum(gx, gy),
            "pow": torch.pow(gxp, gyp), "div": gx / (gy.abs() + 0.1),
            "relu": torch.relu(gx), "sigmoid": torch.sigmoid(gx), "tanh": torch.tanh(gx),
            "exp": torch.exp(gx), "log": torch.log(gxp), "sqrt": torch.sqrt(gxp),
            "abs": torch.abs(gx), "hardsigmoid": F.hardsigmoid(gx),
            "hardswish": F.hardswish(gx), "gelu": F.gelu(gx), "sin": torch.sin(gx),
            "cos": torch.cos(gx), "leaky_relu": F.leaky_relu(gx, 0.02),
            "hardtanh": F.hardtanh(gx, -0.5, 0.5), "elu": F.elu(gx, 0.7),
            "softplus": F.softplus(gx, 2.0), "clamp_min": torch.clamp_min(gx, -0.25),
            "clamp_max": torch.clamp_max(gx, 0.25),
        }
    cpu = {k: v.cpu() for k, v in got.items()}
    yd = y.abs() + 0.1
    compare("maximum", x, y, cpu["maximum"])
    compare("minimum", x, y, cpu["minimum"])
    compare("pow", xp, yp, cpu["pow"])
    compare("div", x, yd, cpu["div"])
    for op in ("relu", "sigmoid", "tanh", "exp", "abs", "hardsigmoid", "hardswish", "gelu",
               "sin", "cos"):
        compare(op, x, None, cpu[op])
    compare("log", xp, None, cpu["log"])
    compare("sqrt", xp, None, cpu["sqrt"])
    compare("leaky_relu", x, None, cpu["leaky_relu"], 0.02)
    compare("clamp", x, None, cpu["hardtanh"], -0.5, 0.5)
    compare("elu", x, None, cpu["elu"], 0.7)
    compare("softplus", x, None, cpu["softplus"], 2.0)
    compare("clamp_min", x, None, cpu["clamp_min"], -0.25)
    compare("clamp_max", x, None, cpu["clamp_max"], 0.25)


@pytest.mark.gpu
def test_jit_chains_write_the_returned_tensors(monkeypatch):
    """sigmoid(a * b) + c: every intermediate and the result land in the
    tensors torch code holds (the reference loses them)."""
    from test_gpu_parity import compare
    monkeypatch.setenv("GPUOS_SCHEDULER_DISABLE_JIT", "0")
    g = torch.Generator().manual_seed(53)
    a, b, c = (torch.randn(4000, generator=g) for _ in range(3))
    ga, gb, gc = a.to(DEV), b.to(DEV), c.to(DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None):
        m = ga * gb
        s = torch.sigmoid(m)
        r = s + gc
        z = r.sum()  # not scheduled (no dim): a synchronous flush runs first
    M = _exact(a, b, "mul")
    assert torch.equal(m.cpu(), M)
    compare("sigmoid", M, None, s.cpu())
    assert torch.equal(r.cpu(), _exact(s.cpu(), c, "add"))
    assert abs(float(z) - float(r.cpu().double().sum())) <= 1e-4 * float(r.cpu().abs().sum())


@pytest.mark.gpu
def test_jit_reductions(monkeypatch):
    monkeypatch.setenv("GPUOS_SCHEDULER_DISABLE_JIT", "0")
    g = torch.Generator().manual_seed(54)
    x = torch.randn(37, 411, generator=g)
    gx = x.to(DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None):
        s1 = gx.sum(dim=1)
        s0 = gx.sum(dim=0, keepdim=True)
        m1 = gx.mean(dim=-1, keepdim=True)
    for got, want in ((s1, x.double().sum(1)), (s0, x.double().sum(0, keepdim=True)),
                      (m1, x.double().mean(-1, keepdim=True))):
        assert got.shape == want.shape
        mag = x.abs().double().sum()
        assert float((got.cpu().double() - want).abs().max()) <= 1e-5 * float(mag)


@pytest.mark.gpu
def test_write_after_read_is_ordered(monkeypatch):
    """An in-place torch op on an input of a pending request waits for it."""
    monkeypatch.delenv("GPUOS_SCHEDULER_DISABLE_JIT", raising=False)
    g = torch.Generator().manual_seed(55)
    a, b = torch.randn(1000, generator=g), torch.randn(1000, generator=g)
    ga, gb = a.to(DEV), b.to(DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None):
        c = ga + gb
        ga.mul_(3.0)  # writes an input of the pending add
    assert torch.equal(c.cpu(), _exact(a, b, "add"))
    assert torch.equal(ga.cpu(), a * 3.0)


def test_pending_extents_cover_views():
    """The byte ranges the scheduler tracks: a slice, a transposed view or a
    narrowed view of a tensor overlaps it; a disjoint slice of the same
    storage does not, nor does another tensor."""
    x = torch.zeros(8, 16)
    table = {}
    S._add(S._extent(x[2:4]), table)
    assert S._overlaps(S._extent(x), table)
    assert S._overlaps(S._extent(x[3]), table)
    assert S._overlaps(S._extent(x.t()[5]), table)        # column 5 crosses rows 2..3
    assert S._overlaps(S._extent(x.narrow(0, 3, 5)), table)
    assert not S._overlaps(S._extent(x[4:]), table)
    assert not S._overlaps(S._extent(x[:2]), table)
    assert not S._overlaps(S._extent(torch.zeros(8, 16)), table)
    assert S._extent(torch.zeros(0)) is None


@pytest.mark.gpu
def test_torch_op_on_a_view_of_a_pending_output_waits(monkeypatch):
    """Reading out[1:] (another data_ptr than out) of a scheduled add before
    any flush sees the add's result."""
    monkeypatch.delenv("GPUOS_SCHEDULER_DISABLE_JIT", raising=False)
    g = torch.Generator().manual_seed(56)
    a, b = torch.randn(3000, generator=g), torch.randn(3000, generator=g)
    ga, gb = a.to(DEV), b.to(DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None):
        c = ga + gb
        tail = c[1:].clone()          # aten::clone of a view: runs in torch
        col = (c.view(30, 100).t()[7]).clone()
    want = _exact(a, b, "add")
    assert torch.equal(tail.cpu(), want[1:])
    assert torch.equal(col.cpu(), want.view(30, 100).t()[7])


@pytest.mark.gpu
def test_torch_write_into_a_view_of_a_pending_input_waits(monkeypatch):
    monkeypatch.delenv("GPUOS_SCHEDULER_DISABLE_JIT", raising=False)
    g = torch.Generator().manual_seed(57)
    a, b = torch.randn(3000, generator=g), torch.randn(3000, generator=g)
    ga, gb = a.to(DEV), b.to(DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None):
        c = ga * gb
        ga[5:].zero_()                # writes a view of the pending mul's input
    assert torch.equal(c.cpu(), _exact(a, b, "mul"))
    assert float(ga[5:].abs().sum()) == 0.0


@pytest.mark.gpu
def test_large_tensors_and_autograd_stay_in_torch(monkeypatch):
    monkeypatch.delenv("GPUOS_SCHEDULER_DISABLE_JIT", raising=False)
    a = torch.randn(5000, device=DEV)
    b = torch.randn(5000, device=DEV)
    with torch.no_grad(), S.scheduler_context(size_threshold=1000, auto_flush_ms=None):
        c = a + b
    assert torch.equal(c, a + b)
    w = torch.randn(100, device=DEV, requires_grad=True)
    with S.scheduler_context(auto_flush_ms=None):
        y = w * 2.0
    y.sum().backward()
    assert torch.equal(w.grad, torch.full_like(w, 2.0))


@pytest.mark.gpu
def test_background_flusher(monkeypatch):
    monkeypatch.delenv("GPUOS_SCHEDULER_DISABLE_JIT", raising=False)
    a = torch.randn(2048, device=DEV)
    b = torch.randn(2048, device=DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=1.0) as s:
        outs = [a * b for _ in range(64)]
        s.flush(sync=True)
    ref = a * b
    for o in outs:
        assert torch.equal(o, ref)
