"""Fused elementwise chains: custom expressions of three and four operands
(gpuos_submit_nary) and the scheduler's composition of chains into one
request (the reference composes only a unary op on one fused node and never
writes the returned tensors: pytorch_ext/scheduler.py:213-222, 349-369).

CPU tests cover the composition and the deferred submission with a stand-in
extension module; GPU tests compare fused chains with the same chains run
op by op, bit for bit where the ops are exact.
"""
import gc

import pytest
import torch

import gpuos_b200.scheduler as S

DEV = "cuda:0"


class FakeExt:
    """Records what the scheduler registers and submits."""

    def __init__(self):
        self.slots = {}
        self.calls = []

    def register_elementwise(self, key, expr, arity):
        self.slots.setdefault(key, (len(self.slots), expr, arity))
        return self.slots[key][0]

    def register_reduce(self, key, op):
        return self.register_elementwise(key, op, 1)

    def expr_of(self, slot):
        return next(e for s, e, _ in self.slots.values() if s == slot)

    def submit_unary(self, slot, a, out):
        self.calls.append(("unary", self.expr_of(slot), [a], out))

    def submit_binary(self, slot, a, b, out):
        self.calls.append(("binary", self.expr_of(slot), [a, b], out))

    def submit_nary(self, slot, ins, out):
        self.calls.append(("nary", self.expr_of(slot), list(ins), out))

    def submit_reduce(self, slot, x, out, axes, keepdim):
        self.calls.append(("reduce", None, [x], out))

    def flush(self, sync=False):
        self.calls.append(("flush", sync, [], None))


def _mode(ext):
    return S._GPUOSSchedulerMode(ext, size_threshold=1 << 16, auto_flush_ms=None,
                                 pending=set(), jit=True, fuse=True)


def test_compose_renames_and_merges_leaves():
    a, b, c, d, e = (torch.zeros(3) for _ in range(5))
    M = S._GPUOSSchedulerMode
    x, lv = M._compose("1.f / (1.f + expf(-A))", [("gpuos_keep_f32((A * B))", [a, b])])
    assert x == "1.f / (1.f + expf(-(gpuos_keep_f32((A * B)))))" and lv[0] is a and lv[1] is b
    y, lv = M._compose("(A + B)", [("gpuos_keep_f32(" + x + ")", [a, b]), ("A", [c])])
    assert y == "((gpuos_keep_f32(" + x + ")) + C)" and lv[2] is c
    # shared leaves are merged (by identity) and renamed in one pass
    w, lv = M._compose("(A * B)", [("gpuos_keep_f32((A - B))", [d, a]),
                                   ("gpuos_keep_f32((A + B))", [a, d])])
    assert w == "((gpuos_keep_f32((A - B))) * (gpuos_keep_f32((B + A))))"
    assert lv[0] is d and lv[1] is a and len(lv) == 2
    # five leaves do not fit a request
    assert M._compose("(A * B)", [("gpuos_keep_f32((A + (B * C)))", [a, b, c]),
                                  ("gpuos_keep_f32((A - B))", [d, e])]) is None


def test_chain_becomes_one_request_and_dead_intermediates_are_skipped():
    ext = FakeExt()
    m = _mode(ext)
    a, b, c = (torch.randn(5) for _ in range(3))
    t = torch.empty(5)
    m._node("bin|aten::mul.Tensor", "(A * B)", [a, b], t)
    s = torch.empty(5)
    m._node("un|aten::sigmoid", "1.f / (1.f + expf(-A))", [t], s)
    r = torch.empty(5)
    m._node("bin|aten::add.Tensor", "(A + B)", [s, c], r)
    del t, s   # the caller keeps only the result
    gc.collect()
    m.submit_nodes()
    assert len(ext.calls) == 1
    kind, expr, ins, out = ext.calls[0]
    assert kind == "nary" and out is r and [x is y for x, y in zip(ins, (a, b, c))] == [True] * 3
    assert expr == ("((gpuos_keep_f32(1.f / (1.f + expf(-(gpuos_keep_f32((A * B))))))) + C)")


def test_held_intermediates_are_written_too():
    ext = FakeExt()
    m = _mode(ext)
    a, b = torch.randn(4), torch.randn(4, dtype=torch.bfloat16)
    t = torch.empty(4)
    m._node("bin|aten::mul.Tensor", "(A * B)", [a, b], t)
    u = torch.empty(4, dtype=torch.bfloat16)
    m._node("un|aten::relu", "(A > 0.f ? A : 0.f)", [t.to(torch.bfloat16)], u)  # not t itself
    v = torch.empty(4)
    m._node("un|aten::exp", "expf(A)", [t], v)
    m.submit_nodes()
    kinds = [(k, e) for k, e, _, _ in ext.calls]
    # t is held: written; u reads a copy (a leaf); v inlines t's expression
    assert kinds[0] == ("binary", "(A * B)")
    assert kinds[1] == ("unary", "(A > 0.f ? A : 0.f)")
    assert kinds[2] == ("binary", "expf((gpuos_keep_f32((A * B))))")


def test_bf16_intermediates_round_as_stored():
    ext = FakeExt()
    m = _mode(ext)
    x, w = torch.randn(8, dtype=torch.bfloat16), torch.randn(8, dtype=torch.bfloat16)
    h = torch.empty(8, dtype=torch.bfloat16)
    m._node("bin|aten::mul.Tensor", "(A * B)", [x, w], h)
    y = torch.empty(8, dtype=torch.bfloat16)
    m._node("bin|aten::mul.Tensor", "(A * B)", [h, h], y)   # h * h: h inlined twice
    del h
    m.submit_nodes()
    assert [(k, e) for k, e, _, _ in ext.calls] == [
        ("binary", "((gpuos_keep_bf16((A * B))) * (gpuos_keep_bf16((A * B))))")]


def test_reduction_submits_deferred_ops_first():
    ext = FakeExt()
    m = _mode(ext)
    a = torch.randn(4, 8)
    sq = torch.empty(4, 8)
    m._node("bin|aten::mul.Tensor", "(A * B)", [a, a], sq)
    m.submit_nodes()   # what the reduction path does before it submits
    assert ext.calls[0][0] == "binary" and ext.calls[0][3] is sq


# ---------------------------------------------------------------- GPU tests
@pytest.mark.gpu
def test_three_and_four_operand_requests():
    import gpuos_b200.cabi as C
    g = torch.Generator(device="cpu").manual_seed(71)
    B, N = 37, 1001
    x = torch.randn(B, N, generator=g)
    w = torch.randn(N, generator=g)
    r = torch.randn(B, 1, generator=g)
    xt = torch.randn(N, B, generator=g).t()           # transposed leaf
    xb = torch.randn(B, N, generator=g).to(torch.bfloat16)
    s = torch.tensor(0.75)                             # 0-dim leaf
    d = {k: v.to(DEV) for k, v in dict(x=x, w=w, r=r, xt=xt, xb=xb, s=s).items()}
    with C.Executor(0, mode=C.MODE_STREAM) as ex:
        k3 = ex.register_elementwise("t3", "gpuos_keep_f32((A * B)) + C", 3)
        k4 = ex.register_elementwise("t4", "gpuos_keep_f32((A * B)) - gpuos_keep_f32((C * D))", 4)
        o1 = torch.empty(B, N, device=DEV)
        o2 = torch.empty(B, N, device=DEV)
        o3 = torch.empty(B, N, device=DEV, dtype=torch.bfloat16)
        o4 = torch.empty(N, B, device=DEV).t()        # strided output
        ex.nary(k3, [d["x"], d["w"], d["r"]], o1)      # [B,N] * [N] + [B,1]
        ex.nary(k4, [d["xt"], d["r"], d["xb"], d["s"]], o2)
        ex.nary(k3, [d["xb"], d["s"], d["w"]], o3)
        ex.nary(k4, [d["x"], d["x"], d["w"], d["r"]], o4)
        with pytest.raises(C.GpuosError):
            ex.nary(k4, [d["x"], d["w"], d["r"]], o1)  # arity mismatch
        ex.flush(sync=True)
    xbf = xb.float()
    assert torch.equal(o1.cpu(), x * w + r)
    assert torch.equal(o2.cpu(), xt * r - xbf * s)
    assert torch.equal(o3.cpu(), (xbf * s + w).to(torch.bfloat16))
    assert torch.equal(o4.cpu(), x * x - w * r)


def _chain(a, b, c, w, rs):
    """Elementwise chains of the decode layer tail and a gating product."""
    h = a + b
    sq = h * h
    m = sq.mean(-1, keepdim=True)
    rstd = torch.rsqrt(m + 1e-6)   # runs in torch (after a flush)
    y = (h * rstd) * w + c
    g = torch.sigmoid(y) * y
    z = torch.maximum(g, rs) - torch.minimum(a, b) / (torch.abs(c) + 0.5)
    return h, g, z


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_fused_chain_equals_unfused(monkeypatch, dtype):
    """The same torch code under the scheduler with fusion on and off: the
    exact operators give identical bits, sigmoid (a transcendental in either
    kernel) agrees to 2 ulp of the result's dtype."""
    monkeypatch.setenv("GPUOS_SCHEDULER_DISABLE_JIT", "0")
    g = torch.Generator(device="cpu").manual_seed(72)
    B, N = 8, 4096
    a, b, c = (torch.randn(B, N, generator=g).to(dtype).to(DEV) for _ in range(3))
    w = torch.randn(N, generator=g).to(dtype).to(DEV)
    rs = torch.randn(B, 1, generator=g).to(dtype).to(DEV)
    outs = {}
    for fuse in ("0", "1"):
        monkeypatch.setenv("GPUOS_SCHEDULER_FUSE", fuse)
        with torch.no_grad(), S.scheduler_context(auto_flush_ms=None) as sch:
            h, gg, z = _chain(a, b, c, w, rs)
            sch.flush(sync=True)
            outs[fuse] = [t.float().cpu() for t in (h, gg, z)]
    eps = torch.finfo(dtype).eps
    (h0, g0, z0), (h1, g1, z1) = outs["0"], outs["1"]
    assert torch.equal(h0, h1)                          # exact ops only
    assert bool(((g0 - g1).abs() <= 2 * eps * g0.abs() + 1e-30).all())
    # z = max(g, rs) - ...: g's difference carries over, plus z's own rounding
    assert bool(((z0 - z1).abs() <= 2 * eps * (g0.abs() + z0.abs()) + 1e-30).all())


@pytest.mark.gpu
def test_fused_chain_is_one_request(monkeypatch):
    """sigmoid(a * b) + c with the intermediates dropped: one request."""
    monkeypatch.setenv("GPUOS_SCHEDULER_DISABLE_JIT", "0")
    monkeypatch.setenv("GPUOS_SCHEDULER_FUSE", "1")
    import gpuos_b200
    ext = gpuos_b200.load()
    g = torch.Generator(device="cpu").manual_seed(73)
    a, b, c = (torch.randn(5000, generator=g) for _ in range(3))
    ga, gb, gc = a.to(DEV), b.to(DEV), c.to(DEV)
    with torch.no_grad(), S.scheduler_context(auto_flush_ms=None) as sch:
        r = torch.sigmoid(ga * gb) + gc
        n0 = ext.peek_queue()["requests"]
        sch.flush(sync=True)
        n1 = ext.peek_queue()["requests"]
    assert n1 - n0 == 1
    m = a * b
    want = 1.0 / (1.0 + torch.exp(-m)) + c
    assert torch.allclose(r.cpu(), want, rtol=2e-6, atol=2e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["stream", "persistent"])
def test_mixed_custom_and_precompiled_batch_is_one_launch(mode):
    """A flush of dependent precompiled, reduction and custom requests runs as
    one batch (in the kernel linked with the custom expressions), in stage
    order."""
    import gpuos_b200.cabi as C
    g = torch.Generator(device="cpu").manual_seed(74)
    B, N = 16, 3000
    x, r, w = torch.randn(B, N, generator=g), torch.randn(B, N, generator=g), torch.randn(N, generator=g)
    d = {k: v.to(DEV) for k, v in dict(x=x, r=r, w=w).items()}
    h, sq, o = (torch.empty(B, N, device=DEV) for _ in range(3))
    m = torch.empty(B, 1, device=DEV)
    md = C.MODE_STREAM if mode == "stream" else C.MODE_PERSISTENT
    with C.Executor(0, mode=md) as ex:
        tail = ex.register_elementwise("mix|tail", "gpuos_keep_f32(A * rsqrtf(B + 1e-6f)) * C", 3)
        mean = ex.register_reduce("mix|mean", "mean")
        ex.flush(sync=True)
        p0 = ex.stats()["published"]
        ex.builtin(C.OP_ADD, d["x"], d["r"], h)
        ex.builtin(C.OP_MUL, h, h, sq)
        ex.reduce(mean, sq, m, [1], True)
        ex.nary(tail, [h, m, d["w"]], o)
        ex.flush(sync=True)
        if md == C.MODE_STREAM:  # (persistent mode runs such a batch on its own launch)
            assert ex.stats()["published"] - p0 == 1
    H = x + r
    assert torch.equal(h.cpu(), H)
    M = (H * H).double().mean(1, keepdim=True)
    assert torch.allclose(m.cpu().double(), M, rtol=1e-5, atol=1e-6)
    want = (H * torch.rsqrt(m.cpu() + 1e-6)) * w
    assert torch.allclose(o.cpu(), want, rtol=1e-5, atol=1e-6)


def test_five_leaves_fall_back_to_a_partial_composition():
    """(a*b + c) * (d - e): inlining both sides needs five leaves; the
    left side is inlined and the right side's result becomes a leaf."""
    ext = FakeExt()
    m = _mode(ext)
    a, b, c, d, e = (torch.randn(6) for _ in range(5))
    ab = torch.empty(6)
    m._node("bin|aten::mul.Tensor", "(A * B)", [a, b], ab)
    l = torch.empty(6)
    m._node("bin|aten::add.Tensor", "(A + B)", [ab, c], l)
    r = torch.empty(6)
    m._node("bin|aten::sub.Tensor", "(A - B)", [d, e], r)
    out = torch.empty(6)
    m._node("bin|aten::mul.Tensor", "(A * B)", [l, r], out)
    del ab, l
    m.submit_nodes()
    calls = [(k, e_, [id(t) for t in ins], o) for k, e_, ins, o in ext.calls]
    # r is written (a leaf of the result); the result inlines l's chain
    assert [c_[0] for c_ in calls] == ["binary", "nary"]
    assert calls[0][3] is r and calls[1][3] is out
    assert calls[1][1] == "((gpuos_keep_f32(((gpuos_keep_f32((A * B))) + C))) * D)"
    assert calls[1][2] == [id(a), id(b), id(c), id(r)]
