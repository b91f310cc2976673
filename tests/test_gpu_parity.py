"""Parity of the CUDA path with the CPU oracle (needs a GPU: -m gpu).

Every test builds its inputs on the CPU from a fixed seed, runs the oracle on
the CPU copies and the executor on device copies of the same bytes, and
compares.  Tolerances (tests/tolerance.py): bit-exact for the exact
operators and casts; documented CUDA ulp bounds, propagated through the
formula, for transcendentals; 1e-5 * sum|x| for fp32 sum/mean.
"""
import ctypes
import hashlib
import json
import time
from pathlib import Path

import numpy as np
import pytest
import torch

import gpuos_b200
import gpuos_b200.cabi as C
import oracle
from gpuos_b200 import workloads as W
from tolerance import EXACT, RED_REL, check_transcendental

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
KAT = json.loads((Path(__file__).parent / "golden" / "kat.json").read_text())
MODES = [C.MODE_PERSISTENT, C.MODE_STREAM]
MODE_IDS = ["persistent", "stream"]
PARAMS = {"leaky_relu": (0.01, 0.0), "clamp": (-0.5, 0.5), "elu": (1.0, 0.0),
          "softplus": (1.0, 0.0), "clamp_min": (-0.25, 0.0), "clamp_max": (0.25, 0.0)}
ALL_OPS = [n for n, v in sorted(oracle.VARIANTS.items(), key=lambda x: x[1]) if v < 32]


@pytest.fixture(params=MODES, ids=MODE_IDS)
def ex(request):
    e = C.Executor(0, mode=request.param)
    yield e
    e.close()


@pytest.fixture(params=["persistent", "stream"])
def ext(request):
    g = gpuos_b200.load()
    g.init(4096, 256, mode=request.param)
    yield g
    g.shutdown()


def gpu(t):
    return t.to(DEV)


def slot_of(e, op):
    """A jump-table slot running operator `op` (registered through the
    reference scheduler's expression string where there is one)."""
    if op in W.EXPR:
        expr, ar = W.EXPR[op]
        return e.register_elementwise(f"t|{op}", expr, ar)
    if op in PARAMS:
        expr, key = W.param_expr(op, *PARAMS[op])
        return e.register_elementwise(key, expr, 1)
    s = e.register_elementwise(f"t|{op}|slot", "(A)", 1)
    e.set_slot(s, C.variant(op), *PARAMS.get(op, (0.0, 0.0)))
    return s


def _bits(t):
    return t.view(torch.int32 if t.dtype == torch.float32 else torch.int16)


def compare(op, a, b, got, p0=0.0, p1=0.0, where=""):
    """got: CPU tensor read back from the GPU; checks it against the oracle.
    Exact operators: bit for bit.  Transcendentals: fp32 results within the
    propagated CUDA ulp bound of the exact value; 16-bit results within one
    output ulp of the oracle's fp32-then-rounded value."""
    ref = torch.empty_like(got)
    oracle.ew(op, a, b, ref, p0, p1)
    if op in EXACT:
        if not torch.equal(_bits(got), _bits(ref)):
            bad = (_bits(got) != _bits(ref)).nonzero()[:5].tolist()
            raise AssertionError(f"{op}{where}: bit mismatch at {bad}")
        return
    if got.dtype != torch.float32:
        diff = (got.double() - ref.double()).abs()
        rel = 2 ** -7 if got.dtype == torch.bfloat16 else 2 ** -10
        step = (ref.double().abs() * rel).clamp_min(1e-30)
        assert bool((diff <= step * 1.01).all()), f"{op}{where}: more than 1 output ulp off"
        return
    ex64 = torch.empty(got.shape, dtype=torch.float64)
    oracle.ew(op, a, b, ex64, p0, p1, exact=True)
    A = torch.broadcast_to(a.float(), got.shape).reshape(-1).numpy()
    B = (torch.broadcast_to(b.float(), got.shape).reshape(-1).numpy() if b is not None
         else np.zeros(got.numel()))
    ok, worst, i = check_transcendental(op, A, B, got.reshape(-1).numpy(),
                                        ex64.reshape(-1).numpy(), p0, p1)
    assert ok, f"{op}{where}: error {worst:.2f}x the bound at flat index {i} (A={A[i]})"


# --------------------------------------------------------------------------
# the reference's own test vectors
# --------------------------------------------------------------------------
def kat_inputs(k):
    i = torch.arange(k["n"], dtype=torch.float32)
    a = torch.tensor(np.float32(k["a"][0])) * i
    b = np.float32(k["b"][0]) + (torch.arange(k["n"]) % k["b"][1]).float()
    return a, b


@pytest.mark.parametrize("name", ["host_mul", "online_add", "online_mul", "dual_add", "dual_mul"])
def test_reference_vectors(ex, name):
    k = KAT[name]
    a, b = kat_inputs(k)
    ga, gb = gpu(a), gpu(b)
    out = torch.full_like(ga, float("nan"))
    ex.builtin({"add": C.OP_ADD, "mul": C.OP_MUL}[k["op"]], ga, gb, out)
    ex.flush(sync=True)
    got = out.cpu().numpy()
    assert [int(x) for x in got[:16].view(np.uint32)] == k["head_bits"]
    assert hashlib.sha256(got.tobytes()).hexdigest() == k["sha256"]


def test_dual_slot_switch(ex):
    """test/dual_slot_switch.cpp: logical slot 0 runs add, is routed to a
    mul in another physical slot, then rolled back."""
    a, b = kat_inputs(KAT["dual_add"])
    ga, gb = gpu(a), gpu(b)
    outs = [torch.empty_like(ga) for _ in range(3)]
    ex.binary(0, ga, gb, outs[0])
    ex.flush(sync=True)
    s = ex.register_elementwise("op_mul", "(A * B)", 2)
    ex.set_alias(0, s)
    ex.binary(0, ga, gb, outs[1])
    ex.flush(sync=True)
    ex.set_alias(0, 0)
    ex.binary(0, ga, gb, outs[2])
    ex.flush(sync=True)
    for o, name in zip(outs, ["dual_add", "dual_mul", "dual_add"]):
        got = o.cpu().numpy()
        assert hashlib.sha256(got.tobytes()).hexdigest() == KAT[name]["sha256"], name


def test_online_switch(ex):
    """test/online_switch.cpp: slot 0 is overwritten in place (add -> mul)."""
    a, b = kat_inputs(KAT["online_add"])
    ga, gb = gpu(a), gpu(b)
    c_add, c_mul = torch.empty_like(ga), torch.empty_like(ga)
    ex.binary(0, ga, gb, c_add)
    ex.flush(sync=True)
    ex.set_slot(0, C.variant("mul"))
    ex.binary(0, ga, gb, c_mul)
    ex.flush(sync=True)
    ex.set_slot(0, C.variant("add"))
    assert hashlib.sha256(c_add.cpu().numpy().tobytes()).hexdigest() == KAT["online_add"]["sha256"]
    assert hashlib.sha256(c_mul.cpu().numpy().tobytes()).hexdigest() == KAT["online_mul"]["sha256"]


def test_reference_task_layout(ex):
    """A request in the reference's 496-byte Task layout (src/common.h:34-46)."""
    n = 1000
    a, b = torch.randn(n), torch.randn(n)
    ga, gb, go = gpu(a), gpu(b), torch.empty(n, device=DEV)
    raw = bytearray(496)

    def tref(off, t):
        d = C.tensor(t)
        raw[off:off + 144] = bytes(d)

    raw[0:4] = (1).to_bytes(4, "little")        # op: jump-table slot 1 (mul)
    raw[8:12] = (1).to_bytes(4, "little")       # ndim
    raw[16:24] = n.to_bytes(8, "little")        # numel
    tref(64, ga)
    tref(208, gb)
    tref(352, go)
    ex.task(bytes(raw))
    ex.flush(sync=True)
    assert torch.equal(go.cpu(), a * b)


# --------------------------------------------------------------------------
# every operator, ragged sizes, aligned and misaligned views
# --------------------------------------------------------------------------
SIZES = [1, 7, 255, 256, 257, 1000, 4097, 33000]


@pytest.mark.parametrize("op", ALL_OPS)
def test_every_operator(op):
    """Every operator on ragged sizes; shift=1 starts the views one element
    into their buffers, so the 16-byte vector path is off and the scalar
    path runs."""
    with C.Executor(0, mode=C.MODE_STREAM) as e:
        s = slot_of(e, op)
        g = torch.Generator().manual_seed(100 + ALL_OPS.index(op))
        binary = op in oracle.BINARY
        cases = []
        for n in SIZES:
            for shift in (0, 1):
                af = torch.randn(n + shift, generator=g)
                bf = torch.randn(n + shift, generator=g)
                if op in ("log", "sqrt", "pow"):
                    af = af.abs() + 1e-3
                if op == "pow":
                    bf = torch.rand(n + shift, generator=g) * 1.5 + 0.5
                if op in ("div", "div0"):
                    bf = torch.sign(bf) * (bf.abs() + 0.1)
                a, b = af[shift:], bf[shift:]
                ga, gb = gpu(af)[shift:], gpu(bf)[shift:]
                go = torch.empty(n + shift, device=DEV)[shift:]
                if binary:
                    e.binary(s, ga, gb, go)
                else:
                    e.unary(s, ga, go)
                # the C ABI does not own tensors: keep the inputs alive until the flush
                cases.append((a, b if binary else None, go, n, shift, ga, gb))
        e.flush(sync=True)
        p0, p1 = PARAMS.get(op, (0.0, 0.0))
        for a, b, go, n, shift, _, _ in cases:
            compare(op, a, b, go.cpu(), p0, p1, where=f" n={n} shift={shift}")


@pytest.mark.parametrize("op", ["add", "mul", "div0", "maximum", "copy", "relu", "clamp"])
@pytest.mark.parametrize("dts", [("f16", "f32", "f32"), ("bf16", "bf16", "bf16"),
                                 ("f16", "f16", "f16"), ("f32", "f32", "bf16"),
                                 ("f32", "f32", "f16")])
def test_dtype_casts_bit_exact(op, dts):
    D = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
    da, db, do = (D[x] for x in dts)
    g = torch.Generator().manual_seed(7)
    with C.Executor(0, mode=C.MODE_PERSISTENT) as e:
        s = slot_of(e, op)
        cases = []
        for n in (33, 4096, 5003):
            a = (torch.randn(n, generator=g) * 3).to(da)
            b = (torch.randn(n, generator=g) * 3).to(db)
            if op == "div0":
                b[::7] = 0
            go = torch.empty(n, dtype=do, device=DEV)
            ga, gb = gpu(a), gpu(b)
            if op in oracle.BINARY:
                e.binary(s, ga, gb, go)
            else:
                e.unary(s, ga, go)
            cases.append((a, b if op in oracle.BINARY else None, go, ga, gb))
        e.flush(sync=True)
        for a, b, go, _, _ in cases:
            ref = torch.empty(go.shape, dtype=do)
            oracle.ew(op, a, b, ref, *PARAMS.get(op, (0.0, 0.0)))
            got = go.cpu()
            assert torch.equal(got.view(torch.int16 if do != torch.float32 else torch.int32),
                               ref.view(torch.int16 if do != torch.float32 else torch.int32)), (op, dts)


@pytest.mark.parametrize("dts", [("f32", "f32", "f32"), ("f16", "f32", "f32"),
                                 ("bf16", "bf16", "bf16")])
def test_vector_rounds_end_inside_the_request(dts):
    """The vector bodies walk a chunk in rounds of up to 8 (light) or 2
    (heavy) groups of 4 elements per lane, each group under its own bound:
    lengths just around the round and chunk boundaries, in one flush of small
    requests (512-element chunks) and one with multi-million-element requests
    (8192-element chunks), flat, with a scalar operand and with a per-row
    operand.  Every result is checked against the oracle and the 64 elements
    after each output must keep their sentinel."""
    D = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
    da, db, do = (D[x] for x in dts)
    g = torch.Generator().manual_seed(17)
    flushes = [
        [3, 4, 5, 124, 127, 128, 131, 1020, 1023, 1024, 1028, 4100, 8190, 8196, 40004, 70001],
        [6_000_003, 1_000_001, 77],
    ]
    with C.Executor(0, mode=C.MODE_STREAM) as e:
        s_exp = slot_of(e, "exp")
        for sizes in flushes:
            cases = []

            def out(n):
                buf = torch.full((n + 64,), 1234.5, dtype=do, device=DEV)
                return buf, buf[:n]

            for n in sizes:
                a = torch.randn(n, generator=g).to(da)
                b = torch.randn(n, generator=g).to(db)
                ga, gb = gpu(a), gpu(b)
                buf, go = out(n)
                e.builtin(C.OP_ADD, ga, gb, go)
                cases.append(("add", a, b, buf, n, ga, gb))
                buf, go = out(n)
                e.unary(s_exp, ga, go)
                cases.append(("exp", a, None, buf, n, ga, None))
                sc = torch.tensor(0.75, dtype=db)
                gsc = gpu(sc)
                buf, go = out(n)
                e.builtin(C.OP_MUL, ga, gsc, go)
                cases.append(("mul", a, sc, buf, n, ga, gsc))
            for R, N in ((1, 4), (3, 132), (37, 1028), (5, 8196)):
                a = torch.randn(R, N, generator=g).to(da)
                b = torch.randn(N, generator=g).to(db)
                ga, gb = gpu(a), gpu(b)
                buf = torch.full((R * N + 64,), 1234.5, dtype=do, device=DEV)
                e.builtin(C.OP_SUB, ga, gb, buf[:R * N].view(R, N))
                cases.append(("sub", a, b, buf, R * N, ga, gb))
            e.flush(sync=True)
            sentinel = torch.full((64,), 1234.5, dtype=do)
            for op, a, b, buf, n, _, _ in cases:
                got = buf.cpu()
                where = f" n={n} {dts}"
                assert torch.equal(_bits(got[n:]), _bits(sentinel)), f"{op}{where}: wrote past the end"
                compare(op, a, b, got[:n].view(a.shape), where=where)


# --------------------------------------------------------------------------
# broadcast, views, strided layouts
# --------------------------------------------------------------------------
_KEEP = []  # device inputs of requests not yet flushed (the C ABI does not own tensors)


def run_one(e, op, a, b, out_shape, out_dtype=torch.float32, out=None, p=(0.0, 0.0)):
    s = slot_of(e, op)
    ga = gpu(a)
    gb = gpu(b) if b is not None else None
    _KEEP.extend([ga, gb])
    go = out if out is not None else torch.empty(out_shape, dtype=out_dtype, device=DEV)
    if b is not None:
        e.binary(s, ga, gb, go)
    else:
        e.unary(s, ga, go)
    return go


def test_broadcast_layouts(ex):
    g = torch.Generator().manual_seed(8)
    B, N = 13, 520
    a = torch.randn(B, N, generator=g)
    row = torch.randn(N, generator=g)
    col = torch.randn(B, 1, generator=g)
    at = torch.randn(N, B, generator=g).t()
    sc = torch.randn((), generator=g)
    cases = [("add", a, row), ("mul", a, col), ("sub", at, row), ("maximum", at, col),
             ("mul", a, sc), ("div", sc, a), ("add", row, col), ("minimum", at, at)]
    outs = []
    for op, x, y in cases:
        shape = torch.broadcast_shapes(x.shape, y.shape)
        outs.append((op, x, y, run_one(ex, op, x, y, shape)))
    ex.flush(sync=True)
    _KEEP.clear()
    for op, x, y, go in outs:
        compare(op, x, y, go.cpu(), where=f" {tuple(x.shape)}x{tuple(y.shape)}")


def test_column_broadcast_is_torch_semantics(ex):
    """[B,N] op [B,1] follows torch (the reference's decomposition gives the
    wrong rows here; the oracle's reference mode reproduces that)."""
    k = KAT["bcast_col"]
    a = torch.tensor(k["a"])
    c = torch.tensor(k["c"]).reshape(-1, 1)
    go = torch.empty(a.shape, device=DEV)
    ga, gc = gpu(a), gpu(c)
    ex.builtin(C.OP_ADD, ga, gc, go)
    ex.flush(sync=True)
    assert go.cpu().tolist() == k["torch"]
    assert go.cpu().tolist() != k["reference"]


def test_strided_and_noncontiguous_out(ex):
    g = torch.Generator().manual_seed(9)
    x = torch.randn(4, 5, 6, 7, generator=g).permute(2, 0, 3, 1)   # 4-D, no collapse
    y = torch.randn(6, 1, 7, 1, generator=g)
    base_out = torch.empty(6, 4, 7, 5 * 2, device=DEV)
    go = base_out[..., ::2]                                           # strided output
    s = slot_of(ex, "mul")
    gx, gy = gpu(x), gpu(y)
    ex.binary(s, gx, gy, go)
    ex.flush(sync=True)
    ref = torch.empty(6, 4, 7, 5)
    oracle.ew("mul", x, y, ref)
    assert torch.equal(go.cpu(), ref)


def test_broadcast_stream(ext):
    st = W.broadcast_mixed(n_req=384, seed=1)
    din, dout = st.device_buffers(DEV)
    views = st.views(din, dout)
    calls = W.Submitter(ext).prepare(st, views)
    for i, (fn, args) in enumerate(calls):
        fn(*args)
        if (i + 1) % st.flush_every == 0:
            ext.flush(sync=False)
    ext.flush(sync=True)
    host_out = dout.cpu()
    for r in st.requests:
        a, b, o = r.a.view(st.host_in), r.b.view(st.host_in), r.out.view(host_out)
        ref = torch.empty(o.shape, dtype=o.dtype)
        oracle.ew(r.op, a, b, ref)
        assert torch.equal(o.view(torch.int16 if o.dtype != torch.float32 else torch.int32),
                           ref.view(torch.int16 if o.dtype != torch.float32 else torch.int32)), r


# --------------------------------------------------------------------------
# whole streams through the reference-facing Python API
# --------------------------------------------------------------------------
def run_stream(ext, st):
    din, dout = st.device_buffers(DEV)
    calls = W.Submitter(ext).prepare(st, st.views(din, dout))
    for i, (fn, args) in enumerate(calls):
        fn(*args)
        if (i + 1) % st.flush_every == 0:
            ext.flush(sync=False)
    ext.flush(sync=True)
    return dout.cpu()


def test_micro_add_mul_stream(ext):
    st = W.micro_add_mul(n_req=256)
    host_out = run_stream(ext, st)
    for r in st.requests:
        ref = torch.empty(r.out.shape)
        oracle.ew(r.op, r.a.view(st.host_in), r.b.view(st.host_in), ref)
        assert torch.equal(r.out.view(host_out), ref)


def test_mixed_stream(ext):
    st = W.mixed_24op(n_req=1024, seed=3)
    host_out = run_stream(ext, st)
    for r in st.requests:
        a = r.a.view(st.host_in)
        b = r.b.view(st.host_in) if r.b is not None else None
        compare(r.op, a, b, r.out.view(host_out).clone(), r.p0, r.p1, where=f" {r.stream_op}")


# --------------------------------------------------------------------------
# reductions
# --------------------------------------------------------------------------
def check_reduce(op, x, got, axes, keepdim):
    ref = torch.empty(got.shape, dtype=got.dtype)
    oracle.reduce(op, x, ref, axes, keepdim)
    cnt = 1
    for a in axes:
        cnt *= x.shape[a]
    if cnt == 0:  # empty reduction: sum 0, mean NaN (torch semantics)
        if op == "mean":
            assert bool(got.isnan().all())
        else:
            assert bool((got == 0).all())
        return
    ex64 = x.double().sum(dim=list(axes), keepdim=keepdim)
    mag = x.double().abs().sum(dim=list(axes), keepdim=keepdim)
    if op == "mean":
        ex64, mag = ex64 / cnt, mag / cnt
    tol = RED_REL * mag + 1e-30
    if got.dtype != torch.float32:
        tol = tol + ex64.abs() * 2 ** -7
    err = (got.double() - ex64).abs()
    assert bool((err <= tol).all()), f"{op} {tuple(x.shape)} axes={axes}: max err/tol " \
                                     f"{float((err / tol).max()):.2f}"
    # the oracle (reference order) sits inside the same bound
    assert bool(((ref.double() - ex64).abs() <= tol).all())


RED_CASES = [((64, 1000), (1,), False), ((3, 8191), (-1,), True), ((5, 9000), (1,), False),
             ((2, 40000), (1,), True), ((300, 70), (1,), False), ((1, 64), (1,), False),
             ((4096, 3), (1,), True), ((8, 16, 32), (0, 1), False), ((8, 16, 32), (1,), True),
             ((7, 0), (1,), False)]


@pytest.mark.parametrize("op", ["sum", "mean"])
@pytest.mark.parametrize("trans", [False, True])
def test_reductions(ex, op, trans):
    g = torch.Generator().manual_seed(10)
    s = ex.register_reduce(f"r|{op}", op)
    pend = []
    for shape, axes, keep in RED_CASES:
        for dt in (torch.float32, torch.bfloat16):
            if trans and len(shape) == 2:
                x = torch.randn(shape[::-1], generator=g).to(dt).t()
            else:
                x = torch.randn(shape, generator=g).to(dt)
            out_shape = list(x.shape)
            for a in sorted(a % x.dim() for a in axes):
                out_shape[a] = 1
            if not keep:
                out_shape = [d for i, d in enumerate(out_shape) if i not in [a % x.dim() for a in axes]]
            go = torch.empty(out_shape, dtype=dt, device=DEV)
            gx = gpu(x)
            ex.reduce(s, gx, go, axes, keep)
            pend.append((x, go, axes, keep, gx))
    ex.flush(sync=True)
    for x, go, axes, keep, _ in pend:
        check_reduce(op, x, go.cpu(), axes, keep)


def test_reduce_stream(ext):
    st = W.lastdim_reduce(n_req=96, seed=2, max_elems=1 << 20)
    host_out = run_stream(ext, st)
    for r in st.requests:
        check_reduce(r.op, r.a.view(st.host_in), r.out.view(host_out).clone(), list(r.axes),
                     r.keepdim)


# --------------------------------------------------------------------------
# hazards inside one flush, errors, lifecycle
# --------------------------------------------------------------------------
def test_dependent_chain_in_one_flush(ex):
    """x = a + b; y = x * c; z = relu(y); a = a - z: read-after-write and
    write-after-read inside a single batch run in submission order."""
    g = torch.Generator().manual_seed(11)
    n = 50000
    a, b, c = (torch.randn(n, generator=g) for _ in range(3))
    ga, gb, gc = gpu(a), gpu(b), gpu(c)
    gx, gy, gz = (torch.empty(n, device=DEV) for _ in range(3))
    relu = slot_of(ex, "relu")
    ex.builtin(C.OP_ADD, ga, gb, gx)
    ex.builtin(C.OP_MUL, gx, gc, gy)
    ex.unary(relu, gy, gz)
    ex.builtin(C.OP_SUB, ga, gz, ga)
    ex.flush(sync=True)
    x = a + b
    y = x * c
    z = torch.relu(y)
    assert torch.equal(gz.cpu(), z)
    assert torch.equal(ga.cpu(), a - z)


def test_chain_across_async_flushes():
    """Consecutive async flushes with a dependency are ordered too."""
    with C.Executor(0, mode=C.MODE_PERSISTENT) as e:
        n = 1 << 18
        x = torch.zeros(n, device=DEV)
        one = torch.ones(n, device=DEV)
        for _ in range(50):
            e.builtin(C.OP_ADD, x, one, x)
            e.flush(sync=False)
        e.flush(sync=True)
        assert bool((x == 50).all())


def test_unregistered_slot_reports_error(ex):
    x = torch.randn(1000, device=DEV)
    y = torch.empty_like(x)
    ex.unary(77, x, y)
    with pytest.raises(C.GpuosError, match="no registered operator"):
        ex.flush(sync=True)
    ex.builtin(C.OP_ADD, x, x, y)           # the executor stays usable
    ex.flush(sync=True)
    assert torch.equal(y, x + x)
    # the failed batch's counter slot comes round again (1024 slots) clean
    z = torch.empty_like(x)
    for i in range(1030):
        ex.builtin(C.OP_MUL if i % 2 else C.OP_ADD, x, x, z)
        ex.flush(sync=False)
    ex.flush(sync=True)
    assert torch.equal(z, x * x)  # the last one (i = 1029) multiplies


def test_bad_requests_rejected_on_host(ex):
    a = torch.randn(4, 5, device=DEV)
    with pytest.raises(C.GpuosError, match="broadcast"):
        ex.builtin(C.OP_ADD, a, torch.randn(3, device=DEV), torch.empty(4, 5, device=DEV))
    with pytest.raises(C.GpuosError):
        ex.builtin(7, a, a, a)


def test_persistent_lifecycle():
    with C.Executor(0, mode=C.MODE_PERSISTENT, idle_ms=30) as e:
        assert e.worker_alive()
        x = torch.randn(10000, device=DEV)
        y = torch.empty_like(x)
        time.sleep(0.3)                       # idle exit after 30 ms
        assert not e.worker_alive()
        e.builtin(C.OP_MUL, x, x, y)
        e.flush(sync=True)                    # relaunched on demand
        assert torch.equal(y, x * x)
        e.set_yield_every(1)                  # exit after every batch
        for _ in range(5):
            e.builtin(C.OP_ADD, x, y, y)
            e.flush(sync=True)
        st = e.stats()
        assert st["relaunches"] >= 5, st
        assert st["errors"] == 0
        assert torch.allclose(y, x * x + 5 * x)


def test_ext_api_surface(ext):
    names = ["init", "shutdown", "abi_version", "set_debug_level", "set_verbose_level",
             "peek_queue", "set_yield_every", "worker_alive", "submit_add", "submit_mul",
             "submit_sub", "submit_div", "flush", "register_elementwise", "submit_unary",
             "submit_binary", "register_reduce", "submit_reduce"]
    for n in names:
        assert hasattr(ext, n), n
    assert ext.abi_version() == 1
    q = ext.peek_queue()
    for k in ("head", "tail", "in_flight", "capacity", "processed", "heartbeat", "quit",
              "host_tail_shadow", "host_pending", "staging", "shard_size"):
        assert k in q, k
    a = torch.arange(16, device=DEV, dtype=torch.float32)
    b = 2 * torch.ones_like(a)
    c = torch.empty_like(a)
    ext.submit_add(a, b, c)
    ext.submit_mul(a, b, c)
    ext.submit_sub(a, b, c)
    ext.submit_div(a, b, c)
    ext.flush(sync=True)
    assert torch.equal(c, a / 2)            # the four ran in submission order
    with pytest.raises(RuntimeError):
        ext.submit_add(a.cpu(), b.cpu(), c.cpu())
    with pytest.raises(TypeError):
        ext.submit_add(a.long(), b, c)


def test_stream_mode_orders_with_torch():
    g = gpuos_b200.load()
    g.init(4096, 256, mode="stream")
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            a = torch.randn(1 << 20, device=DEV)
            b = a * 3                      # produced on s
            c = torch.empty_like(a)
            g.submit_add(a, b, c)
            g.flush(sync=False)            # runs on s after the producer
            d = c * 2                      # consumer on s, no host sync
        s.synchronize()
        assert torch.equal(d, (a + a * 3) * 2)
    finally:
        g.shutdown()


# ---------------------------------------------------------------------------
# Custom expressions (NVRTC): compiled at registration, linked to the batch
# kernel for custom expressions, batched like every other request.
# ---------------------------------------------------------------------------
def _f32_ref(fn, *xs):
    """fn evaluated in float64 on float32 inputs: the exact value the fp32
    result approximates."""
    return fn(*[np.asarray(x, np.float64) for x in xs])


@pytest.mark.parametrize("mode", MODES, ids=MODE_IDS)
def test_custom_expressions(mode):
    with C.Executor(0, mode=mode) as e:
        s2 = e.register_elementwise("cx|quad", "A * A + 2.f * B", 2)
        s1 = e.register_elementwise("cx|wave", "sinf(A) * 0.5f + expf(-A)", 1)
        assert e.register_elementwise("cx|quad", "A * A + 2.f * B", 2) == s2
        g = torch.Generator().manual_seed(77)
        keep = []
        for n, dt in ((1, torch.float32), (4099, torch.float32), (3000, torch.float16),
                      (2048, torch.bfloat16)):
            a = torch.randn(n, generator=g).to(dt)
            b = torch.randn(n, generator=g).to(dt)
            ga, gb = gpu(a), gpu(b)
            o2 = torch.empty(n, device=DEV)
            o1 = torch.empty(n, device=DEV, dtype=dt)
            e.binary(s2, ga, gb, o2)
            e.unary(s1, ga, o1)
            keep.append((a, b, ga, gb, o2, o1))
        # a strided (transposed) operand takes the general path
        x = torch.randn(33, 70, generator=g)
        gx = gpu(x).t()
        ox = torch.empty(70, 33, device=DEV)
        e.unary(s1, gx, ox)
        e.flush(sync=True)
        for a, b, ga, gb, o2, o1 in keep:
            A, B = a.float().numpy(), b.float().numpy()
            want2 = _f32_ref(lambda p, q: p * p + 2.0 * q, A, B)
            got2 = o2.cpu().double().numpy()
            tol2 = (np.abs(A.astype(np.float64)) ** 2 + 2 * np.abs(B)) * 2.0 ** -22
            assert np.all(np.abs(got2 - want2) <= tol2 + 1e-30)
            want1 = _f32_ref(lambda p: np.sin(p) * 0.5 + np.exp(-p), A)
            got1 = o1.cpu().double().numpy()
            ulp_out = 2.0 ** -22 if o1.dtype == torch.float32 else (
                2.0 ** -10 if o1.dtype == torch.float16 else 2.0 ** -7)
            tol1 = (0.5 * np.abs(np.sin(A)) + np.exp(-A.astype(np.float64))) * (2.0 ** -20 + ulp_out)
            assert np.all(np.abs(got1 - want1) <= tol1 + 1e-30)
        wantx = _f32_ref(lambda p: np.sin(p) * 0.5 + np.exp(-p), x.t().numpy())
        tolx = (0.5 * np.abs(np.sin(x.t().numpy())) + np.exp(-x.t().double().numpy())) * 2.0 ** -20
        assert np.all(np.abs(ox.cpu().double().numpy() - wantx) <= tolx)


@pytest.mark.parametrize("mode", MODES, ids=MODE_IDS)
def test_custom_expression_ordering_and_hot_swap(mode):
    """A custom request that reads a precompiled request's output in the same
    flush runs after it (the flush splits into batches in order); a slot can
    be swapped onto a custom expression."""
    with C.Executor(0, mode=mode) as e:
        sc = e.register_elementwise("cx|cube", "A * A * A", 1)
        g = torch.Generator().manual_seed(78)
        a, b = torch.randn(5000, generator=g), torch.randn(5000, generator=g)
        ga, gb = gpu(a), gpu(b)
        t = torch.empty(5000, device=DEV)
        y = torch.empty(5000, device=DEV)
        z = torch.empty(5000, device=DEV)
        e.builtin(C.OP_ADD, ga, gb, t)       # precompiled
        e.unary(sc, t, y)                    # custom, reads t
        e.builtin(C.OP_MUL, y, gb, z)        # precompiled, reads y
        e.flush(sync=True)
        T = (a + b).numpy().astype(np.float64)
        assert np.allclose(y.cpu().double().numpy(), T ** 3, rtol=1e-6, atol=1e-6)
        assert torch.equal(z.cpu(), y.cpu() * b)
        # hot swap: slot 0 (add) onto the custom cube, then back
        v, _, _, _ = e.get_slot(sc)
        assert v >= 64
        e.set_slot(0, v)
        w = torch.empty(5000, device=DEV)
        e.binary(0, ga, gb, w)
        e.flush(sync=True)
        assert np.allclose(w.cpu().double().numpy(), a.double().numpy() ** 3, rtol=1e-6,
                           atol=1e-6)
        e.set_slot(0, C.variant("add"))
        e.binary(0, ga, gb, w)
        e.flush(sync=True)
        assert torch.equal(w.cpu(), a + b)


# ---------------------------------------------------------------------------
# The transformer-decode pointwise chain (bf16): residual add, RMSNorm as
# x*x -> mean(-1) -> +eps -> pow(-0.5) -> * rstd[b,1] -> * w[4096], bias, and
# a SiLU-style gate (sigmoid, mul) on [b, 11008]; several layers in ONE flush,
# so every step depends on the one before.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("B", [1, 8, 64])
@pytest.mark.parametrize("mode", MODES, ids=MODE_IDS)
def test_decode_chain_bf16(mode, B):
    """All 32 layers of the decode configuration, one flush."""
    bf = torch.bfloat16
    H, F, L = 4096, 11008, 32
    g = torch.Generator().manual_seed(91)

    def normal(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).to(bf)

    with C.Executor(0, mode=mode) as e:
        s_sig = slot_of(e, "sigmoid")
        s_pow = slot_of(e, "pow")
        s_mean = e.register_reduce("t|mean", "mean")
        eps = gpu(torch.tensor(1e-6, dtype=bf))
        nhalf = gpu(torch.tensor(-0.5, dtype=bf))
        x = gpu(normal(B, H))
        steps = []
        for _ in range(L):
            res, w, bias = gpu(normal(B, H)), gpu(normal(H)), gpu(normal(H))
            u, u2 = gpu(normal(B, F)), gpu(normal(B, F))
            nan = lambda *s: torch.full(s, float("nan"), dtype=bf, device=DEV)  # noqa: E731
            h, sq, hn, hw, xo = nan(B, H), nan(B, H), nan(B, H), nan(B, H), nan(B, H)
            ms, mse, rstd = nan(B, 1), nan(B, 1), nan(B, 1)
            gt, act = nan(B, F), nan(B, F)
            e.builtin(C.OP_ADD, x, res, h)
            e.builtin(C.OP_MUL, h, h, sq)
            e.reduce(s_mean, sq, ms, [1], True)
            e.builtin(C.OP_ADD, ms, eps, mse)
            e.binary(s_pow, mse, nhalf, rstd)
            e.builtin(C.OP_MUL, h, rstd, hn)         # [b,H] * [b,1]
            e.builtin(C.OP_MUL, hn, w, hw)           # [b,H] * [H]
            e.builtin(C.OP_ADD, hw, bias, xo)
            e.unary(s_sig, u, gt)
            e.builtin(C.OP_MUL, gt, u2, act)
            steps.append(dict(x=x, res=res, w=w, bias=bias, u=u, u2=u2, h=h, sq=sq, ms=ms,
                              mse=mse, rstd=rstd, hn=hn, hw=hw, xo=xo, gt=gt, act=act))
            x = xo
        e.flush(sync=True)
        for st in steps:
            c = {k: v.cpu() for k, v in st.items()}
            # every request against the oracle, from the inputs the GPU gave it
            compare("add", c["x"], c["res"], c["h"])
            compare("mul", c["h"], c["h"], c["sq"])
            ref = torch.empty(B, 1)
            oracle.reduce("mean", c["sq"].float(), ref, [1], True)
            tol = 1e-5 * c["sq"].float().abs().sum(1, keepdim=True) + ref.abs() * 2 ** -8
            assert bool(((c["ms"].float() - ref).abs() <= tol).all())
            compare("add", c["ms"], torch.tensor(1e-6, dtype=bf), c["mse"])
            compare("pow", c["mse"], torch.tensor(-0.5, dtype=bf), c["rstd"])
            compare("mul", c["h"], c["rstd"], c["hn"])
            compare("mul", c["hn"], c["w"], c["hw"])
            compare("add", c["hw"], c["bias"], c["xo"])
            compare("sigmoid", c["u"], None, c["gt"])
            compare("mul", c["gt"], c["u2"], c["act"])
            assert not torch.isnan(c["xo"].float()).any()


@pytest.mark.parametrize("numel", [4096, 1000])
def test_uniform_lean_batch(numel):
    """1024 requests of one shape and light operators flushed at once run as
    one lean launch of the one-shape parameter block (LeanUniBatch); a
    request of another shape, or a heavier operator, ends the run."""
    ops = [C.OP_ADD, C.OP_MUL, C.OP_SUB]
    g = torch.Generator(device="cpu").manual_seed(81)
    a = torch.randn(1024, numel, generator=g)
    b = torch.randn(1024, numel, generator=g)
    da, db = a.to(DEV), b.to(DEV)
    out = torch.empty(1024, numel, device=DEV)
    with C.Executor(0, mode=C.MODE_STREAM) as ex:
        l0 = ex.stats()["lean"]
        for r in range(1024):
            ex.builtin(ops[r % 3], da[r], db[r], out[r])
        ex.flush(sync=True)
        assert ex.stats()["lean"] - l0 == 1
        # 1023 of one shape, then one longer request: two batches
        out2 = torch.empty(1024 * numel + 4, device=DEV)
        for r in range(1023):
            ex.builtin(C.OP_ADD, da[r], db[r], out2[r * numel:(r + 1) * numel])
        big_a = torch.randn(numel + 4, generator=g)
        ex.builtin(C.OP_MUL, big_a.to(DEV), big_a.to(DEV), out2[1023 * numel:])
        ex.flush(sync=True)
        assert ex.stats()["lean"] - l0 == 3
    want = torch.stack([a[r] + b[r] if r % 3 == 0 else a[r] * b[r] if r % 3 == 1 else a[r] - b[r]
                        for r in range(1024)])
    assert torch.equal(out.cpu(), want)
    assert torch.equal(out2[:1023 * numel].cpu(), (a[:1023] + b[:1023]).reshape(-1))
    assert torch.equal(out2[1023 * numel:].cpu(), big_a * big_a)
