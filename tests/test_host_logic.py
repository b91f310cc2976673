"""Host logic of the executor, on CPU (no GPU needed).

* the C ABI library loads and exports every entry point include/gpuos_b200.h
  declares;
* request planning: torch broadcasting, dim coalescing, layout choice, vector
  path legality, chunking and reduction splitting;
* the fast-division constants the kernels use;
* expression matching against the reference scheduler's strings;
* errors come back as status codes / Python exceptions, never as a crash.
"""
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import gpuos_b200
import gpuos_b200.cabi as C
from gpuos_b200 import workloads as W

ROOT = Path(__file__).resolve().parents[1]
HEADER = (ROOT / "include" / "gpuos_b200.h").read_text()


def declared():
    return sorted(set(re.findall(r"^\s*(?:int32_t|const char\*)\s+(gpu(?:os)?_\w+)\(", HEADER, re.M)))


def test_header_symbols_exported():
    L = C.lib()
    names = declared()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(C.SIGNATURES), set(names) ^ set(C.SIGNATURES)


def test_abi_version():
    assert C.lib().gpuos_abi_version() == 1


def test_python_module_surface():
    g = gpuos_b200.load()
    for n in ["init", "shutdown", "abi_version", "set_debug_level", "set_verbose_level",
              "peek_queue", "set_yield_every", "worker_alive", "submit_add", "submit_mul",
              "submit_sub", "submit_div", "flush", "register_elementwise", "submit_unary",
              "submit_binary", "register_reduce", "submit_reduce"]:
        assert hasattr(g, n), n
    assert g.abi_version() == 1


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_no_gpu_is_an_error_not_a_crash():
    g = gpuos_b200.load()
    with pytest.raises(RuntimeError):
        g.init()
    with pytest.raises(C.GpuosError) as e:
        C.Executor(0)
    assert e.value.code == C.ECUDA


# ---- planning -------------------------------------------------------------
def plan(op, a, b, out):
    return C.plan_elementwise(C.variant(op), a, b, out)


def test_plan_contiguous():
    a, b, o = torch.randn(4096), torch.randn(4096), torch.empty(4096)
    p = plan("add", a, b, o)
    assert p["layout"] == 0 and p["flags"] & 2 and p["flags"] & 1   # contig, vec, binary
    assert p["chunk"] == 2048 and p["nchunk"] == 2
    p = plan("add", a[1:], b[1:], o[1:])                              # misaligned: no vec
    assert p["layout"] == 0 and not p["flags"] & 2
    p = plan("exp", torch.randn(100).half(), None, torch.empty(100).half())
    assert p["nchunk"] == 1 and p["flags"] & 2     # 8-byte aligned fp16 views vectorize
    p = plan("exp", torch.randn(101).half()[1:], None, torch.empty(101).half()[1:])
    assert not p["flags"] & 2


def test_plan_coalesces_dims():
    a = torch.randn(8, 16, 32)
    p = plan("mul", a, a, torch.empty(8, 16, 32))
    assert p["layout"] == 0 and p["numel"] == 8 * 16 * 32


def test_plan_broadcast_row_col_scalar():
    A, v, col, sc = torch.randn(8, 64), torch.randn(64), torch.randn(8, 1), torch.randn(())
    O = torch.empty(8, 64)
    p = plan("add", A, v, O)
    assert (p["layout"], p["inner"], p["sa_row"], p["sb_row"], p["sa_in"], p["sb_in"]) == \
        (1, 64, 64, 0, 1, 1)
    assert p["flags"] & 2
    p = plan("mul", A, col, O)
    assert (p["layout"], p["sb_row"], p["sb_in"]) == (1, 1, 0) and p["flags"] & 2
    p = plan("mul", A, sc, O)
    assert p["layout"] == 0 and p["flags"] & 16                       # B scalar
    p = plan("mul", sc, A, O)
    assert p["layout"] == 0 and p["flags"] & 8                        # A scalar


def test_plan_transposed_and_strided():
    At = torch.randn(64, 8).t()
    p = plan("add", At, torch.randn(64), torch.empty(8, 64))
    # a transposed operand: 2-D tiles of whole columns (rows in nseg)
    assert p["layout"] == 3 and p["sa_row"] == 1 and p["sa_in"] == 8 and not p["flags"] & 2
    assert p["nseg"] == 8 and p["inner"] == 64
    x = torch.randn(4, 5, 6, 7).permute(2, 0, 3, 1)
    p = plan("add", x, x, torch.empty(6, 4, 7, 5))
    assert p["layout"] == 1 or p["layout"] == 2
    y = torch.randn(6, 1, 7, 1)
    p = plan("mul", x, y, torch.empty(6, 4, 7, 5))
    assert p["layout"] == 2 and p["has_ext"] == 1


def test_plan_rejects_bad_shapes():
    with pytest.raises(C.GpuosError) as e:
        plan("add", torch.randn(4, 5), torch.randn(3), torch.empty(4, 5))
    assert e.value.code == C.EINVAL and "broadcast" in str(e.value)
    with pytest.raises(C.GpuosError):
        plan("add", torch.randn(2, 4, 5), torch.randn(4, 5), torch.empty(4, 5))


def test_plan_reductions():
    x = torch.randn(100, 3000)
    p = C.plan_reduce(C.variant("sum"), x, torch.empty(100, 1), [-1], True)
    assert (p["kind"], p["layout"], p["nseg"], p["inner"], p["numel"]) == (1, 0, 1, 3000, 100)
    assert p["flags"] & 2 and p["rg"] == 32
    p = C.plan_reduce(C.variant("sum"), torch.randn(5, 40000), torch.empty(5), [1], False)
    assert p["nseg"] == 3 and p["nchunk"] == 15 and p["partials"] == 15 and p["counters"] == 5
    p = C.plan_reduce(C.variant("sum"), torch.randn(64, 64), torch.empty(64), [1], False)
    assert p["rg"] == 4 and p["chunk"] % 8 == 0
    xt = torch.randn(3000, 100).t()
    p = C.plan_reduce(C.variant("mean"), xt, torch.empty(100), [1], False)
    # rows adjacent and 16-byte aligned: lanes read 16 bytes of 4 rows (128 per group)
    assert (p["layout"], p["sa_row"], p["sa_in"], p["rg"]) == (1, 1, 100, 128)
    assert p["flags"] & 2 and p["chunk"] == 128 and p["nseg"] == 24   # 64 KB chunks
    assert p["nchunk"] == 24 and p["partials"] == 24 * 128 and p["counters"] == 1
    xb = torch.randn(3000, 256, dtype=torch.bfloat16).t()    # bf16: 8 rows per lane
    p = C.plan_reduce(C.variant("sum"), xb, torch.empty(256, dtype=torch.bfloat16), [1], False)
    assert p["flags"] & 2 and p["rg"] == 256 and p["chunk"] == 128   # 64 KB chunks
    xo = torch.randn(3000, 99).t()                              # 99 rows: not a multiple of 4
    p = C.plan_reduce(C.variant("mean"), xo, torch.empty(99), [1], False)
    assert (p["layout"], p["rg"]) == (1, 32) and not p["flags"] & 2
    assert p["nseg"] > 1 and p["partials"] == 4 * p["nseg"] * 32
    w = torch.randn(8, 16, 32)
    p = C.plan_reduce(C.variant("sum"), w, torch.empty(32), [0, 1], False)
    assert p["layout"] == 0 or p["layout"] == 1 or p["layout"] == 2
    wp = torch.randn(8, 32, 16).permute(0, 2, 1)     # reduced dims 0 and 2 coalesce
    p = C.plan_reduce(C.variant("sum"), wp, torch.empty(16), [0, 2], False)
    assert (p["layout"], p["inner"], p["sa_in"]) == (1, 256, 16)
    wq = torch.randn(8, 16, 32).permute(2, 0, 1)     # reduced dims 0 and 2 do not
    p = C.plan_reduce(C.variant("sum"), wq, torch.empty(8), [0, 2], False)
    assert p["layout"] == 2 and p["has_ext"] == 1 and p["inner"] == 32 * 16
    # 512 reduced elements per output: a warp per output, 16384 / 512 outputs a chunk
    assert p["rg"] == 1 and p["chunk"] == 32 and p["nchunk"] == 1
    wr = torch.randn(8, 4, 6).permute(2, 0, 1)       # 24 per output: a lane per output
    p = C.plan_reduce(C.variant("sum"), wr, torch.empty(8), [0, 2], False)
    assert p["layout"] == 2 and p["rg"] == 0 and p["chunk"] == 32
    with pytest.raises(C.GpuosError):
        C.plan_reduce(C.variant("sum"), x, torch.empty(7), [1], False)


def test_fast_division_constants():
    """The kernels compute n / N as (umulhi(n, m) + n) >> s for n < 2^31."""
    rng = np.random.default_rng(0)
    divisors = list(range(2, 300)) + [4095, 4096, 4097, 11008, 32768, 65535, 1 << 20,
                                       (1 << 30) - 1, 1000003, 123456789]
    for N in divisors:
        m, s = _magic(N)
        n = np.concatenate([rng.integers(0, 1 << 31, 4000, dtype=np.uint64),
                            np.array([0, 1, N - 1, N, N + 1, (1 << 31) - 1], dtype=np.uint64)])
        q = (((n * np.uint64(m)) >> np.uint64(32)) + n) >> np.uint64(s)
        assert np.array_equal(q, n // np.uint64(N)), N


def _desc(shape, strides, addr=1 << 20):
    d = C.Tensor()
    d.data, d.dtype, d.ndim = addr, C.F32, len(shape)
    for i, (n, st) in enumerate(zip(shape, strides)):
        d.sizes[i], d.strides[i] = n, st
    return d


def _magic(N):
    """fdiv constants the runtime stores in the 2-D record of a [2, N] op [N]
    request (descriptors only: planning never touches the memory)."""
    import ctypes
    a, b, o = _desc((2, N), (N, 1)), _desc((N,), (1,)), _desc((2, N), (N, 1), 1 << 40)
    p = C.Plan()
    C.check(C.lib().gpuos_plan_elementwise(C.variant("add"), 0.0, 0.0, ctypes.byref(a),
                                           ctypes.byref(b), ctypes.byref(o), ctypes.byref(p)))
    r = C.decode_record(bytes(p.record))
    assert r["layout"] in (1, 3) and r["inner"] == N   # ROW2D, or 2-D tiles when N % 4 != 0
    return r["fdiv_m"], r["fdiv_s"]


def test_expression_matching():
    for op, (expr, ar) in W.EXPR.items():
        v, p0, p1 = C.match_expression(expr, ar)
        name = {"div": "div"}.get(op, op)
        assert v == C.variant(name), (op, expr, v)
    for op, p in (("leaky_relu", (0.01,)), ("clamp", (-0.5, 0.5)), ("hardtanh", (-1.0, 1.0)),
                  ("elu", (1.0,)), ("softplus", (2.0,)), ("clamp_min", (-0.25,)),
                  ("clamp_max", (0.75,))):
        expr, key = W.param_expr(op, *p, *([0.0] if len(p) == 1 else []))
        v, p0, p1 = C.match_expression(expr, 1)
        assert v == C.variant("clamp" if op == "hardtanh" else op), (op, expr)
        assert p0 == np.float32(p[0])
        if len(p) > 1:
            assert p1 == np.float32(p[1])
    assert C.match_expression("A*B+1.f", 2)[0] == -1
    assert C.match_expression("(A + B)", 1)[0] == -1       # wrong arity
    assert C.match_expression("(log1pf(expf(1.00000000f*A))/2.00000000f)", 1)[0] == -1


def test_variant_names():
    assert C.variant("add") == 0 and C.variant("div0") == 3 and C.variant("gelu") == 17
    assert C.variant("sum") == 32 and C.variant("mean") == 33 and C.variant("nope") == -1


def test_workload_shapes():
    st = W.mixed_24op(n_req=300, seed=0)
    assert len(st.requests) == 300
    sizes = [r.out.shape[0] for r in st.requests]
    assert min(sizes) >= 256 and max(sizes) <= 32768
    assert {r.stream_op for r in st.requests} <= {m[0] for m in W.MIXED_OPS}
    for r in st.requests:
        if r.stream_op in ("log", "sqrt", "pow"):
            assert float(r.a.view(st.host_in).min()) > 0
        if r.stream_op == "div":
            assert float(r.b.view(st.host_in).abs().min()) >= 0.1
    c1 = W.micro_add_mul(n_req=8)
    assert [r.op for r in c1.requests] == ["add", "mul"] * 4
    assert c1.algo_bytes == 8 * 4096 * 12


def test_custom_expression_compile_check():
    """NVRTC compiles custom expressions on the host (no GPU needed)."""
    L = C.lib()
    assert L.gpuos_jit_check(b"A * A + 2.f * B", 2) == C.OK
    assert L.gpuos_jit_check(b"sinf(A) * 0.5f + expf(-A)", 1) == C.OK
    assert L.gpuos_jit_check(b"A +* B", 2) == C.ENVRTC
    assert "nvrtc" in L.gpuos_last_error().decode()
    assert L.gpuos_jit_check(b"A; }", 1) == C.EINVAL
    assert L.gpuos_jit_check(b"A // c", 1) == C.EINVAL
