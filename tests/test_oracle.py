"""The CPU oracle against the reference's known answers (CPU only).

These pin the oracle before it is trusted as the checker of the CUDA path:
the inputs of the reference's own tests (src/host.cpp, test/online_switch.cpp,
test/dual_slot_switch.cpp), fp16/bf16 rounding computed by numpy/torch, the
[B,1] broadcast example, and independent fp32/fp64 arithmetic.
"""
import hashlib
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tolerance import EXACT, check_transcendental

KAT = json.loads((Path(__file__).parent / "golden" / "kat.json").read_text())


def kat_inputs(k):
    n = k["n"]
    i = np.arange(n, dtype=np.int64)
    a = (np.float32(k["a"][0]) * i.astype(np.float32)).astype(np.float32)
    b = (np.float32(k["b"][0]) + (i % k["b"][1]).astype(np.float32)).astype(np.float32)
    return torch.from_numpy(a), torch.from_numpy(b)


@pytest.mark.parametrize("name", ["host_mul", "online_add", "online_mul", "dual_add", "dual_mul"])
def test_reference_test_vectors(name):
    k = KAT[name]
    a, b = kat_inputs(k)
    out = torch.empty_like(a)
    oracle.ew(k["op"], a, b, out)
    got = out.numpy()
    assert [int(x) for x in got[:16].view(np.uint32)] == k["head_bits"]
    assert hashlib.sha256(got.tobytes()).hexdigest() == k["sha256"]
    # the op_batch path (B != 0 division rule aside) is the same arithmetic
    out2 = torch.empty_like(a)
    oracle.ew({"add": "add", "mul": "mul"}[k["op"]], a, b, out2)
    assert torch.equal(out, out2)


def test_broadcast_column_operand():
    k = KAT["bcast_col"]
    a = torch.tensor(k["a"], dtype=torch.float32)
    c = torch.tensor(k["c"], dtype=torch.float32).reshape(-1, 1)
    out = torch.empty_like(a)
    oracle.ew("add", a, c, out)
    assert out.tolist() == k["torch"]
    oracle.ew("add", a, c, out, refindex=True)  # the reference's own decomposition
    assert out.tolist() == k["reference"]
    assert out[0].tolist() == [100.0, 201.0, 302.0, 103.0]


def test_refindex_agrees_where_reference_is_right():
    g = torch.Generator().manual_seed(0)
    a = torch.randn(6, 40, generator=g)
    row = torch.randn(40, generator=g)
    at = torch.randn(40, 6, generator=g).t()
    for x, y in ((a, row), (at, row), (a, a), (at, at)):
        o1, o2 = torch.empty(6, 40), torch.empty(6, 40)
        oracle.ew("mul", x, y, o1)
        oracle.ew("mul", x, y, o2, refindex=True)
        assert torch.equal(o1, o2)


def test_rounding_fixtures():
    k = KAT["round"]
    L = oracle.lib()
    vals = np.array(k["f32_bits"], dtype=np.uint32).view(np.float32)
    for v, h, bf in zip(vals, k["f16_bits"], k["bf16_bits"]):
        assert L.oracle_f32_to_f16(float(v)) == h, (v, h)
        assert L.oracle_f32_to_bf16(float(v)) == bf, (v, bf)


def test_rounding_exhaustive_against_torch():
    g = torch.Generator().manual_seed(1)
    x = torch.cat([torch.randn(20000, generator=g) * s for s in (1e-6, 1e-3, 1, 1e3, 6e4)])
    xb = x.view(torch.int32) ^ torch.randint(0, 2, x.shape, generator=g, dtype=torch.int32)
    x = xb.view(torch.float32)
    x = x[torch.isfinite(x)]
    for dt in (torch.float16, torch.bfloat16):
        ref = x.to(dt)
        out = torch.empty(x.shape, dtype=dt)
        oracle.ew("copy", x, None, out)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), dt
        back = torch.empty(x.shape, dtype=torch.float32)
        oracle.ew("copy", ref, None, back)
        assert torch.equal(back, ref.float())


def test_reduce_small_exact():
    k = KAT["reduce_small"]
    x = torch.tensor(k["x"], dtype=torch.float32)
    s = torch.empty(3)
    oracle.reduce("sum", x, s, [-1], False)
    assert s.tolist() == k["sum_last"]
    m = torch.empty(3, 1)
    oracle.reduce("mean", x, m, [1], True)
    assert m.reshape(-1).tolist() == k["mean_last"]
    s0 = torch.empty(5)
    oracle.reduce("sum", x, s0, [0], False)
    assert s0.tolist() == k["sum_first"]


def test_reduce_order_is_the_reference_tree():
    # thread-strided partial sums, then the pairwise shared-memory tree
    g = torch.Generator().manual_seed(2)
    x = torch.randn(3, 1000, generator=g)
    out = torch.empty(3)
    oracle.reduce("sum", x, out, [-1], False, threads=256)
    xs = x.numpy()
    for r in range(3):
        part = [np.float32(0)] * 256
        for t in range(256):
            acc = np.float32(0)
            for c in range(t, 1000, 256):
                acc = np.float32(acc + xs[r, c])
            part[t] = acc
        step = 128
        while step:
            for t in range(step):
                part[t] = np.float32(part[t] + part[t + step])
            step //= 2
        assert out[r].item() == float(part[0])


EXACT_NUMPY = {
    "add": lambda a, b: a + b, "mul": lambda a, b: a * b, "sub": lambda a, b: a - b,
    "div": lambda a, b: a / b, "maximum": lambda a, b: np.where(a > b, a, b),
    "minimum": lambda a, b: np.where(a < b, a, b), "relu": lambda a, b: np.where(a > 0, a, 0),
    "abs": lambda a, b: np.abs(a), "sqrt": lambda a, b: np.sqrt(a),
    "hardswish": lambda a, b: a * np.minimum(np.maximum(a / np.float32(6) + np.float32(0.5),
                                                        np.float32(0)), np.float32(1)),
}


@pytest.mark.parametrize("op", sorted(EXACT_NUMPY))
def test_exact_ops_against_numpy(op):
    g = torch.Generator().manual_seed(3)
    a = torch.randn(5000, generator=g)
    b = torch.randn(5000, generator=g)
    if op == "sqrt":
        a = a.abs() + 1e-3
    out = torch.empty(5000)
    oracle.ew(op, a, b, out)
    with np.errstate(all="ignore"):
        ref = EXACT_NUMPY[op](a.numpy(), b.numpy()).astype(np.float32)
    assert np.array_equal(out.numpy().view(np.uint32), ref.view(np.uint32)), op


def test_div0_rule():
    a = torch.tensor([1.0, 2.0, -3.0, 0.0])
    b = torch.tensor([0.0, 4.0, 0.0, 0.0])
    out = torch.empty(4)
    oracle.ew("div0", a, b, out)
    assert out.tolist() == [0.0, 0.5, 0.0, 0.0]
    oracle.ew("div", a[1:2], b[1:2], out[:1])
    assert out[0].item() == 0.5


def test_hardsigmoid_is_one_rounding():
    g = torch.Generator().manual_seed(4)
    a = torch.randn(4000, generator=g) * 4
    out = torch.empty(4000)
    oracle.ew("hardsigmoid", a, None, out)
    x = a.numpy().astype(np.float64)
    fused = (np.float64(np.float32(0.2)) * x + 0.5).astype(np.float32)
    ref = np.minimum(np.maximum(fused, 0), 1).astype(np.float32)
    assert np.array_equal(out.numpy(), ref)


PARAMS = {"leaky_relu": (0.01, 0.0), "clamp": (-0.5, 0.5), "elu": (1.0, 0.0), "softplus": (1.0, 0.0),
          "clamp_min": (-0.25, 0.0), "clamp_max": (0.25, 0.0)}


@pytest.mark.parametrize("op", ["exp", "log", "tanh", "sin", "cos", "pow", "sigmoid", "gelu", "elu",
                                "softplus"])
def test_transcendental_oracle_within_bounds(op):
    g = torch.Generator().manual_seed(5)
    a = torch.randn(20000, generator=g)
    b = torch.rand(20000, generator=g) * 1.5 + 0.5
    if op in ("log", "pow"):
        a = a.abs() + 1e-3
    p0, p1 = PARAMS.get(op, (0.0, 0.0))
    out = torch.empty(20000)
    oracle.ew(op, a, b, out, p0, p1)
    ex = torch.empty(20000, dtype=torch.float64)
    oracle.ew(op, a, b, ex, p0, p1, exact=True)
    ok, worst, i = check_transcendental(op, a.numpy(), b.numpy(), out.numpy(), ex.numpy(), p0, p1)
    # glibc's fp32 functions, not CUDA's: allow 1.5x the CUDA-derived bound
    assert worst <= 1.5, (op, worst, a[i].item(), out[i].item(), ex[i].item())


def test_param_ops():
    assert oracle.op1("leaky_relu", -2.0, 0, 0.01) == np.float32(np.float32(0.01) * np.float32(-2.0))
    assert oracle.op1("clamp", 3.0, 0, -0.5, 0.5) == 0.5
    assert oracle.op1("clamp_min", -3.0, 0, -0.25) == -0.25
    assert oracle.op1("clamp_max", 3.0, 0, 0.25) == 0.25
    assert oracle.op1("elu", 2.0, 0, 1.0) == 2.0
    assert abs(oracle.op1("softplus", 0.0, 0, 1.0) - math.log(2)) < 1e-6


def test_run_matches_single_calls():
    g = torch.Generator().manual_seed(6)
    items, refs = [], []
    for i in range(64):
        n = int(torch.randint(1, 3000, (1,), generator=g))
        a, b = torch.randn(n, generator=g), torch.randn(n, generator=g)
        op = ["add", "mul", "tanh", "gelu"][i % 4]
        out, ref = torch.empty(n), torch.empty(n)
        items.append((0, op, 0.0, 0.0, a, b if op in oracle.BINARY else None, out, None, False))
        oracle.ew(op, a, b if op in oracle.BINARY else None, ref)
        refs.append((out, ref))
    x = torch.randn(30, 70, generator=g)
    rout, rref = torch.empty(30), torch.empty(30)
    items.append((1, "mean", 0.0, 0.0, x, None, rout, [1], False))
    oracle.reduce("mean", x, rref, [1], False)
    refs.append((rout, rref))
    reqs = oracle.make_reqs(items)
    assert oracle.run(reqs, 4) == 4
    for out, ref in refs:
        assert torch.equal(out, ref)


def test_exact_set_is_documented():
    assert {"add", "mul", "sub", "div", "sqrt", "clamp"} <= EXACT
