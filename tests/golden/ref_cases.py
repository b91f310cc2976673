"""The seeded cases whose outputs the reference's own GPU code recorded in
tests/golden/ref_gpu.npz (tests/golden/gen_ref_fixtures.py) — TEST
INFRASTRUCTURE.

Both the generator (run once on a B200 against oracle/_ref) and the parity
test (tests/test_ref_parity.py, against this repository's CUDA path) build
their inputs here, from numpy PCG64 streams seeded per case, so the two sides
see bit-identical inputs without the inputs being stored.

Case groups:
  ops        every operator of the 24-operator stream through the path the
             reference runs it on: add/sub/mul/div through op_batch (the
             builtin path, B == 0 -> 0) and every operator, those four
             included, through the reference's NVRTC elementwise operator
             with the scheduler's expression string.  Per operator: 64
             special values (zeros, denormals, infinities, NaN, the edges of
             expf's range, ...) and three ragged requests with the stream's
             value distribution (pytorch_ext/scheduler.py:145-153, 192-205,
             244-290 for the strings; the mixed-stream configuration for the
             distributions).
  lowp       transcendental operators on fp16 and bf16 tensors (cast-on-store).
  bcast      [B,N] op [N] and [B,N] op [B,1] with half the left operands
             transposed views, for the four dtype pairs of the broadcast
             configuration; op_batch for add/sub/mul/div, the elementwise
             operator for maximum/minimum.  The [B,1] cases record the
             reference's broadcast defect (its index decomposition uses the
             operand's own sizes, src/persistent_kernel.cu:20-31 after
             pytorch_ext/gpuos_ext.cpp:147-165).
  reduce     sum/mean, fp32 and bf16, contiguous rows (the reference's fast
             path) and transposed views and multi-axis reductions (its
             generic path), keepdim both ways (gpuos_ext.cpp:726-806).
  kat        the reference's own test inputs (src/host.cpp:219,
             test/online_switch.cpp:156, test/dual_slot_switch.cpp:138) on
             op_batch.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

UNARY = ["relu", "sigmoid", "tanh", "exp", "log", "sqrt", "abs", "sin", "cos", "gelu",
         "hardsigmoid", "hardswish", "leaky_relu", "hardtanh", "elu", "softplus", "clamp"]
BINARY = ["add", "sub", "mul", "div", "maximum", "minimum", "pow"]
# the executor / oracle operator (and parameters) each expression names
EXEC_OP = {
    "add": ("add", 0.0, 0.0), "sub": ("sub", 0.0, 0.0), "mul": ("mul", 0.0, 0.0),
    "div": ("div", 0.0, 0.0), "maximum": ("maximum", 0.0, 0.0), "minimum": ("minimum", 0.0, 0.0),
    "pow": ("pow", 0.0, 0.0), "relu": ("relu", 0.0, 0.0), "sigmoid": ("sigmoid", 0.0, 0.0),
    "tanh": ("tanh", 0.0, 0.0), "exp": ("exp", 0.0, 0.0), "log": ("log", 0.0, 0.0),
    "sqrt": ("sqrt", 0.0, 0.0), "abs": ("abs", 0.0, 0.0), "sin": ("sin", 0.0, 0.0),
    "cos": ("cos", 0.0, 0.0), "gelu": ("gelu", 0.0, 0.0),
    "hardsigmoid": ("hardsigmoid", 0.0, 0.0), "hardswish": ("hardswish", 0.0, 0.0),
    "leaky_relu": ("leaky_relu", 0.01, 0.0), "hardtanh": ("clamp", -1.0, 1.0),
    "elu": ("elu", 1.0, 0.0), "softplus": ("softplus", 1.0, 0.0), "clamp": ("clamp", -0.5, 0.5),
}
# op_batch's builtin op codes map to these executor operators (div: B == 0 -> 0)
OPBATCH_EXEC = {"add": "add", "sub": "sub", "mul": "mul", "div": "div0"}
# operators whose results are exact (bit-exact comparison); the rest are held
# to 2 fp32 ulp
EXACT = {"add", "sub", "mul", "div", "div0", "maximum", "minimum", "relu", "abs", "clamp", "sqrt",
         "hardtanh", "leaky_relu", "hardsigmoid", "hardswish", "copy"}

TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

SPECIALS = np.array([
    0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 2.0, -2.0, 1e-30, -1e-30, 1e-45, -1e-45, 1.17e-38, -1.17e-38,
    3.0e38, -3.0e38, np.inf, -np.inf, np.nan, 88.72, -88.72, 89.0, -103.0, -87.3, 10.0, -10.0,
    20.0, -20.0, 0.1, -0.1, 1e-7, -1e-7, 3.14159265, -3.14159265, 1e4, -1e4, 1e10, -1e10,
    0.99999, 1.00001, 6.0, -6.0, 3.0, -3.0, 2.5, -2.5, 1.5, -1.5, 0.01, -0.01, 100.0, -100.0,
    1e20, -1e20, 0.7853982, -0.7853982, 1.5707964, 4.0, -4.0, 9.0, 15.5, -15.5, 0.25, -0.25,
], dtype=np.float32)


@dataclass
class Arg:
    shape: tuple            # the logical shape
    dtype: str = "f32"
    dist: str = "normal"
    transposed: bool = False  # 2-D: storage [shape[1], shape[0]] viewed through .t()


@dataclass
class Case:
    name: str
    path: str               # "opbatch", "ew" or "red"
    op: str                 # opbatch: add/sub/mul/div; ew: expression name; red: sum/mean
    a: Arg
    b: Arg | None
    out_shape: tuple
    out_dtype: str
    seed: int
    axes: tuple = ()
    keepdim: bool = False
    meta: dict = field(default_factory=dict)

    @property
    def exec_op(self):
        """(executor operator, p0, p1) this case runs on our side."""
        if self.path == "opbatch":
            return OPBATCH_EXEC[self.op], 0.0, 0.0
        if self.path == "red":
            return self.op, 0.0, 0.0
        return EXEC_OP[self.op]


def _values(rng, n, dist):
    if dist == "normal":
        return rng.standard_normal(n).astype(np.float32)
    if dist == "absplus":            # log / sqrt / pow base: |x| + 1e-3
        return (np.abs(rng.standard_normal(n)) + 1e-3).astype(np.float32)
    if dist == "den":                # div denominators: sign(y) (|y| + 0.1)
        y = rng.standard_normal(n)
        return (np.where(y >= 0, 1.0, -1.0) * (np.abs(y) + 0.1)).astype(np.float32)
    if dist == "powexp":             # pow exponent U[0.5, 2]
        return (rng.random(n) * 1.5 + 0.5).astype(np.float32)
    if dist == "u1":
        return (rng.random(n) * 2 - 1).astype(np.float32)
    if dist == "u2":                 # broadcast configuration: U[-2, 2]
        return (rng.random(n) * 4 - 2).astype(np.float32)
    if dist == "u2den":
        y = rng.random(n) * 4 - 2
        return np.where(np.abs(y) < 0.05, 0.5, y).astype(np.float32)
    if dist == "specials":
        return SPECIALS[:n].copy()
    if dist == "specials_perm":
        return SPECIALS[rng.permutation(len(SPECIALS))][:n].copy()
    if dist.startswith("kat"):
        # kat:scale:mod:offset -> A[i] = scale * i (mod == 0) or offset + (i % mod)
        _, scale, mod, off = dist.split(":")
        i = np.arange(n, dtype=np.int64)
        if int(mod) == 0:
            return (np.float32(float(scale)) * i.astype(np.float32)).astype(np.float32)
        return (np.float32(float(off)) + (i % int(mod)).astype(np.float32)).astype(np.float32)
    raise KeyError(dist)


def make_tensor(arg: Arg, rng, device) -> torch.Tensor:
    """A tensor with `arg`'s shape, dtype, values and layout (values drawn as
    fp32, then rounded to the dtype)."""
    n = int(np.prod(arg.shape)) if arg.shape else 1
    v = torch.from_numpy(_values(rng, n, arg.dist))
    dt = TDT[arg.dtype]
    if arg.transposed:
        R, C = arg.shape
        base = v.reshape(C, R).to(dt).to(device)
        return base.t()
    return v.reshape(arg.shape).to(dt).to(device)


def make_inputs(case: Case, device):
    rng = np.random.default_rng(case.seed)
    a = make_tensor(case.a, rng, device)
    b = make_tensor(case.b, rng, device) if case.b is not None else None
    return a, b


def _dist_a(op):
    return "absplus" if op in ("log", "sqrt", "pow") else "normal"


def _dist_b(op):
    return {"div": "den", "pow": "powexp"}.get(op, "normal")


def cases():
    out = []
    seed = 1000
    sizes = (257, 1031, 2053)

    def add(**kw):
        nonlocal seed
        seed += 1
        out.append(Case(seed=seed, **kw))

    # ops: every operator through the elementwise JIT operator; add/sub/mul/div
    # also through op_batch
    for op in BINARY + UNARY:
        paths = ["ew"] + (["opbatch"] if op in ("add", "sub", "mul", "div") else [])
        for path in paths:
            binary = op in BINARY
            add(name=f"ops/{path}/{op}/specials", path=path, op=op,
                a=Arg((64,), dist="specials"),
                b=Arg((64,), dist="specials_perm") if binary else None,
                out_shape=(64,), out_dtype="f32")
            for n in sizes:
                add(name=f"ops/{path}/{op}/n{n}", path=path, op=op, a=Arg((n,), dist=_dist_a(op)),
                    b=Arg((n,), dist=_dist_b(op)) if binary else None,
                    out_shape=(n,), out_dtype="f32")
    # lowp: transcendental operators on fp16 / bf16 (C5's bf16 sigmoid / pow)
    for op in ("sigmoid", "exp", "tanh", "gelu", "pow", "softplus"):
        for dt in ("f16", "bf16"):
            binary = op in BINARY
            add(name=f"lowp/{op}/{dt}", path="ew", op=op, a=Arg((1031,), dt, _dist_a(op)),
                b=Arg((1031,), dt, _dist_b(op)) if binary else None,
                out_shape=(1031,), out_dtype=dt)
    # bcast: the broadcast configuration's shapes and dtype pairs, smaller
    pairs = [("f32", "f32"), ("f16", "f32"), ("bf16", "bf16"), ("f16", "f16")]
    promote = {("f32", "f32"): "f32", ("f16", "f32"): "f32", ("bf16", "bf16"): "bf16",
               ("f16", "f16"): "f16"}
    rng = np.random.default_rng(77)
    for da, db in pairs:
        for op in ("add", "sub", "mul", "div", "maximum", "minimum"):
            path = "opbatch" if op in ("add", "sub", "mul", "div") else "ew"
            for col in (False, True):
                for trans in (False, True):
                    B = int(rng.integers(1, 9))
                    N = int(rng.integers(64, 161))
                    bshape = (B, 1) if col else (N,)
                    add(name=f"bcast/{da}{db}/{op}/{'col' if col else 'row'}/{'t' if trans else 'c'}",
                        path=path, op=op, a=Arg((B, N), da, "u2", trans),
                        b=Arg(bshape, db, "u2den" if op == "div" else "u2"),
                        out_shape=(B, N), out_dtype=promote[(da, db)],
                        meta={"d1": col and B > 1})
    # reduce
    shapes = [(1, 64), (7, 1000), (33, 5000), (100, 300), (3, 20000), (64, 4096)]
    for op in ("sum", "mean"):
        for dt in ("f32", "bf16"):
            for (R, C) in shapes:
                for trans in (False, True):
                    keep = (R + C + trans) % 2 == 0
                    add(name=f"reduce/{op}/{dt}/{R}x{C}/{'t' if trans else 'c'}", path="red", op=op,
                        a=Arg((R, C), dt, "normal", trans), b=None,
                        out_shape=(R, 1) if keep else (R,), out_dtype=dt, axes=(1,), keepdim=keep)
        for axes, keep in (((0, 1), False), ((0, 1), True), ((0, 2), False)):
            shp = (4, 6, 50)
            o = tuple(1 if i in axes else s for i, s in enumerate(shp)) if keep else \
                tuple(s for i, s in enumerate(shp) if i not in axes)
            add(name=f"reduce/{op}/f32/4x6x50/axes{''.join(map(str, axes))}{'k' if keep else ''}",
                path="red", op=op, a=Arg(shp), b=None, out_shape=o, out_dtype="f32",
                axes=axes, keepdim=keep)
    # kat: the reference tests' inputs on op_batch
    for name, op, da, dbb in (("host_mul", "mul", "kat:0.5:0:0", "kat:0:7:2"),
                              ("online_add", "add", "kat:0.5:0:0", "kat:0:5:1"),
                              ("online_mul", "mul", "kat:0.5:0:0", "kat:0:5:1"),
                              ("dual_add", "add", "kat:0.3:0:0", "kat:0:9:2"),
                              ("dual_mul", "mul", "kat:0.3:0:0", "kat:0:9:2")):
        add(name=f"kat/{name}", path="opbatch", op=op, a=Arg((4096,), dist=da),
            b=Arg((4096,), dist=dbb), out_shape=(4096,), out_dtype="f32")
    names = [c.name for c in out]
    assert len(names) == len(set(names))
    return out
