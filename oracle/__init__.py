"""CPU oracle for the aggregated small-op path — TEST INFRASTRUCTURE ONLY.

A ctypes wrapper around liboracle.so (oracle.c), the plain-C restatement of
the reference's algorithm (see oracle.h for what is restated and where it
comes from).  Only tests/, __graft_entry__.smoke() and the CPU-baseline legs
of bench.py import this package, as the checker or as the timed CPU
baseline.  Tensors passed in are CPU torch tensors used as plain buffers; all
arithmetic happens in C.

Parity pins: tests/test_oracle.py checks this oracle against the known-answer
inputs of the reference's own tests and against tests/golden/*.json.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

VARIANTS = {
    "add": 0, "mul": 1, "sub": 2, "div0": 3, "div": 4, "maximum": 5, "minimum": 6,
    "pow": 7, "relu": 8, "sigmoid": 9, "tanh": 10, "exp": 11, "log": 12, "sqrt": 13,
    "abs": 14, "hardsigmoid": 15, "hardswish": 16, "gelu": 17, "sin": 18, "cos": 19,
    "leaky_relu": 20, "clamp": 21, "elu": 22, "softplus": 23, "clamp_min": 24,
    "clamp_max": 25, "copy": 26, "sum": 32, "mean": 33,
}
BINARY = {"add", "mul", "sub", "div0", "div", "maximum", "minimum", "pow"}
DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 4}


class OrTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8)]


class OrReq(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("variant", ctypes.c_int32), ("p0", ctypes.c_float),
                ("p1", ctypes.c_float), ("has_b", ctypes.c_int32), ("naxes", ctypes.c_int32),
                ("keepdim", ctypes.c_int32), ("axes", ctypes.c_int32 * 8), ("pad", ctypes.c_int32),
                ("a", OrTensor), ("b", OrTensor), ("out", OrTensor)]


_lib = None


def build():
    """Compile liboracle.so with the committed Makefile (gcc, no GPU)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.POINTER
        L.oracle_op1.restype = ctypes.c_float
        L.oracle_op1.argtypes = [ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                 ctypes.c_float]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        L.oracle_f16_to_f32.restype = ctypes.c_float
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_bf16_to_f32.restype = ctypes.c_float
        L.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_op1_exact.restype = ctypes.c_double
        L.oracle_op1_exact.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_double,
                                       ctypes.c_double, ctypes.c_double]
        for fn in (L.oracle_ew, L.oracle_ew_refindex, L.oracle_ew_exact):
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.c_int, ctypes.c_float, ctypes.c_float, P(OrTensor), P(OrTensor),
                           P(OrTensor)]
        L.oracle_reduce.restype = ctypes.c_int
        L.oracle_reduce.argtypes = [ctypes.c_int, P(OrTensor), P(OrTensor), P(ctypes.c_int32),
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_run.restype = ctypes.c_int
        L.oracle_run.argtypes = [P(OrReq), ctypes.c_int, ctypes.c_int]
        _lib = L
    return _lib


def desc(t: torch.Tensor) -> OrTensor:
    if t.device.type != "cpu":
        raise ValueError("the oracle works on CPU tensors")
    if t.dtype not in DTYPES:
        raise TypeError(f"unsupported dtype {t.dtype}")
    d = OrTensor()
    d.data = t.data_ptr() if t.numel() else None
    d.dtype = DTYPES[t.dtype]
    d.ndim = t.dim()
    for i in range(t.dim()):
        d.sizes[i] = t.size(i)
        d.strides[i] = t.stride(i)
    return d


def _vid(op) -> int:
    return VARIANTS[op] if isinstance(op, str) else int(op)


def ew(op, a, b, out, p0=0.0, p1=0.0, refindex=False, exact=False):
    """out = op(a[, b]) with torch broadcasting (refindex=True: the
    reference's own per-operand index decomposition; exact=True: the same
    formula in double precision into a float64 `out`)."""
    L = lib()
    fn = L.oracle_ew_exact if exact else (L.oracle_ew_refindex if refindex else L.oracle_ew)
    da, do = desc(a), desc(out)
    db = desc(b) if b is not None else None
    rc = fn(_vid(op), p0, p1, ctypes.byref(da), ctypes.byref(db) if db is not None else None,
            ctypes.byref(do))
    if rc != 0:
        raise ValueError("oracle: shapes do not broadcast")
    return out


def reduce(op, x, out, axes, keepdim, threads=256):
    L = lib()
    arr = (ctypes.c_int32 * 8)(*list(axes)[:8])
    rc = L.oracle_reduce(1 if _vid(op) == VARIANTS["mean"] else 0, ctypes.byref(desc(x)),
                         ctypes.byref(desc(out)), arr, len(axes), int(bool(keepdim)), threads)
    if rc != 0:
        raise ValueError("oracle: bad reduction axes")
    return out


def op1(op, a, b=0.0, p0=0.0, p1=0.0) -> float:
    return lib().oracle_op1(_vid(op), a, b, p0, p1)


def make_reqs(items):
    """items: list of (kind, op, p0, p1, a, b, out, axes, keepdim) with CPU tensors."""
    arr = (OrReq * len(items))()
    for i, (kind, op, p0, p1, a, b, out, axes, keepdim) in enumerate(items):
        q = arr[i]
        q.kind = kind
        q.variant = _vid(op)
        q.p0, q.p1 = p0, p1
        q.a = desc(a)
        q.has_b = 1 if b is not None else 0
        if b is not None:
            q.b = desc(b)
        q.out = desc(out)
        axes = list(axes or [])
        q.naxes = len(axes)
        for j, ax in enumerate(axes):
            q.axes[j] = ax
        q.keepdim = int(bool(keepdim))
    return arr


def run(reqs, nthreads=0) -> int:
    """Execute a request array from make_reqs; returns the threads used."""
    return lib().oracle_run(reqs, len(reqs), nthreads)
