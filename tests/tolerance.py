"""Tolerances of the parity tests, written out per operator.

* Exact operators (IEEE add/sub/mul/div/sqrt, comparisons, min/max, clamps,
  casts, and hardsigmoid/hardswish whose formulas are exact IEEE operations
  once the fused multiply-add is placed as the CUDA compiler places it) must
  match the oracle bit for bit.
* Transcendental operators are measured against the exact (double precision)
  value of the same formula: a CUDA math function contributes at most its
  documented maximum ulp error (CUDA Math API, single precision: expf 2,
  logf 1, log1pf 1, tanhf 2, sinf 2, cosf 2, powf 4), every fp32 operation
  half an ulp, propagated through the formula to the result.
* fp32 sum/mean: |got - exact| <= 1e-5 * sum|x| (relative error 1e-5 of the
  magnitude being summed).
"""
import numpy as np

EXACT = {"add", "mul", "sub", "div0", "div", "maximum", "minimum", "relu", "abs", "hardsigmoid",
         "hardswish", "leaky_relu", "clamp", "clamp_min", "clamp_max", "copy", "sqrt"}
TRANSCENDENTAL = {"exp", "log", "tanh", "sin", "cos", "pow", "sigmoid", "gelu", "elu", "softplus"}
CUDA_ULP = {"exp": 2.0, "log": 1.0, "log1p": 1.0, "tanh": 2.0, "sin": 2.0, "cos": 2.0, "pow": 4.0}
RED_REL = 1e-5


def ulp32(x):
    """float64 array: the fp32 ulp at |x|."""
    f = np.abs(np.asarray(x, dtype=np.float64)).astype(np.float32)
    return np.spacing(f).astype(np.float64)


def bound(op, A, B, exact, got, p0=0.0, p1=0.0):
    """Largest allowed |got - exact| for an fp32 result (float64 arrays)."""
    A = np.asarray(A, np.float64)
    B = np.asarray(B, np.float64)
    u = np.maximum(ulp32(exact), ulp32(got))
    if op in ("exp", "log", "tanh", "sin", "cos", "pow"):
        return (CUDA_ULP[op] + 0.01) * u
    if op == "sigmoid":
        e = np.exp(-A)
        s = 1.0 + e
        return 1.25 * ((CUDA_ULP["exp"] * ulp32(e) + 0.5 * ulp32(s)) / (s * s) + 0.5 * u)
    if op == "gelu":
        c1, c2 = float(np.float32(0.044715)), float(np.float32(0.79788456))
        p = c1 * A * A
        z = A + p * A
        uu = c2 * z
        t = np.tanh(uu)
        dz = np.abs(p * A) * 2.0 ** -22 + 0.5 * ulp32(z)
        du = c2 * dz + 0.5 * ulp32(uu)
        dt = (1.0 - t * t) * du + CUDA_ULP["tanh"] * ulp32(t)
        d1 = dt + 0.5 * ulp32(1.0 + t)
        return 1.5 * (0.5 * np.abs(A) * d1 + 0.5 * ulp32(0.5 * A) * np.abs(1.0 + t) + u)
    if op == "elu":
        e = np.exp(np.minimum(A, 0.0))
        d = CUDA_ULP["exp"] * ulp32(e) + 0.5 * ulp32(e - 1.0)
        return np.where(A > 0, 0.0, 1.25 * (abs(p0) * d + 0.5 * u))
    if op == "softplus":
        x = p0 * A
        e = np.exp(x)
        dx = 0.5 * ulp32(x)
        de = e * dx + CUDA_ULP["exp"] * ulp32(e)
        l = np.log1p(e)
        dl = de / (1.0 + e) + CUDA_ULP["log1p"] * ulp32(l)
        return 1.25 * (dl / abs(p0) + 0.5 * u)
    raise KeyError(op)


def check_transcendental(op, A, B, got, exact, p0=0.0, p1=0.0):
    """(ok, worst ratio of error to bound, index of worst element)."""
    got = np.asarray(got, np.float64).reshape(-1)
    exact = np.asarray(exact, np.float64).reshape(-1)
    A = np.asarray(A, np.float64).reshape(-1)
    B = np.asarray(B, np.float64).reshape(-1)
    err = np.abs(got - exact)
    both_inf = np.isinf(got) & np.isinf(exact) & (np.sign(got) == np.sign(exact))
    both_nan = np.isnan(got) & np.isnan(exact)
    err = np.where(both_inf | both_nan, 0.0, err)
    b = bound(op, A, B, exact, got, p0, p1) + 1e-45
    ratio = err / b
    i = int(np.nanargmax(ratio)) if ratio.size else 0
    worst = float(ratio[i]) if ratio.size else 0.0
    return bool(np.all(ratio <= 1.0)), worst, i


def ulp_distance_f32(a, b):
    """elementwise distance in fp32 ulps between two float32 arrays"""
    ai = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    bi = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7fffffff), ai)
    bi = np.where(bi < 0, -(bi & 0x7fffffff), bi)
    return np.abs(ai - bi)
