"""Seeded synthetic request streams with the shapes, sizes and value
distributions of the reference's benchmark configurations.

  micro_add_mul   1024 fp32 requests alternating add/mul, 4096 contiguous
                  elements each, U[-1, 1]
  mixed_24op      16384 fp32 requests over the 24 operators below, sizes
                  log-uniform in [256, 32768], N(0, 1) with the domain
                  transforms of each operator, flushed in batches of 512
  broadcast_mixed 8192 [B,N] op [N] / [B,N] op [B,1] requests, half of the
                  left operands transposed views, mixed dtypes
  lastdim_reduce  4096 sum/mean requests over the last dim of [R, C],
                  half transposed, fp32 and bf16

All tensors of a stream are views into one byte slab, so a stream moves
between host and device with one copy each way.  Nothing here executes a
request: `submit` hands every request to a gpuos_ext-compatible module.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

# The reference scheduler's expression strings (pytorch_ext/scheduler.py:
# 145-153, 192-205, 244-290): the operator contract of register_elementwise.
EXPR = {
    "add": ("(A + B)", 2), "sub": ("(A - B)", 2), "mul": ("(A * B)", 2), "div": ("(A / B)", 2),
    "maximum": ("(A > B ? A : B)", 2), "minimum": ("(A < B ? A : B)", 2),
    "pow": ("powf(A, B)", 2),
    "relu": ("(A > 0.f ? A : 0.f)", 1), "sigmoid": ("1.f / (1.f + expf(-A))", 1),
    "tanh": ("tanhf(A)", 1), "exp": ("expf(A)", 1), "log": ("logf(A)", 1),
    "sqrt": ("sqrtf(A)", 1), "abs": ("fabsf(A)", 1),
    "hardsigmoid": ("fminf(fmaxf(0.2f*A + 0.5f, 0.f), 1.f)", 1),
    "hardswish": ("A * fminf(fmaxf(A/6.f + 0.5f, 0.f), 1.f)", 1),
    "gelu": ("0.5f * A * (1.f + tanhf(0.79788456f*(A + 0.044715f*A*A*A)))", 1),
    "sin": ("sinf(A)", 1), "cos": ("cosf(A)", 1),
}


def param_expr(op: str, p0: float, p1: float = 0.0):
    """Expression string (and key) the reference scheduler builds for a
    parametric operator (scheduler.py:244-290)."""
    f = lambda v: f"{float(v):.8f}f"  # noqa: E731
    if op == "leaky_relu":
        return f"(A >= 0.f ? A : {f(p0)}*A)", f"leaky_relu|f32|{p0:.8f}"
    if op in ("clamp", "hardtanh"):
        return f"fminf(fmaxf(A, {f(p0)}), {f(p1)})", f"{op}|f32|{p0:.8f}|{p1:.8f}"
    if op == "elu":
        return f"(A > 0.f ? A : {f(p0)}*(expf(A) - 1.f))", f"elu|f32|{p0:.8f}"
    if op == "softplus":
        return f"(log1pf(expf({f(p0)}*A))/{f(p0)})", f"softplus|f32|{p0:.8f}"
    if op == "clamp_min":
        return f"fmaxf(A, {f(p0)})", f"clamp_min|f32|{p0:.8f}"
    if op == "clamp_max":
        return f"fminf(A, {f(p0)})", f"clamp_max|f32|{p0:.8f}"
    raise KeyError(op)


# oracle / executor operator name of each stream operator, and its parameters
MIXED_OPS = [
    ("add", "add", 0.0, 0.0), ("sub", "sub", 0.0, 0.0), ("mul", "mul", 0.0, 0.0),
    ("div", "div0", 0.0, 0.0), ("maximum", "maximum", 0.0, 0.0), ("minimum", "minimum", 0.0, 0.0),
    ("pow", "pow", 0.0, 0.0), ("relu", "relu", 0.0, 0.0), ("sigmoid", "sigmoid", 0.0, 0.0),
    ("tanh", "tanh", 0.0, 0.0), ("exp", "exp", 0.0, 0.0), ("log", "log", 0.0, 0.0),
    ("sqrt", "sqrt", 0.0, 0.0), ("abs", "abs", 0.0, 0.0), ("sin", "sin", 0.0, 0.0),
    ("cos", "cos", 0.0, 0.0), ("gelu", "gelu", 0.0, 0.0), ("hardsigmoid", "hardsigmoid", 0.0, 0.0),
    ("hardswish", "hardswish", 0.0, 0.0), ("leaky_relu", "leaky_relu", 0.01, 0.0),
    ("hardtanh", "clamp", -1.0, 1.0), ("elu", "elu", 1.0, 0.0), ("softplus", "softplus", 1.0, 0.0),
    ("clamp", "clamp", -0.5, 0.5),
]
BINARY = {"add", "sub", "mul", "div", "maximum", "minimum", "pow"}
BUILTIN_SUBMIT = {"add": "submit_add", "sub": "submit_sub", "mul": "submit_mul", "div": "submit_div"}

_ESZ = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}


class Slab:
    """Bump allocator of tensor views inside one byte buffer."""

    def __init__(self):
        self.chunks = []
        self.size = 0

    def alloc(self, nbytes: int, align: int = 256) -> int:
        off = (self.size + align - 1) // align * align
        self.size = off + nbytes
        return off


@dataclass
class TensorSpec:
    off: int
    dtype: torch.dtype
    shape: tuple
    strides: tuple

    def view(self, buf: torch.Tensor) -> torch.Tensor:
        n = 1
        for s, st in zip(self.shape, self.strides):
            n += (s - 1) * st if s > 0 else 0
        nb = n * _ESZ[self.dtype]
        return buf[self.off:self.off + nb].view(self.dtype).as_strided(self.shape, self.strides)

    @property
    def nbytes_unique(self) -> int:
        n = 1
        for s, st in zip(self.shape, self.strides):
            if st != 0:
                n *= s
        return n * _ESZ[self.dtype]


@dataclass
class Request:
    stream_op: str          # the name in the stream definition
    op: str                 # oracle / executor operator name
    p0: float
    p1: float
    a: TensorSpec
    b: TensorSpec | None
    out: TensorSpec
    kind: str = "ew"        # "ew" or "reduce"
    axes: tuple = ()
    keepdim: bool = False

    @property
    def algo_bytes(self) -> int:
        """unique input elements + output elements, times element sizes"""
        n = self.a.nbytes_unique + self.out.nbytes_unique
        if self.b is not None:
            n += self.b.nbytes_unique
        return n


@dataclass
class Stream:
    name: str
    requests: list
    in_bytes: int
    out_bytes: int
    host_in: torch.Tensor       # byte slab with the inputs (CPU)
    flush_every: int
    meta: dict = field(default_factory=dict)

    @property
    def algo_bytes(self) -> int:
        return sum(r.algo_bytes for r in self.requests)

    def batch_spans(self):
        """Per flush group of `flush_every` requests: the byte ranges
        (in_lo, in_hi, out_lo, out_hi) of the two slabs its tensors cover.
        Slabs are allocated in request order, so the groups' ranges follow
        one another."""
        return self.batch_spans_of(self.requests)

    def batch_spans_of(self, requests):
        def span(t: TensorSpec):
            n = 1
            for sz, st in zip(t.shape, t.strides):
                n += (sz - 1) * st if sz > 0 else 0
            return t.off, t.off + n * _ESZ[t.dtype]
        res = []
        fe = self.flush_every
        for i in range(0, len(requests), fe):
            ilo = olo = 1 << 62
            ihi = ohi = 0
            for r in requests[i:i + fe]:
                for t in (r.a, r.b):
                    if t is not None:
                        lo, hi = span(t)
                        ilo, ihi = min(ilo, lo), max(ihi, hi)
                lo, hi = span(r.out)
                olo, ohi = min(olo, lo), max(ohi, hi)
            res.append((ilo, ihi, olo, ohi))
        return res

    def head(self, n: int) -> "Stream":
        """The stream of its first n requests, with the slabs cut to what those
        requests use (slabs are allocated in request order)."""
        reqs = self.requests[:n]
        spans = self.batch_spans_of(reqs)
        in_end = max(s[1] for s in spans) if reqs else 0
        out_end = max(s[3] for s in spans) if reqs else 0
        host = self.host_in[:in_end] if self.host_in is not None else None
        return Stream(self.name, reqs, in_end, out_end, host, self.flush_every, dict(self.meta))

    def device_buffers(self, device, pin=False):
        """(inputs, outputs) byte slabs on `device` with the inputs copied (or,
        for a stream built without host values, drawn on the device)."""
        dout = torch.zeros(self.out_bytes, dtype=torch.uint8, device=device)
        if self.host_in is None:
            return self.device_inputs(device), dout
        din = self.host_in.to(device)
        return din, dout

    def device_inputs(self, device, seed=0):
        """The input slab drawn on the device: every input view gets the
        stream's value distribution (meta["dist"]: "normal" or "u2"), from a
        device generator.  For timing runs of streams too large to draw on
        the host; the values differ from the host-built stream's."""
        din = torch.empty(self.in_bytes, dtype=torch.uint8, device=device)
        g = torch.Generator(device=device).manual_seed(seed)
        dist = self.meta.get("dist", "normal")
        for r in self.requests:
            for t in (r.a, r.b):
                if t is None:
                    continue
                v = t.view(din)
                x = torch.randn(v.shape, generator=g, device=device) if dist == "normal" else \
                    torch.rand(v.shape, generator=g, device=device) * 4 - 2
                v.copy_(x)
        return din

    def views(self, din, dout):
        """per request (a, b, out) tensor views into the two slabs"""
        res = []
        for r in self.requests:
            a = r.a.view(din)
            b = r.b.view(din) if r.b is not None else None
            res.append((a, b, r.out.view(dout)))
        return res


def _contig(off, dtype, shape):
    st, acc = [], 1
    for s in reversed(shape):
        st.append(acc)
        acc *= s
    return TensorSpec(off, dtype, tuple(shape), tuple(reversed(st)))


def _fill(buf: torch.Tensor, spec: TensorSpec, values: torch.Tensor):
    spec.view(buf).copy_(values.reshape(spec.shape))


def micro_add_mul(n_req=1024, numel=4096, seed=0) -> Stream:
    g = torch.Generator().manual_seed(seed)
    si, so = Slab(), Slab()
    reqs = []
    for i in range(n_req):
        op = "add" if i % 2 == 0 else "mul"
        a = _contig(si.alloc(numel * 4), torch.float32, (numel,))
        b = _contig(si.alloc(numel * 4), torch.float32, (numel,))
        o = _contig(so.alloc(numel * 4), torch.float32, (numel,))
        reqs.append(Request(op, op, 0.0, 0.0, a, b, o))
    buf = torch.empty(si.size, dtype=torch.uint8)
    for r in reqs:
        _fill(buf, r.a, torch.rand(numel, generator=g) * 2 - 1)
        _fill(buf, r.b, torch.rand(numel, generator=g) * 2 - 1)
    return Stream("micro_add_mul", reqs, si.size, so.size, buf, flush_every=n_req,
                  meta={"requests": n_req, "numel": numel, "dtype": "f32"})


def mixed_24op(n_req=16384, seed=0, lo=256, hi=32768, flush_every=512) -> Stream:
    g = torch.Generator().manual_seed(seed)
    sizes = torch.exp(torch.rand(n_req, generator=g, dtype=torch.float64) *
                      (math.log(hi) - math.log(lo)) + math.log(lo)).floor().long().clamp(lo, hi)
    ops = torch.randint(0, len(MIXED_OPS), (n_req,), generator=g)
    si, so = Slab(), Slab()
    reqs = []
    for i in range(n_req):
        n = int(sizes[i])
        sop, op, p0, p1 = MIXED_OPS[int(ops[i])]
        a = _contig(si.alloc(n * 4), torch.float32, (n,))
        b = _contig(si.alloc(n * 4), torch.float32, (n,)) if sop in BINARY else None
        o = _contig(so.alloc(n * 4), torch.float32, (n,))
        reqs.append(Request(sop, op, p0, p1, a, b, o))
    buf = torch.empty(si.size, dtype=torch.uint8)
    for r in reqs:
        n = r.a.shape[0]
        x = torch.randn(n, generator=g)
        if r.stream_op in ("log", "sqrt"):
            x = x.abs() + 1e-3
        if r.stream_op == "pow":
            x = x.abs() + 1e-3
        _fill(buf, r.a, x)
        if r.b is not None:
            y = torch.randn(n, generator=g)
            if r.stream_op == "div":
                y = torch.sign(y) * (y.abs() + 0.1)
                y[y == 0] = 0.1
            if r.stream_op == "pow":
                y = torch.rand(n, generator=g) * 1.5 + 0.5
            _fill(buf, r.b, y)
    return Stream("mixed_24op", reqs, si.size, so.size, buf, flush_every=flush_every,
                  meta={"requests": n_req, "sizes": [lo, hi], "dtype": "f32", "ops": 24})


BCAST_DTYPES = [(torch.float32, torch.float32), (torch.float16, torch.float32),
                (torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16)]
BCAST_OPS = [("add", "add"), ("sub", "sub"), ("mul", "mul"), ("div", "div0"),
             ("maximum", "maximum"), ("minimum", "minimum")]


def broadcast_mixed(n_req=8192, seed=0, flush_every=512, fill=True) -> Stream:
    g = torch.Generator().manual_seed(seed)
    si, so = Slab(), Slab()
    reqs = []
    for i in range(n_req):
        B = int(torch.randint(1, 65, (1,), generator=g))
        N = int(torch.randint(64, 4097, (1,), generator=g))
        col = bool(torch.randint(0, 2, (1,), generator=g))
        trans = bool(torch.randint(0, 2, (1,), generator=g))
        da, db = BCAST_DTYPES[int(torch.randint(0, 4, (1,), generator=g))]
        sop, op = BCAST_OPS[int(torch.randint(0, 6, (1,), generator=g))]
        dout = torch.promote_types(da, db)
        if trans:
            base = si.alloc(B * N * _ESZ[da])
            a = TensorSpec(base, da, (B, N), (1, B))      # [N, B] storage seen as [B, N]
        else:
            a = _contig(si.alloc(B * N * _ESZ[da]), da, (B, N))
        if col:
            b = _contig(si.alloc(B * _ESZ[db]), db, (B, 1))
        else:
            b = _contig(si.alloc(N * _ESZ[db]), db, (N,))
        o = _contig(so.alloc(B * N * _ESZ[dout]), dout, (B, N))
        reqs.append(Request(sop, op, 0.0, 0.0, a, b, o))
    if not fill:
        return Stream("broadcast_mixed", reqs, si.size, so.size, None, flush_every=flush_every,
                      meta={"requests": n_req, "dist": "u2", "dtype": "f32/f16/bf16"})
    buf = torch.empty(si.size, dtype=torch.uint8)
    for r in reqs:
        B, N = r.out.shape
        _fill(buf, r.a, (torch.rand(B * N, generator=g) * 4 - 2).to(r.a.dtype))
        nb = B if r.b.shape == (B, 1) else N
        y = (torch.rand(nb, generator=g) * 4 - 2)
        if r.stream_op == "div":
            y = torch.where(y.abs() < 0.05, torch.full_like(y, 0.5), y)
        _fill(buf, r.b, y.to(r.b.dtype))
    return Stream("broadcast_mixed", reqs, si.size, so.size, buf, flush_every=flush_every,
                  meta={"requests": n_req, "dist": "u2", "dtype": "f32/f16/bf16"})


def lastdim_reduce(n_req=4096, seed=0, flush_every=512, max_elems=1 << 24, fill=True) -> Stream:
    g = torch.Generator().manual_seed(seed)
    si, so = Slab(), Slab()
    reqs = []
    for i in range(n_req):
        R = int(math.exp(float(torch.rand(1, generator=g)) * math.log(4096)))
        C = int(math.exp(float(torch.rand(1, generator=g)) * (math.log(32768) - math.log(64)) +
                         math.log(64)))
        R = max(1, min(R, max_elems // C))
        dt = torch.float32 if bool(torch.randint(0, 2, (1,), generator=g)) else torch.bfloat16
        trans = bool(torch.randint(0, 2, (1,), generator=g))
        mean = bool(torch.randint(0, 2, (1,), generator=g))
        keep = bool(torch.randint(0, 2, (1,), generator=g))
        off = si.alloc(R * C * _ESZ[dt])
        x = TensorSpec(off, dt, (R, C), (1, R)) if trans else _contig(off, dt, (R, C))
        o = _contig(so.alloc(R * _ESZ[dt]), dt, (R, 1) if keep else (R,))
        op = "mean" if mean else "sum"
        reqs.append(Request(op, op, 0.0, 0.0, x, None, o, kind="reduce", axes=(1,), keepdim=keep))
    if not fill:
        return Stream("lastdim_reduce", reqs, si.size, so.size, None, flush_every=flush_every,
                      meta={"requests": n_req, "dist": "normal", "dtype": "f32/bf16"})
    buf = torch.empty(si.size, dtype=torch.uint8)
    for r in reqs:
        R, C = r.a.shape
        _fill(buf, r.a, torch.randn(R * C, generator=g).to(r.a.dtype))
    return Stream("lastdim_reduce", reqs, si.size, so.size, buf, flush_every=flush_every,
                  meta={"requests": n_req, "dist": "normal", "dtype": "f32/bf16"})


STREAMS = {
    "micro_add_mul": micro_add_mul,
    "mixed_24op": mixed_24op,
    "broadcast_mixed": broadcast_mixed,
    "lastdim_reduce": lastdim_reduce,
}


class Submitter:
    """Routes requests through a gpuos_ext-compatible module the way the
    reference's benchmark harness does: add/sub/mul/div through submit_*
    (op_batch), every other operator through a register_elementwise slot
    with the reference scheduler's expression string, reductions through
    register_reduce / submit_reduce."""

    def __init__(self, ext):
        self.ext = ext
        self.slots = {}

    def slot_for(self, r: Request) -> int:
        key = (r.stream_op, r.p0, r.p1, r.kind)
        s = self.slots.get(key)
        if s is None:
            if r.kind == "reduce":
                s = self.ext.register_reduce(f"reduce_{r.op}", r.op)
            elif r.stream_op in EXPR:
                expr, ar = EXPR[r.stream_op]
                s = self.ext.register_elementwise(f"{r.stream_op}|f32", expr, ar)
            else:
                expr, k = param_expr(r.op if r.stream_op != "hardtanh" else "hardtanh", r.p0, r.p1)
                s = self.ext.register_elementwise(k, expr, 1)
            self.slots[key] = s
        return s

    def prepare(self, stream: Stream, views):
        """Resolve slots and bind the submit call of every request once."""
        ext = self.ext
        calls = []
        for r, (a, b, o) in zip(stream.requests, views):
            if r.kind == "reduce":
                calls.append((ext.submit_reduce, (self.slot_for(r), a, o, list(r.axes), r.keepdim)))
            elif r.stream_op in BUILTIN_SUBMIT:
                calls.append((getattr(ext, BUILTIN_SUBMIT[r.stream_op]), (a, b, o)))
            elif b is not None:
                calls.append((ext.submit_binary, (self.slot_for(r), a, b, o)))
            else:
                calls.append((ext.submit_unary, (self.slot_for(r), a, o)))
        return calls
