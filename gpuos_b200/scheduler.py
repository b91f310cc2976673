"""TorchDispatch scheduler: route small CUDA tensor ops to the aggregated
executor while the context is active.

Same interface as the reference's ``pytorch_ext/scheduler.py``:
``GPUOSScheduler(capacity=8192, threads_per_block=256, size_threshold=1 << 16,
auto_flush_ms=2.0)`` (``__enter__`` initialises the executor, ``flush(sync)``,
``__exit__`` flushes synchronously and shuts down), ``scheduler_context(...)``,
and the environment switch ``GPUOS_SCHEDULER_DISABLE_JIT`` (default ``'1'``,
scheduler.py:19; read when the context is entered).

* JIT switch off (the reference's default): only ``aten::add/sub/mul/div.Tensor``
  of two CUDA tensors are scheduled, through ``submit_add/sub/mul/div``
  (scheduler.py:125-143); everything else runs in torch.
* JIT switch on: the binary ops ``maximum``, ``minimum``, ``pow.Tensor_Tensor``,
  the unary ops, the parametric ones (``leaky_relu``, ``hardtanh``, ``elu``,
  ``softplus``, ``clamp*``) and ``sum.dim_IntList`` / ``mean.dim`` are also
  scheduled, with the reference's expression strings (scheduler.py:145-153,
  192-205, 244-290) registered through ``register_elementwise``.

Every scheduled op writes the tensor it returns.  The reference defers
binary and unary results into "fused" nodes that it later computes into a
freshly allocated tensor, so the returned tensor never receives the result
(scheduler.py:118, 157-160, 349-358), and it composes only a unary op on top
of one node (scheduler.py:213-222).  Here, with the JIT switch on (and
``GPUOS_SCHEDULER_FUSE`` not ``'0'``), an elementwise op whose input is the
result of an earlier elementwise op that has not been submitted yet inlines
that op's expression: ``torch.sigmoid(a * b) + c`` becomes one request,
``(gpuos_keep_f32(1.f / (1.f + expf(-(gpuos_keep_f32((A * B))))))) + C``
over the leaves a, b, c (up to four leaves: operands A..D of a custom
expression).  Each inlined intermediate is rounded as the unfused chain
would have stored it (``gpuos_keep_<dtype>``: its dtype's rounding, and for
fp32 no contraction into the consuming operation), so a fused chain gives
the unfused chain's values.  The ops are submitted when something needs
them: a reduction or a torch op that reads their memory, a flush, the end of
the context.  An intermediate whose tensor the caller no longer holds by then
is not written at all; one that is still held is written as well.  Without
fusion the executor still orders each request after the earlier requests of
the flush whose outputs it reads.

An op that is not scheduled and reads memory a pending request writes, or
writes memory a pending request reads or writes, forces a synchronous flush
first.  Pending requests are tracked by the byte ranges of their tensors in
their storages, so a slice, a transpose or any other view of a pending
tensor counts (the reference compares data_ptr values of pending outputs
only, scheduler.py:55-99, which misses views that start elsewhere).  Tensors larger than ``size_threshold``
elements, ops under autograd, CPU tensors, and ``add``/``sub`` with
``alpha != 1`` (which the reference ignores) run in torch.
"""
from __future__ import annotations

import contextlib
import os
import re
import sys
import threading
from typing import Any, Dict, List, Optional, Set, Tuple

import torch

from . import load as _load

def _jit_disabled() -> bool:
    return os.environ.get("GPUOS_SCHEDULER_DISABLE_JIT", "1") not in ("0", "false", "False")


def _fuse_enabled() -> bool:
    return os.environ.get("GPUOS_SCHEDULER_FUSE", "1") not in ("0", "false", "False")


_LETTERS = "ABCD"
_TOKEN = re.compile(r"\b([A-D])\b")
_KEEP = {torch.float32: "gpuos_keep_f32", torch.float16: "gpuos_keep_f16",
         torch.bfloat16: "gpuos_keep_bf16"}
_MAX_EXPR = 4000  # characters: an operand used twice doubles the text


def _rename(expr: str, mapping: Dict[str, str]) -> str:
    """Rename the operand letters of `expr` in one pass."""
    return _TOKEN.sub(lambda m: mapping.get(m.group(1), m.group(1)), expr)


class _Node:
    """An elementwise op not yet submitted: `expr` over the operand letters
    A.. (one per leaf tensor), writing `out`."""
    __slots__ = ("expr", "leaves", "out")

    def __init__(self, expr: str, leaves: List[torch.Tensor], out: torch.Tensor):
        self.expr = expr
        self.leaves = leaves
        self.out = out

_BINARY_BUILTIN = {
    "aten::add.Tensor": "submit_add",
    "aten::sub.Tensor": "submit_sub",
    "aten::mul.Tensor": "submit_mul",
    "aten::div.Tensor": "submit_div",
}
# scheduler.py:145-153
_BINARY_EXPR = {
    "aten::add.Tensor": "(A + B)",
    "aten::sub.Tensor": "(A - B)",
    "aten::mul.Tensor": "(A * B)",
    "aten::div.Tensor": "(A / B)",
    "aten::maximum": "(A > B ? A : B)",
    "aten::minimum": "(A < B ? A : B)",
    "aten::pow.Tensor_Tensor": "powf(A, B)",
}
# scheduler.py:192-205
_UNARY_EXPR = {
    "aten::relu": "(A > 0.f ? A : 0.f)",
    "aten::sigmoid": "1.f / (1.f + expf(-A))",
    "aten::tanh": "tanhf(A)",
    "aten::exp": "expf(A)",
    "aten::log": "logf(A)",
    "aten::sqrt": "sqrtf(A)",
    "aten::abs": "fabsf(A)",
    "aten::hardsigmoid": "fminf(fmaxf(0.2f*A + 0.5f, 0.f), 1.f)",
    "aten::hardswish": "A * fminf(fmaxf(A/6.f + 0.5f, 0.f), 1.f)",
    "aten::gelu": "0.5f * A * (1.f + tanhf(0.79788456f*(A + 0.044715f*A*A*A)))",
    "aten::sin": "sinf(A)",
    "aten::cos": "cosf(A)",
}
_PARAM_UNARY = ("aten::leaky_relu", "aten::hardtanh", "aten::elu", "aten::softplus",
                "aten::clamp", "aten::clamp_min", "aten::clamp_max")
_REDUCE = {"aten::sum.dim_IntList": "sum", "aten::mean.dim": "mean"}


def _scheduled_names(jit: bool) -> Set[str]:
    names = set(_BINARY_BUILTIN)
    if jit:
        names |= set(_BINARY_EXPR) | set(_UNARY_EXPR) | set(_PARAM_UNARY) | set(_REDUCE)
    return names


def _param_expr(name: str, args, kwargs) -> Optional[tuple]:
    """(key, expr) of a parametric unary op, or None to run it in torch
    (scheduler.py:244-290)."""
    def arg(i, key, default):
        v = kwargs.get(key, args[i] if len(args) > i else default)
        return float(default if v is None else v)

    if name == "aten::leaky_relu":
        ns = arg(1, "negative_slope", 0.01)
        return f"leaky_relu|f32|{ns:.8f}", f"(A >= 0.f ? A : {ns:.8f}f*A)"
    if name == "aten::hardtanh":
        mn, mx = arg(1, "min_val", -1.0), arg(2, "max_val", 1.0)
        return f"hardtanh|f32|{mn:.8f}|{mx:.8f}", f"fminf(fmaxf(A, {mn:.8f}f), {mx:.8f}f)"
    if name == "aten::elu":
        al = arg(1, "alpha", 1.0)
        return f"elu|f32|{al:.8f}", f"(A > 0.f ? A : {al:.8f}f*(expf(A) - 1.f))"
    if name == "aten::softplus":
        be = arg(1, "beta", 1.0)
        return f"softplus|f32|{be:.8f}", f"(log1pf(expf({be:.8f}f*A))/{be:.8f}f)"
    if name == "aten::clamp":
        mn, mx = kwargs.get("min"), kwargs.get("max")
        if mn is None or mx is None:
            return None
        mn, mx = float(mn), float(mx)
        return f"clamp|f32|{mn:.8f}|{mx:.8f}", f"fminf(fmaxf(A, {mn:.8f}f), {mx:.8f}f)"
    if name == "aten::clamp_min":
        mn = arg(1, "min", 0.0)
        return f"clamp_min|f32|{mn:.8f}", f"fmaxf(A, {mn:.8f}f)"
    if name == "aten::clamp_max":
        mx = arg(1, "max", 0.0)
        return f"clamp_max|f32|{mx:.8f}", f"fminf(A, {mx:.8f}f)"
    return None


def _extent(t: torch.Tensor) -> Optional[Tuple[int, int, int]]:
    """(storage address, first byte, one past the last byte) a tensor view
    covers in its storage, or None for an empty tensor."""
    if t.numel() == 0:
        return None
    lo = hi = t.storage_offset()
    for n, st in zip(t.shape, t.stride()):
        if n > 1:
            if st >= 0:
                hi += (n - 1) * st
            else:
                lo += (n - 1) * st
    es = t.element_size()
    return t.untyped_storage().data_ptr(), lo * es, (hi + 1) * es


def _overlaps(e, table) -> bool:
    if e is None:
        return False
    for lo, hi in table.get(e[0], ()):
        if e[1] < hi and lo < e[2]:
            return True
    return False


def _add(e, table):
    if e is not None:
        table.setdefault(e[0], []).append((e[1], e[2]))


class _GPUOSSchedulerMode(torch.utils._python_dispatch.TorchDispatchMode):
    def __init__(self, ext, *, size_threshold: int, auto_flush_ms: Optional[float],
                 pending: Set[int], jit: bool, fuse: bool = False):
        super().__init__()
        self.ext = ext
        self.fuse = jit and fuse
        # elementwise ops not yet submitted, by id of the tensor they return,
        # in the order they were made (with their slots)
        self._nodes: Dict[int, Tuple[_Node, int]] = {}
        self.size_threshold = size_threshold
        self.auto_flush_ms = auto_flush_ms
        self.pending = pending  # data_ptr of every output not yet flushed synchronously
        self.pending_in: Set[int] = set()  # data_ptr of their inputs
        # byte ranges the pending requests write / read, per storage
        self._w: Dict[int, List[Tuple[int, int]]] = {}
        self._r: Dict[int, List[Tuple[int, int]]] = {}
        self.jit = jit
        self._names = _scheduled_names(jit)
        self._stop = threading.Event()
        self._bg: Optional[threading.Thread] = None
        if auto_flush_ms and auto_flush_ms > 0:
            self._bg = threading.Thread(target=self._flusher, daemon=True)
            self._bg.start()

    def close(self):
        self._stop.set()
        if self._bg is not None:
            self._bg.join(timeout=1.0)

    def _flusher(self):
        # publish what is queued every auto_flush_ms (scheduler.py:40-51)
        while not self._stop.wait(self.auto_flush_ms / 1000.0):
            try:
                self.ext.flush(sync=False)
            except Exception:  # a failed batch surfaces at the next synchronous flush
                pass

    # ---- helpers -------------------------------------------------------------
    def _small_cuda(self, *ts) -> bool:
        if torch.is_grad_enabled():
            return False
        for t in ts:
            if not isinstance(t, torch.Tensor) or not t.is_cuda or t.numel() > self.size_threshold:
                return False
        return True

    def _reads_pending(self, args, kwargs) -> bool:
        """Does any CUDA tensor among the arguments overlap what a pending
        request writes?"""
        def walk(o: Any) -> bool:
            if isinstance(o, torch.Tensor):
                return o.is_cuda and _overlaps(_extent(o), self._w)
            if isinstance(o, (list, tuple)):
                return any(walk(i) for i in o)
            if isinstance(o, dict):
                return any(walk(v) for v in o.values())
            return False
        return walk(args) or walk(kwargs)

    def _writes_pending(self, func, args, kwargs) -> bool:
        """Does the op write memory a pending request reads or writes?"""
        for i, a in enumerate(func._schema.arguments):
            v = kwargs.get(a.name) if a.kwarg_only or i >= len(args) else args[i]
            if a.alias_info is not None and a.alias_info.is_write:
                ts = v if isinstance(v, (list, tuple)) else [v]
                for t in ts:
                    if isinstance(t, torch.Tensor) and t.is_cuda:
                        e = _extent(t)
                        if _overlaps(e, self._w) or _overlaps(e, self._r):
                            return True
        return False

    def _done(self, out: torch.Tensor, *inputs) -> torch.Tensor:
        self.pending.add(out.data_ptr())
        _add(_extent(out), self._w)
        for t in inputs:
            self.pending_in.add(t.data_ptr())
            _add(_extent(t), self._r)
        return out

    # ---- fused chains --------------------------------------------------------
    def _operand(self, t: torch.Tensor, expand: bool):
        """(expression, leaves) standing for tensor `t`: the expression of the
        unsubmitted op that returned it, rounded as its dtype stores it, or
        the tensor itself."""
        if expand:
            e = self._nodes.get(id(t))
            if e is not None and e[0].out is t and t.dtype in _KEEP:
                return f"{_KEEP[t.dtype]}({e[0].expr})", e[0].leaves
        return "A", [t]

    @staticmethod
    def _compose(expr: str, operands) -> Optional[Tuple[str, List[torch.Tensor]]]:
        """Substitute the operand letters of an op's expression (A, B) by the
        operands' expressions, merging their leaves (at most four)."""
        leaves: List[torch.Tensor] = []
        mapping: Dict[str, str] = {}
        for letter, (sub, sl) in zip("AB", operands):
            ren: Dict[str, str] = {}
            for k, t in enumerate(sl):
                idx = next((j for j, u in enumerate(leaves) if u is t), None)
                if idx is None:
                    leaves.append(t)
                    idx = len(leaves) - 1
                if idx >= len(_LETTERS):
                    return None
                ren[_LETTERS[k]] = _LETTERS[idx]
            mapping[letter] = "(" + _rename(sub, ren) + ")" if sub != "A" else ren["A"]
        out = _TOKEN.sub(lambda m: mapping.get(m.group(1), m.group(1)), expr)
        if len(out) > _MAX_EXPR:
            return None
        return out, leaves

    def _node(self, key: str, expr: str, inputs: List[torch.Tensor], out: torch.Tensor):
        """Defer the elementwise op `expr` over `inputs` writing `out`,
        inlining the unsubmitted ops its inputs come from where the operands
        (at most four leaves) and the JIT allow."""
        ext = self.ext
        tries = [(True,) * len(inputs)]
        if len(inputs) == 2:
            tries += [(True, False), (False, True)]
        def deferred(t):
            e = self._nodes.get(id(t))
            return e is not None and e[0].out is t and t.dtype in _KEEP

        for expand in tries:
            if not any(x and deferred(t) for t, x in zip(inputs, expand)):
                continue  # nothing to inline
            c = self._compose(expr, [self._operand(t, x) for t, x in zip(inputs, expand)])
            if c is None:
                continue
            cexpr, leaves = c
            try:
                slot = ext.register_elementwise(f"fused|{len(leaves)}|{cexpr}", cexpr, len(leaves))
            except Exception:  # NVRTC missing or out of custom slots: do not inline
                continue
            self._nodes[id(out)] = (_Node(cexpr, leaves, out), slot)
            return self._done(out, *leaves)
        slot = ext.register_elementwise(key, expr, len(inputs))
        self._nodes[id(out)] = (_Node(expr, list(inputs), out), slot)
        return self._done(out, *inputs)

    def submit_nodes(self):
        """Submit the deferred ops in the order they were made.  An op whose
        returned tensor nobody else holds any more (only this node refers to
        it) was inlined into the ops that read it, or is unused: it is not
        written."""
        if not self._nodes:
            return
        nodes = list(self._nodes.values())
        self._nodes.clear()
        ext = self.ext
        for node, slot in nodes:
            # references: node.out, and getrefcount's own argument
            if sys.getrefcount(node.out) <= 2:
                continue
            lv = node.leaves
            if len(lv) == 1:
                ext.submit_unary(slot, lv[0], node.out)
            elif len(lv) == 2:
                ext.submit_binary(slot, lv[0], lv[1], node.out)
            else:
                ext.submit_nary(slot, lv, node.out)
        del nodes

    def sync(self):
        self.submit_nodes()
        self.ext.flush(sync=True)
        self.clear_pending()

    def clear_pending(self):
        self.pending.clear()
        self.pending_in.clear()
        self._w.clear()
        self._r.clear()

    def _out_for(self, kwargs, shape, dtype, device) -> Optional[torch.Tensor]:
        out = kwargs.get("out")
        if out is None:
            return torch.empty(shape, dtype=dtype, device=device)
        if not out.is_cuda or out.device != device or tuple(out.shape) != tuple(shape):
            return None
        return out

    # ---- dispatch ------------------------------------------------------------
    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        name = func.name()
        if name in self._names:
            r = self._schedule(name, func, args, kwargs)
            if r is not None:
                return r
        # runs in torch: pending requests it depends on must be done first
        if self.pending and (self._reads_pending(args, kwargs) or
                             self._writes_pending(func, args, kwargs)):
            self.sync()
        return func(*args, **kwargs)

    def _schedule(self, name, func, args, kwargs):
        ext = self.ext
        if name in _BINARY_EXPR:
            if len(args) < 2:
                return None
            a, b = args[0], args[1]
            if not self._small_cuda(a, b) or a.device != b.device:
                return None
            alpha = kwargs.get("alpha", 1)
            if alpha is not None and alpha != 1:
                return None
            try:
                shape = torch.broadcast_shapes(tuple(a.shape), tuple(b.shape))
            except RuntimeError:
                return None
            out = self._out_for(kwargs, shape, torch.result_type(a, b), a.device)
            if out is None:
                return None
            if not self.jit:
                getattr(ext, _BINARY_BUILTIN[name])(a, b, out)
            elif self.fuse:
                return self._node(f"bin|{name}", _BINARY_EXPR[name], [a, b], out)
            else:
                slot = ext.register_elementwise(f"bin|{name}", _BINARY_EXPR[name], 2)
                ext.submit_binary(slot, a, b, out)
            return self._done(out, a, b)
        if name in _UNARY_EXPR or name in _PARAM_UNARY:
            x = args[0]
            if not self._small_cuda(x):
                return None
            if name in _UNARY_EXPR:
                key, expr = f"un|{name}", _UNARY_EXPR[name]
                if name == "aten::gelu" and kwargs.get("approximate", "none") not in ("none", "tanh"):
                    return None
            else:
                ke = _param_expr(name, args, kwargs)
                if ke is None:
                    return None
                key, expr = ke
            out = self._out_for(kwargs, x.shape, x.dtype, x.device)
            if out is None:
                return None
            if self.fuse:
                return self._node(key, expr, [x], out)
            slot = ext.register_elementwise(key, expr, 1)
            ext.submit_unary(slot, x, out)
            return self._done(out, x)
        if name in _REDUCE:
            x = args[0]
            if not self._small_cuda(x):
                return None
            dim = kwargs.get("dim", args[1] if len(args) > 1 else None)
            keepdim = bool(kwargs.get("keepdim", args[2] if len(args) > 2 else False))
            if kwargs.get("dtype") is not None or (len(args) > 3 and args[3] is not None):
                return None
            if dim is None:
                return None
            dims = [dim] if isinstance(dim, int) else list(dim)
            nd = x.dim()
            axes = sorted({int(d) + nd if int(d) < 0 else int(d) for d in dims})
            if not axes or axes[0] < 0 or axes[-1] >= nd:
                return None
            shape = [1 if i in axes else s for i, s in enumerate(x.shape)] if keepdim else \
                [s for i, s in enumerate(x.shape) if i not in axes]
            out = torch.empty(shape, dtype=x.dtype, device=x.device)
            op = _REDUCE[name]
            self.submit_nodes()  # its input may be a deferred op's result
            slot = ext.register_reduce(f"reduce_{op}", op)
            ext.submit_reduce(slot, x, out, axes, keepdim)
            return self._done(out, x)
        return None


class GPUOSScheduler:
    """Context manager: initialise the executor, route small CUDA ops to it,
    flush and shut down on exit (scheduler.py:369-404)."""

    def __init__(self, *, capacity: int = 8192, threads_per_block: int = 256,
                 size_threshold: int = 1 << 16, auto_flush_ms: Optional[float] = 2.0):
        self.ext = _load()
        self.capacity = capacity
        self.threads_per_block = threads_per_block
        self.size_threshold = size_threshold
        self.auto_flush_ms = auto_flush_ms
        self._mode: Optional[_GPUOSSchedulerMode] = None
        self._pending: Set[int] = set()

    def __enter__(self):
        self.ext.init(self.capacity, self.threads_per_block)
        self._mode = _GPUOSSchedulerMode(self.ext, size_threshold=self.size_threshold,
                                         auto_flush_ms=self.auto_flush_ms,
                                         pending=self._pending, jit=not _jit_disabled(),
                                         fuse=_fuse_enabled())
        self._mode.__enter__()
        return self

    def flush(self, sync: bool = False):
        if self._mode is not None:
            self._mode.submit_nodes()
        self.ext.flush(sync=sync)
        if sync:
            self._pending.clear()
            if self._mode is not None:
                self._mode.clear_pending()

    def __exit__(self, exc_type, exc, tb):
        try:
            if self._mode is not None:
                self._mode.close()
                self._mode.submit_nodes()
                self._mode.__exit__(exc_type, exc, tb)
        finally:
            self._mode = None
            try:
                self.ext.flush(sync=True)
            finally:
                self._pending.clear()
                self.ext.shutdown()
        return False


@contextlib.contextmanager
def scheduler_context(*, capacity: int = 8192, threads_per_block: int = 256,
                      size_threshold: int = 1 << 16, auto_flush_ms: Optional[float] = 2.0):
    sched = GPUOSScheduler(capacity=capacity, threads_per_block=threads_per_block,
                           size_threshold=size_threshold, auto_flush_ms=auto_flush_ms)
    with sched:
        yield sched
