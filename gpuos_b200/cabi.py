"""ctypes binding of the C ABI in include/gpuos_b200.h.

This is the binding a Python caller that cannot (or does not want to) load
the torch extension uses; it is also how the parity tests drive the
executor "through the C ABI".  Every function returns a status code; `check`
turns a negative status into an exception carrying gpuos_last_error().
"""
from __future__ import annotations

import ctypes
import struct
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgpuos_b200.so"

OK, EINVAL, ECUDA, ETIMEOUT, ESTATE, EUNSUPPORTED, EDEVICE, ENVRTC = 0, -1, -2, -3, -4, -5, -6, -7
F32, F16, BF16 = 0, 1, 2
MODE_PERSISTENT, MODE_STREAM = 0, 1
OP_ADD, OP_MUL, OP_SUB, OP_DIV = 0, 1, 2, 3


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8)]


class Options(ctypes.Structure):
    _fields_ = [("capacity", ctypes.c_int32), ("threads_per_block", ctypes.c_int32),
                ("mode", ctypes.c_int32), ("blocks_per_sm", ctypes.c_int32),
                ("idle_ms", ctypes.c_double), ("sync_timeout_s", ctypes.c_double),
                ("max_batch", ctypes.c_int32), ("wait_limit_us", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 6)]


class Stats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "published", "staged", "processed", "retired", "heartbeat", "requests", "pending",
        "errors", "relaunches", "dev_ns", "lean", "chain")] + [(n, ctypes.c_int32) for n in (
            "capacity", "max_batch", "mode", "worker_alive", "quit", "grid", "block", "device")]


class Plan(ctypes.Structure):
    _fields_ = [("record", ctypes.c_uint8 * 128), ("nchunk", ctypes.c_uint32),
                ("has_ext", ctypes.c_uint32), ("partials", ctypes.c_uint64),
                ("counters", ctypes.c_uint64)]


# exported symbol -> (restype, argtypes); every declaration of the header
P = ctypes.POINTER
_VP = ctypes.c_void_p
SIGNATURES = {
    "gpuos_abi_version": (ctypes.c_int32, []),
    "gpuos_last_error": (ctypes.c_char_p, []),
    "gpuos_executor_create": (ctypes.c_int32, [ctypes.c_int32, P(Options), P(_VP)]),
    "gpuos_executor_destroy": (ctypes.c_int32, [_VP]),
    "gpuos_submit_builtin": (ctypes.c_int32, [_VP, ctypes.c_int32, P(Tensor), P(Tensor), P(Tensor)]),
    "gpuos_submit_unary": (ctypes.c_int32, [_VP, ctypes.c_int32, P(Tensor), P(Tensor)]),
    "gpuos_submit_binary": (ctypes.c_int32, [_VP, ctypes.c_int32, P(Tensor), P(Tensor), P(Tensor)]),
    "gpuos_submit_nary": (ctypes.c_int32, [_VP, ctypes.c_int32, ctypes.c_int32, P(Tensor), P(Tensor)]),
    "gpuos_register_elementwise": (ctypes.c_int32, [_VP, ctypes.c_char_p, ctypes.c_char_p,
                                                    ctypes.c_int32, P(ctypes.c_int32)]),
    "gpuos_register_reduce": (ctypes.c_int32, [_VP, ctypes.c_char_p, ctypes.c_char_p,
                                               P(ctypes.c_int32)]),
    "gpuos_submit_reduce": (ctypes.c_int32, [_VP, ctypes.c_int32, P(Tensor), P(Tensor),
                                             P(ctypes.c_int32), ctypes.c_int32, ctypes.c_int32]),
    "gpuos_submit_task": (ctypes.c_int32, [_VP, _VP]),
    "gpuos_flush": (ctypes.c_int32, [_VP, ctypes.c_int32, _VP, P(ctypes.c_uint64)]),
    "gpuos_wait": (ctypes.c_int32, [_VP, ctypes.c_uint64, ctypes.c_double]),
    "gpuos_set_alias": (ctypes.c_int32, [_VP, ctypes.c_int32, ctypes.c_int32]),
    "gpuos_set_slot": (ctypes.c_int32, [_VP, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                        ctypes.c_float]),
    "gpuos_get_slot": (ctypes.c_int32, [_VP, ctypes.c_int32, P(ctypes.c_int32), P(ctypes.c_float),
                                        P(ctypes.c_float), P(ctypes.c_int32)]),
    "gpuos_variant_by_name": (ctypes.c_int32, [ctypes.c_char_p]),
    "gpuos_set_timing": (ctypes.c_int32, [_VP, ctypes.c_int32]),
    "gpuos_take_timings": (ctypes.c_int32, [_VP, P(ctypes.c_float), ctypes.c_uint64,
                                            P(ctypes.c_uint64)]),
    "gpuos_set_yield_every": (ctypes.c_int32, [_VP, ctypes.c_uint64]),
    "gpuos_set_debug_level": (ctypes.c_int32, [_VP, ctypes.c_int32]),
    "gpuos_worker_alive": (ctypes.c_int32, [_VP]),
    "gpuos_debug_stall_next_batch": (ctypes.c_int32, [_VP]),
    "gpu_set_op_table_async": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_uint64, _VP]),
    "gpu_set_alias_async": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_int32, _VP]),
    "gpuos_plan_elementwise": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_float, ctypes.c_float,
                                                P(Tensor), P(Tensor), P(Tensor), P(Plan)]),
    "gpuos_plan_reduce": (ctypes.c_int32, [ctypes.c_int32, P(Tensor), P(Tensor), P(ctypes.c_int32),
                                           ctypes.c_int32, ctypes.c_int32, P(Plan)]),
    "gpuos_jit_check": (ctypes.c_int32, [ctypes.c_char_p, ctypes.c_int32]),
    "gpuos_reduce_rows_noalloc": (ctypes.c_int32, [ctypes.c_int32, _VP, ctypes.c_int32,
                                                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                   _VP, ctypes.c_int32, _VP]),
    "gpuos_match_expression": (ctypes.c_int32, [ctypes.c_char_p, ctypes.c_int32,
                                                P(ctypes.c_int32), P(ctypes.c_float),
                                                P(ctypes.c_float)]),
    "gpuos_get_stats": (ctypes.c_int32, [_VP, P(Stats)]),
    "gpuos_ipc_server_create": (ctypes.c_int32, [ctypes.c_char_p, ctypes.c_int32, ctypes.c_uint64,
                                                 ctypes.c_int32, ctypes.c_int32, P(Options),
                                                 P(_VP)]),
    "gpuos_ipc_server_destroy": (ctypes.c_int32, [_VP]),
    "gpuos_ipc_server_stats": (ctypes.c_int32, [_VP, P(ctypes.c_uint64), P(ctypes.c_uint64),
                                                P(ctypes.c_uint64), P(ctypes.c_int32)]),
    "gpuos_ipc_connect": (ctypes.c_int32, [ctypes.c_char_p, ctypes.c_double, P(_VP)]),
    "gpuos_ipc_disconnect": (ctypes.c_int32, [_VP]),
    "gpuos_ipc_pool": (ctypes.c_int32, [_VP, P(_VP), P(ctypes.c_uint64), P(ctypes.c_uint64),
                                        P(ctypes.c_uint64), P(ctypes.c_int32)]),
    "gpuos_ipc_submit_builtin": (ctypes.c_int32, [_VP, ctypes.c_int32, P(Tensor), P(Tensor),
                                                  P(Tensor)]),
    "gpuos_ipc_submit_slot": (ctypes.c_int32, [_VP, ctypes.c_int32, ctypes.c_int32, P(Tensor),
                                               P(Tensor)]),
    "gpuos_ipc_submit_reduce": (ctypes.c_int32, [_VP, ctypes.c_int32, P(Tensor), P(Tensor),
                                                 P(ctypes.c_int32), ctypes.c_int32,
                                                 ctypes.c_int32]),
    "gpuos_ipc_flush": (ctypes.c_int32, [_VP, ctypes.c_int32]),
    "gpuos_ipc_register": (ctypes.c_int32, [_VP, ctypes.c_int32, ctypes.c_char_p, ctypes.c_char_p,
                                            ctypes.c_int32, P(ctypes.c_int32)]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OSError(f"{LIB_PATH} is not built (python -m gpuos_b200._build)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class GpuosError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"gpuos status {code}: {msg}")
        self.code = code


def check(rc):
    if rc < 0:
        raise GpuosError(rc, lib().gpuos_last_error().decode(errors="replace"))
    return rc


_DT = None


def tensor(t) -> Tensor:
    """gpuos_tensor describing a torch tensor (any device; nothing is copied)."""
    global _DT
    if _DT is None:
        import torch
        _DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
    d = Tensor()
    d.data = t.data_ptr() if t.numel() else None
    d.dtype = _DT[t.dtype]
    d.ndim = t.dim()
    for i in range(t.dim()):
        d.sizes[i] = t.size(i)
        d.strides[i] = t.stride(i)
    return d


# Req field layout (gpuos_b200/csrc/gpuos_abi.h)
_REQ = struct.Struct("<HBBBBBBff II q QQQ q qqq qq IIIIII")
REQ_FIELDS = ("op kind layout dta dtb dto flags p0 p1 chunk nseg numel a b o inner "
              "sa_row sb_row so_row sa_in sb_in ext part cnt fdiv_m fdiv_s rg").split()
assert _REQ.size == 128


def decode_record(raw: bytes) -> dict:
    return dict(zip(REQ_FIELDS, _REQ.unpack(bytes(raw))))


def plan_elementwise(variant, a, b, out, p0=0.0, p1=0.0) -> dict:
    p = Plan()
    da, do = tensor(a), tensor(out)
    db = tensor(b) if b is not None else None
    check(lib().gpuos_plan_elementwise(variant, p0, p1, ctypes.byref(da),
                                       ctypes.byref(db) if db is not None else None,
                                       ctypes.byref(do), ctypes.byref(p)))
    r = decode_record(bytes(p.record))
    r.update(nchunk=p.nchunk, has_ext=p.has_ext, partials=p.partials, counters=p.counters)
    return r


def plan_reduce(variant, x, out, axes, keepdim) -> dict:
    p = Plan()
    arr = (ctypes.c_int32 * 8)(*list(axes)[:8])
    check(lib().gpuos_plan_reduce(variant, ctypes.byref(tensor(x)), ctypes.byref(tensor(out)),
                                  arr, len(axes), int(bool(keepdim)), ctypes.byref(p)))
    r = decode_record(bytes(p.record))
    r.update(nchunk=p.nchunk, has_ext=p.has_ext, partials=p.partials, counters=p.counters)
    return r


def match_expression(expr: str, arity: int):
    v, p0, p1 = ctypes.c_int32(), ctypes.c_float(), ctypes.c_float()
    check(lib().gpuos_match_expression(expr.encode(), arity, ctypes.byref(v), ctypes.byref(p0),
                                       ctypes.byref(p1)))
    return v.value, p0.value, p1.value


class Executor:
    """Thin owner of one gpuos_executor handle."""

    def __init__(self, device=0, mode=MODE_PERSISTENT, capacity=4096, threads_per_block=256,
                 max_batch=0, idle_ms=0.0, wait_limit_us=0, sync_timeout_s=0.0):
        o = Options()
        o.capacity, o.threads_per_block, o.mode = capacity, threads_per_block, mode
        o.max_batch, o.idle_ms = max_batch, idle_ms
        o.wait_limit_us, o.sync_timeout_s = wait_limit_us, sync_timeout_s
        h = ctypes.c_void_p()
        check(lib().gpuos_executor_create(device, ctypes.byref(o), ctypes.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            h, self.h = self.h, None
            check(lib().gpuos_executor_destroy(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def builtin(self, op, a, b, out):
        check(lib().gpuos_submit_builtin(self.h, op, ctypes.byref(tensor(a)),
                                         ctypes.byref(tensor(b)), ctypes.byref(tensor(out))))

    def unary(self, slot, a, out):
        check(lib().gpuos_submit_unary(self.h, slot, ctypes.byref(tensor(a)),
                                       ctypes.byref(tensor(out))))

    def binary(self, slot, a, b, out):
        check(lib().gpuos_submit_binary(self.h, slot, ctypes.byref(tensor(a)),
                                        ctypes.byref(tensor(b)), ctypes.byref(tensor(out))))

    def nary(self, slot, inputs, out):
        """out = expr(A, B, C, D) of slot `slot` over 1 to 4 input tensors."""
        arr = (Tensor * len(inputs))(*[tensor(t) for t in inputs])
        check(lib().gpuos_submit_nary(self.h, slot, len(inputs), arr, ctypes.byref(tensor(out))))

    def register_elementwise(self, key, expr, arity) -> int:
        s = ctypes.c_int32()
        check(lib().gpuos_register_elementwise(self.h, key.encode(), expr.encode(), arity,
                                               ctypes.byref(s)))
        return s.value

    def register_reduce(self, key, op) -> int:
        s = ctypes.c_int32()
        check(lib().gpuos_register_reduce(self.h, key.encode(), op.encode(), ctypes.byref(s)))
        return s.value

    def reduce(self, slot, x, out, axes, keepdim):
        arr = (ctypes.c_int32 * 8)(*list(axes)[:8])
        check(lib().gpuos_submit_reduce(self.h, slot, ctypes.byref(tensor(x)),
                                        ctypes.byref(tensor(out)), arr, len(axes),
                                        int(bool(keepdim))))

    def task(self, raw: bytes):
        buf = ctypes.create_string_buffer(bytes(raw), len(raw))
        check(lib().gpuos_submit_task(self.h, buf))

    def flush(self, sync=False, stream=None) -> int:
        t = ctypes.c_uint64()
        check(lib().gpuos_flush(self.h, int(bool(sync)), stream, ctypes.byref(t)))
        return t.value

    def wait(self, ticket, timeout_s=0.0):
        check(lib().gpuos_wait(self.h, ticket, timeout_s))

    def set_alias(self, logical, physical):
        check(lib().gpuos_set_alias(self.h, logical, physical))

    def set_slot(self, slot, variant, p0=0.0, p1=0.0):
        check(lib().gpuos_set_slot(self.h, slot, variant, p0, p1))

    def get_slot(self, slot):
        """(variant, p0, p1, alias) of a slot."""
        v, a = ctypes.c_int32(), ctypes.c_int32()
        p0, p1 = ctypes.c_float(), ctypes.c_float()
        check(lib().gpuos_get_slot(self.h, slot, ctypes.byref(v), ctypes.byref(p0),
                                   ctypes.byref(p1), ctypes.byref(a)))
        return v.value, p0.value, p1.value, a.value

    def set_timing(self, on: bool):
        check(lib().gpuos_set_timing(self.h, int(bool(on))))

    def take_timings(self, cap: int = 1 << 16) -> list:
        """Kernel durations (ms) recorded since the last call."""
        buf = (ctypes.c_float * cap)()
        n = ctypes.c_uint64()
        check(lib().gpuos_take_timings(self.h, buf, cap, ctypes.byref(n)))
        return list(buf[:min(n.value, cap)])

    def stall_next_batch(self):
        """Fault injection: the next batch with stage barriers waits for a
        chunk that never comes, until its bounded wait runs out."""
        check(lib().gpuos_debug_stall_next_batch(self.h))

    def set_yield_every(self, n):
        check(lib().gpuos_set_yield_every(self.h, n))

    def worker_alive(self) -> bool:
        return check(lib().gpuos_worker_alive(self.h)) == 1

    def stats(self) -> dict:
        s = Stats()
        check(lib().gpuos_get_stats(self.h, ctypes.byref(s)))
        return {n: getattr(s, n) for n, _ in Stats._fields_}


def variant(name: str) -> int:
    return lib().gpuos_variant_by_name(name.encode())
