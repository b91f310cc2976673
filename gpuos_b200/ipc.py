"""Several processes sharing one GPU's executor (C ABI ``gpuos_ipc_*``).

The reference gives every process its own persistent kernel and leaves the
sharing of a GPU to MPS (benchmarks/bench_mps.py:54-92, each worker process
calling ``gpuos_ext.init``, ``submit_add`` and ``flush``).  Here a
:class:`Server` owns the GPU's executor and a device pool exported with CUDA
IPC; each :class:`Client` process allocates its tensors in its own region of
that pool (:meth:`Client.empty`) and submits with the reference module's
calls (``submit_add`` .. ``submit_div``, ``register_elementwise``,
``register_reduce``, ``submit_unary``, ``submit_binary``, ``submit_reduce``,
``flush``), plus ``submit_nary``.  The server drains every client's ring into
the one executor, so the requests of different processes share batches.

A client flush first synchronizes the client's current CUDA stream, so the
work that produced its inputs is done before the server's kernels read them;
results may be read after ``flush(sync=True)`` returns.  Tensors from
:meth:`Client.empty` do not own their memory: they are valid while the client
is connected and the server runs.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

from . import cabi as C

MB_ELEMENTWISE, MB_REDUCE = 1, 2


class Server:
    """The executor of one GPU, shared through shared memory ``/<name>``.
    ``device=-1`` runs in record mode (no GPU: requests are counted and every
    flush completes at once)."""

    def __init__(self, name: str, device: int = 0, pool_bytes: int = 1 << 30,
                 max_clients: int = 8, ring_entries: int = 4096,
                 mode: int = C.MODE_STREAM):
        self.name = name
        h = ctypes.c_void_p()
        opt = C.Options()
        opt.mode = mode
        C.check(C.lib().gpuos_ipc_server_create(name.encode(), device, pool_bytes, max_clients,
                                                ring_entries, ctypes.byref(opt), ctypes.byref(h)))
        self.h = h

    def stats(self) -> dict:
        r, cf, lf = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        n = ctypes.c_int32()
        C.check(C.lib().gpuos_ipc_server_stats(self.h, ctypes.byref(r), ctypes.byref(cf),
                                               ctypes.byref(lf), ctypes.byref(n)))
        return {"requests": r.value, "client_flushes": cf.value, "launch_flushes": lf.value,
                "clients": n.value}

    def close(self):
        if self.h:
            h, self.h = self.h, None
            C.check(C.lib().gpuos_ipc_server_destroy(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


class _CudaArray:
    """The minimal __cuda_array_interface__ torch.as_tensor accepts."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class Client:
    """One process's connection to a :class:`Server`."""

    def __init__(self, name: str, timeout_s: float = 60.0):
        h = ctypes.c_void_p()
        C.check(C.lib().gpuos_ipc_connect(name.encode(), timeout_s, ctypes.byref(h)))
        self.h = h
        base, size, roff, rbytes = ctypes.c_void_p(), ctypes.c_uint64(), ctypes.c_uint64(), \
            ctypes.c_uint64()
        dev = ctypes.c_int32()
        C.check(C.lib().gpuos_ipc_pool(h, ctypes.byref(base), ctypes.byref(size), ctypes.byref(roff),
                                       ctypes.byref(rbytes), ctypes.byref(dev)))
        self.base = base.value or 0
        self.pool_bytes = size.value
        self.device = dev.value
        self._next = roff.value
        self._end = roff.value + rbytes.value

    # ---- memory ------------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        """Address (in this process) of `nbytes` of this client's region."""
        off = (self._next + 255) // 256 * 256
        if off + nbytes > self._end:
            raise MemoryError(f"client region of the pool exhausted ({nbytes} bytes asked)")
        self._next = off + nbytes
        return self.base + off

    def empty(self, shape: Sequence[int], dtype=None):
        """A contiguous tensor in this client's region of the pool."""
        import torch
        dtype = dtype or torch.float32
        n = 1
        for s in shape:
            n *= int(s)
        esz = torch.empty((), dtype=dtype).element_size()
        ptr = self.alloc(max(n, 1) * esz)
        typestr = {torch.float32: "<f4", torch.float16: "<f2", torch.bfloat16: "<i2"}[dtype]
        t = torch.as_tensor(_CudaArray(ptr, shape, typestr), device=f"cuda:{self.device}")
        return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t

    def reset(self):
        """Forget every allocation (the caller no longer uses those tensors)."""
        roff, rb = ctypes.c_uint64(), ctypes.c_uint64()
        C.check(C.lib().gpuos_ipc_pool(self.h, None, None, ctypes.byref(roff), ctypes.byref(rb),
                                       None))
        self._next = roff.value

    # ---- the reference module's calls ----------------------------------------
    def _builtin(self, op, a, b, out):
        C.check(C.lib().gpuos_ipc_submit_builtin(self.h, op, ctypes.byref(C.tensor(a)),
                                                 ctypes.byref(C.tensor(b)),
                                                 ctypes.byref(C.tensor(out))))

    def submit_add(self, a, b, out):
        self._builtin(C.OP_ADD, a, b, out)

    def submit_mul(self, a, b, out):
        self._builtin(C.OP_MUL, a, b, out)

    def submit_sub(self, a, b, out):
        self._builtin(C.OP_SUB, a, b, out)

    def submit_div(self, a, b, out):
        self._builtin(C.OP_DIV, a, b, out)

    def _register(self, kind, key, expr, arity) -> int:
        slot = ctypes.c_int32()
        C.check(C.lib().gpuos_ipc_register(self.h, kind, key.encode(), expr.encode(), arity,
                                           ctypes.byref(slot)))
        return slot.value

    def register_elementwise(self, key: str, expr: str, arity: int) -> int:
        return self._register(MB_ELEMENTWISE, key, expr, arity)

    def register_reduce(self, key: str, op_name: str) -> int:
        return self._register(MB_REDUCE, key, op_name, 1)

    def submit_nary(self, slot: int, inputs, out):
        arr = (C.Tensor * len(inputs))(*[C.tensor(t) for t in inputs])
        C.check(C.lib().gpuos_ipc_submit_slot(self.h, slot, len(inputs), arr,
                                              ctypes.byref(C.tensor(out))))

    def submit_unary(self, slot: int, a, out):
        self.submit_nary(slot, [a], out)

    def submit_binary(self, slot: int, a, b, out):
        self.submit_nary(slot, [a, b], out)

    def submit_reduce(self, slot: int, x, out, axes, keepdim: bool):
        ax = (ctypes.c_int32 * max(1, len(axes)))(*[int(a) for a in axes])
        C.check(C.lib().gpuos_ipc_submit_reduce(self.h, slot, ctypes.byref(C.tensor(x)),
                                                ctypes.byref(C.tensor(out)), ax, len(axes),
                                                1 if keepdim else 0))

    def flush(self, sync: bool = False):
        if self.device >= 0:
            import torch
            torch.cuda.current_stream(self.device).synchronize()
        C.check(C.lib().gpuos_ipc_flush(self.h, 1 if sync else 0))

    def close(self):
        if self.h:
            h, self.h = self.h, None
            C.check(C.lib().gpuos_ipc_disconnect(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False
