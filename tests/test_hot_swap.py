"""Jump-table hot swap against published batches (needs a GPU: -m gpu).

The reference's worker reads g_op_alias -> g_op_table when it starts a Task
(src/persistent_kernel.cu:168-175), so an update reaches Tasks already in the
queue.  The persistent worker here does the same from its device copy of the
table (acquire loads when it starts a slot request).  To make "published but
not yet started" hold, the slot request is published behind a long batch (a
chain of eight dependent 256 MB requests, about a millisecond) whose output
it reads, so it starts only after that batch: the swap, made right after the
publication, lands while it waits.  In stream mode a request's slot is
resolved when it is flushed, so the same swap does not change it.

The reference-named shims gpu_set_op_table_async / gpu_set_alias_async act on
the executor most recently created on the current device.
"""
import ctypes

import pytest
import torch

import gpuos_b200.cabi as C

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _setup(ex, n=1 << 16):
    g = torch.Generator(device=DEV).manual_seed(5)
    a = torch.randn(n, device=DEV, generator=g)
    b = torch.randn(n, device=DEV, generator=g)
    c, d, o = torch.empty_like(a), torch.empty_like(a), torch.empty_like(a)
    return a, b, c, d, o


@pytest.mark.parametrize("mode", [C.MODE_PERSISTENT, C.MODE_STREAM], ids=["persistent", "stream"])
def test_swap_after_publish(mode):
    with C.Executor(0, mode=mode) as ex:
        s = ex.register_elementwise("swap|mul", "(A * B)", 2)
        n = 1 << 26                          # 256 MB per tensor
        g = torch.Generator(device=DEV).manual_seed(6)
        a = torch.randn(n, device=DEV, generator=g)
        b = torch.randn(n, device=DEV, generator=g)
        xs = [torch.empty_like(a) for _ in range(8)]
        o = torch.empty_like(a)
        # batch 1: eight dependent requests (eight stages, about a millisecond)
        prev = a
        for k, x in enumerate(xs):
            ex.builtin(C.OP_ADD if k % 2 == 0 else C.OP_MUL, prev, b, x)
            prev = x
        ex.flush(sync=False)
        # batch 2 reads batch 1's last output, so it starts after batch 1
        ex.binary(s, xs[-1], b, o)
        ex.flush(sync=False)
        ex.set_slot(s, C.variant("add"))     # swap while the request waits
        ex.flush(sync=True)
        want = a
        for k in range(8):
            want = want + b if k % 2 == 0 else want * b
        assert torch.equal(xs[-1], want)
        if mode == C.MODE_PERSISTENT:
            assert torch.equal(o, want + b)  # the swapped operator ran
        else:
            assert torch.equal(o, want * b)  # resolved at flush: the old one ran


def test_reference_named_shims():
    with C.Executor(0, mode=C.MODE_PERSISTENT) as ex:
        L = C.lib()
        a, b, _, _, o = _setup(ex)
        s_mul = ex.register_elementwise("shim|mul", "(A * B)", 2)
        s_add = ex.register_elementwise("shim|add", "(A + B)", 2)
        # dual slot: route logical s_mul to the physical add slot, then back
        assert L.gpu_set_alias_async(s_mul, s_add, None) == 0
        ex.binary(s_mul, a, b, o)
        ex.flush(sync=True)
        assert torch.equal(o, a + b)
        assert L.gpu_set_alias_async(s_mul, s_mul, None) == 0
        ex.binary(s_mul, a, b, o)
        ex.flush(sync=True)
        assert torch.equal(o, a * b)
        # online: overwrite what physical slot s_mul runs
        assert L.gpu_set_op_table_async(s_mul, C.variant("sub"), None) == 0
        ex.binary(s_mul, a, b, o)
        ex.flush(sync=True)
        assert torch.equal(o, a - b)
        # out of range: cudaErrorInvalidValue
        assert L.gpu_set_alias_async(1000, 0, ctypes.c_void_p(0)) == 1
