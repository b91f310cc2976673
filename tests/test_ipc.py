"""Multi-process sharing of one executor (gpuos_b200.ipc, C ABI gpuos_ipc_*).

The reference's multi-process pattern (benchmarks/bench_mps.py:54-92) gives
every process its own persistent kernel.  Here client processes feed one
server's executor through rings in shared memory.  CPU tests run the
protocol against a server in record mode (no GPU): rings that wrap, flush
markers, the registration mailbox, errors, and a client that dies without
disconnecting.  GPU tests run real client processes on cuda:0 against a
server in this process and check every result.
"""
import ctypes
import multiprocessing as mp
import os
import time

import pytest
import torch

import gpuos_b200.cabi as C
import gpuos_b200.ipc as I

DEV = "cuda:0"


def _name(tag):
    return f"gpuos-test-{tag}-{os.getpid()}-{time.monotonic_ns() % 1000000}"


def _desc(addr, n, dtype=C.F32):
    t = C.Tensor()
    t.data = addr
    t.dtype = dtype
    t.ndim = 1
    t.sizes[0] = n
    t.strides[0] = 1
    return t


def _record_client(name, k, n, q):
    """A client process of a record-mode server: n requests, a flush every k."""
    try:
        with I.Client(name, timeout_s=30) as c:
            a = _desc(c.base + 1024, 64)
            o = _desc(c.base + 4096, 64)
            slot = c.register_elementwise(f"k{os.getpid()}", "(A > 0.f ? A : 0.f)", 1)
            for i in range(n):
                C.check(C.lib().gpuos_ipc_submit_builtin(c.h, C.OP_ADD, ctypes.byref(a),
                                                         ctypes.byref(a), ctypes.byref(o)))
                if (i + 1) % k == 0:
                    c.flush(sync=(i // k) % 2 == 0)
            c.submit_unary(slot, torch.empty(0), torch.empty(0))  # empty: no memory needed
            c.flush(sync=True)
        q.put(("ok", os.getpid()))
    except Exception as e:  # reported to the parent
        q.put(("error", repr(e)))


def test_record_mode_rings_flushes_and_mailbox():
    name = _name("rec")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with I.Server(name, device=-1, pool_bytes=1 << 20, max_clients=4, ring_entries=8) as s:
        ps = [ctx.Process(target=_record_client, args=(name, 7, 100, q)) for _ in range(3)]
        for p in ps:
            p.start()
        res = [q.get(timeout=120) for _ in ps]
        for p in ps:
            p.join(timeout=60)
        assert all(r[0] == "ok" for r in res), res
        st = s.stats()
        # 100 builtin requests and one empty unary request per client
        assert st["requests"] == 3 * 101
        # 14 flushes of every 7 requests, the last one, and the disconnect's
        assert 3 * 15 <= st["client_flushes"] <= 3 * 16
        assert 1 <= st["launch_flushes"] <= st["client_flushes"]


def test_record_mode_rejects_tensors_outside_the_pool():
    name = _name("oob")
    with I.Server(name, device=-1, pool_bytes=1 << 16, max_clients=1, ring_entries=4) as s:
        with I.Client(name, timeout_s=10) as c:
            inside = _desc(c.base, 16)
            tail = _desc(c.base + (1 << 16) - 32, 16)     # runs 32 bytes past the end
            C.check(C.lib().gpuos_ipc_submit_builtin(c.h, C.OP_MUL, ctypes.byref(inside),
                                                     ctypes.byref(tail), ctypes.byref(inside)))
            with pytest.raises(C.GpuosError) as e:
                c.flush(sync=True)
            assert e.value.code == C.EINVAL and "outside the shared pool" in str(e.value)
            c.flush(sync=True)                            # the error was reported once
            with pytest.raises(C.GpuosError):             # the client side checks too
                C.check(C.lib().gpuos_ipc_submit_builtin(c.h, C.OP_MUL, ctypes.byref(inside),
                                                         ctypes.byref(_desc(64, 4)),
                                                         ctypes.byref(inside)))
        assert s.stats()["requests"] == 0


def _die_connected(name):
    c = I.Client(name, timeout_s=10)
    os._exit(0)  # leave without disconnecting


def test_dead_client_slot_is_freed():
    name = _name("dead")
    ctx = mp.get_context("spawn")
    with I.Server(name, device=-1, pool_bytes=1 << 20, max_clients=1, ring_entries=4) as s:
        p = ctx.Process(target=_die_connected, args=(name,))
        p.start()
        p.join(timeout=60)
        t0 = time.time()
        while True:  # the server notices within about 50 ms
            try:
                c = I.Client(name, timeout_s=5)
                break
            except C.GpuosError as e:
                assert e.code == C.ESTATE
                assert time.time() - t0 < 10
                time.sleep(0.05)
        c.close()


def test_no_server_and_bad_names():
    with pytest.raises(C.GpuosError):
        I.Client(_name("none"), timeout_s=1)
    with pytest.raises(C.GpuosError):
        I.Server("bad/name", device=-1)
    name = _name("dup")
    with I.Server(name, device=-1, pool_bytes=1 << 16):
        with pytest.raises(C.GpuosError):
            I.Server(name, device=-1, pool_bytes=1 << 16)    # the name is taken


# ---------------------------------------------------------------- GPU tests
def _gpu_client(name, seed, q):
    """A client process on cuda:0: builtins, a custom expression of three
    operands, a reduction; checked against torch in the same process."""
    try:
        import torch
        torch.cuda.set_device(0)
        g = torch.Generator(device="cuda").manual_seed(seed)
        with I.Client(name, timeout_s=120) as c:
            n = 100_000
            a, b, w = (c.empty([n]) for _ in range(3))
            a.copy_(torch.randn(n, device="cuda", generator=g))
            b.copy_(torch.randn(n, device="cuda", generator=g))
            w.copy_(torch.randn(n, device="cuda", generator=g))
            s1, p1, f1 = c.empty([n]), c.empty([n]), c.empty([n])
            x = c.empty([64, 1000], torch.bfloat16)
            x.copy_(torch.randn(64, 1000, device="cuda", generator=g))
            m = c.empty([64, 1], torch.bfloat16)
            c.submit_add(a, b, s1)
            c.submit_mul(s1, w, p1)                       # reads s1: ordered after it
            k3 = c.register_elementwise("ipc|fma3", "gpuos_keep_f32((A * B)) + C", 3)
            c.submit_nary(k3, [a, b, w], f1)
            r = c.register_reduce("ipc|mean", "mean")
            c.submit_reduce(r, x, m, [1], True)
            c.flush(sync=True)
            ok = (torch.equal(s1, a + b) and torch.equal(p1, (a + b) * w) and
                  torch.equal(f1, a * b + w))
            want = x.float().mean(1, keepdim=True)
            ok = ok and bool(((m.float() - want).abs() <= 1e-2 * want.abs() + 1e-3).all())
        q.put(("ok" if ok else "mismatch", seed))
    except Exception as e:
        q.put(("error", repr(e)))


@pytest.mark.gpu
def test_clients_share_one_executor():
    name = _name("gpu")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with I.Server(name, device=0, pool_bytes=256 << 20, max_clients=4, ring_entries=64) as s:
        ps = [ctx.Process(target=_gpu_client, args=(name, 100 + i, q)) for i in range(3)]
        for p in ps:
            p.start()
        res = [q.get(timeout=600) for _ in ps]
        for p in ps:
            p.join(timeout=120)
        assert all(r[0] == "ok" for r in res), res
        st = s.stats()
        assert st["requests"] == 3 * 4
        assert st["launch_flushes"] <= st["client_flushes"]


def test_record_mode_four_input_requests_and_mailbox_limits():
    name = _name("nary")
    with I.Server(name, device=-1, pool_bytes=1 << 20, max_clients=2, ring_entries=4) as s:
        with I.Client(name, timeout_s=10) as c:
            ts = [_desc(c.base + 4096 * k, 256) for k in range(5)]
            arr = (C.Tensor * 4)(*ts[:4])
            for _ in range(6):                               # wraps the 4-entry ring
                C.check(C.lib().gpuos_ipc_submit_slot(c.h, 3, 4, arr, ctypes.byref(ts[4])))
            c.flush(sync=True)
            assert s.stats()["requests"] == 6
            with pytest.raises(C.GpuosError):                # five inputs: rejected
                C.check(C.lib().gpuos_ipc_submit_slot(c.h, 3, 5, arr, ctypes.byref(ts[4])))
            with pytest.raises(C.GpuosError) as e:           # longer than the mailbox holds
                c.register_elementwise("k" * 300, "(A + B)", 2)
            assert e.value.code == C.EINVAL
            assert c.register_elementwise("ok", "(A + B)", 2) >= 0
