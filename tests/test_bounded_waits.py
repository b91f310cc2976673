"""Failure detection without a GPU fault (needs a GPU: -m gpu).

Every wait inside the kernels is bounded by %globaltimer, and every host wait
by a timeout.  These tests make both kinds run out on purpose, in the only
forms that cannot hurt the GPU: a stage wait that nothing will ever satisfy
(gpuos_debug_stall_next_batch), which the kernel abandons after
wait_limit_us, reporting ERR_STAGE_TIMEOUT; and a host wait shorter than the
work in front of it.  Afterwards the executor must still run requests
correctly.  (The reference has no timeouts: its flush(sync=True) spins for
ever if the worker stops, pytorch_ext/gpuos_ext.cpp:601-621.)
"""
import time

import pytest
import torch

import gpuos_b200.cabi as C

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
EDEVICE, ETIMEOUT = -6, -3


def _chain(ex, n=4096):
    """c = a + b, then d = c * b: one batch with a stage barrier."""
    a = torch.randn(n, device=DEV)
    b = torch.randn(n, device=DEV)
    c = torch.empty_like(a)
    d = torch.empty_like(a)
    ex.builtin(C.OP_ADD, a, b, c)
    ex.builtin(C.OP_MUL, c, b, d)
    return a, b, c, d


@pytest.mark.parametrize("mode", [C.MODE_PERSISTENT, C.MODE_STREAM], ids=["persistent", "stream"])
def test_stage_wait_runs_out_and_reports(mode):
    with C.Executor(0, mode=mode, wait_limit_us=5000) as ex:
        # a clean chain first: the limit does not get in the way of real waits
        a, b, c, d = _chain(ex)
        ex.flush(sync=True)
        assert torch.equal(d, (a + b) * b)
        # now the last stage waits for a chunk that never comes
        _chain(ex)
        ex.stall_next_batch()
        t0 = time.perf_counter()
        with pytest.raises(C.GpuosError) as e:
            ex.flush(sync=True)
        el = time.perf_counter() - t0
        assert e.value.code == EDEVICE
        assert "stage barrier wait timed out" in str(e.value)
        assert el < 5.0, f"the 5 ms device wait took {el:.2f} s to surface"
        # the executor is still usable, and the error was reported once
        a, b, c, d = _chain(ex)
        ex.flush(sync=True)
        assert torch.equal(d, (a + b) * b)
        assert ex.stats()["errors"] >= 1


def test_host_wait_times_out_then_completes():
    with C.Executor(0, mode=C.MODE_STREAM) as ex:
        cur = torch.cuda.current_stream()
        a = torch.randn(1 << 16, device=DEV)
        b = torch.randn(1 << 16, device=DEV)
        o = torch.empty_like(a)
        torch.cuda._sleep(200_000_000)  # holds the stream for a while (~0.1 s)
        ex.builtin(C.OP_ADD, a, b, o)
        ticket = ex.flush(sync=False, stream=cur.cuda_stream)
        with pytest.raises(C.GpuosError) as e:
            ex.wait(ticket, 1e-3)
        assert e.value.code == ETIMEOUT
        ex.wait(ticket, 30.0)
        assert torch.equal(o, a + b)


@pytest.mark.parametrize("mode", [C.MODE_PERSISTENT, C.MODE_STREAM], ids=["persistent", "stream"])
def test_device_time_is_accounted(mode):
    """stats.dev_ns grows by the device time of completed batches (first CTA
    in -> last chunk) for the persistent worker and lean stream batches."""
    with C.Executor(0, mode=mode) as ex:
        a = torch.randn(1 << 20, device=DEV)
        b = torch.randn(1 << 20, device=DEV)
        o = torch.empty_like(a)
        before = ex.stats()["dev_ns"]
        for _ in range(4):
            ex.builtin(C.OP_ADD, a, b, o)
            ex.flush(sync=True)
        after = ex.stats()
        assert torch.equal(o, a + b)
        d = after["dev_ns"] - before
        assert 0 < d < 4 * 50_000_000, d   # a 12 MB batch: microseconds, not 50 ms
        if mode == C.MODE_STREAM:
            assert after["lean"] >= 4
