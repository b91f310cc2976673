"""The reference's own scheduler, unchanged, over this module (needs a GPU).

The reference's pytorch_ext/scheduler.py imports a top-level module named
`gpuos_ext` (scheduler.py:9-16) and calls only its API.  Here
sys.modules["gpuos_ext"] is gpuos_b200.load(), and the reference's file is
loaded as it is from oracle/_ref/scheduler.py, where oracle/build_ref.py
places it next to the tree (set GPUOS_REF_SCHEDULER to use another copy).
In its default mode (GPUOS_SCHEDULER_DISABLE_JIT unset: JIT off), it routes
add/sub/mul/div on small CUDA tensors to submit_add/sub/mul/div
(scheduler.py:125-143) and flushes synchronously before any other op reads a
pending output (scheduler.py:53-98); results are checked against the oracle.
"""
import importlib.util
import os
import sys
from pathlib import Path

import pytest
import torch

import gpuos_b200
import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ROOT = Path(__file__).resolve().parents[1]
REF_SCHED = Path(os.environ.get("GPUOS_REF_SCHEDULER", ROOT / "oracle" / "_ref" / "scheduler.py"))


@pytest.fixture
def ref_scheduler(monkeypatch):
    if not REF_SCHED.exists():
        pytest.skip("the reference's scheduler.py is not next to the tree (oracle/build_ref.py)")
    monkeypatch.delenv("GPUOS_SCHEDULER_DISABLE_JIT", raising=False)
    monkeypatch.setitem(sys.modules, "gpuos_ext", gpuos_b200.load())
    spec = importlib.util.spec_from_file_location("gpuos_reference_scheduler", REF_SCHED)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.gpuos_ext is sys.modules["gpuos_ext"]
    return mod


def _exact(a, b, op):
    out = torch.empty(torch.broadcast_shapes(a.shape, b.shape), dtype=torch.float32)
    oracle.ew(op, a, b, out)
    return out


def test_reference_scheduler_runs_unchanged(ref_scheduler):
    g = torch.Generator().manual_seed(61)
    a, b = torch.randn(2000, generator=g), torch.randn(2000, generator=g)
    d = torch.sign(b) * (b.abs() + 0.1)
    ga, gb, gd = a.to(DEV), b.to(DEV), d.to(DEV)
    with torch.no_grad(), ref_scheduler.scheduler_context(auto_flush_ms=None):
        c = ga + gb                  # submit_add
        e = c * gb                   # submit_mul, reads a pending output
        f = e - ga                   # submit_sub
        h = f / gd                   # submit_div (op_batch's B == 0 -> 0 rule)
        r = torch.relu(h)            # not scheduled: the scheduler flushes first
    C0 = _exact(a, b, "add")
    E0 = _exact(C0, b, "mul")
    F0 = _exact(E0, a, "sub")
    H0 = _exact(F0, d, "div0")
    for got, want in ((c, C0), (e, E0), (f, F0), (h, H0)):
        assert torch.equal(got.cpu(), want)
    assert torch.equal(r.cpu(), torch.relu(H0))


def test_reference_scheduler_broadcast_and_background_flush(ref_scheduler):
    g = torch.Generator().manual_seed(62)
    x = torch.randn(16, 300, generator=g)
    w = torch.randn(300, generator=g)
    gx, gw = x.to(DEV), w.to(DEV)
    with torch.no_grad(), ref_scheduler.scheduler_context(auto_flush_ms=1.0) as s:
        outs = [gx * gw for _ in range(32)]
        s.flush(sync=True)
    want = _exact(x, w, "mul")
    for o in outs:
        assert torch.equal(o.cpu(), want)
