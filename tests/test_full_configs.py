"""The benchmark configurations at their full sizes (needs a GPU: -m gpu).

Each stream runs through the reference-facing Python API (gpuos_ext, as the
bench drives it: submit_* per request, flush every `flush_every`) and its
whole output slab is checked against the oracle (tests/stream_check.py):
  add/mul      1024 requests x 4096 fp32 elements
  mixed_24op   16,384 requests, 24 operators, sizes log-uniform [256, 32768]
  broadcast    8,192 [B,N] op [N] / [B,1] requests, mixed dtypes, half transposed
  reduce       4,096 sum/mean requests up to 2^24 elements each, half transposed
The transformer-decode chain at batch 1, 8 and 64 with all 32 layers is in
tests/test_gpu_parity.py (test_decode_chain_bf16).
"""
import pytest
import torch

import gpuos_b200
from gpuos_b200 import workloads as W
from stream_check import check_stream

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def run(ext, st):
    din, dout = st.device_buffers(DEV)
    calls = W.Submitter(ext).prepare(st, st.views(din, dout))
    for i, (fn, args) in enumerate(calls):
        fn(*args)
        if (i + 1) % st.flush_every == 0:
            ext.flush(sync=False)
    ext.flush(sync=True)
    out = dout.cpu()
    del din, dout
    return out


@pytest.fixture(scope="module")
def streams():
    return {}


def _stream(cache, name):
    if name not in cache:
        cache[name] = W.STREAMS[name]()
    return cache[name]


@pytest.mark.parametrize("mode", ["stream", "persistent"])
@pytest.mark.parametrize("name", ["micro_add_mul", "mixed_24op", "broadcast_mixed"])
def test_full_size_stream(streams, name, mode):
    st = _stream(streams, name)
    ext = gpuos_b200.load()
    ext.init(8192, 256, mode=mode)
    try:
        out = run(ext, st)
    finally:
        ext.shutdown()
    s = check_stream(st, out)
    assert s["exact"] + s["transcendental"] == len(st.requests)


def test_full_size_reductions():
    st = W.lastdim_reduce()
    assert len(st.requests) == 4096
    assert max(r.a.shape[0] * r.a.shape[1] for r in st.requests) <= 1 << 24
    ext = gpuos_b200.load()
    ext.init(8192, 256, mode="stream")
    try:
        out = run(ext, st)
    finally:
        ext.shutdown()
    s = check_stream(st, out)
    assert s["reduce"] == 4096
    torch.cuda.empty_cache()
