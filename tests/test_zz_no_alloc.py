"""gpuos_reduce_rows_noalloc: the row reduction that allocates nothing.

Its results are checked against the executor's own reduction entry point
(gpuos_submit_reduce + gpuos_flush) and against the double-precision sum of
the same inputs, within the reduction tolerance of the parity tests
(|got - want| <= 1e-5 * sum|x| per row, plus one output ulp for 16-bit
outputs), on two calls in a row: the second call reuses the static scratch
the first one left behind.  A warmed call must leave the device's free memory
unchanged.  The file is named to run last, and passes alone in a fresh
process.
"""
import ctypes

import pytest
import torch

import gpuos_b200.cabi as C
from tolerance import RED_REL

DEV = "cuda:0"
SUM, MEAN = C.variant("sum"), C.variant("mean")
DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def noalloc(variant, x, out):
    rows, cols = x.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    C.check(C.lib().gpuos_reduce_rows_noalloc(variant, ctypes.c_void_p(x.data_ptr()), DT[x.dtype],
                                              rows, cols, x.stride(0),
                                              ctypes.c_void_p(out.data_ptr()), DT[out.dtype],
                                              stream))


def executor_reduce(variant, x, out_dtype):
    out = torch.empty(x.shape[0], dtype=out_dtype, device=DEV)
    with C.Executor(0, mode=C.MODE_STREAM) as e:
        s = e.register_reduce("zz|" + ("sum" if variant == SUM else "mean"),
                              "sum" if variant == SUM else "mean")
        e.reduce(s, x, out, [1], False)
        e.flush(sync=True)
    return out


def exact(variant, x):
    """The double-precision sum (or mean) of every row, on the CPU."""
    d = x.double().cpu()
    return d.sum(dim=1) if variant == SUM else d.mean(dim=1)


def assert_close(got, want, x):
    tol = RED_REL * x.float().abs().sum(dim=1).double().cpu()
    if got.dtype != torch.float32:
        # one rounding of the fp32 result to the 16-bit output type on top
        tol = tol + want.double().abs().cpu() * 2.0 ** -7
    err = (got.double().cpu() - want.double().cpu()).abs()
    assert bool((err <= tol + 1e-30).all()), float((err - tol).max())


@pytest.mark.gpu
def test_noalloc_matches_executor_on_two_calls():
    g = torch.Generator(device="cpu").manual_seed(7)
    # call 1: 300 rows of 20,000 fp32 columns, split into 3 segments each
    x1 = torch.randn(300, 20000, generator=g).to(DEV)
    # call 2: 1,000 bf16 rows of 9,000 columns (2 segments) in a padded layout,
    # reusing the counters and partial sums call 1 left in the static array
    x2 = torch.randn(1000, 9008, generator=g).to(torch.bfloat16).to(DEV)[:, :9000]
    o1 = torch.empty(300, dtype=torch.float32, device=DEV)
    o2 = torch.empty(1000, dtype=torch.float32, device=DEV)
    noalloc(SUM, x1, o1)
    noalloc(MEAN, x2, o2)
    torch.cuda.synchronize()
    w1 = executor_reduce(SUM, x1, torch.float32)
    w2 = executor_reduce(MEAN, x2, torch.float32)
    assert_close(o1, w1, x1)
    assert_close(o2, w2, x2)
    assert_close(o1.cpu(), exact(SUM, x1), x1.cpu())
    assert_close(o2.cpu(), exact(MEAN, x2), x2.cpu())
    # and once more on the first input, now after call 2's scratch contents
    o3 = torch.empty(300, dtype=torch.float32, device=DEV)
    noalloc(SUM, x1, o3)
    torch.cuda.synchronize()
    assert_close(o3, w1, x1)
    assert_close(o3.cpu(), exact(SUM, x1), x1.cpu())


@pytest.mark.gpu
def test_noalloc_allocates_nothing_and_handles_unaligned_bf16():
    """A warmed call leaves the device's free memory as it was; a bf16 input
    one element off 16-byte alignment with rows longer than a segment (the
    scalar path with split rows) matches the double-precision sums."""
    g = torch.Generator(device="cpu").manual_seed(9)
    base = torch.randn(300 * 9001 + 1, generator=g).to(torch.bfloat16).to(DEV)
    x = base[1:].view(300, 9001)                 # odd offset and odd row stride
    o = torch.empty(300, dtype=torch.bfloat16, device=DEV)
    noalloc(SUM, x, o)                            # warm: device set-up on first use
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        noalloc(SUM, x, o)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert_close(o.cpu(), exact(SUM, x), x.cpu())
    assert_close(o, executor_reduce(SUM, x, torch.bfloat16), x)


@pytest.mark.gpu
def test_noalloc_short_rows_and_half_output():
    g = torch.Generator(device="cpu").manual_seed(8)
    x = torch.randn(4097, 333, generator=g).to(torch.float16).to(DEV)
    o = torch.empty(4097, dtype=torch.float16, device=DEV)
    noalloc(MEAN, x, o)
    torch.cuda.synchronize()
    assert_close(o, executor_reduce(MEAN, x, torch.float16), x)
    assert_close(o.cpu(), exact(MEAN, x), x.cpu())


def test_noalloc_rejects_sizes_beyond_the_scratch():
    # 65,537 split rows need more counters than the static array holds; the
    # check comes before any device work, so it runs without a GPU too
    with pytest.raises(C.GpuosError) as e:
        C.check(C.lib().gpuos_reduce_rows_noalloc(SUM, ctypes.c_void_p(16), 0, 65537, 8193, 8193,
                                                  ctypes.c_void_p(16), 0, None))
    assert e.value.code == C.EINVAL
    assert "static scratch" in str(e.value)
    with pytest.raises(C.GpuosError) as e:
        C.check(C.lib().gpuos_reduce_rows_noalloc(SUM, ctypes.c_void_p(16), 0, 20000, 90000, 90000,
                                                  ctypes.c_void_p(16), 0, None))
    assert e.value.code == C.EINVAL
