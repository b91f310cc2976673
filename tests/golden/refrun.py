"""Run the reference's own device code on a GPU — PARITY CHECKER ONLY.

Loads what oracle/build_ref.py built into oracle/_ref/ (the reference's
op_batch compiled from src/persistent_kernel.cu, and its NVRTC elementwise
and reduce operators as PTX) and runs reference Tasks on them: one CTA of
256 threads per Task, as the reference's persistent worker runs a Task
(src/persistent_kernel.cu:133-200, default threads_per_block 256,
pytorch_ext/gpuos_ext.cpp:863).  No persistent kernel, queue or device
function pointer is involved, so nothing here waits on anything.

Tasks are built the way the reference's extension builds them from tensors
(pytorch_ext/gpuos_ext.cpp):
  fill_tensorref        :147-165   right-aligned sizes, stride 0 for size 1
  build_binary_task     :167-184   output contiguous
  build_unary_task      :186-201   in1 = null, sizes 1, strides 0
  build_reduce_task     :827-845   in0 = the input's own sizes and strides
  flush's shard Tasks   :586-599   op 10, numel = sub-Task count, in0.data =
                                   the sub-Task array
Before any launch, every offset the reference's index decomposition
(linear_to_offset, src/persistent_kernel.cu:20-31) can form for a Task is
checked on the CPU against the bytes its tensor's storage holds.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
REF_DIR = ROOT / "oracle" / "_ref"

DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
OPBATCH_CODE = {"add": 0, "mul": 1, "sub": 2, "div": 3}
BATCH_SLOT = 10
THREADS = 256


class TensorRef(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8)]


class Task(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("flags", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("numel", ctypes.c_int64), ("rrank", ctypes.c_int32),
                ("r_axes", ctypes.c_int32 * 8), ("r_keepdim", ctypes.c_int32),
                ("in0", TensorRef), ("in1", TensorRef), ("out0", TensorRef)]


assert ctypes.sizeof(TensorRef) == 144 and ctypes.sizeof(Task) == 496
assert Task.numel.offset == 16 and Task.rrank.offset == 24 and Task.in0.offset == 64
assert Task.in1.offset == 208 and Task.out0.offset == 352


def available() -> bool:
    return (REF_DIR / "manifest.json").exists() and (REF_DIR / "libref_opbatch.so").exists()


def manifest() -> dict:
    return json.loads((REF_DIR / "manifest.json").read_text())


# ---- Task building (the reference's host code, restated) --------------------
def _storage_span(t: torch.Tensor):
    """First and one-past-last byte of t's storage."""
    st = t.untyped_storage()
    return st.data_ptr(), st.data_ptr() + st.nbytes()


def fill_tensorref(tr: TensorRef, ten: torch.Tensor, out_sizes):
    out_ndim = len(out_sizes)
    tr.data = ten.data_ptr()
    tr.dtype = DT.get(ten.dtype, 0)
    tr.ndim = out_ndim
    in_nd = ten.dim()
    for d in range(out_ndim):
        od, i = out_ndim - 1 - d, in_nd - 1 - d
        size_in = ten.size(i) if i >= 0 else 1
        stride_in = ten.stride(i) if i >= 0 else 0
        tr.sizes[od] = size_in
        tr.strides[od] = 0 if size_in == 1 else stride_in


def _out_contig(tr: TensorRef, out: torch.Tensor):
    tr.data = out.data_ptr()
    tr.dtype = DT.get(out.dtype, 0)
    tr.ndim = out.dim()
    stride = 1
    for d in range(out.dim() - 1, -1, -1):
        tr.sizes[d] = out.size(d)
        tr.strides[d] = stride
        stride *= out.size(d)


def binary_task(op: int, a, b, out) -> Task:
    t = Task()
    t.op, t.flags, t.ndim, t.numel = op, 0, out.dim(), out.numel()
    _out_contig(t.out0, out)
    fill_tensorref(t.in0, a, list(out.shape))
    fill_tensorref(t.in1, b, list(out.shape))
    return t


def unary_task(op: int, x, out) -> Task:
    t = Task()
    t.op, t.flags, t.ndim, t.numel = op, 0, out.dim(), out.numel()
    _out_contig(t.out0, out)
    fill_tensorref(t.in0, x, list(out.shape))
    t.in1.data = None
    t.in1.dtype = t.in0.dtype
    t.in1.ndim = out.dim()
    for i in range(out.dim()):
        t.in1.sizes[i], t.in1.strides[i] = 1, 0
    return t


def reduce_task(op: int, x, out, axes, keepdim: bool) -> Task:
    t = Task()
    t.op, t.flags, t.ndim, t.numel = op, 0, out.dim(), out.numel()
    t.rrank, t.r_keepdim = len(axes), 1 if keepdim else 0
    for i, ax in enumerate(axes):
        t.r_axes[i] = ax
    t.in0.data, t.in0.dtype, t.in0.ndim = x.data_ptr(), DT.get(x.dtype, 0), x.dim()
    for i in range(x.dim()):
        t.in0.sizes[i], t.in0.strides[i] = x.size(i), x.stride(i)
    _out_contig(t.out0, out)
    t.in1.data = None
    t.in1.ndim = out.dim()
    for i in range(out.dim()):
        t.in1.sizes[i], t.in1.strides[i] = 1, 0
    return t


def _esz(code: int) -> int:
    return 4 if code == 0 else 2


def check_bounds(t: Task, tensors):
    """Every element offset linear_to_offset can form for each TensorRef of
    t (indices in [0, size_d) per dim, so 0 .. sum (size_d - 1) * stride_d
    for the nonnegative strides used here) stays inside the storage of the
    tensor it points into."""
    spans = [_storage_span(x) for x in tensors]
    refs = [t.in0, t.out0] + ([t.in1] if t.in1.data else [])
    for tr in refs:
        lo = hi = 0
        for d in range(tr.ndim):
            n = max(tr.sizes[d], 1)
            s = tr.strides[d]
            if s < 0:
                lo += (n - 1) * s
            else:
                hi += (n - 1) * s
        e = _esz(tr.dtype)
        first, last = tr.data + lo * e, tr.data + hi * e + e
        if not any(s0 <= first and last <= s1 for s0, s1 in spans):
            raise AssertionError(f"reference Task would read outside its tensors: {first:#x}..{last:#x}")


# ---- running ---------------------------------------------------------------
class _Cuda:
    """The few driver calls needed to load PTX and launch (libcuda.so.1)."""

    def __init__(self):
        L = ctypes.CDLL("libcuda.so.1")
        self.L = L
        for n in ("cuModuleLoadData", "cuModuleGetFunction", "cuLaunchKernel", "cuModuleUnload",
                  "cuInit", "cuGetErrorString"):
            getattr(L, n).restype = ctypes.c_int
        self.check(L.cuInit(0), "cuInit")

    def check(self, r, what):
        if r != 0:
            s = ctypes.c_char_p()
            self.L.cuGetErrorString(r, ctypes.byref(s))
            raise RuntimeError(f"{what}: CUDA driver error {r} ({s.value})")

    def load(self, ptx: bytes):
        mod = ctypes.c_void_p()
        self.check(self.L.cuModuleLoadData(ctypes.byref(mod), ctypes.c_char_p(ptx)),
                   "cuModuleLoadData")
        fn = ctypes.c_void_p()
        self.check(self.L.cuModuleGetFunction(ctypes.byref(fn), mod, b"gpuos_ref_run"),
                   "cuModuleGetFunction")
        return mod, fn

    def launch(self, fn, grid: int, block: int, stream: int, tasks_ptr: int):
        arg = ctypes.c_void_p(tasks_ptr)
        params = (ctypes.c_void_p * 1)(ctypes.addressof(arg))
        self.check(self.L.cuLaunchKernel(fn, grid, 1, 1, block, 1, 1, 0, ctypes.c_void_p(stream),
                                         params, None), "cuLaunchKernel")


class Reference:
    """The reference's operators, loaded once: module name -> kernel."""

    def __init__(self):
        if not available():
            raise RuntimeError("oracle/_ref is not built (python oracle/build_ref.py)")
        torch.cuda.init()
        torch.empty(1, device="cuda")  # the primary context is current from here on
        self.cu = _Cuda()
        self.fns = {}
        self.mods = []
        self.lib = ctypes.CDLL(str(REF_DIR / "libref_opbatch.so"))
        self.lib.gpuos_ref_launch_op_batch.restype = ctypes.c_int
        self.lib.gpuos_ref_launch_op_batch.argtypes = [ctypes.c_void_p, ctypes.c_int,
                                                       ctypes.c_int, ctypes.c_void_p]
        assert self.lib.gpuos_ref_task_size() == 496
        self.keep = []

    def fn(self, module: str):
        f = self.fns.get(module)
        if f is None:
            mod, f = self.cu.load((REF_DIR / f"{module}.ptx").read_bytes())
            self.mods.append(mod)
            self.fns[module] = f
        return f

    @staticmethod
    def to_device(tasks) -> torch.Tensor:
        n = len(tasks)
        arr = (Task * n)(*tasks)
        host = torch.frombuffer(bytearray(arr), dtype=torch.uint8)
        return host.cuda()

    def run_tasks(self, module: str, tasks, stream=None):
        """One CTA per Task of `module` (an ew_* or red_* operator)."""
        if not tasks:
            return
        dev = self.to_device(tasks)
        self.keep.append(dev)
        s = stream if stream is not None else torch.cuda.current_stream()
        self.cu.launch(self.fn(module), len(tasks), THREADS, s.cuda_stream, dev.data_ptr())

    def run_op_batch(self, subs, shard=512, stream=None):
        """The builtin path: sub-Tasks (op 0..3) in shards of `shard`, one
        CTA per shard, as flush() enqueues them."""
        if not subs:
            return
        d_subs = self.to_device(subs)
        shards = []
        for start in range(0, len(subs), shard):
            cnt = min(shard, len(subs) - start)
            b = Task()
            b.op, b.flags, b.ndim, b.numel = BATCH_SLOT, 0, 1, cnt
            b.in0.data = d_subs.data_ptr() + start * ctypes.sizeof(Task)
            b.in0.dtype, b.in0.ndim = 0, 1
            b.in0.sizes[0], b.in0.strides[0] = cnt, 1
            b.in1.data = None
            b.out0.data = None
            shards.append(b)
        d_sh = self.to_device(shards)
        self.keep += [d_subs, d_sh]
        s = stream if stream is not None else torch.cuda.current_stream()
        r = self.lib.gpuos_ref_launch_op_batch(d_sh.data_ptr(), len(shards), THREADS,
                                               ctypes.c_void_p(s.cuda_stream))
        if r:
            raise RuntimeError(f"op_batch launch failed: cudaError {r}")

    def release(self):
        """Drop the Task arrays kept alive for launches (after a sync)."""
        self.keep.clear()
