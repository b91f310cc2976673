"""Build the parity checker from the reference's own sources — TEST
INFRASTRUCTURE ONLY.

    python oracle/build_ref.py            # reference at $GPUOS_REFERENCE or /root/reference

Everything lands in oracle/_ref/ (git-ignored; it travels with the tree to a
GPU box, where the reference's sources are not present):

  libref_opbatch.so   the reference's op_batch (src/persistent_kernel.cu:81-112),
                      compiled by nvcc from src/persistent_kernel.cu where it
                      lies, with the flags of pytorch_ext/setup.py:27-28 and the
                      B200 gencode, plus the one-CTA-per-shard launcher
                      oracle/ref_opbatch_harness.cu.
  ew_<op>.ptx         the reference's JIT elementwise operator for each
                      expression of the reference scheduler's table, and
  red_<sum|mean>.ptx  its JIT reduce operator: the source text that
                      build_elementwise_src / build_reduce_src
                      (pytorch_ext/gpuos_ext.cpp:625-679, 710-812) generate,
                      compiled by NVRTC with the options of nvrtc_compile_ptx
                      (gpuos_ext.cpp:203-232) for compute_100 (what arch_opt()
                      picks on a B200), as PTX.  The driver JIT-compiles that
                      PTX when it is loaded, as the reference's
                      cuModuleLoadDataEx does (gpuos_ext.cpp:243).  Appended
                      to each generated source is a one-line kernel that runs
                      op_impl / op_reduce on one CTA per Task (the reference's
                      worker does the same through a device function pointer,
                      src/persistent_kernel.cu:168-177).
  scheduler.py        the reference's pytorch_ext/scheduler.py, unchanged, for
                      the drop-in test (tests/test_ref_scheduler_dropin.py).
  manifest.json       sha256 of every reference file used, the NVRTC version.

The generated sources are assembled from the string literals of those two
functions in gpuos_ext.cpp, read from the file itself; the recipe checks that
the literals it expects are there and fails loudly otherwise.  No source text
of the reference is written anywhere (only PTX and the compiled library), and
nothing here is committed except this recipe and the launcher.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
REF = Path(os.environ.get("GPUOS_REFERENCE", "/root/reference"))

# The reference scheduler's expression table (pytorch_ext/scheduler.py:145-153,
# 192-205, 244-290) for the operators of the 24-operator stream, keyed by the
# name the fixtures use.  The parametric ones carry the parameters the stream
# uses, formatted as the scheduler formats them (f"{float(v):.8f}f").
# Every string is checked to occur in scheduler.py (the parametric ones as
# their format templates).
EXPRESSIONS = {
    "add": ("(A + B)", 2), "sub": ("(A - B)", 2), "mul": ("(A * B)", 2), "div": ("(A / B)", 2),
    "maximum": ("(A > B ? A : B)", 2), "minimum": ("(A < B ? A : B)", 2),
    "pow": ("powf(A, B)", 2),
    "relu": ("(A > 0.f ? A : 0.f)", 1), "sigmoid": ("1.f / (1.f + expf(-A))", 1),
    "tanh": ("tanhf(A)", 1), "exp": ("expf(A)", 1), "log": ("logf(A)", 1),
    "sqrt": ("sqrtf(A)", 1), "abs": ("fabsf(A)", 1),
    "hardsigmoid": ("fminf(fmaxf(0.2f*A + 0.5f, 0.f), 1.f)", 1),
    "hardswish": ("A * fminf(fmaxf(A/6.f + 0.5f, 0.f), 1.f)", 1),
    "gelu": ("0.5f * A * (1.f + tanhf(0.79788456f*(A + 0.044715f*A*A*A)))", 1),
    "sin": ("sinf(A)", 1), "cos": ("cosf(A)", 1),
    "leaky_relu": ("(A >= 0.f ? A : 0.01000000f*A)", 1),
    "hardtanh": ("fminf(fmaxf(A, -1.00000000f), 1.00000000f)", 1),
    "elu": ("(A > 0.f ? A : 1.00000000f*(expf(A) - 1.f))", 1),
    "softplus": ("(log1pf(expf(1.00000000f*A))/1.00000000f)", 1),
    "clamp": ("fminf(fmaxf(A, -0.50000000f), 0.50000000f)", 1),
}
# parametric expressions: the f-string each one comes from in scheduler.py and
# the parameters the stream uses; the recipe checks that formatting the
# template with them gives the string above
PARAM_TEMPLATES = {
    "leaky_relu": ("(A >= 0.f ? A : {ns:.8f}f*A)", {"ns": 0.01}),
    "hardtanh": ("fminf(fmaxf(A, {mn:.8f}f), {mx:.8f}f)", {"mn": -1.0, "mx": 1.0}),
    "elu": ("(A > 0.f ? A : {alpha:.8f}f*(expf(A) - 1.f))", {"alpha": 1.0}),
    "softplus": ("(log1pf(expf({beta:.8f}f*A))/{beta:.8f}f)", {"beta": 1.0}),
    "clamp": ("fminf(fmaxf(A, {mn:.8f}f), {mx:.8f}f)", {"mn": -0.5, "mx": 0.5}),
}

# the one-CTA-per-Task launchers appended to the generated sources (our code)
EW_LAUNCHER = '\nextern "C" __global__ void gpuos_ref_run(const Task* tasks) { op_impl(tasks[blockIdx.x]); }\n'
RED_LAUNCHER = '\nextern "C" __global__ void gpuos_ref_run(const Task* tasks) { op_reduce(tasks[blockIdx.x]); }\n'


def sha(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


# ---- reading the generator functions' string literals -----------------------
_TOKEN = re.compile(r'R"\((.*?)\)"|"((?:[^"\\\n]|\\.)*)"', re.S)


def _unescape(s: str) -> str:
    return s.encode("latin-1").decode("unicode_escape")


def function_literals(text: str, signature: str, end_marker: str):
    """The string literals (raw and plain, in order) of one function body."""
    i = text.index(signature)
    j = text.index(end_marker, i)
    body = text[i + len(signature):j]
    out = []
    for m in _TOKEN.finditer(body):
        if m.group(1) is not None:
            out.append(("raw", m.group(1)))
        else:
            out.append(("str", _unescape(m.group(2))))
    return out


def elementwise_source(lits, expr: str, arity: int) -> str:
    """build_elementwise_src(expr, arity), gpuos_ext.cpp:625-679."""
    kinds = [k for k, _ in lits]
    vals = [v for _, v in lits]
    want_kinds = ["raw", "raw", "str", "str", "str", "str", "str", "str", "raw"]
    if kinds != want_kinds or vals[2:8] != ["        float R = ", "(", ")", "(", ")", ";\n"]:
        raise SystemExit("build_elementwise_src no longer has the expected literals: "
                         f"{kinds} {vals[2:8]}")
    src = vals[0]
    if arity == 2:
        src += vals[1]
    src += vals[2] + "(" + expr + ")" + ";\n"
    src += vals[8]
    return src


def reduce_source(lits, op_name: str) -> str:
    """build_reduce_src(op_name), gpuos_ext.cpp:710-812."""
    kinds = [k for k, _ in lits]
    vals = [v for _, v in lits]
    want = ["raw", "str", "str", "raw", "str", "str", "raw"]
    if kinds != want or vals[1] != "mean" or vals[4] != "mean" or \
            vals[2] != "              outv = outv / (float)red_N;\n" or \
            vals[5] != "        acc = acc / (float)red_N;\n":
        raise SystemExit(f"build_reduce_src no longer has the expected literals: {kinds}")
    mean = op_name == "mean"
    return vals[0] + (vals[2] if mean else "") + vals[3] + (vals[5] if mean else "") + vals[6]


# ---- NVRTC, as nvrtc_compile_ptx (gpuos_ext.cpp:216-232) calls it -----------
def nvrtc():
    for cand in (CUDA_HOME / "lib64" / "libnvrtc.so.12", CUDA_HOME / "lib64" / "libnvrtc.so"):
        if cand.exists():
            L = ctypes.CDLL(str(cand))
            break
    else:
        raise SystemExit("NVRTC not found under CUDA_HOME")
    L.nvrtcGetErrorString.restype = ctypes.c_char_p
    return L


def nvrtc_ptx(L, src: str, name: str, arch: str) -> bytes:
    prog = ctypes.c_void_p()
    r = L.nvrtcCreateProgram(ctypes.byref(prog), src.encode(), name.encode(), 0, None, None)
    if r:
        raise SystemExit(f"nvrtcCreateProgram: {r}")
    opts = [f"--gpu-architecture={arch}", "--std=c++17", "--relocatable-device-code=true",
            "-rdc=true", "--device-as-default-execution-space",
            f"-I{CUDA_HOME / 'include'}", "-I/usr/include"]
    arr = (ctypes.c_char_p * len(opts))(*[o.encode() for o in opts])
    res = L.nvrtcCompileProgram(prog, len(opts), arr)
    n = ctypes.c_size_t()
    L.nvrtcGetProgramLogSize(prog, ctypes.byref(n))
    log = ctypes.create_string_buffer(n.value)
    L.nvrtcGetProgramLog(prog, log)
    if res:
        raise SystemExit(f"NVRTC failed for {name}: {L.nvrtcGetErrorString(res).decode()}\n"
                         f"{log.value.decode(errors='replace')}")
    L.nvrtcGetPTXSize(prog, ctypes.byref(n))
    ptx = ctypes.create_string_buffer(n.value)
    L.nvrtcGetPTX(prog, ptx)
    L.nvrtcDestroyProgram(ctypes.byref(prog))
    return ptx.raw.rstrip(b"\0") + b"\0"


def nvrtc_version(L) -> str:
    a, b = ctypes.c_int(), ctypes.c_int()
    L.nvrtcVersion(ctypes.byref(a), ctypes.byref(b))
    return f"{a.value}.{b.value}"


def main() -> int:
    ext = REF / "pytorch_ext" / "gpuos_ext.cpp"
    pk = REF / "src" / "persistent_kernel.cu"
    sched = REF / "pytorch_ext" / "scheduler.py"
    for p in (ext, pk, sched, REF / "src" / "common.h"):
        if not p.exists():
            print(f"reference source missing: {p}; oracle/_ref not built", file=sys.stderr)
            return 1
    OUT.mkdir(exist_ok=True)
    text = ext.read_text()
    stext = sched.read_text()
    # the option strings of nvrtc_compile_ptx, as the file has them
    for opt in ('"--std=c++17"', '"--relocatable-device-code=true"', '"-rdc=true"',
                '"--device-as-default-execution-space"', "compute_%d%d"):
        if opt not in text:
            raise SystemExit(f"nvrtc_compile_ptx no longer passes {opt}")
    for name, (expr, _) in EXPRESSIONS.items():
        if name in PARAM_TEMPLATES:
            tmpl, params = PARAM_TEMPLATES[name]
            if f"f'{tmpl}'" not in stext or tmpl.format(**params) != expr:
                raise SystemExit(f"scheduler.py no longer builds {name} as {tmpl}")
        elif expr not in stext:
            raise SystemExit(f"scheduler.py no longer has the expression {expr!r} ({name})")

    ew_lits = function_literals(text, "static std::string build_elementwise_src(",
                                "static int ensure_elementwise_registered(")
    red_lits = function_literals(text, "static std::string build_reduce_src(",
                                 "static int ensure_reduce_registered(")
    L = nvrtc()
    arch = "compute_100"  # arch_opt() on a compute-capability 10.0 device
    built = {}
    for name, (expr, arity) in EXPRESSIONS.items():
        src = elementwise_source(ew_lits, expr, arity) + EW_LAUNCHER
        ptx = nvrtc_ptx(L, src, "batch.cu", arch)
        (OUT / f"ew_{name}.ptx").write_bytes(ptx)
        built[f"ew_{name}"] = {"expr": expr, "arity": arity}
    for op in ("sum", "mean"):
        ptx = nvrtc_ptx(L, reduce_source(red_lits, op) + RED_LAUNCHER, "batch.cu", arch)
        (OUT / f"red_{op}.ptx").write_bytes(ptx)
        built[f"red_{op}"] = {"op": op}

    # op_batch: nvcc on the reference's own translation unit
    nvcc = CUDA_HOME / "bin" / "nvcc"
    lib = OUT / "libref_opbatch.so"
    cmd = [str(nvcc), "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC", "-shared",
           "-I", str(REF / "src"), str(HERE / "ref_opbatch_harness.cu"), "-o", str(lib)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise SystemExit("nvcc failed on the reference's persistent_kernel.cu")

    shutil.copyfile(sched, OUT / "scheduler.py")
    manifest = {
        "sha256": {"pytorch_ext/gpuos_ext.cpp": sha(ext), "src/persistent_kernel.cu": sha(pk),
                   "src/common.h": sha(REF / "src" / "common.h"),
                   "pytorch_ext/scheduler.py": sha(sched)},
        "nvrtc": nvrtc_version(L), "nvrtc_arch": arch,
        "nvcc_flags": cmd[1:8],
        "modules": built,
    }
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1))
    print(f"oracle/_ref: {len(built)} JIT modules, libref_opbatch.so, scheduler.py")
    return 0


if __name__ == "__main__":
    sys.exit(main())
