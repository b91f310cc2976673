"""Record the reference's own GPU outputs as fixtures — TEST INFRASTRUCTURE.

    python oracle/build_ref.py                    # here, where the reference's sources are
    python tests/golden/gen_ref_fixtures.py OUTDIR   # on a B200 (oracle/_ref travels)

Runs every case of tests/golden/ref_cases.py on the reference's own device
code (tests/golden/refrun.py: its op_batch, and its NVRTC elementwise and
reduce operators, one CTA per Task) and writes
  OUTDIR/ref_gpu.npz    the raw bytes of every case's output
  OUTDIR/ref_gpu.json   the cases, the reference files' sha256, the GPU, and
                        digests of the reference's outputs for the
                        exact-result operators of the whole 16,384-request
                        mixed stream
  OUTDIR/ref_rate.json  the reference's device-side rate on that stream
which are then copied into tests/golden/.  Nothing here waits on anything:
no persistent kernel runs, so synchronising the device is safe.

The rate: the reference runs the mixed stream as one op_batch shard per
flush of 512 for add/sub/mul/div (one CTA, the sub-Tasks one after another)
and one Task per request for every other operator (one CTA each).  Here each
flush's shard and its per-operator Task groups are launched at once on 9
streams, with no host cost between them: no enqueue round trip per Task
(pytorch_ext/gpuos_ext.cpp:297-319) and no 5 ms polling in flush
(:601-621).  That is more parallel than the reference's worker (one CTA per
SM) and free of its host costs, so the figure is an upper bound on the
reference's rate.
"""
from __future__ import annotations

import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

import ref_cases as RC  # noqa: E402
import refrun as RR  # noqa: E402


def run_cases(ref: RR.Reference, dev="cuda"):
    results = {}
    opb, ew, red = [], {}, {}
    live = []
    for c in RC.cases():
        a, b = RC.make_inputs(c, dev)
        out = torch.full(c.out_shape, float("nan"), dtype=RC.TDT[c.out_dtype], device=dev)
        if c.path == "opbatch":
            t = RR.binary_task(RR.OPBATCH_CODE[c.op], a, b, out)
            opb.append(t)
        elif c.path == "ew":
            t = RR.binary_task(20, a, b, out) if b is not None else RR.unary_task(20, a, out)
            ew.setdefault(f"ew_{c.op}", []).append(t)
        else:
            t = RR.reduce_task(20, a, out, list(c.axes), c.keepdim)
            red.setdefault(f"red_{c.op}", []).append(t)
        RR.check_bounds(t, [x for x in (a, b, out) if x is not None])
        live.append((c, a, b, out))
    ref.run_op_batch(opb)
    for m, ts in list(ew.items()) + list(red.items()):
        ref.run_tasks(m, ts)
    torch.cuda.synchronize()
    ref.release()
    for c, a, b, out in live:
        results[c.name] = out.contiguous().view(torch.uint8).cpu().numpy().reshape(-1).copy()
    return results


def mixed_stream_tasks(ref, stream, din, dout):
    """Per flush group: (op_batch sub-Tasks, {module: Tasks}) of the stream."""
    from gpuos_b200 import workloads as W
    views = stream.views(din, dout)
    groups = []
    fe = stream.flush_every
    for i in range(0, len(stream.requests), fe):
        subs, per = [], {}
        for r, (a, b, o) in zip(stream.requests[i:i + fe], views[i:i + fe]):
            if r.stream_op in W.BUILTIN_SUBMIT:
                t = RR.binary_task(RR.OPBATCH_CODE[r.stream_op], a, b, o)
                subs.append(t)
            elif b is not None:
                t = RR.binary_task(20, a, b, o)
                per.setdefault(f"ew_{r.stream_op}", []).append(t)
            else:
                t = RR.unary_task(20, a, o)
                per.setdefault(f"ew_{r.stream_op}", []).append(t)
            RR.check_bounds(t, [din, dout])
        groups.append((subs, per))
    return groups


def mixed_stream(ref, dev="cuda", reps=3):
    from gpuos_b200 import workloads as W
    stream = W.mixed_24op(seed=0)
    din, dout = stream.device_buffers(dev)
    groups = mixed_stream_tasks(ref, stream, din, dout)
    # the Task arrays, on the device once (their copies are not timed)
    staged = []
    for subs, per in groups:
        d_subs = ref.to_device(subs) if subs else None
        shards = None
        if subs:
            b = RR.Task()
            b.op, b.ndim, b.numel = RR.BATCH_SLOT, 1, len(subs)
            b.in0.data = d_subs.data_ptr()
            b.in0.ndim = 1
            b.in0.sizes[0], b.in0.strides[0] = len(subs), 1
            shards = ref.to_device([b])
        mods = [(m, ref.to_device(ts), len(ts)) for m, ts in per.items()]
        staged.append((d_subs, shards, mods))
    streams = [torch.cuda.Stream() for _ in range(9)]
    main = torch.cuda.current_stream()
    for m in {m for _, _, mods in staged for m, _, _ in mods}:
        ref.fn(m)

    def once():
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(main)
        for s in streams:
            s.wait_event(e0)
        for _, shards, mods in staged:
            if shards is not None:
                r = ref.lib.gpuos_ref_launch_op_batch(shards.data_ptr(), 1, RR.THREADS,
                                                      streams[0].cuda_stream)
                assert r == 0, r
            for k, (m, dt, n) in enumerate(mods):
                s = streams[1 + k % 8]
                ref.cu.launch(ref.fn(m), n, RR.THREADS, s.cuda_stream, dt.data_ptr())
        for s in streams:
            ev = torch.cuda.Event()
            ev.record(s)
            main.wait_event(ev)
        e1.record(main)
        e1.synchronize()
        return e0.elapsed_time(e1) / 1e3

    once()
    times = [once() for _ in range(reps)]
    best = min(times)
    out = dout.cpu()
    # digests of the exact-result operators' outputs, per operator in stream order
    digests = {}
    for r in stream.requests:
        if r.op in RC.EXACT or r.stream_op in RC.EXACT:
            t = r.out.view(out)
            digests.setdefault(r.stream_op, hashlib.sha256())
            digests[r.stream_op].update(t.contiguous().view(torch.uint8).numpy().tobytes())
    n = len(stream.requests)
    rate = {
        "workload": "mixed_24op: 16384 requests, 24 ops, f32, sizes log-uniform [256, 32768], "
                    "flush every 512",
        "requests": n, "seconds": best, "all_seconds": times,
        "requests_per_s": n / best,
        "algo_gbs": stream.algo_bytes / best / 1e9,
        "how": "reference device code only (op_batch shard + one CTA per JIT Task per flush "
               "group, launched at once on 9 streams, no host enqueue cost): an upper bound "
               "on the reference's rate",
    }
    return rate, {k: v.hexdigest() for k, v in digests.items()}


def main():
    # default: this directory, where the committed fixtures live
    outdir = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent
    outdir.mkdir(parents=True, exist_ok=True)
    ref = RR.Reference()
    t0 = time.time()
    res = run_cases(ref)
    np.savez_compressed(outdir / "ref_gpu.npz", **{k.replace("/", "__"): v for k, v in res.items()})
    rate, digests = mixed_stream(ref)
    props = torch.cuda.get_device_properties(0)
    meta = {
        "generated_by": "tests/golden/gen_ref_fixtures.py on the reference's device code "
                        "(oracle/build_ref.py)",
        "gpu": props.name, "torch": torch.__version__,
        "reference": RR.manifest()["sha256"], "nvrtc": RR.manifest()["nvrtc"],
        "cases": [c.name for c in RC.cases()],
        "mixed_24op_exact_digests": digests,
        "seconds": round(time.time() - t0, 1),
    }
    (outdir / "ref_gpu.json").write_text(json.dumps(meta, indent=1))
    (outdir / "ref_rate.json").write_text(json.dumps(rate, indent=1))
    print(json.dumps(rate))
    print(f"{len(res)} cases recorded")


if __name__ == "__main__":
    main()
