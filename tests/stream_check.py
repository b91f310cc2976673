"""Whole-stream checks of the CUDA path against the oracle (test helper).

check_stream(stream, host_out) runs the oracle (oracle.run, all host cores)
over every request of a stream from tests/../gpuos_b200/workloads.py and
compares the GPU's output slab with it under the parity tolerances of
tests/tolerance.py:
  * exact operators and every cast: bit for bit;
  * transcendental operators: within CUDA's documented ulp bounds propagated
    through the formula, against the formula evaluated in double precision
    (one vectorised check per operator over all its requests);
  * sum/mean: |got - oracle| <= 2e-5 * sum|x| (each is within 1e-5 * sum|x|
    of the exact sum; plus one output ulp for 16-bit outputs).
Returns a summary dict; raises AssertionError listing the first failures.
"""
from __future__ import annotations

import numpy as np
import torch

import oracle
from tolerance import EXACT, RED_REL, check_transcendental


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int32 if t.dtype == torch.float32 else torch.int16)


def oracle_out(stream) -> torch.Tensor:
    out = torch.zeros(stream.out_bytes, dtype=torch.uint8)
    items = [(0 if r.kind == "ew" else 1, r.op, r.p0, r.p1, r.a.view(stream.host_in),
              r.b.view(stream.host_in) if r.b is not None else None, r.out.view(out),
              list(r.axes), r.keepdim) for r in stream.requests]
    oracle.run(oracle.make_reqs(items), 0)
    return out


def check_stream(stream, host_out: torch.Tensor, limit_fail: int = 20) -> dict:
    ref = oracle_out(stream)
    fails = []
    n_exact = n_tr = n_red = 0
    by_op = {}
    for i, r in enumerate(stream.requests):
        got = r.out.view(host_out)
        want = r.out.view(ref)
        a = r.a.view(stream.host_in)
        if r.kind == "reduce":
            # the GPU and the oracle are each within 1e-5 * sum|x| of the exact
            # sum, so they are within twice that of each other
            n_red += 1
            mag = a.float().abs().sum(dim=list(r.axes), keepdim=r.keepdim).double()
            cnt = 1
            for ax in r.axes:
                cnt *= a.shape[ax]
            if r.op == "mean" and cnt:
                mag = mag / cnt
            tol = 2 * RED_REL * mag + 1e-30
            if got.dtype != torch.float32:
                tol = tol + want.double().abs() * 2 ** -7
            err = (got.double() - want.double()).abs()
            if not bool((err <= tol).all()):
                fails.append(f"request {i} ({r.op} {tuple(a.shape)}): err/tol "
                             f"{float((err / tol).max()):.2f}")
            continue
        if r.op in EXACT or got.dtype != torch.float32:
            n_exact += 1
            if got.dtype != torch.float32 and r.op not in EXACT:
                # a transcendental rounded to 16 bits: within one output ulp
                diff = (got.double() - want.double()).abs()
                step = 2 ** -7 if got.dtype == torch.bfloat16 else 2 ** -10
                if not bool((diff <= want.double().abs() * step * 1.01 + 1e-30).all()):
                    fails.append(f"request {i} ({r.stream_op}): more than 1 output ulp off")
            elif not torch.equal(_bits(got.contiguous()), _bits(want.contiguous())):
                bad = (_bits(got.contiguous()) != _bits(want.contiguous())).nonzero()[:3].tolist()
                fails.append(f"request {i} ({r.stream_op}): not bit-exact at {bad}")
            continue
        n_tr += 1
        b = r.b.view(stream.host_in) if r.b is not None else None
        ex = torch.empty(got.shape, dtype=torch.float64)
        oracle.ew(r.op, a, b, ex, r.p0, r.p1, exact=True)
        d = by_op.setdefault((r.op, r.p0, r.p1), ([], [], [], []))
        d[0].append(torch.broadcast_to(a.float(), got.shape).reshape(-1).numpy())
        d[1].append(torch.broadcast_to(b.float(), got.shape).reshape(-1).numpy() if b is not None
                    else np.zeros(got.numel(), np.float32))
        d[2].append(got.reshape(-1).numpy())
        d[3].append(ex.reshape(-1).numpy())
        if len(fails) >= limit_fail:
            break
    worst = {}
    for (op, p0, p1), (A, B, G, E) in by_op.items():
        ok, w, j = check_transcendental(op, np.concatenate(A), np.concatenate(B),
                                        np.concatenate(G), np.concatenate(E), p0, p1)
        worst[op] = round(w, 3)
        if not ok:
            fails.append(f"{op}: error {w:.2f}x the bound at element {j} of its requests")
    assert not fails, "\n".join(fails[:limit_fail])
    return {"exact": n_exact, "transcendental": n_tr, "reduce": n_red, "worst_ratio": worst}
