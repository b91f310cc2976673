"""Generate tests/golden/kat.json: known-answer vectors for the oracle and the
CUDA path.

The inputs are the reference's own test inputs:
  src/host.cpp:204,219             N = 1<<16, A[i] = 0.5 i, B[i] = 2 + (i % 7); C = A * B
  test/online_switch.cpp:150,156   N = 1<<15, A[i] = 0.5 i, B[i] = 1 + (i % 5); add, then mul
  test/dual_slot_switch.cpp:137-138 N = 1<<15, A[i] = 0.3 i, B[i] = 2 + (i % 9); add, mul, add
plus the [B,N] op [B,1] broadcast example whose wrong result the reference's
index decomposition (src/persistent_kernel.cu:20-31 after
pytorch_ext/gpuos_ext.cpp:147-165) gives, and fp16 / bf16 rounding cases.

Expected values are computed here with numpy float32 / torch arithmetic, an
implementation independent of the C oracle, so the fixtures pin the oracle.
Re-run:  python tests/golden/gen_golden.py
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "kat.json"


def bits(a: np.ndarray) -> list:
    return [int(x) for x in a.view(np.uint32)]


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def vec(n, scale, mod, off):
    i = np.arange(n, dtype=np.int64)
    A = (np.float32(scale) * i.astype(np.float32)).astype(np.float32)
    B = (np.float32(off) + (i % mod).astype(np.float32)).astype(np.float32)
    return A, B


def main():
    kat = {}
    # host.cpp: C = A * B
    A, B = vec(1 << 16, 0.5, 7, 2.0)
    C = (A * B).astype(np.float32)
    kat["host_mul"] = {"n": 1 << 16, "a": [0.5, "i"], "b": [2.0, 7], "op": "mul",
                       "head_bits": bits(C[:16]), "sha256": digest(C)}
    # online_switch.cpp: add then mul
    A, B = vec(1 << 15, 0.5, 5, 1.0)
    kat["online_add"] = {"n": 1 << 15, "a": [0.5, "i"], "b": [1.0, 5], "op": "add",
                         "head_bits": bits((A + B)[:16]), "sha256": digest((A + B).astype(np.float32))}
    kat["online_mul"] = {"n": 1 << 15, "a": [0.5, "i"], "b": [1.0, 5], "op": "mul",
                         "head_bits": bits((A * B)[:16]), "sha256": digest((A * B).astype(np.float32))}
    # dual_slot_switch.cpp: add, mul (after the alias switch), add (after rollback)
    A, B = vec(1 << 15, 0.3, 9, 2.0)
    for name, op, r in (("dual_add", "add", A + B), ("dual_mul", "mul", A * B)):
        r = r.astype(np.float32)
        kat[name] = {"n": 1 << 15, "a": [0.3, "i"], "b": [2.0, 9], "op": op,
                     "head_bits": bits(r[:16]), "sha256": digest(r)}
    # [B,N] + [B,1]: a[b, n] = n + 10 b, c[b] = 100 (b + 1)
    Bn, N = 3, 4
    a = (np.arange(N, dtype=np.float32)[None, :] + 10 * np.arange(Bn, dtype=np.float32)[:, None])
    c = (100.0 * (np.arange(Bn, dtype=np.float32) + 1))[:, None].astype(np.float32)
    correct = (a + c).astype(np.float32)
    # the reference decomposes the linear index over the [B,1] operand's own
    # sizes: offset = idx % B
    idx = np.arange(Bn * N)
    ref = (a.reshape(-1) + c.reshape(-1)[idx % Bn]).reshape(Bn, N).astype(np.float32)
    kat["bcast_col"] = {"B": Bn, "N": N, "a": a.tolist(), "c": c.reshape(-1).tolist(),
                        "torch": correct.tolist(), "reference": ref.tolist()}
    # rounding: fp32 -> fp16 (numpy, IEEE RNE) and fp32 -> bf16 (torch, RNE)
    vals = np.array([0.0, -0.0, 1.0, 1.0009765625, 1.00048828125, 1.000732421875, 65504.0,
                     65519.99, 65520.0, 1e-8, 2.9802322387695312e-08, 5.960464477539063e-08,
                     6.103515625e-05, 3.14159265, -2.71828182, 1e30, -1e-30, 0.1, 1.00390625,
                     1.005859375, 1.0078125, 3.3895314e38, 255.5, -1234.5678], dtype=np.float32)
    f16 = vals.astype(np.float16).view(np.uint16)
    bf16 = torch.from_numpy(vals.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    kat["round"] = {"f32_bits": bits(vals), "f16_bits": [int(x) for x in f16],
                    "bf16_bits": [int(x) for x in bf16]}
    # small exact reductions: integers, so every order gives the same sum
    x = (np.arange(15, dtype=np.float32).reshape(3, 5) - 7).astype(np.float32)
    kat["reduce_small"] = {"x": x.tolist(), "sum_last": x.sum(-1).tolist(),
                           "mean_last": (x.sum(-1) / np.float32(5)).astype(np.float32).tolist(),
                           "sum_first": x.sum(0).tolist()}
    OUT.write_text(json.dumps(kat, indent=1))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
