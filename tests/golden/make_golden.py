"""Generates tests/golden/*.npz: seeded inputs and the CPU oracle's outputs for
the quantized path.

The reference (Kotlin) cannot run on this machine and ships no golden vectors
for quantized results, so these fixtures record the oracle (oracle/kt_oracle.c,
a restatement of Engine/kotensor/src/main/kotlin/QuantizedTensor.kt:256-324 and
MatMul.kt:460-1003) on the shapes of the reference's own tests
(QuantizationTest.kt:77-108, DecodeKernelTest.kt:48-78) plus rounding and
clamping edge cases.  They pin the oracle against regressions and give the GPU
parity tests fixed inputs/outputs.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

# (m, k, n) of QuantizationTest.testDequantizingMatmulMatchesDequantizedWeights, minus the
# 256x1537 case (checked live on the GPU box instead, it would make the fixture large).
MATMUL_SHAPES = [(1, 70, 300), (1, 64, 64), (5, 130, 577), (40, 96, 33)]
# (k, n) of DecodeKernelTest.testSingleRowKernelsAgreeBitForBit that stay small.
DECODE_SHAPES = [(200, 33), (450, 129), (2, 17)]
QUANTIZATIONS = [(8, 64), (4, 64), (4, 32), (8, 1000)]


def edge_matrix() -> np.ndarray:
    """Rows x columns with rounding ties, clamps, zero / one-signed columns, tiny and huge values."""
    rng = np.random.default_rng(99)
    rows, cols = 67, 23
    w = ((rng.random((rows, cols), dtype=np.float32) - 0.5) * 0.2).astype(np.float32)
    w[:, 0] = 0.0                                    # all-zero column: scale 1, q 0
    w[:, 1] = np.abs(w[:, 1]) + 0.01                 # all positive: INT4 min clamps to 0
    w[:, 2] = -np.abs(w[:, 2]) - 0.01                # all negative: INT4 max clamps to 0
    w[:, 3] = np.float32(1e-36)                      # INT8 scale 7.9e-39 is subnormal (no flush to zero)
    w[::2, 3] = 0.0
    w[:, 4] = np.linspace(-3e30, 3e30, rows, dtype=np.float32)  # huge
    w[:, 5] = np.float32(127.0) * np.arange(rows, dtype=np.float32) / 64.0  # products near .5 ties
    w[:, 6] = np.float32(0.49999997)
    w[0, 6] = 1.0
    w[:, 7] = (np.arange(rows, dtype=np.float32) - 33.0) * np.float32(0.5)  # exact x.5 multiples
    w[:, 8] = -0.0
    return w


def main() -> None:
    O.build()
    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(2)
    for (m, k, n) in MATMUL_SHAPES:
        a = (rng.random((m, k), dtype=np.float32) - 0.5).astype(np.float32)
        w = ((rng.random((k, n), dtype=np.float32) - 0.5) * 0.2).astype(np.float32)
        dy = (rng.random((m, n), dtype=np.float32) - 0.5).astype(np.float32)
        key = f"mm_{m}_{k}_{n}"
        out[f"{key}/a"], out[f"{key}/w"], out[f"{key}/dy"] = a, w, dy
        for bits, g in QUANTIZATIONS:
            t = O.quantize(w, bits, g)
            qk = f"{key}/int{bits}g{g}"
            out[f"{qk}/qdata"], out[f"{qk}/scales"] = t.qdata, t.scales
            if t.zeros is not None:
                out[f"{qk}/zeros"] = t.zeros
            out[f"{qk}/y"] = O.multiply_quantized(a, t, accumulate=False)
            out[f"{qk}/y_acc"] = O.multiply_quantized(a, t, c=np.ones((m, n), np.float32), accumulate=True,
                                                      alpha=0.5)
            out[f"{qk}/dx"] = O.multiply_by_quantized_transposed(dy, t, accumulate=False)
    rng = np.random.default_rng(8)
    for (k, n) in DECODE_SHAPES:
        w = ((rng.random((k, n), dtype=np.float32) - 0.5) * 0.2).astype(np.float32)
        a = (rng.random((1, k), dtype=np.float32) - 0.5).astype(np.float32)
        key = f"dec_{k}_{n}"
        out[f"{key}/a"], out[f"{key}/w"] = a, w
        for bits, g in [(4, 64), (4, 32), (8, 64)]:
            t = O.quantize(w, bits, g)
            qk = f"{key}/int{bits}g{g}"
            out[f"{qk}/qdata"], out[f"{qk}/scales"] = t.qdata, t.scales
            if t.zeros is not None:
                out[f"{qk}/zeros"] = t.zeros
            out[f"{qk}/y"] = O.multiply_quantized(a, t, accumulate=False)
    w = edge_matrix()
    out["edge/w"] = w
    for bits, g in [(8, 64), (4, 64), (4, 16), (8, 1), (4, 1), (8, 100), (4, 5)]:
        t = O.quantize(w, bits, g)
        qk = f"edge/int{bits}g{g}"
        out[f"{qk}/qdata"], out[f"{qk}/scales"] = t.qdata, t.scales
        if t.zeros is not None:
            out[f"{qk}/zeros"] = t.zeros
    np.savez_compressed(os.path.join(HERE, "quantized_path.npz"), **out)
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main()
