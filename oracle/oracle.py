"""ctypes wrapper over the CPU oracle (oracle/libkt_oracle.so).

TEST INFRASTRUCTURE ONLY.  The parity tests, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg import this module as the checker; the product
(``kotensor_b200``) never imports it.  The C restatement it wraps follows
Engine/kotensor/src/main/kotlin/QuantizedTensor.kt:172-324 and
Engine/kotensor/src/main/kotlin/MatMul.kt:460-1003 (citations per function in
kt_oracle.c).  Parity status: pinned to the reference's known-answer tests
(properties only); the reference ships no golden quantized outputs and cannot
run here, so outputs beyond those properties are "parity unpinned".
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libkt_oracle.so")
_lib = None

KTO_OK, KTO_ERR_ARG, KTO_ERR_NAN = 0, 1, 2


def build() -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE, "libkt_oracle.so"], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i32, i64, f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        L.kto_groups.argtypes, L.kto_groups.restype = [i32, i32], i32
        L.kto_bytes_per_row.argtypes, L.kto_bytes_per_row.restype = [i32, i32], i32
        L.kto_size_in_bytes.argtypes, L.kto_size_in_bytes.restype = [i32, i32, i32, i32], i64
        L.kto_round.argtypes, L.kto_round.restype = [f32, ctypes.POINTER(i32)], i32
        L.kto_quantize.argtypes, L.kto_quantize.restype = [P, i32, i32, i32, i32, P, P, P], i32
        L.kto_raw_value.argtypes, L.kto_raw_value.restype = [P, i32, i32, i32, i32], i32
        L.kto_value.argtypes, L.kto_value.restype = [P, P, P, i32, i32, i32, i32, i32], f32
        L.kto_dequantize.argtypes, L.kto_dequantize.restype = [P, P, P, i32, i32, i32, i32, P], None
        L.kto_dequantize_row.argtypes, L.kto_dequantize_row.restype = [P, P, P, i32, i32, i32, i32, i32, P], None
        L.kto_multiply_quantized.argtypes = [P, P, P, P, i32, i32, i32, i32, P, i32, i32, f32, i32]
        L.kto_multiply_quantized.restype = i32
        L.kto_multiply_by_quantized_transposed.argtypes = [P, P, P, P, i32, i32, i32, i32, P, i32, i32, i32]
        L.kto_multiply_by_quantized_transposed.restype = i32
        L.kto_multiply_dequantized_f64.argtypes = [P, P, P, P, i32, i32, i32, i32, P, i32]
        L.kto_multiply_dequantized_f64.restype = None
        _lib = L
    return _lib


def _p(arr):
    return None if arr is None else arr.ctypes.data_as(ctypes.c_void_p)


def jround(x: float) -> int:
    """Kotlin Float.roundToInt(); raises ValueError on NaN like Kotlin."""
    out = ctypes.c_int32()
    if lib().kto_round(ctypes.c_float(x), ctypes.byref(out)) != KTO_OK:
        raise ValueError("Cannot round NaN value.")
    return out.value


@dataclass
class OracleQTensor:
    """Host copy of a QuantizedTensor in the reference's byte layout."""
    qdata: np.ndarray   # uint8 [rows * bytesPerRow]
    scales: np.ndarray  # float32 [groups * columns]
    zeros: np.ndarray | None  # uint8 [groups * columns] (INT4 only)
    rows: int
    columns: int
    bits: int
    group_size: int

    @property
    def groups(self) -> int:
        return lib().kto_groups(self.rows, self.group_size)

    @property
    def bytes_per_row(self) -> int:
        return lib().kto_bytes_per_row(self.bits, self.columns)

    @property
    def stored_columns(self) -> int:
        return self.columns + self.columns % 2 if self.bits == 4 else self.columns

    @property
    def size_in_bytes(self) -> int:
        return lib().kto_size_in_bytes(self.bits, self.group_size, self.rows, self.columns)

    def raw_value(self, row: int, column: int) -> int:
        return lib().kto_raw_value(_p(self.qdata), self.bits, self.columns, row, column)

    def value(self, row: int, column: int) -> float:
        return lib().kto_value(_p(self.qdata), _p(self.scales), _p(self.zeros), self.bits, self.group_size,
                               self.columns, row, column)

    def dequantize_row(self, row: int) -> np.ndarray:
        out = np.empty(self.columns, np.float32)
        lib().kto_dequantize_row(_p(self.qdata), _p(self.scales), _p(self.zeros), self.bits, self.group_size,
                                 self.rows, self.columns, row, _p(out))
        return out

    def dequantize(self) -> np.ndarray:
        out = np.empty((self.rows, self.columns), np.float32)
        lib().kto_dequantize(_p(self.qdata), _p(self.scales), _p(self.zeros), self.bits, self.group_size,
                             self.rows, self.columns, _p(out))
        return out


def quantize(data: np.ndarray, bits: int, group_size: int = 64) -> OracleQTensor:
    """QuantizedTensor.quantize(data, rows, columns, Quantization(bits, groupSize))."""
    data = np.ascontiguousarray(data, dtype=np.float32)
    rows, columns = data.shape
    L = lib()
    groups = L.kto_groups(rows, group_size)
    bpr = L.kto_bytes_per_row(bits, columns)
    qdata = np.zeros(rows * bpr, np.uint8)
    scales = np.zeros(groups * columns, np.float32)
    zeros = np.zeros(groups * columns, np.uint8) if bits == 4 else None
    st = L.kto_quantize(_p(data), rows, columns, bits, group_size, _p(qdata), _p(scales), _p(zeros))
    if st == KTO_ERR_NAN:
        raise ValueError("Cannot round NaN value.")
    if st != KTO_OK:
        raise ValueError(f"invalid quantization arguments bits={bits} group={group_size} shape={data.shape}")
    return OracleQTensor(qdata, scales, zeros, rows, columns, bits, group_size)


def multiply_quantized(a: np.ndarray, w: OracleQTensor, c: np.ndarray | None = None, m: int | None = None,
                       accumulate: bool = False, alpha: float = 1.0, threads: int = 1) -> np.ndarray:
    """MatMul.multiplyQuantized(a, W, c, m, accumulate, alpha) (scalar reference arithmetic)."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    if m is None:
        m = a.size // w.rows
    if c is None:
        c = np.zeros(m * w.columns, np.float32)
    c = np.ascontiguousarray(c, dtype=np.float32).reshape(-1).copy()
    st = lib().kto_multiply_quantized(_p(a), _p(w.qdata), _p(w.scales), _p(w.zeros), w.bits, w.group_size,
                                      w.rows, w.columns, _p(c), m, int(accumulate), float(alpha), threads)
    if st != KTO_OK:
        raise ValueError("invalid arguments")
    return c.reshape(m, w.columns)


def multiply_by_quantized_transposed(dy: np.ndarray, w: OracleQTensor, dx: np.ndarray | None = None,
                                     m: int | None = None, accumulate: bool = False,
                                     threads: int = 1) -> np.ndarray:
    """MatMul.multiplyByQuantizedTransposed(dy, W, dx, m, accumulate)."""
    dy = np.ascontiguousarray(dy, dtype=np.float32).reshape(-1)
    if m is None:
        m = dy.size // w.columns
    if dx is None:
        dx = np.zeros(m * w.rows, np.float32)
    dx = np.ascontiguousarray(dx, dtype=np.float32).reshape(-1).copy()
    st = lib().kto_multiply_by_quantized_transposed(_p(dy), _p(w.qdata), _p(w.scales), _p(w.zeros), w.bits,
                                                    w.group_size, w.rows, w.columns, _p(dx), m, int(accumulate),
                                                    threads)
    if st != KTO_OK:
        raise ValueError("invalid arguments")
    return dx.reshape(m, w.rows)


def multiply_dequantized_f64(a: np.ndarray, w: OracleQTensor) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    m = a.size // w.rows
    c = np.zeros(m * w.columns, np.float64)
    lib().kto_multiply_dequantized_f64(_p(a), _p(w.qdata), _p(w.scales), _p(w.zeros), w.bits, w.group_size,
                                       w.rows, w.columns, _p(c), m)
    return c.reshape(m, w.columns)
