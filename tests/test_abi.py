"""CPU checks of the C ABI: libkt_cuda.so loads, exports every function that
include/kt_cuda.h declares, the Python signatures cover the header, and the
host-side argument checks behave like the reference's require(...) calls.
No compute call is made here (no GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = set()
    for fname in os.listdir(os.path.join(ROOT, "include")):
        if not fname.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fname)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(kt_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol(kt):
    lib = kt.load_library()
    declared = header_functions()
    assert {"kt_init", "kt_quantize", "kt_qmatmul", "kt_qmatmul_t", "kt_qweight_upload"} <= declared
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_the_header(kt):
    from kotensor_b200 import _lib
    declared = header_functions()
    assert declared <= set(_lib.SIGNATURES), sorted(declared - set(_lib.SIGNATURES))


def test_version_and_quantization_checks(kt):
    lib = kt.load_library()
    assert lib.kt_version() >= 1
    assert lib.kt_check_quantization(8, 64) == 0
    assert lib.kt_check_quantization(4, 1) == 0
    assert lib.kt_check_quantization(3, 64) == 1
    assert b"bits must be 4 or 8" in lib.kt_last_error()
    assert lib.kt_check_quantization(4, 0) == 1
    assert b"groupSize must be positive" in lib.kt_last_error()


def test_python_quantization_mirror(kt):
    """Quantization(3) is rejected (QuantizationTest.kt:73); INT8/INT4 constants exist."""
    with pytest.raises(ValueError):
        kt.Quantization(3)
    with pytest.raises(ValueError):
        kt.Quantization(4, 0)
    assert (kt.Quantization.INT8.bits, kt.Quantization.INT8.group_size) == (8, 64)
    assert (kt.Quantization.INT4.bits, kt.Quantization.INT4.group_size) == (4, 64)
    assert repr(kt.Quantization(4, 32)) == "int4/g32"


def test_null_arguments_are_rejected_without_a_device(kt):
    lib = kt.load_library()
    assert lib.kt_qmatmul(None, None, None, None, 1, 0, ctypes.c_float(1.0), None, None) == 1
    assert lib.kt_quantize(None, 8, 64, 4, 4, None, None, None) == 1
    out = ctypes.c_void_p()
    assert lib.kt_init(-1, ctypes.byref(out)) != 0


def test_product_package_does_not_import_the_oracle():
    """The oracle is test infrastructure: nothing under kotensor_b200/ may import it."""
    pkg = os.path.join(ROOT, "kotensor_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".h", ".cuh", ".cpp")):
                text = open(os.path.join(dirpath, f), errors="replace").read()
                assert "oracle" not in re.sub(r"#.*|//.*", "", text).lower().replace("oracle_", ""), f


def test_matmul_argument_checks_follow_the_reference(kt):
    """MatMul.multiplyQuantized's require(...) checks and messages (MatMul.kt:470-473) and
    multiplyByQuantizedTransposed's (MatMul.kt:963-965), raised on the host before any
    device work; m == 0 is a no-op."""
    import numpy as np
    from types import SimpleNamespace
    w = SimpleNamespace(rows=4, columns=8)  # K = 4, N = 8: only the shape is read before the checks pass
    with pytest.raises(ValueError, match="Negative row count -1"):
        kt.MatMul.multiply_quantized(np.zeros(4, np.float32), w, np.zeros(8, np.float32), -1)
    with pytest.raises(ValueError, match="a has 7 elements, needs 2 × 4"):
        kt.MatMul.multiply_quantized(np.zeros(7, np.float32), w, np.zeros(16, np.float32), 2)
    with pytest.raises(ValueError, match="c has 15 elements, needs 2 × 8"):
        kt.MatMul.multiply_quantized(np.zeros(8, np.float32), w, np.zeros(15, np.float32), 2)
    kt.MatMul.multiply_quantized(np.zeros(0, np.float32), w, np.zeros(0, np.float32), 0)
    with pytest.raises(ValueError, match="dy has 15 elements, needs 2 × 8"):
        kt.MatMul.multiply_by_quantized_transposed(np.zeros(15, np.float32), w, np.zeros(8, np.float32), 2)
    with pytest.raises(ValueError, match="dx has 7 elements, needs 2 × 4"):
        kt.MatMul.multiply_by_quantized_transposed(np.zeros(16, np.float32), w, np.zeros(7, np.float32), 2)
    kt.MatMul.multiply_by_quantized_transposed(np.zeros(0, np.float32), w, np.zeros(0, np.float32), 0)


def test_quantized_tensor_constructor_checks_follow_the_reference(kt):
    """QuantizedTensor's init require(...) checks and messages (QuantizedTensor.kt:63-70),
    raised on the host before any device work."""
    import numpy as np
    QT = kt.QuantizedTensor
    with pytest.raises(ValueError, match=r"needs a 2-D shape, got \[4, 0\]"):
        QT.from_arrays(np.zeros(0, np.uint8), np.zeros(0, np.float32), None, (4, 0), 8, 64)
    with pytest.raises(ValueError, match="bits must be 4 or 8"):
        QT.from_arrays(np.zeros(16, np.uint8), np.zeros(4, np.float32), None, (4, 4), 3, 64)
    # INT4 split-half packing: 5 columns take 3 bytes per row
    with pytest.raises(ValueError, match="qdata has 10 bytes, expected 12"):
        QT.from_arrays(np.zeros(10, np.uint8), np.zeros(5, np.float32), np.zeros(5, np.uint8), (4, 5), 4, 64)
    with pytest.raises(ValueError, match="scales has 4 entries, expected 10"):
        QT.from_arrays(np.zeros(12, np.uint8), np.zeros(4, np.float32), np.zeros(10, np.uint8), (4, 5), 4, 2)
    with pytest.raises(ValueError, match="zeros has 5 entries, expected 10"):
        QT.from_arrays(np.zeros(12, np.uint8), np.zeros(10, np.float32), np.zeros(5, np.uint8), (4, 5), 4, 2)
    with pytest.raises(ValueError, match="4-bit tensors need zero points"):
        QT.from_arrays(np.zeros(12, np.uint8), np.zeros(5, np.float32), None, (4, 5), 4, 64)
