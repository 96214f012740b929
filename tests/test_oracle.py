"""CPU tests of the oracle (oracle/kt_oracle.c) -- the checker every GPU parity
test relies on.

Each test ports a known-answer or property test of the reference's own suite
(Engine/kotensor/src/test/kotlin/QuantizationTest.kt, DecodeKernelTest.kt) to
the oracle, so the oracle is pinned to everything the reference pins for this
path.  An independent numpy restatement of the quantizer cross-checks the C
oracle byte for byte, and the committed golden fixtures pin it against
regressions.
"""
import numpy as np
import pytest


def uniform(rng, shape, scale):
    return ((rng.random(shape, dtype=np.float32) * 2 - 1) * scale).astype(np.float32)


# ----------------------------------------------------------------- numpy restatement

def np_java_round(x):
    """Math.round(float) vectorised (ties toward +inf, saturating); x has no NaN."""
    x = np.asarray(x, np.float32)
    f = np.floor(x)
    r = np.where((x - f) >= np.float32(0.5), f + np.float32(1), f)
    r = np.clip(r.astype(np.float64), -2147483648.0, 2147483647.0)
    return r.astype(np.int64)


def np_quantize(w, bits, g):
    """QuantizedTensor.quantize (QuantizedTensor.kt:261-324) restated with numpy float32 ops."""
    rows, cols = w.shape
    groups = (rows + g - 1) // g
    half = (cols + cols % 2) // 2 if bits == 4 else cols
    scales = np.zeros((groups, cols), np.float32)
    zeros = np.zeros((groups, cols), np.uint8)
    qv = np.zeros((rows, cols), np.int64)
    for gi in range(groups):
        blk = w[gi * g:(gi + 1) * g]
        if bits == 8:
            max_abs = np.maximum(np.abs(blk).max(axis=0), np.float32(0))
            scale = np.where(max_abs > 0, max_abs / np.float32(127), np.float32(1)).astype(np.float32)
            inv = (np.float32(1) / scale).astype(np.float32)
            q = np.clip(np_java_round(blk * inv), -127, 127)
        else:
            mn = np.minimum(blk.min(axis=0), np.float32(0))
            mx = np.maximum(blk.max(axis=0), np.float32(0))
            rng_ = (mx - mn).astype(np.float32)
            scale = np.where(rng_ > 0, rng_ / np.float32(15), np.float32(1)).astype(np.float32)
            zero = np.clip(np_java_round((-mn) / scale), 0, 15)
            zeros[gi] = zero
            inv = (np.float32(1) / scale).astype(np.float32)
            q = np.clip(np_java_round(blk * inv) + zero, 0, 15)
        scales[gi] = scale
        qv[gi * g:(gi + 1) * g] = q
    if bits == 8:
        qdata = qv.astype(np.int8).view(np.uint8).reshape(-1)
        return qdata, scales.reshape(-1), None
    packed = np.zeros((rows, half), np.uint8)
    packed |= qv[:, :half].astype(np.uint8)
    hi = qv[:, half:].astype(np.uint8)
    packed[:, :hi.shape[1]] |= (hi << 4).astype(np.uint8)
    return packed.reshape(-1), scales.reshape(-1), zeros.reshape(-1)


# ----------------------------------------------------------------- tests

def test_java_round_semantics(oracle):
    cases = {0.5: 1, -0.5: 0, 1.5: 2, -1.5: -1, 2.5: 3, -2.5: -2, 0.49999997: 0, -0.49999997: 0,
             126.5: 127, -126.5: -126, 3e9: 2147483647, -3e9: -2147483648, float("inf"): 2147483647,
             float("-inf"): -2147483648, 8388609.0: 8388609, -0.0: 0}
    for x, want in cases.items():
        assert oracle.jround(x) == want, x
    with pytest.raises(ValueError):
        oracle.jround(float("nan"))


def test_quantize_dequantize_error_bounds(oracle):
    """QuantizationTest.testQuantizeDequantizeErrorBounds (QuantizationTest.kt:38-74)."""
    rng = np.random.default_rng(1)
    rows, cols = 100, 37
    w = uniform(rng, (rows, cols), 0.3)
    int8 = oracle.quantize(w, 8, 64)
    assert int8.bits == 8 and int8.groups == 2 and int8.zeros is None
    assert int8.qdata.size == rows * cols
    assert np.abs(w - int8.dequantize()).max() <= 0.3 / 127 + 1e-6
    int4 = oracle.quantize(w, 4, 32)
    assert int4.groups == 4 and int4.stored_columns == 38 and int4.bytes_per_row == 19
    assert int4.qdata.size == rows * 19 and int4.zeros.size == 4 * cols
    deq = int4.dequantize()
    assert np.abs(w - deq).max() <= 0.6 / 15 / 2 + 1e-6
    for r in range(0, rows, 7):
        for c in range(cols):
            assert 0 <= int4.raw_value(r, c) <= 15
            assert int4.value(r, c) == deq[r, c]
    z = np.zeros((rows, cols), np.float32)
    assert np.abs(oracle.quantize(z, 4, 64).dequantize()).max() == 0
    assert np.abs(oracle.quantize(z, 8, 64).dequantize()).max() == 0
    assert int8.size_in_bytes == rows * cols + 2 * cols * 4
    assert int4.size_in_bytes == rows * 19 + 4 * cols * 4 + 4 * cols


@pytest.mark.parametrize("bits,g", [(8, 64), (4, 64), (4, 32), (8, 1000), (4, 1), (8, 1), (4, 7)])
@pytest.mark.parametrize("shape", [(100, 37), (64, 64), (130, 577), (3, 1), (1, 2)])
def test_c_oracle_matches_numpy_restatement(oracle, bits, g, shape):
    rng = np.random.default_rng(hash((bits, g, shape)) % 2**32)
    w = uniform(rng, shape, 0.2)
    t = oracle.quantize(w, bits, g)
    q, s, z = np_quantize(w, bits, g)
    assert np.array_equal(t.qdata, q)
    assert np.array_equal(t.scales.view(np.uint32), s.view(np.uint32))
    if bits == 4:
        assert np.array_equal(t.zeros, z)


def test_edge_matrix_matches_numpy_restatement(oracle, golden):
    w = golden["edge/w"]
    for bits, g in [(8, 64), (4, 64), (4, 16), (8, 1), (4, 1), (8, 100), (4, 5)]:
        t = oracle.quantize(w, bits, g)
        q, s, z = np_quantize(w, bits, g)
        assert np.array_equal(t.qdata, q), (bits, g)
        assert np.array_equal(t.scales.view(np.uint32), s.view(np.uint32)), (bits, g)
        if bits == 4:
            assert np.array_equal(t.zeros, z), (bits, g)


def test_oracle_reproduces_golden_fixtures(oracle, golden):
    """Regression pin: the committed fixtures are reproduced bit for bit."""
    checked = 0
    for key in golden:
        if not key.endswith("/qdata"):
            continue
        base = key[: -len("/qdata")]
        shape_key, qname = base.rsplit("/", 1)
        bits = int(qname[3]) if qname[4] == "g" else int(qname[3:5])
        g = int(qname.split("g", 1)[1])
        w = golden[f"{shape_key}/w"]
        t = oracle.quantize(w, bits, g)
        assert np.array_equal(t.qdata, golden[f"{base}/qdata"]), base
        assert np.array_equal(t.scales.view(np.uint32), golden[f"{base}/scales"].view(np.uint32)), base
        if bits == 4:
            assert np.array_equal(t.zeros, golden[f"{base}/zeros"]), base
        if f"{base}/y" in golden:
            a = golden[f"{shape_key}/a"]
            y = oracle.multiply_quantized(a, t, accumulate=False)
            assert np.array_equal(y.view(np.uint32), golden[f"{base}/y"].view(np.uint32)), base
        checked += 1
    assert checked >= 30


@pytest.mark.parametrize("m,k,n", [(1, 70, 300), (1, 64, 64), (5, 130, 577), (40, 96, 33), (1, 256, 1537)])
@pytest.mark.parametrize("bits,g", [(8, 64), (4, 64), (4, 32), (8, 1000)])
def test_dequantizing_matmul_matches_dequantized_weights(oracle, m, k, n, bits, g):
    """QuantizationTest.testDequantizingMatmulMatchesDequantizedWeights (QuantizationTest.kt:77-108)."""
    rng = np.random.default_rng(2)
    a = (rng.random((m, k), dtype=np.float32) - 0.5).astype(np.float32)
    w = ((rng.random((k, n), dtype=np.float32) - 0.5) * 0.2).astype(np.float32)
    t = oracle.quantize(w, bits, g)
    deq = t.dequantize()
    expected = a.astype(np.float64) @ deq.astype(np.float64)
    actual = oracle.multiply_quantized(a, t, accumulate=False)
    assert np.abs(expected - actual).max() < 1e-4
    acc = oracle.multiply_quantized(a, t, c=np.ones((m, n), np.float32), accumulate=True, alpha=0.5)
    assert np.abs(acc - (1.0 + 0.5 * expected)).max() < 1e-4
    dy = (rng.random((m, n), dtype=np.float32) - 0.5).astype(np.float32)
    dx = oracle.multiply_by_quantized_transposed(dy, t, accumulate=False)
    assert np.abs(dx - dy.astype(np.float64) @ deq.T.astype(np.float64)).max() < 1e-3


def test_parallel_quantized_kernel_matches_serial(oracle):
    """QuantizationTest.testParallelQuantizedKernelMatchesSerial (QuantizationTest.kt:111-134)."""
    rng = np.random.default_rng(4)
    k, n = 300, 2100
    a = (rng.random(k, dtype=np.float32) - 0.5).astype(np.float32)
    t = oracle.quantize((rng.random((k, n), dtype=np.float32) - 0.5).astype(np.float32), 4, 64)
    serial = oracle.multiply_quantized(a, t, threads=1)
    parallel = oracle.multiply_quantized(a, t, threads=4)
    assert np.array_equal(serial.view(np.uint32), parallel.view(np.uint32))
    batched = oracle.multiply_quantized(np.tile(a, 3), t, m=3)
    assert np.abs(batched - serial).max() < 1e-4


@pytest.mark.parametrize("k,n", [(130, 9001), (300, 2100), (200, 33), (70, 300), (450, 129), (2, 17)])
def test_single_row_kernels_agree_bit_for_bit(oracle, k, n):
    """DecodeKernelTest.testSingleRowKernelsAgreeBitForBit (DecodeKernelTest.kt:48-78):
    every thread count gives identical bits, within 1e-4 of the fp32 product."""
    rng = np.random.default_rng(8)
    w = ((rng.random((k, n), dtype=np.float32) - 0.5) * 0.2).astype(np.float32)
    a = (rng.random(k, dtype=np.float32) - 0.5).astype(np.float32)
    for bits, g in [(4, 64), (4, 32), (8, 64)]:
        t = oracle.quantize(w, bits, g)
        ref = a.astype(np.float64) @ t.dequantize().astype(np.float64)
        first = None
        for threads in (1, 4, 3):
            y = oracle.multiply_quantized(a, t, threads=threads)[0]
            assert np.abs(ref - y).max() < 1e-4
            if first is None:
                first = y
            assert np.array_equal(first.view(np.uint32), y.view(np.uint32))


def test_single_row_kernel_accumulates_with_alpha(oracle):
    """DecodeKernelTest.testSingleRowKernelAccumulatesWithAlpha (DecodeKernelTest.kt:80-91)."""
    rng = np.random.default_rng(9)
    k, n = 96, 8200
    t = oracle.quantize((rng.random((k, n), dtype=np.float32) - 0.5).astype(np.float32), 4, 64)
    a = (rng.random(k, dtype=np.float32) - 0.5).astype(np.float32)
    plain = oracle.multiply_quantized(a, t)
    acc = oracle.multiply_quantized(a, t, c=np.full((1, n), 2.0, np.float32), accumulate=True, alpha=-0.5)
    assert np.abs(acc - (2.0 - 0.5 * plain)).max() < 1e-4


def test_memory_footprint_follows_bits_per_weight(oracle):
    """QuantizationTest.testMemoryFootprintFollowsBitsPerWeight (QuantizationTest.kt:326-341), per tensor."""
    for k, n in [(64, 64), (64, 128), (128, 64)]:
        assert 1.0 <= oracle.lib().kto_size_in_bytes(8, 64, k, n) / (k * n) <= 1.2
        assert 0.5 <= oracle.lib().kto_size_in_bytes(4, 64, k, n) / (k * n) <= 0.7


@pytest.mark.parametrize("bits", [4, 8])
def test_nan_and_overflowing_inverse_are_rejected(oracle, bits):
    """Float.roundToInt() throws on NaN (QuantizedTensor.kt:291, :308, :315)."""
    w = np.zeros((8, 4), np.float32)
    w[3, 1] = np.nan
    with pytest.raises(ValueError):
        oracle.quantize(w, bits, 4)
    w = np.zeros((8, 4), np.float32)
    w[2, 2] = np.inf  # scale = inf, inverse = 0, inf * 0 = NaN
    with pytest.raises(ValueError):
        oracle.quantize(w, bits, 4)


def test_tiny_group_overflows_inverse_like_the_reference(oracle):
    """A group whose max is 1e-40 has scale 7.9e-43 and 1/scale = inf; the zero in
    the same group gives 0 * inf = NaN, so the reference throws (INT8)."""
    w = np.zeros((4, 1), np.float32)
    w[1, 0] = np.float32(1e-40)
    with pytest.raises(ValueError):
        oracle.quantize(w, 8, 4)
