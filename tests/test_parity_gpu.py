"""GPU parity tests: every CUDA entry point of libkt_cuda.so against the CPU
oracle (oracle/kt_oracle.c) and the committed golden fixtures.

Bars (from the reference's north star):
  * packed bytes, scales and zeros: bit-exact;
  * dequantize: bit-exact (one fp32 multiply, as QuantizedTensor.kt:201/210);
  * matmul on the fp32-accumulate kernels (m <= 8 and the generic kernel):
    max|y - y_ref| <= 1e-3 * max|y_ref|;
  * matmul on the bf16 tensor-core kernel (m >= 9, aligned shapes): <= 2e-2 * max|y_ref|;
  * results are deterministic (identical bits on repeated calls).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-3
TOL_BF16 = 2e-2


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def tol_for(qt, m):
    from kotensor_b200 import _lib
    return TOL_BF16 if qt.matmul_path(m) == _lib.KT_PATH_TENSOR_CORE else TOL_FP32


def qname_parts(qname):
    bits = int(qname[3]) if qname[4] == "g" else int(qname[3:5])
    return bits, int(qname.split("g", 1)[1])


def golden_cases(golden):
    for key in sorted(golden):
        if key.endswith("/qdata"):
            base = key[: -len("/qdata")]
            shape_key, qname = base.rsplit("/", 1)
            bits, g = qname_parts(qname)
            yield base, shape_key, bits, g


# ----------------------------------------------------------------- quantizer

def test_quantize_matches_golden_bit_for_bit(kt, golden):
    n = 0
    for base, shape_key, bits, g in golden_cases(golden):
        w = golden[f"{shape_key}/w"]
        qt = kt.QuantizedTensor.quantize(dev(w), kt.Quantization(bits, g))
        q, s, z = qt.download()
        assert np.array_equal(q, golden[f"{base}/qdata"]), base
        assert np.array_equal(s.view(np.uint32), golden[f"{base}/scales"].view(np.uint32)), base
        if bits == 4:
            assert np.array_equal(z, golden[f"{base}/zeros"]), base
        n += 1
    assert n >= 30


@pytest.mark.parametrize("shape", [(2048, 2048), (256, 1537), (1000, 577), (4096, 1024), (3, 5), (130, 9001)])
@pytest.mark.parametrize("bits,g", [(8, 64), (4, 64), (4, 32), (8, 1000), (4, 1)])
def test_quantize_matches_oracle_bit_for_bit(kt, oracle, shape, bits, g):
    rng = np.random.default_rng(hash((shape, bits, g)) % 2**32)
    w = (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float32)
    ref = oracle.quantize(w, bits, g)
    qt = kt.QuantizedTensor.quantize(dev(w), kt.Quantization(bits, g))
    q, s, z = qt.download()
    assert (qt.rows, qt.columns, qt.groups, qt.bytes_per_row, qt.size_in_bytes) == (
        ref.rows, ref.columns, ref.groups, ref.bytes_per_row, ref.size_in_bytes)
    assert np.array_equal(q, ref.qdata)
    assert np.array_equal(s.view(np.uint32), ref.scales.view(np.uint32))
    if bits == 4:
        assert np.array_equal(z, ref.zeros)


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_reports_nan_like_the_reference(kt, bits):
    for bad in (np.nan, np.inf, -np.inf):
        w = np.zeros((8, 40), np.float32)
        w[5, 33] = bad
        with pytest.raises(ValueError, match="NaN"):
            kt.QuantizedTensor.quantize(dev(w), kt.Quantization(bits, 4))
    # the context stays usable after the error
    ok = kt.QuantizedTensor.quantize(dev(np.ones((8, 40), np.float32)), kt.Quantization(bits, 4))
    assert ok.rows == 8


def test_quantize_rejects_bad_arguments(kt):
    with pytest.raises(ValueError):
        kt.QuantizedTensor.quantize(dev(np.zeros((4, 4), np.float32)), kt.Quantization(8), rows=4, columns=5)
    with pytest.raises(ValueError):
        kt.QuantizedTensor.from_arrays(np.zeros(16, np.uint8), np.zeros(4, np.float32), None, (4, 4), 4, 64)
    with pytest.raises(ValueError):
        kt.QuantizedTensor.from_arrays(np.zeros(15, np.uint8), np.zeros(4, np.float32), None, (4, 4), 8, 64)


def test_upload_download_round_trip(kt, oracle):
    rng = np.random.default_rng(5)
    w = (rng.random((300, 101), dtype=np.float32) - 0.5).astype(np.float32)
    for bits, g in [(4, 16), (8, 64)]:
        ref = oracle.quantize(w, bits, g)
        qt = kt.QuantizedTensor.from_arrays(ref.qdata, ref.scales, ref.zeros, (300, 101), bits, g)
        q, s, z = qt.download()
        assert np.array_equal(q, ref.qdata) and np.array_equal(s, ref.scales)
        if bits == 4:
            assert np.array_equal(z, ref.zeros)
        assert qt.raw_value(7, 100) == ref.raw_value(7, 100)
        assert qt.value(7, 100) == ref.value(7, 100)


# ----------------------------------------------------------------- dequantize

@pytest.mark.parametrize("bits,g", [(8, 64), (4, 64), (4, 32), (4, 5)])
def test_dequantize_bit_exact(kt, oracle, bits, g):
    rng = np.random.default_rng(6)
    w = (rng.random((257, 131), dtype=np.float32) - 0.5).astype(np.float32)
    ref = oracle.quantize(w, bits, g)
    qt = kt.QuantizedTensor.from_arrays(ref.qdata, ref.scales, ref.zeros, (257, 131), bits, g)
    got = qt.dequantize().cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.dequantize().view(np.uint32))
    rows = torch.tensor([0, 256, 64, 3, 3], dtype=torch.int32)
    got_rows = qt.dequantize_rows(rows).cpu().numpy()
    for i, r in enumerate(rows.tolist()):
        assert np.array_equal(got_rows[i].view(np.uint32), ref.dequantize_row(r).view(np.uint32))
    with pytest.raises(ValueError):
        qt.dequantize_rows(torch.tensor([257], dtype=torch.int32))


# ----------------------------------------------------------------- matmul

def run_matmul(kt, qt, a, c0=None, accumulate=False, alpha=1.0, bias=None):
    m = a.shape[0]
    c = dev(c0.copy()) if c0 is not None else torch.zeros((m, qt.columns), device="cuda")
    kt.MatMul.multiply_quantized(dev(a), qt, c, m, accumulate=accumulate, alpha=alpha,
                                 bias=dev(bias) if bias is not None else None)
    return c.cpu().numpy()


def test_matmul_matches_golden(kt, golden):
    for base, shape_key, bits, g in golden_cases(golden):
        if f"{base}/y" not in golden:
            continue
        a = golden[f"{shape_key}/a"]
        m, k = a.shape
        n = golden[f"{base}/y"].shape[1]
        z = golden.get(f"{base}/zeros")
        qt = kt.QuantizedTensor.from_arrays(golden[f"{base}/qdata"], golden[f"{base}/scales"], z, (k, n), bits, g)
        tol = tol_for(qt, m)
        y = run_matmul(kt, qt, a)
        assert rel_err(y, golden[f"{base}/y"]) <= tol, base
        if f"{base}/y_acc" in golden:
            y2 = run_matmul(kt, qt, a, c0=np.ones((m, n), np.float32), accumulate=True, alpha=0.5)
            assert rel_err(y2, golden[f"{base}/y_acc"]) <= tol, base


SHAPES = [(2048, 2048), (4096, 1024), (2048, 5632), (5632, 2048), (768, 32000), (896, 4864), (4864, 896),
          (896, 128), (1024, 128), (64, 64), (256, 1537), (130, 9001), (300, 2100), (200, 33), (2, 17), (96, 8200)]


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 6, 8])
def test_matmul_matches_oracle(kt, oracle, k, n, bits, m):
    rng = np.random.default_rng(hash((k, n, bits, m)) % 2**32)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    a = rng.standard_normal((m, k), dtype=np.float32)
    ref_t = oracle.quantize(w, bits, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), bits, 64)
    ref = oracle.multiply_quantized(a, ref_t, threads=8)
    y = run_matmul(kt, qt, a)
    assert rel_err(y, ref) <= tol_for(qt, m)
    c0 = rng.standard_normal((m, n), dtype=np.float32)
    y2 = run_matmul(kt, qt, a, c0=c0, accumulate=True, alpha=-0.5)
    ref2 = oracle.multiply_quantized(a, ref_t, c=c0, accumulate=True, alpha=-0.5, threads=8)
    assert rel_err(y2, ref2) <= tol_for(qt, m)


@pytest.mark.parametrize("bits", [4, 8])
def test_matmul_is_deterministic(kt, oracle, bits):
    rng = np.random.default_rng(11)
    k, n = 4096, 4096
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    qt = kt.QuantizedTensor.quantize(dev(w), kt.Quantization(bits))
    for m in (1, 3, 8):
        a = dev(rng.standard_normal((m, k), dtype=np.float32))
        outs = []
        for _ in range(3):
            c = torch.zeros((m, n), device="cuda")
            kt.MatMul.multiply_quantized(a, qt, c, m, accumulate=False)
            outs.append(c.cpu().numpy().view(np.uint32))
        assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_full_size_int4_ffn_shape_against_oracle(kt, oracle):
    """BASELINE config 2's largest weight (K=4096, N=14336, INT4 g64) at m=1."""
    rng = np.random.default_rng(1234)
    k, n = 4096, 14336
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    a = rng.standard_normal((1, k), dtype=np.float32)
    qt = kt.QuantizedTensor.quantize(dev(w), kt.Quantization(4))
    ref_t = oracle.quantize(w, 4, 64)
    q, s, z = qt.download()
    assert np.array_equal(q, ref_t.qdata) and np.array_equal(s, ref_t.scales) and np.array_equal(z, ref_t.zeros)
    ref = oracle.multiply_quantized(a, ref_t, threads=8)
    y = run_matmul(kt, qt, a)
    assert rel_err(y, ref) <= TOL_FP32
    # linearity: y(a1 + a2) == y(a1) + y(a2) within the same tolerance
    a2 = rng.standard_normal((1, k), dtype=np.float32)
    y12 = run_matmul(kt, qt, (a + a2).astype(np.float32))
    assert rel_err(y12, run_matmul(kt, qt, a) + run_matmul(kt, qt, a2)) <= 2 * TOL_FP32


def test_bias_and_quantized_linear(kt, oracle):
    rng = np.random.default_rng(12)
    k, n, m = 896, 896, 3
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    bias = rng.standard_normal(n, dtype=np.float32)
    x = rng.standard_normal((m, k), dtype=np.float32)
    layer = kt.QuantizedLinear.from_linear(dev(w), dev(bias), kt.Quantization.INT4)
    ref_t = oracle.quantize(w, 4, 64)
    ref = oracle.multiply_quantized(x, ref_t) + bias[None, :]
    y = layer.forward(dev(x)).cpu().numpy()
    assert rel_err(y, ref) <= TOL_FP32
    out = torch.empty((m, n), device="cuda")
    layer.forward_into(dev(x), out)
    assert np.array_equal(out.cpu().numpy(), y)
    assert layer.size_in_bytes == ref_t.size_in_bytes + n * 4


def test_host_entry_point(kt, oracle):
    rng = np.random.default_rng(13)
    k, n = 1024, 2048
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 8, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, None, (k, n), 8, 64)
    a = rng.standard_normal((2, k), dtype=np.float32)
    c = np.ones((2, n), np.float32)
    kt.MatMul.multiply_quantized(a, qt, c, 2, accumulate=True, alpha=2.0)
    ref = oracle.multiply_quantized(a, ref_t, c=np.ones((2, n), np.float32), accumulate=True, alpha=2.0)
    assert rel_err(c, ref) <= TOL_FP32


def test_zero_rows_is_a_noop_and_shapes_are_checked(kt):
    qt = kt.QuantizedTensor.quantize(dev(np.ones((64, 64), np.float32)), kt.Quantization.INT8)
    c = torch.full((1, 64), 3.0, device="cuda")
    kt.MatMul.multiply_quantized(torch.zeros((0, 64), device="cuda"), qt, c, 0)
    assert float(c[0, 0]) == 3.0
    with pytest.raises(ValueError):
        kt.MatMul.multiply_quantized(torch.zeros((1, 63), device="cuda"), qt, c, 1)
    with pytest.raises(ValueError):
        kt.MatMul.multiply_quantized(torch.zeros((1, 64), device="cuda"), qt, c, -1)


# ----------------------------------------------------------------- backward

def test_transposed_matches_golden(kt, golden):
    for base, shape_key, bits, g in golden_cases(golden):
        if f"{base}/dx" not in golden:
            continue
        dy = golden[f"{shape_key}/dy"]
        m, n = dy.shape
        k = golden[f"{shape_key}/a"].shape[1]
        qt = kt.QuantizedTensor.from_arrays(golden[f"{base}/qdata"], golden[f"{base}/scales"],
                                            golden.get(f"{base}/zeros"), (k, n), bits, g)
        dx = torch.zeros((m, k), device="cuda")
        kt.MatMul.multiply_by_quantized_transposed(dev(dy), qt, dx, m, accumulate=False)
        assert rel_err(dx.cpu().numpy(), golden[f"{base}/dx"]) <= TOL_FP32, base


@pytest.mark.parametrize("bits,g", [(8, 64), (4, 64), (4, 32), (4, 5)])
@pytest.mark.parametrize("shape", [(256, 1537), (1000, 577), (130, 9)])
def test_dequantize_column_matches_the_oracle(kt, oracle, bits, g, shape):
    """dequantizeColumn (QuantizedTensor.kt:235-241): every column of odd-width INT4
    and INT8 weights, bit-identical to the oracle's dequantize(); out of range raises."""
    rng = np.random.default_rng(sum(shape) + bits + g)
    w = (rng.standard_normal(shape, dtype=np.float32) * 0.05).astype(np.float32)
    ref = oracle.quantize(w, bits, g)
    qt = kt.QuantizedTensor.from_arrays(ref.qdata, ref.scales, ref.zeros, shape, bits, g)
    want = ref.dequantize()
    cols = list(range(shape[1]))[::-1]
    got = qt.dequantize_columns(cols).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(want.T[cols]).view(np.uint32))
    assert np.array_equal(qt.dequantize_column(0).cpu().numpy().view(np.uint32),
                          np.ascontiguousarray(want[:, 0]).view(np.uint32))
    with pytest.raises(ValueError):
        qt.dequantize_column(shape[1])
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k,n,m", [(4096, 1024, 1), (2048, 5632, 4), (896, 4864, 9), (300, 2101, 2)])
@pytest.mark.parametrize("bits", [4, 8])
def test_transposed_matches_oracle(kt, oracle, k, n, m, bits):
    rng = np.random.default_rng(14)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, bits, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), bits, 64)
    dy = rng.standard_normal((m, n), dtype=np.float32)
    dx0 = rng.standard_normal((m, k), dtype=np.float32)
    dx = dev(dx0.copy())
    kt.MatMul.multiply_by_quantized_transposed(dev(dy), qt, dx, m, accumulate=True)
    ref = oracle.multiply_by_quantized_transposed(dy, ref_t, dx=dx0, accumulate=True, threads=8)
    assert rel_err(dx.cpu().numpy(), ref) <= TOL_FP32


# (bits, K, N, m, group): at m >= 16, INT4 with N % 128 == 0 and INT8 with
# N % 64 == 0 run the tcgen05 transposed kernel -- one or several 128-token
# tiles, ragged K (partial 128-row tiles and partial groups), group sizes
# 32 / 64 / 128 / 256, split-K over N.
@pytest.mark.parametrize("bits,k,n,m,g", [(4, 4096, 14336, 16, 64), (4, 1000, 1024, 17, 32), (4, 2048, 5632, 100, 128),
                                          (4, 896, 4864, 40, 64), (4, 520, 256, 300, 256), (4, 384, 2048, 130, 32),
                                          (8, 4096, 14336, 16, 64), (8, 1000, 576, 17, 32), (8, 2048, 5632, 100, 128),
                                          (8, 520, 64, 300, 256), (8, 384, 2048, 130, 64)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_transposed_tensor_core_matches_oracle(kt, oracle, bits, k, n, m, g, accumulate):
    from kotensor_b200 import _lib
    rng = np.random.default_rng(k + n + m)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, bits, g)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), bits, g)
    assert qt.transposed_path(m) == _lib.KT_PATH_TENSOR_CORE
    dy = rng.standard_normal((m, n), dtype=np.float32)
    dx0 = rng.standard_normal((m, k), dtype=np.float32)
    dx = dev(dx0.copy()) if accumulate else torch.full((m, k), float("nan"), device="cuda")
    kt.MatMul.multiply_by_quantized_transposed(dev(dy), qt, dx, m, accumulate=accumulate)
    ref = oracle.multiply_by_quantized_transposed(dy, ref_t, dx=dx0 if accumulate else None,
                                                  accumulate=accumulate, threads=8)
    got = dx.cpu().numpy()
    assert np.isfinite(got).all()
    # the accumulated part is compared on dx alone so that dx0 cannot hide an error
    assert rel_err(got - (dx0 if accumulate else 0), ref - (dx0 if accumulate else 0)) <= TOL_BF16
    # deterministic: a second product gives the same bits
    dx2 = dev(dx0.copy()) if accumulate else torch.zeros((m, k), device="cuda")
    kt.MatMul.multiply_by_quantized_transposed(dev(dy), qt, dx2, m, accumulate=accumulate)
    assert torch.equal(dx, dx2)
    assert kt.Context.get().take_error() == 0


def test_transposed_path_selection(kt, oracle):
    from kotensor_b200 import _lib
    rng = np.random.default_rng(3)
    for bits, n, g, m, want in [(4, 1024, 64, 16, _lib.KT_PATH_TENSOR_CORE), (4, 1024, 64, 15, _lib.KT_PATH_GENERIC),
                                (8, 1024, 64, 64, _lib.KT_PATH_TENSOR_CORE), (8, 1000, 64, 64, _lib.KT_PATH_GENERIC),
                                (8, 1024, 64, 15, _lib.KT_PATH_GENERIC), (4, 1000, 64, 64, _lib.KT_PATH_GENERIC),
                                (4, 960, 64, 64, _lib.KT_PATH_GENERIC), (4, 1024, 96, 64, _lib.KT_PATH_GENERIC)]:
        w = (rng.standard_normal((256, n)) * 0.02).astype(np.float32)
        t = oracle.quantize(w, bits, g)
        qt = kt.QuantizedTensor.from_arrays(t.qdata, t.scales, t.zeros, (256, n), bits, g)
        assert qt.transposed_path(m) == want, (bits, n, g, m)


def test_no_kernel_reported_a_timeout(kt):
    """Every bounded wait inside the kernels completed in the calls above."""
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("lane_bytes,cluster_k", [(16, 1), (16, 8), (8, 3), (4, 8), (4, 1)])
def test_every_launch_shape_matches_the_oracle(kt, oracle, lane_bytes, cluster_k):
    """The tuning knob changes the launch shape only, never the tolerance."""
    lib = kt.load_library()
    rng = np.random.default_rng(21)
    k, n = 2048, 5632
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, 64)
    try:
        lib.kt_set_gemv_tuning(lane_bytes, cluster_k)
        for m in (1, 2, 5):
            a = rng.standard_normal((m, k), dtype=np.float32)
            y = run_matmul(kt, qt, a)
            assert rel_err(y, oracle.multiply_quantized(a, ref_t, threads=8)) <= TOL_FP32
    finally:
        lib.kt_set_gemv_tuning(0, 0)
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k_splits", [1, 2, 5, 37])
@pytest.mark.parametrize("k,n,g", [(2048, 5632, 64), (4864, 896, 64), (1024, 4096, 32), (960, 2048, 96)])
def test_int4_tensor_core_gemv_matches_the_oracle(kt, oracle, k_splits, k, n, g):
    """The INT4 m <= 8 tensor-core GEMV at several K-split counts (slices that
    start and end inside groups, empty slices), ragged last tiles (896 columns)
    and group sizes 32 / 64 / 96, within the fp32 tolerance."""
    from kotensor_b200 import _lib
    lib = kt.load_library()
    rng = np.random.default_rng(k + n + g)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, g)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, g)
    assert qt.matmul_path(1) == _lib.KT_PATH_GEMV_MMA
    try:
        lib.kt_set_gemv_mma_tuning(k_splits)
        for m in (1, 2, 4, 6, 8):
            a = (rng.standard_normal((m, k), dtype=np.float32) * np.float32(3.0)).astype(np.float32)
            a[0, : k // 3] *= np.float32(1e-3)  # a wide dynamic range inside one row
            c0 = rng.standard_normal((m, n), dtype=np.float32)
            y = run_matmul(kt, qt, a, c0=c0, accumulate=True, alpha=0.75)
            ref = oracle.multiply_quantized(a, ref_t, c=c0, accumulate=True, alpha=0.75, threads=8)
            assert rel_err(y, ref) <= TOL_FP32, (m, rel_err(y, ref))
    finally:
        lib.kt_set_gemv_mma_tuning(0)
    assert kt.Context.get().take_error() == 0


def test_int4_tensor_core_gemv_huge_and_tiny_activations(kt, oracle):
    """x rows scaled by 1e30 and 1e-30: the per-slice power-of-two scaling keeps
    the fp16 split in range."""
    rng = np.random.default_rng(33)
    k, n = 2048, 2048
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, 64)
    for s in (1e30, 1e-30, 0.0):
        a = (rng.standard_normal((2, k), dtype=np.float32) * np.float32(s)).astype(np.float32)
        y = run_matmul(kt, qt, a)
        ref = oracle.multiply_quantized(a, ref_t, threads=8)
        if s == 0.0:
            assert not np.any(y)
        else:
            assert rel_err(y, ref) <= TOL_FP32, s


def test_int4_tensor_core_gemv_split_k_workspace_is_reused_safely(kt, oracle):
    """Launches with few column tiles and many K-splits alternate with launches
    with many tiles on one stream's workspace: no launch's partial tiles may
    disturb another's arrival counters."""
    from kotensor_b200 import _lib
    rng = np.random.default_rng(44)
    cases = []
    for k, n in [(5632, 2048), (768, 32000), (4096, 1024), (1024, 16384)]:
        w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
        ref_t = oracle.quantize(w, 4, 64)
        qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, 64)
        assert qt.matmul_path(1) == _lib.KT_PATH_GEMV_MMA
        cases.append((qt, ref_t, k))
    for _ in range(2):
        for qt, ref_t, k in cases:
            for m in (1, 4):
                a = rng.standard_normal((m, k), dtype=np.float32)
                y = run_matmul(kt, qt, a)
                assert rel_err(y, oracle.multiply_quantized(a, ref_t, threads=8)) <= TOL_FP32, (k, m)
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k,n,g", [(2048, 5632, 64), (4096, 1024, 64), (896, 4864, 64), (960, 2048, 96),
                                   (1024, 4096, 32), (4864, 896, 64)])
@pytest.mark.parametrize("m", [9, 16, 24, 40, 64, 128, 200, 256, 512])
def test_int4_tensor_core_gemm_matches_the_oracle(kt, oracle, m, k, n, g):
    """The bf16 tcgen05 GEMMs (m >= 9): A in tensor memory for m <= 128
    (partial token tiles at 9, 24, 40), A in shared memory above (partial token
    tiles at 200, two token tiles at 512), a K that is not a multiple of the
    64-row stage (960), group sizes 32 / 64 / 96, accumulate / alpha / bias,
    within the bf16 tolerance."""
    from kotensor_b200 import _lib
    rng = np.random.default_rng(k * 3 + n + m + g)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, g)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, g)
    assert qt.matmul_path(m) == _lib.KT_PATH_TENSOR_CORE
    a = rng.standard_normal((m, k), dtype=np.float32)
    c0 = rng.standard_normal((m, n), dtype=np.float32)
    bias = rng.standard_normal(n, dtype=np.float32)
    y = run_matmul(kt, qt, a, c0=c0, accumulate=True, alpha=0.5, bias=bias)
    ref = oracle.multiply_quantized(a, ref_t, c=c0, accumulate=True, alpha=0.5, threads=8) + bias[None, :]
    assert rel_err(y, ref) <= TOL_BF16, rel_err(y, ref)
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k,n,g", [(2048, 2048, 64), (4096, 1024, 64), (960, 2048, 96), (1024, 4096, 32)])
@pytest.mark.parametrize("m", [9, 64, 200, 512])
def test_int8_tensor_core_gemm_matches_the_oracle(kt, oracle, m, k, n, g):
    """The tcgen05 bf16 GEMM on INT8 weights (BASELINE config 1 at M = 64 and
    around it), accumulate / alpha / bias, within the bf16 tolerance."""
    from kotensor_b200 import _lib
    rng = np.random.default_rng(k * 5 + n + m + g)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 8, g)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, None, (k, n), 8, g)
    assert qt.matmul_path(m) == _lib.KT_PATH_TENSOR_CORE
    a = rng.standard_normal((m, k), dtype=np.float32)
    c0 = rng.standard_normal((m, n), dtype=np.float32)
    bias = rng.standard_normal(n, dtype=np.float32)
    y = run_matmul(kt, qt, a, c0=c0, accumulate=True, alpha=0.5, bias=bias)
    ref = oracle.multiply_quantized(a, ref_t, c=c0, accumulate=True, alpha=0.5, threads=8) + bias[None, :]
    assert rel_err(y, ref) <= TOL_BF16, rel_err(y, ref)
    assert kt.Context.get().take_error() == 0


BENCH_SHAPES = [(2048, 5632), (5632, 2048), (4096, 14336), (14336, 4096)]  # BASELINE config 2 (K, N)


@pytest.mark.parametrize("k,n", BENCH_SHAPES)
def test_bench_weights_gemv_against_oracle(kt, oracle, k, n):
    """The four weights bench.py times, quantized on the
    device (bit-exact) and multiplied at m = 1 on the integer tensor-core GEMV,
    plus m = 4 and m = 5 / 8 (two token groups in one launch) on the fp16 one."""
    from kotensor_b200 import _lib
    rng = np.random.default_rng(k + 3 * n)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    qt = kt.QuantizedTensor.quantize(dev(w), kt.Quantization(4))
    ref_t = oracle.quantize(w, 4, 64)
    q, s, z = qt.download()
    assert np.array_equal(q, ref_t.qdata) and np.array_equal(s.view(np.uint32), ref_t.scales.view(np.uint32))
    assert np.array_equal(z, ref_t.zeros)
    assert qt.matmul_path(1) == _lib.KT_PATH_GEMV_MMA
    for m in (1, 4, 5, 8):
        assert qt.matmul_path(m) == _lib.KT_PATH_GEMV_MMA
        a = rng.standard_normal((m, k), dtype=np.float32)
        y = run_matmul(kt, qt, a)
        assert rel_err(y, oracle.multiply_quantized(a, ref_t, threads=8)) <= TOL_FP32, m
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k,n", [(4096, 14336), (14336, 4096)])
@pytest.mark.parametrize("m", [16, 128, 512])
def test_bench_weights_gemm_against_oracle(kt, oracle, k, n, m):
    """The prefill / batched-decode GEMM on the Llama-8B FFN weights bench.py
    times (BASELINE config 2 at M = 16, 128, 512), within the bf16 tolerance."""
    from kotensor_b200 import _lib
    rng = np.random.default_rng(k + n + m)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, 64)
    assert qt.matmul_path(m) == _lib.KT_PATH_TENSOR_CORE
    a = rng.standard_normal((m, k), dtype=np.float32)
    y = run_matmul(kt, qt, a)
    assert rel_err(y, oracle.multiply_quantized(a, ref_t, threads=8)) <= TOL_BF16
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k,n", [(4096, 6144), (4096, 4096), (14336, 4096)])
def test_llama_prefill_gemm_against_oracle(kt, oracle, k, n):
    """The GEMM of a 1,024-token prompt block on the Llama-3-8B-shaped
    projections bench.py's prefill runs (q|k|v, output, down: 256-token tiles,
    the output and down products split over K and summed by the reduction
    kernel), plus RMSNorm fused into its bf16 pre-pass, within the bf16
    tolerance of the oracle."""
    import ctypes
    from kotensor_b200 import _lib
    lib = kt.load_library()
    m = 1024
    rng = np.random.default_rng(k + 2 * n)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, 64)
    assert qt.matmul_path(m) == _lib.KT_PATH_TENSOR_CORE
    a = rng.standard_normal((m, k), dtype=np.float32)
    y = run_matmul(kt, qt, a)
    y_ref = oracle.multiply_quantized(a, ref_t, threads=16)
    assert rel_err(y, y_ref) <= TOL_BF16
    # RMSNorm in the pre-pass (kt_rmsnorm_qmatmul at m = 1024) against the float64 norm then the oracle
    nwh = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    x, nw = dev(a), dev(nwh)
    out = torch.empty((m, n), device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    _lib.check(lib.kt_rmsnorm_qmatmul(kt.Context.get().handle, qt.handle, p(x), p(nw), 1e-6, None, p(out), m, 0,
                                      None, s))
    torch.cuda.synchronize()
    ad = a.astype(np.float64)
    an = (ad / np.sqrt((ad * ad).mean(axis=1, keepdims=True) + 1e-6) * nwh).astype(np.float32)
    assert rel_err(out.cpu().numpy(), oracle.multiply_quantized(an, ref_t, threads=16)) <= TOL_BF16
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k,n", BENCH_SHAPES)
@pytest.mark.parametrize("factor,count", [(50.0, 1), (100.0, 1), (100.0, 4), (75.0, 16)])
def test_int4_gemv_with_outlier_channels(kt, oracle, k, n, factor, count):
    """LLM-style activations: a few channels at 50-100x the row's rms inside one
    1,024-row slice.  The m = 1 kernel rounds x to 15 bits relative to the
    largest |x| among each warp's rows, so an outlier coarsens its neighbours'
    rounding; the result must stay within the fp32 tolerance."""
    rng = np.random.default_rng(int(factor) * count + k)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), 4, 64)
    a = rng.standard_normal((1, k), dtype=np.float32)
    rms = float(np.sqrt(np.mean(a.astype(np.float64) ** 2)))
    base = int(rng.integers(0, k // 1024)) * 1024
    idx = base + rng.choice(1024, count, replace=False)
    a[0, idx] = (np.where(rng.random(count) < 0.5, -1.0, 1.0) * factor * rms).astype(np.float32)
    y = run_matmul(kt, qt, a)
    ref = oracle.multiply_quantized(a, ref_t, threads=8)
    assert rel_err(y, ref) <= TOL_FP32, rel_err(y, ref)
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k,h", [(896, 4864), (4096, 14336), (2048, 5632), (768, 2048), (512, 1024)])
@pytest.mark.parametrize("m", [1, 3, 16, 64])
def test_swiglu_epilogue_equals_matmul_then_silu(kt, oracle, k, h, m):
    """kt_qmatmul_swiglu on a fused gate | up weight [K x 2H]: at m = 1 the
    silu(gate) * up product is formed in the INT4 GEMV's epilogue (every
    split-K route: one CTA per tile, clusters, partials in global memory), at
    m >= 9 in the tcgen05 GEMM's split-K reduction where the GEMM splits K; it
    must equal kt_qmatmul followed by kt_silu_mul_rows bit for bit; other m take
    that route themselves.  Within the tolerance of the path against the oracle."""
    import ctypes
    from kotensor_b200 import _lib
    lib = kt.load_library()
    rng = np.random.default_rng(k + h + m)
    w = (rng.standard_normal((k, 2 * h), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 4, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, 2 * h), 4, 64)
    a = rng.standard_normal((m, k), dtype=np.float32)
    bias = (rng.standard_normal(2 * h, dtype=np.float32) * 0.1).astype(np.float32)
    ad, bd = dev(a), dev(bias)
    h_ = kt.Context.get().handle
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    gu = torch.empty((m, 2 * h), device="cuda")
    want = torch.empty((m, h), device="cuda")
    _lib.check(lib.kt_qmatmul(h_, qt.handle, p(ad), p(gu), m, 0, 1.0, p(bd), s))
    _lib.check(lib.kt_silu_mul_rows(h_, p(gu), p(want), m, h, s))
    for _ in range(2):
        got = torch.full((m, h), float("nan"), device="cuda")
        _lib.check(lib.kt_qmatmul_swiglu(h_, qt.handle, p(ad), p(gu), p(got), m, 1.0, p(bd), s))
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    g_u = oracle.multiply_quantized(a, ref_t, threads=8) + bias[None, :]
    g, u = g_u[:, :h].astype(np.float64), g_u[:, h:].astype(np.float64)
    ref = g / (1.0 + np.exp(-g)) * u
    assert rel_err(got.cpu().numpy(), ref) <= tol_for(qt, m)
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("bits,k,n", [(4, 896, 1152), (4, 4096, 6144), (4, 896, 9728), (4, 4096, 28672),
                                      (8, 768, 2304)])
@pytest.mark.parametrize("m", [1, 3, 6, 16])
@pytest.mark.parametrize("swiglu", [False, True])
def test_rmsnorm_prologue_matches_rmsnorm_then_matmul(kt, oracle, bits, k, n, m, swiglu):
    """kt_rmsnorm_qmatmul(_swiglu): RMSNorm(x) . W + bias (then silu(gate) * up).
    On INT4 (m = 1 integer GEMV, m = 3 and 6 fp16 GEMV, one and two token
    groups) the norm is applied while the GEMV stages x (each CTA sums the
    rows' squares itself), at m = 16 in the tcgen05 GEMM's bf16 pre-pass;
    INT8 m = 2..8: kt_rmsnorm then the matmul.  Within 1e-5 of the separate
    kernels on the fp32 paths (the squares are added in another order; bf16
    tolerance on the GEMM, where a last-bit change of the scale can move a
    bf16 rounding) and within the path's tolerance of the oracle; accumulate
    into c included."""
    import ctypes
    from kotensor_b200 import _lib
    lib = kt.load_library()
    rng = np.random.default_rng(k + n + m + bits + swiglu)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, bits, 64)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, ref_t.zeros, (k, n), bits, 64)
    xh = (rng.standard_normal((m, k), dtype=np.float32) * 3).astype(np.float32)
    nwh = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    bh = (0.1 * rng.standard_normal(n)).astype(np.float32)
    x, nw, bias = dev(xh), dev(nwh), dev(bh)
    h_ = kt.Context.get().handle
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    xn = torch.empty((m, k), device="cuda")
    gu = torch.empty((m, n), device="cuda")
    out_n = n // 2 if swiglu else n
    c0 = torch.randn((m, out_n), device="cuda")
    want = c0.clone()
    _lib.check(lib.kt_rmsnorm(h_, p(x), p(nw), p(xn), m, k, 1e-6, s))
    if swiglu:
        _lib.check(lib.kt_qmatmul_swiglu(h_, qt.handle, p(xn), p(gu), p(want), m, 1.0, p(bias), s))
    else:
        _lib.check(lib.kt_qmatmul(h_, qt.handle, p(xn), p(want), m, 1, 1.0, p(bias), s))
    got = c0.clone()
    if swiglu:
        _lib.check(lib.kt_rmsnorm_qmatmul_swiglu(h_, qt.handle, p(x), p(nw), 1e-6, p(xn), p(gu), p(got), m, p(bias), s))
    else:
        _lib.check(lib.kt_rmsnorm_qmatmul(h_, qt.handle, p(x), p(nw), 1e-6, p(xn), p(got), m, 1, p(bias), s))
    torch.cuda.synchronize()
    tol = tol_for(qt, m)
    assert ((got - want).abs().max() / want.abs().max()).item() <= (1e-5 if tol == TOL_FP32 else tol)
    # against the oracle: RMSNorm in float64, the quantized product
    xd = xh.astype(np.float64)
    xnh = (xd / np.sqrt((xd * xd).mean(axis=1, keepdims=True) + 1e-6) * nwh).astype(np.float32)
    y = oracle.multiply_quantized(xnh, ref_t, threads=8) + bh[None, :]
    if swiglu:
        g, u = y[:, :n // 2].astype(np.float64), y[:, n // 2:].astype(np.float64)
        ref = g / (1.0 + np.exp(-g)) * u
    else:
        ref = c0.cpu().numpy() + y
    assert rel_err(got.cpu().numpy(), ref) <= tol
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("k_splits", [0, 1, 2, 5, 37])
@pytest.mark.parametrize("k,n,g", [(2048, 2048, 64), (768, 32000, 64), (4096, 1024, 32), (960, 2304, 96),
                                   (14336, 4096, 64)])
def test_int8_tensor_core_gemv_matches_the_oracle(kt, oracle, k_splits, k, n, g):
    """INT8 weights at m = 1 on the integer tensor-core GEMV (signed-byte MMAs,
    128 output columns per tile): every K-split count (clusters and partials in
    global memory), accumulate / alpha / bias, a wide dynamic range, within the
    fp32 tolerance of the oracle; BASELINE config 1's 2048 x 2048 included."""
    from kotensor_b200 import _lib
    lib = kt.load_library()
    rng = np.random.default_rng(k + n + g + k_splits)
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref_t = oracle.quantize(w, 8, g)
    qt = kt.QuantizedTensor.from_arrays(ref_t.qdata, ref_t.scales, None, (k, n), 8, g)
    assert qt.matmul_path(1) == _lib.KT_PATH_GEMV_MMA
    try:
        lib.kt_set_gemv_mma_tuning(k_splits)
        a = (rng.standard_normal((1, k), dtype=np.float32) * np.float32(3.0)).astype(np.float32)
        a[0, : k // 3] *= np.float32(1e-3)
        c0 = rng.standard_normal((1, n), dtype=np.float32)
        bias = rng.standard_normal(n, dtype=np.float32)
        y = run_matmul(kt, qt, a, c0=c0, accumulate=True, alpha=0.75, bias=bias)
        ref = oracle.multiply_quantized(a, ref_t, c=c0, accumulate=True, alpha=0.75, threads=8) + bias[None, :]
        assert rel_err(y, ref) <= TOL_FP32, rel_err(y, ref)
    finally:
        lib.kt_set_gemv_mma_tuning(0)
    assert kt.Context.get().take_error() == 0
