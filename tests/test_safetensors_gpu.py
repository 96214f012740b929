"""Safetensors files into and out of HBM (kt_st_read_*_device, kt_qweight_load,
kt_st_write with device tensors) against the oracle restatement of
SafeTensors.kt / Transformer.saveQuantized and the golden dtype fixture.

Reference behaviour ported (Engine/kotensor/src/test/kotlin/):
  QuantizationTest.testSaveAndLoadQuantizedModelRoundTrip   (bytes, scales, zeros, biases and outputs equal)
  MappedModelTest.testMemoryMappedModelMatchesHeapModelExactly (a loaded model decodes exactly like the source)
  MappedModelTest.testTiedModelRoundTripsThroughFilesWithoutAnEmbeddingCopy
  MappedModelTest.testMapReturnsTheTensorBytes              (device bytes equal readRaw)
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import safetensors_oracle as SO  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def st(kt):
    from kotensor_b200 import safetensors
    return safetensors


def _same_f32(got, exp):
    nan = np.isnan(exp)
    return np.array_equal(np.isnan(got), nan) and np.array_equal(got[~nan].view(np.uint32),
                                                                  exp[~nan].view(np.uint32))


def test_device_conversion_matches_golden_fixture(st):
    path = os.path.join(GOLDEN, "dtypes.safetensors")
    with np.load(os.path.join(GOLDEN, "dtypes_expected.npz")) as z, st.SafeTensorsFile(path) as f:
        for name in f.names:
            got = f.load(name).cpu().numpy().reshape(-1)
            assert _same_f32(got, z[name]), name
        # NaN payloads of binary16 kept bit for bit (halfToFloat, SafeTensors.kt:179-198)
        halves = f.load("halves").cpu().numpy().reshape(-1).view(np.uint32)
        want = np.array([SO.half_to_float(b) for b in range(65536)], np.float32).view(np.uint32)
        assert np.array_equal(halves, want)


@pytest.mark.parametrize("dtype", ["F16", "BF16", "I64", "F64", "F32", "I8"])
def test_multi_chunk_device_reads(st, tmp_path, dtype):
    """Tensors larger than the staging buffers, at an odd offset in the file."""
    rng = np.random.default_rng(len(dtype))
    esize = SO.BYTES_PER_ELEMENT[dtype]
    count = (41 << 20) // esize + 7
    raw = rng.integers(0, 256, count * esize, dtype=np.uint8)
    path = tmp_path / "big.safetensors"
    st.save_entries(path, [st.SafeTensorsEntry("pad", "U8", [5], np.arange(5, dtype=np.uint8)),
                           st.SafeTensorsEntry("x", dtype, [count], raw)])
    with st.SafeTensorsFile(path) as f:
        got = f.load("x").cpu().numpy()
        dev = torch.zeros(raw.size + 16, dtype=torch.uint8, device="cuda")
        f.read_raw_into("x", dev)
        torch.cuda.synchronize()
        assert np.array_equal(dev[:raw.size].cpu().numpy(), raw)
        assert int(dev[raw.size:].sum()) == 0
    if dtype == "F16":
        exp = raw.view("<f2").astype(np.float32)  # numpy's binary16 conversion keeps NaN payloads as well
    else:
        with np.errstate(over="ignore", invalid="ignore"):
            exp = SO.to_float32(dtype, raw.tobytes())
    assert _same_f32(got, exp)


def test_reads_check_the_destination(st, tmp_path):
    path = tmp_path / "s.safetensors"
    st.save_entries(path, [st.SafeTensorsEntry("x", "F32", [4, 4], np.ones((4, 4), np.float32)),
                           st.SafeTensorsEntry("u", "U16", [2], np.zeros(2, np.uint16))])
    with st.SafeTensorsFile(path) as f:
        with pytest.raises(ValueError, match="Destination too small"):
            f.read_into("x", torch.empty(15, device="cuda"))
        with pytest.raises(ValueError, match="Destination too small"):
            f.read_raw_into("x", torch.empty(63, dtype=torch.uint8, device="cuda"))
        with pytest.raises(ValueError, match="Unsupported safetensors dtype"):
            f.load("u")
        with pytest.raises(ValueError, match="No tensor named"):
            f.load("nope")


def _weight_entries(name, q):
    out = [(f"{name}.qweight", "I8" if q.bits == 8 else "U8", [q.rows, q.bytes_per_row], q.qdata.tobytes()),
           (f"{name}.scales", "F32", [q.groups, q.columns], q.scales.tobytes())]
    if q.bits == 4:
        out.append((f"{name}.zeros", "U8", [q.groups, q.columns], q.zeros.tobytes()))
    return out


@pytest.mark.parametrize("bits,group,k,n", [(8, 64, 192, 300), (4, 64, 256, 333), (4, 32, 100, 64), (8, 1000, 70, 9)])
def test_qweight_load_and_save(kt, oracle, st, tmp_path, bits, group, k, n):
    """mapFrom into HBM: the device weight holds the file's bytes and multiplies
    like the uploaded weight; written back from HBM, the file is byte-identical."""
    rng = np.random.default_rng(k + n)
    w = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    q = oracle.quantize(w, bits, group)
    entries = [("other", "F32", [3], np.ones(3, np.float32).tobytes())] + _weight_entries("layer.w", q)
    path = tmp_path / "q.safetensors"
    SO.save_entries(str(path), entries, {"kotensor.quantization.bits": str(bits)})
    with st.SafeTensorsFile(path) as f:
        loaded = f.load_quantized("layer.w", kt.Quantization(bits, group), k, n)
    qd, sd, zd = loaded.download()
    assert qd.tobytes() == q.qdata.tobytes() and sd.tobytes() == q.scales.tobytes()
    assert (zd is None) == (bits == 8) and (zd is None or zd.tobytes() == q.zeros.tobytes())
    uploaded = kt.QuantizedTensor.from_arrays(q.qdata, q.scales, q.zeros, (k, n), bits, group)
    for m in (1, 4, 16):
        a = torch.randn(m, k, device="cuda")
        c1, c2 = torch.zeros(m, n, device="cuda"), torch.zeros(m, n, device="cuda")
        kt.MatMul.multiply_quantized(a, loaded, c1, m, accumulate=False)
        kt.MatMul.multiply_quantized(a, uploaded, c2, m, accumulate=False)
        assert torch.equal(c1, c2)
    out = tmp_path / "q2.safetensors"
    st.save_entries(out, [st.SafeTensorsEntry("other", "F32", [3], torch.ones(3, device="cuda"))]
                    + st.quantized_entries("layer.w", loaded), {"kotensor.quantization.bits": str(bits)})
    assert out.read_bytes() == path.read_bytes()


def test_qweight_load_checks_sizes_like_map_from(kt, oracle, st, tmp_path):
    rng = np.random.default_rng(0)
    q = oracle.quantize((rng.standard_normal((128, 64)) * 0.02).astype(np.float32), 4, 64)
    good = _weight_entries("w", q)
    cases = {
        "qweight": ([(good[0][0], "U8", [1], b"\x00")] + good[1:], "w.qweight has 1 bytes, expected 4096"),
        "scales": ([good[0], ("w.scales", "F16", [2, 64], b"\x00" * 256), good[2]], "w.scales is F16"),
        "zeros": (good[:2] + [("w.zeros", "U8", [2], b"\x00\x00")], "w.zeros has 2 bytes, expected 128"),
        "missing": (good[:2], "No tensor named 'w.zeros'"),
    }
    for case, (entries, message) in cases.items():
        path = tmp_path / f"{case}.safetensors"
        SO.save_entries(str(path), entries)
        with st.SafeTensorsFile(path) as f, pytest.raises(ValueError, match=message):
            f.load_quantized("w", kt.Quantization(4, 64), 128, 64)


def test_device_tensors_write_through_staging(st, tmp_path):
    """Device tensors larger than the staging buffers write the same bytes as host ones."""
    t = torch.randn(5 << 20, device="cuda")  # 20 MiB
    s = torch.arange(77, dtype=torch.int32, device="cuda")
    path = tmp_path / "d.safetensors"
    st.save_entries(path, [st.SafeTensorsEntry.of("t", t), st.SafeTensorsEntry("s", "I32", [77], s)], {"a": "b"})
    expect = SO.encode([("t", "F32", [5 << 20], t.cpu().numpy().tobytes()),
                        ("s", "I32", [77], s.cpu().numpy().tobytes())], {"a": "b"})
    assert path.read_bytes() == expect
    back = st.load(path)
    assert torch.equal(back["t"], t) and torch.equal(back["s"], s.float())


CONFIGS = {
    "int8_untied": dict(vocab=300, dim=128, layers=2, heads=4, kv_heads=2, hidden=320, bits=8, group_size=64),
    "int4_scaled_rope_bias": dict(vocab=500, dim=192, layers=2, heads=3, kv_heads=1, hidden=384, bits=4,
                                  group_size=32, rope_theta=500000.0, rope_scaling=(8.0, 1.0, 4.0, 8192),
                                  qkv_bias=True, eps=1e-5),
    "int4_tied": dict(vocab=640, dim=128, layers=3, heads=2, kv_heads=2, hidden=256, bits=4, group_size=64,
                      tied=True, rope_theta=1000000.0, qkv_bias=True),
}


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_quantized_model_file_round_trip(kt, oracle, st, tmp_path, name):
    """A file laid out as Transformer.saveQuantized writes it loads into a device
    decoder that decodes exactly like one built from the same weights in memory,
    matches the CPU decode step, and writes the same file back byte for byte."""
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    cfg_o = DO.DecoderConfig(**CONFIGS[name])
    weights = DO.DecoderWeights.random(cfg_o, seed=len(name))
    path_a = tmp_path / "a.safetensors"
    SO.save_quantized(str(path_a), weights)
    loaded = D.DeviceDecoder.load_quantized(path_a, max_seq=48)
    assert loaded.cfg.tied == cfg_o.tied and loaded.cfg.rope_scaling == cfg_o.rope_scaling
    assert np.float32(loaded.cfg.eps) == np.float32(cfg_o.eps)
    built = D.DeviceDecoder(D.DecoderConfig(**CONFIGS[name]), weights, max_seq=48)
    ref = DO.OracleDecoder(weights, max_seq=48)
    prompt = [4, 8, 15, 16, 23, 42]
    for t in prompt:
        la, lb = loaded.step(t), built.step(t)
        assert torch.equal(la, lb)
        lr = ref.step(t)
        scale = np.abs(lr).max()
        assert np.abs(la.cpu().numpy() - lr).max() <= 1e-3 * scale
    loaded.reset()
    built.reset()
    assert loaded.generate(prompt, 8) == built.generate(prompt, 8)
    path_b = tmp_path / "b.safetensors"
    loaded.save_quantized(path_b)
    assert path_b.read_bytes() == path_a.read_bytes()
    assert kt.Context.get().take_error() == 0


def test_loading_reports_missing_metadata_and_tensors(kt, oracle, st, tmp_path):
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    cfg = DO.DecoderConfig(**CONFIGS["int8_untied"])
    meta, entries = SO.quantized_model_entries(DO.DecoderWeights.random(cfg, seed=1))
    no_meta = tmp_path / "nometa.safetensors"
    SO.save_entries(str(no_meta), entries, {k: v for k, v in meta.items() if k != "kotensor.numHeads"})
    with pytest.raises(ValueError, match="has no kotensor.numHeads metadata"):
        D.load_quantized_weights(no_meta)
    missing = tmp_path / "missing.safetensors"
    SO.save_entries(str(missing), [e for e in entries if e[0] != "finalNorm.weight"], meta)
    with pytest.raises(ValueError, match="is missing finalNorm.weight"):
        D.load_quantized_weights(missing)
