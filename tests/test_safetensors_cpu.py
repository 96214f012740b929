"""CPU checks of the safetensors files (no GPU): the native header reader and
writer of libkt_cuda.so (kt_st_open / kt_st_write, host memory only) against
the oracle restatement of SafeTensors.kt, and the oracle against the `safetensors`
package and the golden dtype fixture.

Reference behaviour ported (Engine/kotensor/src/test/kotlin/):
  QuantizationTest.testSaveAndLoadQuantizedModelRoundTrip  (file layout, metadata first, I8/U8 qweight)
  MappedModelTest.testTiedModelRoundTripsThroughFilesWithoutAnEmbeddingCopy (no embedding.* entries)
  HuggingFaceImportTest dtype fixture                        (F16 / BF16 / F32 conversion)
  Phase5Test.testSafeTensorsSaveAndLoad                     (save / load round trip)
"""
import json
import os
import struct

import numpy as np
import pytest

from oracle import safetensors_oracle as SO

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
# The reference's own fixtures (src/test/resources/hf), copied unchanged by
# tests/golden/make_hf_golden.py.
REF_FIXTURES = os.path.join(GOLDEN, "hf")


@pytest.fixture(scope="module")
def st(kt):
    from kotensor_b200 import safetensors
    return safetensors


def _same_f32(got, exp):
    nan = np.isnan(exp)
    return np.array_equal(np.isnan(got), nan) and np.array_equal(got[~nan].view(np.uint32),
                                                                  exp[~nan].view(np.uint32))


def test_oracle_conversion_matches_golden_fixture():
    path = os.path.join(GOLDEN, "dtypes.safetensors")
    entries, meta, _ = SO.parse(path)
    assert meta == {"format": "pt", "note": "kotensor dtype fixture"}
    with np.load(os.path.join(GOLDEN, "dtypes_expected.npz")) as z:
        for name, (dtype, shape, s, e) in entries.items():
            with np.errstate(over="ignore"):
                got = SO.to_float32(dtype, SO.read_raw(path, name))
            assert _same_f32(got, z[name]), name


def test_oracle_conversion_matches_reference_known_answers():
    """The reference's own dtype fixture and its expected values (HuggingFaceImportTest)."""
    d = os.path.join(REF_FIXTURES, "dtypes")
    expected = json.load(open(os.path.join(d, "expected.json")))
    path = os.path.join(d, "dtypes.safetensors")
    entries, meta, _ = SO.parse(path)
    for name, values in expected.items():
        got = SO.to_float32(entries[name][0], SO.read_raw(path, name))
        assert np.array_equal(got, np.array(values, np.float32)), name


def test_half_to_float_matches_binary16_for_every_pattern():
    bits = np.arange(65536, dtype=np.uint16)
    ours = np.array([SO.half_to_float(int(b)) for b in bits], np.float32)
    ref = bits.view(np.float16).astype(np.float32)
    assert _same_f32(ours, ref)


def _fixture_files():
    files = [os.path.join(GOLDEN, "dtypes.safetensors")]
    for sub in sorted(os.listdir(REF_FIXTURES)):
        for f in sorted(os.listdir(os.path.join(REF_FIXTURES, sub))):
            if f.endswith(".safetensors"):
                files.append(os.path.join(REF_FIXTURES, sub, f))
    return files


@pytest.mark.parametrize("path", _fixture_files(), ids=os.path.basename)
def test_native_reader_matches_oracle_and_safetensors_package(st, path):
    from safetensors import safe_open
    entries, meta, data_start = SO.parse(path)
    with st.SafeTensorsFile(path) as f:
        assert f.names == list(entries)
        assert f.metadata == meta
        for name, (dtype, shape, s, e) in entries.items():
            got = f.entry(name)
            assert (got.dtype, list(got.shape), got.byte_offset, got.byte_length) == (dtype, shape, s, e - s)
            assert f.read_raw(name).tobytes() == SO.read_raw(path, name)
    with safe_open(path, "pt") as g:
        assert sorted(g.keys()) == sorted(entries)
        assert (g.metadata() or {}) == meta
        for name in g.keys():
            assert list(g.get_slice(name).get_shape()) == entries[name][1]


def _entries(rng):
    return [
        ("block.0.attention.wQ.qweight", "U8", [3, 5], rng.integers(0, 256, 15, dtype=np.uint8).tobytes()),
        ("scales", "F32", [2, 2], rng.standard_normal(4).astype(np.float32).tobytes()),
        ("quo\"te\\back\nslash\ttab\x01ctl", "I8", [4], bytes([1, 255, 3, 128])),
        ("ünïcödé", "F32", [], np.float32(2.5).tobytes()),
        ("empty", "F32", [0, 3], b""),
        ("big", "I64", [1, 2, 3], rng.integers(-2**62, 2**62, 6, dtype=np.int64).tobytes()),
    ]


@pytest.mark.parametrize("meta", [None, {}, {"kotensor.normEps": "1.0E-6", "k\"e\ty": "v\\a\nl\x1f", "ü": "ß"}])
def test_native_writer_writes_the_reference_bytes(st, tmp_path, meta):
    entries = _entries(np.random.default_rng(5))
    path = tmp_path / "w.safetensors"
    st.save_entries(path, [st.SafeTensorsEntry(n, d, s, np.frombuffer(b, np.uint8)) for n, d, s, b in entries], meta)
    blob = path.read_bytes()
    assert blob == SO.encode(entries, meta)
    size = struct.unpack("<q", blob[:8])[0]
    assert size % 8 == 0 and blob[8 + size - 1:8 + size] in (b" ", b"}")
    from safetensors import safe_open
    with safe_open(str(path), "np") as g:
        assert (g.metadata() or {}) == (meta or {})
        assert g.get_tensor("big").tobytes() == entries[-1][3]


def test_save_and_load_round_trip_host(st, tmp_path):
    """Phase5Test.testSafeTensorsSaveAndLoad on host memory: F32 entries back bit for bit."""
    rng = np.random.default_rng(3)
    tensors = {"w1": rng.standard_normal((4, 6)).astype(np.float32), "b": rng.standard_normal(6).astype(np.float32)}
    path = tmp_path / "p.safetensors"
    st.save(path, tensors)
    with st.SafeTensorsFile(path) as f:
        for name, a in tensors.items():
            assert f.entry(name).dtype == "F32" and f.entry(name).shape == a.shape
            assert np.array_equal(f.read_raw(name).view(np.float32).reshape(a.shape), a)


def test_multi_chunk_host_read(st, tmp_path):
    """Reads larger than one parallel slice come back byte for byte."""
    data = np.random.default_rng(9).integers(0, 256, (37 << 20) + 13, dtype=np.uint8)
    path = tmp_path / "big.safetensors"
    st.save_entries(path, [st.SafeTensorsEntry("pad", "U8", [3], np.arange(3, dtype=np.uint8)),
                           st.SafeTensorsEntry("x", "U8", [data.size], data)])
    with st.SafeTensorsFile(path) as f:
        assert np.array_equal(f.read_raw("x"), data)
        with pytest.raises(ValueError, match="No tensor named"):
            f.read_raw("nope")


def _write_raw(path, header: bytes, data: bytes = b"", size=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<q", len(header) if size is None else size) + header + data)


@pytest.mark.parametrize("case,header,data,size,error", [
    ("zero size", b"", b"", 0, ValueError),
    ("huge size", b"{}", b"", (100 << 20) + 1, ValueError),
    ("not an object", b"[1, 2]  ", b"", None, ValueError),
    ("no dtype", b'{"a":{"shape":[1],"data_offsets":[0,1]}}', b"x", None, ValueError),
    ("no offsets", b'{"a":{"dtype":"U8","shape":[1]}}', b"x", None, ValueError),
    ("past eof", b'{"a":{"dtype":"U8","shape":[9],"data_offsets":[0,9]}}', b"x", None, ValueError),
    ("reversed", b'{"a":{"dtype":"U8","shape":[1],"data_offsets":[1,0]}}', b"x", None, ValueError),
    ("trailing", b'{"a":1} x', b"", None, ValueError),
    ("truncated header", b'{"a":1}', b"", 64, OSError),
])
def test_malformed_files_fail_like_the_reference(st, tmp_path, case, header, data, size, error):
    path = tmp_path / "bad.safetensors"
    _write_raw(path, header, data, size)
    with pytest.raises(error):
        st.SafeTensorsFile(path)
    with pytest.raises((ValueError, OSError, json.JSONDecodeError)):
        SO.parse(str(path))


@pytest.mark.parametrize("case,header", [
    # an end offset whose sum with the data start overflows int64 must not pass the bounds check
    ("end near 2^63", b'{"a":{"dtype":"U8","shape":[1],"data_offsets":[0,9223372036854775800]}}'),
    ("negative dimension", b'{"a":{"dtype":"U8","shape":[-1],"data_offsets":[0,1]}}'),
    ("dimension beyond int32", b'{"a":{"dtype":"U8","shape":[4294967297],"data_offsets":[0,1]}}'),
])
def test_native_reader_rejects_out_of_range_numbers(st, tmp_path, case, header):
    path = tmp_path / "bad.safetensors"
    _write_raw(path, header, b"x")
    with pytest.raises(ValueError):
        st.SafeTensorsFile(path)


def test_missing_file_is_an_io_error(st, tmp_path):
    with pytest.raises(OSError):
        st.SafeTensorsFile(tmp_path / "absent.safetensors")


def test_header_tolerance_matches_the_reference_reader(st, tmp_path):
    """Non-object members are skipped, metadata values that are not strings keep
    their JSON text, a repeated key keeps its first position and last value, and
    escapes (\\u with surrogate pairs) decode to UTF-8."""
    header = (b'{"skip":5,"__metadata__":{"a":"1","n":42,"a":"2"},'
              b'"t\\u00e9\\ud83d\\ude00":{"dtype":"U8","shape":[2],"data_offsets":[0,2]},'
              b'"t2":{"dtype":"U8","shape":[1],"data_offsets":[0,1]},'
              b'"t2":{"dtype":"I8","shape":[1],"data_offsets":[1,2]}}')
    path = tmp_path / "tol.safetensors"
    _write_raw(path, header, b"ab")
    with st.SafeTensorsFile(path) as f:
        assert f.names == ["té\U0001F600", "t2"]
        assert f.metadata == {"a": "2", "n": "42"}
        assert f.entry("t2").dtype == "I8" and f.read_raw("t2").tobytes() == b"b"


def test_java_float_string(st):
    known = [(1e-6, "1.0E-6"), (1e-5, "1.0E-5"), (10000.0, "10000.0"), (500000.0, "500000.0"),
             (1e6, "1000000.0"), (1e7, "1.0E7"), (8.0, "8.0"), (0.001, "0.001"), (9.765625e-4, "9.765625E-4"),
             (0.1, "0.1"), (-2.5, "-2.5"), (3.4028235e38, "3.4028235E38"), (1.4e-45, "1.4E-45"), (0.0, "0.0"),
             (-0.0, "-0.0"), (1234567.0, "1234567.0")]
    for x, text in known:
        assert st.java_float_string(x) == text, x
        assert SO.java_float_str(x) == text, x
    vals = np.random.default_rng(1).standard_normal(3000).astype(np.float32) * np.float32(10.0) ** \
        np.random.default_rng(2).integers(-12, 12, 3000).astype(np.float32)
    for v in vals:
        text = st.java_float_string(v)
        assert text == SO.java_float_str(v)
        assert np.float32(text.replace("E", "e")) == v


@pytest.mark.parametrize("bits,tied", [(8, False), (4, False), (4, True)])
def test_oracle_quantized_model_file_layout(st, tmp_path, bits, tied):
    """Transformer.saveQuantized's layout: kotensor.* metadata first, 16 quantized
    tensors for 2 layers (untied), I8 / U8 qweights, no embedding.* when tied,
    and a file smaller than the fp32 parameters."""
    from oracle.decoder_oracle import DecoderConfig, DecoderWeights
    cfg = DecoderConfig(vocab=48, dim=32, layers=2, heads=4, kv_heads=2, hidden=80, bits=bits, group_size=16,
                        tied=tied, rope_scaling=(8.0, 1.0, 4.0, 8192))
    w = DecoderWeights.random(cfg, seed=31)
    path = tmp_path / "m.safetensors"
    SO.save_quantized(str(path), w)
    with st.SafeTensorsFile(path) as f:
        assert next(iter(f.metadata)).split(".")[0] == "kotensor"
        assert f.metadata["kotensor.ropeScaling"] == "8.0,1.0,4.0,8192"
        assert f.metadata["kotensor.normEps"] == "1.0E-6"
        assert f.metadata.get("kotensor.tiedEmbedding") == ("true" if tied else None)
        quantized = [n[:-len(".qweight")] for n in f.names if n.endswith(".qweight")]
        assert len(quantized) == (15 if tied else 16)
        assert f.entry("block.0.attention.wQ.qweight").dtype == ("I8" if bits == 8 else "U8")
        assert not tied or not any(n.startswith("embedding.") for n in f.names)
        kv = cfg.kv_heads * cfg.head_dim
        params = cfg.vocab * cfg.dim * (1 if tied else 2) + cfg.layers * (
            2 * cfg.dim * cfg.dim + 2 * cfg.dim * kv + 3 * cfg.dim * cfg.hidden)
        assert os.path.getsize(path) < params * 4
