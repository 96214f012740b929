"""CPU restatement of Kotensor's safetensors files.  TEST INFRASTRUCTURE ONLY:
the file-format parity tests use it as the checker; the product never imports it.

Follows (paths inside the Kotensor project, Engine/kotensor/src/main/kotlin/):
  SafeTensorsFile header parse        SafeTensors.kt:33-69
  Entry.bytesPerElement               SafeTensors.kt:23-30
  readRaw / readInto / convert        SafeTensors.kt:90-98, :110-170
  halfToFloat                         SafeTensors.kt:179-198
  SafeTensors.saveEntries, jsonString SafeTensors.kt:220-264
  Transformer.saveQuantized           Transformer.kt:402-431
  namedParameters / namedProjections  Transformer.kt:268-282, :316-335
  namedQuantizedTensors               Transformer.kt:354-359
Kotlin's Float.toString (the metadata's normEps, ropeTheta and RoPE scaling
values) is restated from its specification: the shortest decimal that rounds
to the float, plain notation for 1e-3 <= |v| < 1e7, else d.dddE<exp>.

Pinned by the `safetensors` package (an independent implementation of the
format): files written here read back through it with the same names, dtypes,
shapes, bytes and metadata, and files it writes parse here identically.
"""
from __future__ import annotations

import json
import struct
from typing import Optional

import numpy as np

BYTES_PER_ELEMENT = {"F32": 4, "I32": 4, "U32": 4, "F16": 2, "BF16": 2, "I16": 2, "U16": 2,
                     "F64": 8, "I64": 8, "U64": 8, "I8": 1, "U8": 1, "BOOL": 1}


def json_string(text: str) -> str:
    """SafeTensors.jsonString (SafeTensors.kt:251-264)."""
    out = ['"']
    for c in text:
        if c == '"':
            out.append('\\"')
        elif c == '\\':
            out.append('\\\\')
        elif c == '\n':
            out.append('\\n')
        elif c == '\r':
            out.append('\\r')
        elif c == '\t':
            out.append('\\t')
        elif ord(c) < 0x20:
            out.append('\\u%04x' % ord(c))
        else:
            out.append(c)
    out.append('"')
    return "".join(out)


def encode(entries: list, metadata: Optional[dict] = None) -> bytes:
    """The bytes SafeTensors.saveEntries writes (SafeTensors.kt:220-249).
    entries: (name, dtype, shape, data bytes) in order."""
    parts = []
    if metadata:
        pairs = ",".join(f"{json_string(k)}:{json_string(v)}" for k, v in metadata.items())
        parts.append('"__metadata__":{' + pairs + '}')
    offset = 0
    for name, dtype, shape, data in entries:
        end = offset + len(data)
        parts.append(f'{json_string(name)}:{{"dtype":"{dtype}","shape":[{",".join(str(int(d)) for d in shape)}],'
                     f'"data_offsets":[{offset},{end}]}}')
        offset = end
    header = ("{" + ",".join(parts) + "}").encode("utf-8")
    padding = (8 - len(header) % 8) % 8
    return struct.pack("<q", len(header) + padding) + header + b" " * padding + b"".join(bytes(d) for d in
                                                                                         (e[3] for e in entries))


def save_entries(path: str, entries: list, metadata: Optional[dict] = None) -> None:
    with open(path, "wb") as f:
        f.write(encode(entries, metadata))


def _linked(pairs):
    """LinkedHashMap put semantics: a repeated key keeps its first position."""
    d = {}
    for k, v in pairs:
        d[k] = v
    return d


def parse(path: str):
    """SafeTensorsFile.init (SafeTensors.kt:33-69): (entries, metadata, data_start),
    entries name -> (dtype, shape, start, end) in header order."""
    with open(path, "rb") as f:
        blob = f.read()
    size = struct.unpack("<q", blob[:8])[0]
    if not 1 <= size <= (100 << 20):
        raise ValueError(f"Invalid safetensors header size {size} in {path}")
    if 8 + size > len(blob):
        raise OSError("header runs past the end of the file")
    header = json.loads(blob[8:8 + size].decode("utf-8"), object_pairs_hook=_linked)
    if not isinstance(header, dict):
        raise ValueError(f"safetensors header of {path} is not a JSON object")
    data_start = 8 + size
    entries, metadata = {}, {}
    for name, body in header.items():
        if not isinstance(body, dict):
            continue
        if name == "__metadata__":
            for k, v in body.items():
                metadata[k] = v if isinstance(v, str) else json.dumps(v)
            continue
        dtype = body.get("dtype")
        if not isinstance(dtype, str):
            raise ValueError(f"Tensor {name} has no dtype")
        shape = [int(d) for d in body.get("shape", [])] if isinstance(body.get("shape"), list) else []
        offsets = body.get("data_offsets")
        if not isinstance(offsets, list):
            raise ValueError(f"Tensor {name} has no data_offsets")
        start, end = int(offsets[0]), int(offsets[1])
        if start < 0 or end < start or data_start + end > len(blob):
            raise ValueError(f"Tensor {name} data range [{start}, {end}) exceeds file {len(blob)}")
        entries[name] = (dtype, shape, start, end)
    return entries, metadata, data_start


def read_raw(path: str, name: str) -> bytes:
    entries, _, data_start = parse(path)
    _, _, start, end = entries[name]
    with open(path, "rb") as f:
        f.seek(data_start + start)
        return f.read(end - start)


def half_to_float(bits: int) -> np.float32:
    """SafeTensorsFile.halfToFloat (SafeTensors.kt:179-198), from the binary16 definition."""
    sign = (bits >> 15) & 1
    exponent = (bits >> 10) & 0x1F
    mantissa = bits & 0x3FF
    if exponent == 0x1F:
        out = (sign << 31) | 0x7F800000 | (mantissa << 13)
    elif exponent != 0:
        out = (sign << 31) | ((exponent - 15 + 127) << 23) | (mantissa << 13)
    elif mantissa == 0:
        out = sign << 31
    else:
        shifted, shifts = mantissa, -1
        while True:
            shifts += 1
            shifted <<= 1
            if shifted & 0x400:
                break
        out = (sign << 31) | ((127 - 15 - shifts) << 23) | ((shifted & 0x3FF) << 13)
    return np.array([out], np.uint32).view(np.float32)[0]


def to_float32(dtype: str, raw: bytes) -> np.ndarray:
    """SafeTensorsFile.convert (SafeTensors.kt:136-170) for a whole tensor."""
    b = np.frombuffer(raw, np.uint8)
    if dtype == "F32":
        return b.view("<f4").astype(np.float32)
    if dtype == "BF16":
        return (b.view("<u2").astype(np.uint32) << 16).view(np.float32)
    if dtype == "F16":
        return np.array([half_to_float(int(h)) for h in b.view("<u2")], np.float32)
    if dtype == "F64":
        return b.view("<f8").astype(np.float32)
    if dtype == "I8":
        return b.view(np.int8).astype(np.float32)
    if dtype in ("U8", "BOOL"):
        return b.astype(np.float32)
    if dtype == "I16":
        return b.view("<i2").astype(np.float32)
    if dtype == "I32":
        return b.view("<i4").astype(np.float32)
    if dtype == "I64":
        return b.view("<i8").astype(np.float32)
    raise ValueError(f"Unsupported safetensors dtype '{dtype}'")


def java_float_str(x) -> str:
    """Kotlin/Java Float.toString."""
    f = np.float32(x)
    if np.isnan(f):
        return "NaN"
    if np.isinf(f):
        return "Infinity" if f > 0 else "-Infinity"
    if f == 0:
        return "-0.0" if np.signbit(f) else "0.0"
    sign = "-" if f < 0 else ""
    a = np.float32(abs(f))
    mant, exp = np.format_float_scientific(a, unique=True, trim="k").split("e")
    digits = mant.replace(".", "").rstrip("0") or "0"
    if len(digits) == 1:
        # a one-digit shortest decimal is replaced by the closest two-digit one
        mant, exp = np.format_float_scientific(a, precision=1, unique=False).split("e")
        digits = mant.replace(".", "").rstrip("0") or "0"
    e = int(exp)
    if 1e-3 <= float(a) < 1e7:
        if e >= 0:
            whole = digits[:e + 1].ljust(e + 1, "0")
            frac = digits[e + 1:] or "0"
        else:
            whole, frac = "0", "0" * (-e - 1) + digits
        return f"{sign}{whole}.{frac}"
    return f"{sign}{digits[0]}.{digits[1:] or '0'}E{e}"


PROJECTIONS = [("attention.wQ", "wq", "bq"), ("attention.wK", "wk", "bk"), ("attention.wV", "wv", "bv"),
               ("attention.wOut", "wo", "bo"), ("ffn.wGate", "wg", "bg"), ("ffn.wUp", "wu", "bu"),
               ("ffn.wDown", "wd", "bd")]


def quantized_model_entries(weights):
    """(metadata, entries) of Transformer.saveQuantized (Transformer.kt:402-431)
    for decoder weights (oracle.decoder_oracle.DecoderWeights)."""
    cfg = weights.cfg
    meta = {
        "kotensor.vocabularySize": str(cfg.vocab),
        "kotensor.dimension": str(cfg.dim),
        "kotensor.numLayers": str(cfg.layers),
        "kotensor.numHeads": str(cfg.heads),
        "kotensor.hiddenDimension": str(cfg.hidden),
        "kotensor.numKeyValueHeads": str(cfg.kv_heads),
        "kotensor.normEps": java_float_str(cfg.eps),
        "kotensor.ropeTheta": java_float_str(cfg.rope_theta),
    }
    if cfg.rope_scaling is not None:
        f, lo, hi, orig = cfg.rope_scaling
        meta["kotensor.ropeScaling"] = f"{java_float_str(f)},{java_float_str(lo)},{java_float_str(hi)},{int(orig)}"
    meta["kotensor.quantization.bits"] = str(cfg.bits)
    meta["kotensor.quantization.groupSize"] = str(cfg.group_size)
    if cfg.tied:
        meta["kotensor.tiedEmbedding"] = "true"

    def f32(name, a, shape):
        return (name, "F32", shape, np.ascontiguousarray(a, np.float32).tobytes())

    entries = []
    for l, L in enumerate(weights.layers):
        entries.append(f32(f"block.{l}.norm1.weight", L["norm1"], [1, cfg.dim]))
        entries.append(f32(f"block.{l}.norm2.weight", L["norm2"], [1, cfg.dim]))
    entries.append(f32("finalNorm.weight", weights.final_norm, [1, cfg.dim]))
    projections = []
    for l, L in enumerate(weights.layers):
        for suffix, wk, bk in PROJECTIONS:
            projections.append((f"block.{l}.{suffix}", L[wk], L[bk]))
    projections.append(("lmHead", weights.head, weights.head_bias))
    for name, w, b in projections:
        entries.append(f32(f"{name}.bias", b, [1, w.columns]))
    quantized = ([] if cfg.tied else [("embedding", weights.embedding)]) + [(n, w) for n, w, _ in projections]
    for name, w in quantized:
        bpr, groups = w.bytes_per_row, w.groups
        entries.append((f"{name}.qweight", "I8" if w.bits == 8 else "U8", [w.rows, bpr],
                        np.ascontiguousarray(w.qdata).view(np.uint8).tobytes()))
        entries.append(f32(f"{name}.scales", w.scales, [groups, w.columns]))
        if w.bits == 4:
            entries.append((f"{name}.zeros", "U8", [groups, w.columns], np.ascontiguousarray(w.zeros).tobytes()))
    return meta, entries


def save_quantized(path: str, weights) -> None:
    meta, entries = quantized_model_entries(weights)
    save_entries(path, entries, meta)
