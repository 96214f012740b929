"""Kotensor's safetensors model files, read straight into HBM and written from it
(the C ABI's kt_st_* entry points; parsing and file I/O are native code).

Reference (paths inside the Kotensor project, Engine/kotensor/src/main/kotlin/):
  SafeTensorsFile (entries, metadata, load, readInto, readRaw)   SafeTensors.kt:12-178
  SafeTensorsEntry.of / SafeTensors.save / saveEntries / load   SafeTensors.kt:200-278
  QuantizedTensor.mapFrom (here: into HBM)                      QuantizedTensor.kt:109-126

Where the reference returns a FloatArray, this module returns a CUDA float32
tensor filled by the library (bytes copied from the file through pinned
staging buffers, converted to float32 on the GPU).  ``read_raw`` is the one
host-memory read, as in the reference.  Errors: a failed ``require`` raises
ValueError, an unreadable file OSError.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Iterable, Optional, Sequence

import numpy as np

from . import _lib
from .quantized import Context, Quantization, QuantizedTensor, _stream_of

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None

BYTES_PER_ELEMENT = {"F32": 4, "I32": 4, "U32": 4, "F16": 2, "BF16": 2, "I16": 2, "U16": 2,
                     "F64": 8, "I64": 8, "U64": 8, "I8": 1, "U8": 1, "BOOL": 1}


@dataclass(frozen=True)
class Entry:
    """SafeTensorsFile.Entry (SafeTensors.kt:14-31)."""
    name: str
    dtype: str
    shape: tuple
    byte_offset: int
    byte_length: int

    @property
    def element_count(self) -> int:
        count = 1
        for d in self.shape:
            count *= d
        if count > 2**31 - 1:
            raise ValueError(f"Tensor {self.name} has {count} elements, more than a FloatArray can hold")
        return count

    @property
    def bytes_per_element(self) -> int:
        if self.dtype not in BYTES_PER_ELEMENT:
            raise ValueError(f"Unsupported safetensors dtype '{self.dtype}' for tensor {self.name}")
        return BYTES_PER_ELEMENT[self.dtype]


def _device_ctx(device: Optional[int]) -> Context:
    return Context.get(device)


class SafeTensorsFile:
    """An open safetensors file (kt_st_open): the parsed header and the file's
    staging buffers.  Use as a context manager or call ``close()``."""

    def __init__(self, path):
        self.path = str(path)
        h = ctypes.c_void_p()
        _lib.check(_lib.load().kt_st_open(self.path.encode(), ctypes.byref(h)))
        self._handle = h
        lib = _lib.load()
        entries = {}
        for i in range(lib.kt_st_tensor_count(h)):
            name = lib.kt_st_tensor_name(h, i).decode()
            info = _lib.KtStEntryInfo()
            _lib.check(lib.kt_st_entry(h, name.encode(), ctypes.byref(info)))
            entries[name] = Entry(name, info.dtype.decode(), tuple(info.shape[d] for d in range(info.rank)),
                                  int(info.offset), int(info.bytes))
        self.entries = entries
        meta = {}
        for i in range(lib.kt_st_metadata_count(h)):
            k, v = ctypes.c_char_p(), ctypes.c_char_p()
            _lib.check(lib.kt_st_metadata_at(h, i, ctypes.byref(k), ctypes.byref(v)))
            meta[k.value.decode()] = v.value.decode()
        self.metadata = meta

    # -- header
    @property
    def names(self) -> list:
        return list(self.entries)

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def entry(self, name: str) -> Entry:
        if name not in self.entries:
            raise ValueError(f"No tensor named '{name}' in {self.path}")
        return self.entries[name]

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._handle:
            raise ValueError(f"{self.path} is closed")
        return self._handle

    # -- reads
    def read_raw(self, name: str) -> np.ndarray:
        """readRaw(name): the tensor's bytes in host memory (uint8)."""
        e = self.entry(name)
        out = np.empty(e.byte_length, np.uint8)
        _lib.check(_lib.load().kt_st_read_raw(self.handle, name.encode(), out.ctypes.data_as(ctypes.c_void_p),
                                              out.size))
        return out

    def read_raw_into(self, name: str, dest) -> None:
        """The tensor's bytes into a CUDA tensor of at least that many bytes,
        on the tensor's current stream."""
        if not (torch is not None and isinstance(dest, torch.Tensor) and dest.is_cuda and dest.is_contiguous()):
            raise ValueError("dest must be a contiguous CUDA tensor")
        ctx = _device_ctx(dest.device.index)
        _lib.check(_lib.load().kt_st_read_raw_device(ctx.handle, self.handle, name.encode(),
                                                     ctypes.c_void_p(dest.data_ptr()),
                                                     dest.numel() * dest.element_size(), _stream_of(dest)))

    def read_into(self, name: str, dest) -> None:
        """readInto(name, dest) (SafeTensors.kt:86-88): float32 values into a CUDA
        float32 tensor with room for them, converted from the stored dtype on the GPU."""
        if not (torch is not None and isinstance(dest, torch.Tensor) and dest.is_cuda and dest.is_contiguous()
                and dest.dtype == torch.float32):
            raise ValueError("dest must be a contiguous CUDA float32 tensor")
        ctx = _device_ctx(dest.device.index)
        _lib.check(_lib.load().kt_st_read_f32_device(ctx.handle, self.handle, name.encode(),
                                                     ctypes.c_void_p(dest.data_ptr()), dest.numel(),
                                                     _stream_of(dest)))

    def load(self, name: str, device: Optional[int] = None):
        """load(name) (SafeTensors.kt:79-84): a CUDA float32 tensor of the entry's shape."""
        e = self.entry(name)
        ctx = _device_ctx(device)
        out = torch.empty(e.shape, dtype=torch.float32, device=f"cuda:{ctx.device}")
        self.read_into(name, out)
        return out

    def load_quantized(self, name: str, quantization: Quantization, rows: int, columns: int,
                       device: Optional[int] = None) -> QuantizedTensor:
        """A device QuantizedTensor from <name>.qweight / .scales / .zeros
        (QuantizedTensor.mapFrom's checks, QuantizedTensor.kt:109-126)."""
        ctx = _device_ctx(device)
        h = ctypes.c_void_p()
        stream = ctypes.c_void_p(torch.cuda.current_stream(ctx.device).cuda_stream)
        _lib.check(_lib.load().kt_qweight_load(ctx.handle, self.handle, name.encode(), quantization.bits,
                                               quantization.group_size, int(rows), int(columns), stream,
                                               ctypes.byref(h)))
        return QuantizedTensor(h, ctx)

    # -- lifetime
    def close(self) -> None:
        if self._handle:
            _lib.load().kt_st_close(self._handle)
            self._handle = ctypes.c_void_p()

    def __enter__(self) -> "SafeTensorsFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class SafeTensorsEntry:
    """SafeTensorsEntry(name, dtype, shape, bytes) (SafeTensors.kt:200-209).
    ``data`` is a numpy array (host) or a contiguous CUDA tensor whose bytes are
    written as they are."""
    name: str
    dtype: str
    shape: Sequence[int]
    data: object

    @staticmethod
    def of(name: str, tensor) -> "SafeTensorsEntry":
        """SafeTensorsEntry.of(name, tensor): float32 values as F32."""
        if torch is not None and isinstance(tensor, torch.Tensor):
            t = tensor.detach().to(torch.float32).contiguous()
            return SafeTensorsEntry(name, "F32", list(t.shape), t)
        a = np.ascontiguousarray(tensor, dtype=np.float32)
        return SafeTensorsEntry(name, "F32", list(a.shape), a)


class _DeviceBytes:
    """Device memory owned elsewhere (a QuantizedTensor's arrays) as entry data."""

    def __init__(self, ptr: int, nbytes: int, device: int):
        self.ptr, self.nbytes, self.device = ptr, nbytes, device


def _entry_bytes(e: SafeTensorsEntry):
    """(pointer, byte count, device index or None, keep-alive) of an entry's data."""
    d = e.data
    if isinstance(d, _DeviceBytes):
        return d.ptr, d.nbytes, d.device, d
    if torch is not None and isinstance(d, torch.Tensor):
        if not d.is_contiguous():
            raise ValueError(f"tensor {e.name} is not contiguous")
        if d.is_cuda:
            return d.data_ptr(), d.numel() * d.element_size(), d.device.index, d
        d = d.numpy()
    if isinstance(d, (bytes, bytearray, memoryview)):
        d = np.frombuffer(bytes(d), np.uint8)
    a = np.ascontiguousarray(d)
    return a.ctypes.data, a.nbytes, None, a


def save_entries(path, entries: Iterable[SafeTensorsEntry], metadata: Optional[dict] = None) -> None:
    """SafeTensors.saveEntries(file, entries, metadata) (SafeTensors.kt:220-249)."""
    entries = list(entries)
    metadata = dict(metadata or {})
    keep = []
    arr = (_lib.KtStTensor * max(1, len(entries)))()
    device = None
    for i, e in enumerate(entries):
        ptr, nbytes, dev_index, ref = _entry_bytes(e)
        shape = (ctypes.c_int64 * max(1, len(e.shape)))(*[int(s) for s in e.shape])
        name, dtype = e.name.encode(), e.dtype.encode()
        keep += [ref, shape, name, dtype]
        arr[i] = _lib.KtStTensor(name, dtype, len(e.shape), ctypes.cast(shape, ctypes.POINTER(ctypes.c_int64)),
                                 ctypes.c_void_p(ptr), nbytes, int(dev_index is not None))
        if dev_index is not None:
            if device is not None and device != dev_index:
                raise ValueError("all device tensors of one file must be on one device")
            device = dev_index
    keys = (ctypes.c_char_p * max(1, len(metadata)))(*[k.encode() for k in metadata])
    values = (ctypes.c_char_p * max(1, len(metadata)))(*[str(v).encode() for v in metadata.values()])
    ctx, stream = None, None
    if device is not None:
        ctx = _device_ctx(device).handle
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    _lib.check(_lib.load().kt_st_write(ctx, str(path).encode(), arr, len(entries), keys, values, len(metadata),
                                       stream))


def save(path, tensors: dict, metadata: Optional[dict] = None) -> None:
    """SafeTensors.save(file, tensors, metadata): every tensor as F32."""
    save_entries(path, [SafeTensorsEntry.of(n, t) for n, t in tensors.items()], metadata)


def load(path, device: Optional[int] = None) -> dict:
    """SafeTensors.load(file): every tensor as a CUDA float32 tensor."""
    with SafeTensorsFile(path) as f:
        return {name: f.load(name, device) for name in f.names}


def quantized_entries(name: str, weight: QuantizedTensor) -> list:
    """The entries Transformer.saveQuantized writes for one quantized weight
    (Transformer.kt:423-428), reading the device arrays in place."""
    info = weight._info
    groups, columns = weight.groups, weight.columns

    def dev(ptr, nbytes):
        return _DeviceBytes(ptr, nbytes, weight.device)

    out = [SafeTensorsEntry(f"{name}.qweight", "I8" if weight.bits == 8 else "U8",
                            [weight.rows, weight.bytes_per_row], dev(info.qdata, weight.rows * weight.bytes_per_row)),
           SafeTensorsEntry(f"{name}.scales", "F32", [groups, columns], dev(info.scales, groups * columns * 4))]
    if weight.bits == 4:
        out.append(SafeTensorsEntry(f"{name}.zeros", "U8", [groups, columns], dev(info.zeros, groups * columns)))
    return out


def java_float_string(x: float) -> str:
    """Kotlin's Float.toString, used for the kotensor.* metadata values: the
    shortest decimal that rounds back to the float (two digits when one would
    do), plain for 1e-3 <= |v| < 1e7, else <d.ddd>E<exponent>."""
    f = np.float32(x)
    if np.isnan(f):
        return "NaN"
    if np.isinf(f):
        return "Infinity" if f > 0 else "-Infinity"
    if f == 0:
        return "-0.0" if np.signbit(f) else "0.0"
    a = np.float32(abs(f))
    text = np.format_float_scientific(a, unique=True, trim="k")
    digits = text.split("e")[0].replace(".", "").rstrip("0") or "0"
    if len(digits) < 2:
        text = np.format_float_scientific(a, precision=1, unique=False)
        digits = text.split("e")[0].replace(".", "").rstrip("0") or "0"
    exp = int(text.split("e")[1])
    sign = "-" if f < 0 else ""
    if 1e-3 <= float(a) < 1e7:
        if exp >= 0:
            return f"{sign}{digits[:exp + 1].ljust(exp + 1, '0')}.{digits[exp + 1:] or '0'}"
        return f"{sign}0.{'0' * (-exp - 1)}{digits}"
    return f"{sign}{digits[0]}.{digits[1:] or '0'}E{exp}"
