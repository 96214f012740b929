"""Host-side mirror of Kotensor's quantized-weight and MatMul operator surface,
running on the B200 through the C ABI (include/kt_cuda.h).

Reference (paths inside the Kotensor project, Engine/kotensor/):
  Quantization                       src/main/kotlin/QuantizedTensor.kt:10-25
  QuantizedTensor                    src/main/kotlin/QuantizedTensor.kt:27-326
  MatMul.multiplyQuantized           src/main/kotlin/MatMul.kt:460-486
  MatMul.multiplyByQuantizedTransposed src/main/kotlin/MatMul.kt:954-981
  QuantizedLinear                    src/main/kotlin/QuantizedLinear.kt:3-46
  Tensor.matmulDequant(Into)         src/main/kotlin/Tensor.kt:162-188

Names follow the reference (snake_case), argument meaning and error behaviour
are the same: a failed ``require`` raises ValueError (the reference's
IllegalArgumentException), a device failure raises KtError
(IllegalStateException), ``m == 0`` is a no-op.

Tensors: device arguments are CUDA ``torch.Tensor`` s (torch supplies device
memory and the current stream only; every computation is a kernel of
libkt_cuda.so).  ``MatMul`` also accepts numpy host arrays, which take the
C ABI's host-buffer entry point (the literal FloatArray signature).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np

from . import _lib

try:  # torch is the device-memory plumbing for the device entry points
    import torch
except ImportError:  # pragma: no cover - the package needs torch for device tensors
    torch = None


# ---------------------------------------------------------------- context

class Context:
    """One kt_ctx per CUDA device (the reference's MatMul singleton holds its
    thread pool the same way, MatMul.kt:30-57)."""

    _by_device: dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        self.device = device
        self.handle = ctypes.c_void_p()
        _lib.check(_lib.load().kt_init(device, ctypes.byref(self.handle)))

    @classmethod
    def get(cls, device: Optional[int] = None) -> "Context":
        if device is None:
            device = torch.cuda.current_device() if torch is not None and torch.cuda.is_available() else 0
        ctx = cls._by_device.get(device)
        if ctx is None:
            ctx = cls._by_device[device] = Context(device)
        return ctx

    def take_error(self) -> int:
        """Reads and clears the device error word (non-zero: a bounded wait in a
        kernel timed out and that call's output is invalid)."""
        out = ctypes.c_int32()
        _lib.check(_lib.load().kt_ctx_take_error(self.handle, ctypes.byref(out)))
        return out.value

    def close(self) -> None:
        if self.handle:
            _lib.load().kt_destroy(self.handle)
            self.handle = ctypes.c_void_p()
            Context._by_device.pop(self.device, None)


def _stream_of(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _is_device(t) -> bool:
    return torch is not None and isinstance(t, torch.Tensor) and t.is_cuda


def _require_f32_device(name: str, t) -> None:
    if not _is_device(t):
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous float32 tensor")


# ---------------------------------------------------------------- Quantization

class Quantization:
    """Quantization(bits, group_size=64), QuantizedTensor.kt:10-25.  The checks
    are the reference's two require(...) calls (the C ABI repeats them in
    kt_check_quantization)."""

    INT8: "Quantization"
    INT4: "Quantization"

    def __init__(self, bits: int, group_size: int = 64):
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        if group_size <= 0:
            raise ValueError("groupSize must be positive")
        self.bits = int(bits)
        self.group_size = int(group_size)

    def __repr__(self) -> str:
        return f"int{self.bits}/g{self.group_size}"

    def __eq__(self, other) -> bool:
        return isinstance(other, Quantization) and (self.bits, self.group_size) == (other.bits, other.group_size)

    def __hash__(self) -> int:
        return hash((self.bits, self.group_size))


Quantization.INT8 = Quantization(8)
Quantization.INT4 = Quantization(4)


# ---------------------------------------------------------------- QuantizedTensor

class QuantizedTensor:
    """Device-resident twin of the reference QuantizedTensor (QuantizedTensor.kt:27-326).

    Byte layout in HBM equals the reference's: qdata [rows x bytesPerRow]
    (INT4 split-half nibbles), scales fp32 [groups x columns], zeros u8
    [groups x columns] for INT4.
    """

    def __init__(self, handle: ctypes.c_void_p, ctx: Context):
        self._handle = handle
        self._ctx = ctx
        info = _lib.KtInfo()
        _lib.check(_lib.load().kt_qweight_info_get(handle, ctypes.byref(info)))
        self._info = info
        self._rows, self._columns = int(info.rows), int(info.columns)

    # -- construction
    @staticmethod
    def from_arrays(qdata: np.ndarray, scales: np.ndarray, zeros: Optional[np.ndarray], shape: Sequence[int],
                    bits: int, group_size: int, device: Optional[int] = None) -> "QuantizedTensor":
        """QuantizedTensor(qdata, scales, zeros, shape, bits, groupSize) (QuantizedTensor.kt:36-70)
        from host arrays in the reference layout; validated like the reference constructor."""
        if len(shape) != 2 or shape[0] <= 0 or shape[1] <= 0:
            raise ValueError(f"QuantizedTensor needs a 2-D shape, got {list(shape)}")
        rows, columns = int(shape[0]), int(shape[1])
        Quantization(bits, group_size)
        groups = (rows + group_size - 1) // group_size
        bpr = (columns + columns % 2) // 2 if bits == 4 else columns
        qdata = np.ascontiguousarray(qdata).view(np.uint8).reshape(-1)
        scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        if qdata.size != rows * bpr:
            raise ValueError(f"qdata has {qdata.size} bytes, expected {rows * bpr}")
        if scales.size != groups * columns:
            raise ValueError(f"scales has {scales.size} entries, expected {groups * columns}")
        if zeros is not None:
            zeros = np.ascontiguousarray(zeros).view(np.uint8).reshape(-1)
            if zeros.size != groups * columns:
                raise ValueError(f"zeros has {zeros.size} entries, expected {groups * columns}")
        if bits == 4 and zeros is None:
            raise ValueError("4-bit tensors need zero points")
        ctx = Context.get(device)
        h = ctypes.c_void_p()
        zp = zeros.ctypes.data_as(ctypes.c_void_p) if zeros is not None and bits == 4 else None
        _lib.check(_lib.load().kt_qweight_upload(ctx.handle, bits, group_size, rows, columns,
                                                 qdata.ctypes.data_as(ctypes.c_void_p),
                                                 scales.ctypes.data_as(ctypes.c_void_p), zp, ctypes.byref(h)))
        return QuantizedTensor(h, ctx)

    @staticmethod
    def quantize(data, quantization: Quantization, rows: Optional[int] = None,
                 columns: Optional[int] = None) -> "QuantizedTensor":
        """QuantizedTensor.quantize(data, rows, columns, quantization) (QuantizedTensor.kt:256-278),
        run by the device quantize/pack kernel.  ``data`` is a CUDA float32 tensor
        [rows, columns] (or flat with rows/columns given) or a host array, which
        is first copied to the device."""
        if not _is_device(data):
            arr = np.ascontiguousarray(data, dtype=np.float32)
            if arr.ndim == 2 and rows is None:
                rows, columns = arr.shape
            data = torch.from_numpy(arr.reshape(-1)).cuda()
        if rows is None:
            if data.dim() != 2:
                raise ValueError(f"Only 2-D tensors can be quantized, got {list(data.shape)}")
            rows, columns = data.shape
        if data.numel() != rows * columns:
            raise ValueError(f"data has {data.numel()} elements, expected {rows} × {columns}")
        data = data.contiguous()
        if data.dtype != torch.float32:
            raise ValueError("data must be float32")
        ctx = Context.get(data.device.index)
        h = ctypes.c_void_p()
        _lib.check(_lib.load().kt_quantize(ctx.handle, quantization.bits, quantization.group_size, int(rows),
                                           int(columns), ctypes.c_void_p(data.data_ptr()), _stream_of(data),
                                           ctypes.byref(h)))
        return QuantizedTensor(h, ctx)

    def close(self) -> None:
        if self._handle:
            _lib.load().kt_qweight_free(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- bookkeeping (QuantizedTensor.kt:45-49, :97-98)
    handle = property(lambda self: self._handle)
    bits = property(lambda self: self._info.bits)
    group_size = property(lambda self: self._info.group_size)
    rows = property(lambda self: self._rows)
    columns = property(lambda self: self._columns)
    groups = property(lambda self: self._info.groups)
    stored_columns = property(lambda self: self._info.stored_columns)
    bytes_per_row = property(lambda self: self._info.bytes_per_row)
    size_in_bytes = property(lambda self: self._info.size_in_bytes)
    shape = property(lambda self: (self.rows, self.columns))

    @property
    def device(self) -> int:
        return self._ctx.device

    # -- host copies in the reference layout
    def download(self) -> tuple[np.ndarray, np.ndarray, Optional[np.ndarray]]:
        q = np.empty(self.rows * self.bytes_per_row, np.uint8)
        s = np.empty(self.groups * self.columns, np.float32)
        z = np.empty(self.groups * self.columns, np.uint8) if self.bits == 4 else None
        _lib.check(_lib.load().kt_qweight_download(self._handle, q.ctypes.data_as(ctypes.c_void_p),
                                                   s.ctypes.data_as(ctypes.c_void_p),
                                                   z.ctypes.data_as(ctypes.c_void_p) if z is not None else None))
        return q, s, z

    @property
    def qdata(self) -> np.ndarray:
        return self.download()[0]

    @property
    def scales(self) -> np.ndarray:
        return self.download()[1]

    @property
    def zeros(self) -> Optional[np.ndarray]:
        return self.download()[2]

    # -- dequantize (QuantizedTensor.kt:172-249)
    def dequantize(self):
        """dequantize(): a CUDA float32 tensor [rows, columns]."""
        out = torch.empty((self.rows, self.columns), dtype=torch.float32, device=f"cuda:{self.device}")
        _lib.check(_lib.load().kt_dequantize(self._ctx.handle, self._handle, ctypes.c_void_p(out.data_ptr()),
                                             _stream_of(out)))
        return out

    def dequantize_rows(self, rows):
        """dequantizeRow for each index in ``rows`` (an int32 CUDA tensor): [len(rows), columns]."""
        idx = rows.to(device=f"cuda:{self.device}", dtype=torch.int32).contiguous()
        out = torch.empty((idx.numel(), self.columns), dtype=torch.float32, device=idx.device)
        status = torch.zeros(1, dtype=torch.int32, device=idx.device)
        _lib.check(_lib.load().kt_dequantize_rows(self._ctx.handle, self._handle, ctypes.c_void_p(idx.data_ptr()),
                                                  idx.numel(), ctypes.c_void_p(out.data_ptr()),
                                                  ctypes.c_void_p(status.data_ptr()), _stream_of(out)))
        if int(status.item()) != 0:
            raise ValueError(f"row index out of range for {self.rows} rows")
        return out

    def dequantize_columns(self, columns):
        """dequantizeColumn for each index in ``columns`` (QuantizedTensor.kt:235-241;
        an int32 CUDA tensor or a sequence): [len(columns), rows], bit-identical."""
        idx = torch.as_tensor(columns).to(device=f"cuda:{self.device}", dtype=torch.int32).contiguous().reshape(-1)
        out = torch.empty((idx.numel(), self.rows), dtype=torch.float32, device=idx.device)
        if idx.numel() == 0:
            return out
        status = torch.zeros(1, dtype=torch.int32, device=idx.device)
        _lib.check(_lib.load().kt_dequantize_column(self._ctx.handle, self._handle, ctypes.c_void_p(idx.data_ptr()),
                                                    idx.numel(), ctypes.c_void_p(out.data_ptr()),
                                                    ctypes.c_void_p(status.data_ptr()), _stream_of(out)))
        if int(status.item()) != 0:
            raise ValueError(f"column index out of range for {self.columns} columns")
        return out

    def dequantize_column(self, column: int):
        return self.dequantize_columns([column])[0]

    def dequantize_row(self, row: int):
        import torch as _t
        return self.dequantize_rows(_t.tensor([row], dtype=_t.int32))[0]

    def matmul_path(self, m: int) -> int:
        """The kernel family kt_qmatmul runs for m rows (kotensor_b200._lib.KT_PATH_*)."""
        out = ctypes.c_int32()
        _lib.check(_lib.load().kt_qmatmul_path(self._handle, int(m), ctypes.byref(out)))
        return out.value

    def transposed_path(self, m: int) -> int:
        """The kernel family kt_qmatmul_t runs for m rows of dy (KT_PATH_TENSOR_CORE or KT_PATH_GENERIC)."""
        out = ctypes.c_int32()
        _lib.check(_lib.load().kt_qmatmul_t_path(self._handle, int(m), ctypes.byref(out)))
        return out.value

    def raw_value(self, row: int, column: int) -> int:
        """rawValue(row, column), QuantizedTensor.kt:172-180."""
        q = self.qdata
        if self.bits == 8:
            return int(q.view(np.int8)[row * self.bytes_per_row + column])
        half = self.bytes_per_row
        byte = int(q[row * half + column % half])
        return byte & 0xF if column < half else (byte >> 4) & 0xF

    def value(self, row: int, column: int) -> float:
        """value(row, column), QuantizedTensor.kt:182-186."""
        return float(self.dequantize_row(row)[column].item())


# ---------------------------------------------------------------- MatMul

class MatMul:
    """MatMul's quantized entry points (MatMul.kt:460-486, :954-981)."""

    @staticmethod
    def multiply_quantized(a, weight: QuantizedTensor, c, m: int, accumulate: bool = True, alpha: float = 1.0,
                           bias=None) -> None:
        """c[m x N] = (accumulate ? c : 0) + alpha * a[m x K] . dequant(W) (+ bias).

        ``a``/``c`` are CUDA float32 tensors (device entry point, torch's current
        stream) or numpy float32 arrays (host entry point, synchronous)."""
        k, n = weight.rows, weight.columns
        if m < 0:
            raise ValueError(f"Negative row count {m}")
        if _numel(a) < m * k:
            raise ValueError(f"a has {_numel(a)} elements, needs {m} × {k}")
        if _numel(c) < m * n:
            raise ValueError(f"c has {_numel(c)} elements, needs {m} × {n}")
        if m == 0:
            return
        L = _lib.load()
        if _is_device(a):
            _require_f32_device("a", a)
            _require_f32_device("c", c)
            if bias is not None:
                _require_f32_device("bias", bias)
            _lib.check(L.kt_qmatmul(weight._ctx.handle, weight.handle, ctypes.c_void_p(a.data_ptr()),
                                    ctypes.c_void_p(c.data_ptr()), m, int(bool(accumulate)), float(alpha),
                                    ctypes.c_void_p(bias.data_ptr()) if bias is not None else None, _stream_of(c)))
            return
        a_h = a if (type(a) is np.ndarray and a.dtype == np.float32 and a.flags.c_contiguous) else \
            np.ascontiguousarray(a, dtype=np.float32)
        if not (isinstance(c, np.ndarray) and c.dtype == np.float32 and c.flags.c_contiguous):
            raise ValueError("c must be a contiguous float32 numpy array")
        b_h = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        st = L.kt_qmatmul_host(weight._ctx.handle, weight.handle, a_h.ctypes.data, c.ctypes.data, m,
                               1 if accumulate else 0, alpha, b_h.ctypes.data if b_h is not None else None)
        if st:
            _lib.check(st)

    @staticmethod
    def multiply_by_quantized_transposed(dy, weight: QuantizedTensor, dx, m: int, accumulate: bool = True) -> None:
        """dx[m x K] = (accumulate ? dx : 0) + dy[m x N] . dequant(W)^T (device tensors)."""
        k, n = weight.rows, weight.columns
        if _numel(dy) < m * n:
            raise ValueError(f"dy has {_numel(dy)} elements, needs {m} × {n}")
        if _numel(dx) < m * k:
            raise ValueError(f"dx has {_numel(dx)} elements, needs {m} × {k}")
        if m <= 0:
            if m < 0:
                raise ValueError(f"Negative row count {m}")
            return
        _require_f32_device("dy", dy)
        _require_f32_device("dx", dx)
        _lib.check(_lib.load().kt_qmatmul_t(weight._ctx.handle, weight.handle, ctypes.c_void_p(dy.data_ptr()),
                                            ctypes.c_void_p(dx.data_ptr()), m, int(bool(accumulate)),
                                            _stream_of(dx)))


def _numel(t) -> int:
    if _is_device(t):
        return t.numel()
    return int(np.asarray(t).size)


# ---------------------------------------------------------------- QuantizedLinear

class QuantizedLinear:
    """QuantizedLinear(inSize, outSize, quantization), QuantizedLinear.kt:3-46:
    forward(x) = x . dequant(W) + bias; forwardInto(x, out) writes into out."""

    def __init__(self, in_size: int, out_size: int, quantization: Quantization, device: Optional[int] = None):
        self.in_size = in_size
        self.out_size = out_size
        self.quantization = quantization
        dev = Context.get(device).device
        self._weight: Optional[QuantizedTensor] = None
        self.bias = torch.zeros((1, out_size), dtype=torch.float32, device=f"cuda:{dev}")

    @property
    def weight(self) -> QuantizedTensor:
        if self._weight is None:
            raise ValueError("weight is not set")
        return self._weight

    @weight.setter
    def weight(self, value: QuantizedTensor) -> None:
        if value.rows != self.in_size or value.columns != self.out_size:
            raise ValueError(f"Quantized weight is {value.rows} × {value.columns}, layer is "
                             f"{self.in_size} × {self.out_size}")
        self._weight = value

    def forward(self, x):
        if x.dim() != 2 or x.shape[1] != self.in_size:
            raise ValueError(f"{x.shape[1] if x.dim() == 2 else x.shape} != {self.in_size}")
        out = torch.empty((x.shape[0], self.out_size), dtype=torch.float32, device=x.device)
        return self.forward_into(x, out)

    def forward_into(self, x, out):
        m = x.shape[0]
        if tuple(out.shape) != (m, self.out_size):
            raise ValueError(f"out shape {list(out.shape)} != [{m}, {self.out_size}]")
        MatMul.multiply_quantized(x.contiguous(), self.weight, out, m, accumulate=False, alpha=1.0, bias=self.bias)
        return out

    __call__ = forward

    @property
    def size_in_bytes(self) -> int:
        return self.weight.size_in_bytes + self.out_size * 4

    @staticmethod
    def from_linear(weight, bias, quantization: Quantization) -> "QuantizedLinear":
        """QuantizedLinear.fromLinear: quantizes an fp32 [in, out] weight on the device."""
        in_size, out_size = weight.shape
        layer = QuantizedLinear(in_size, out_size, quantization, device=weight.device.index)
        layer.weight = QuantizedTensor.quantize(weight, quantization)
        if bias is not None:
            layer.bias.copy_(bias.reshape(1, out_size))
        return layer
