"""Tensor parallelism for the quantized matmul: one process per GPU, weights
sharded per layer, an NCCL all-reduce where the product has a real exchange.

The reference runs on one host and has no counterpart; the layout of a shard
is the reference's own (QuantizedTensor.kt:27-98) for the shard's shape.

  row-parallel    (split K at whole groups; attention out, FFN down):
                  c = (acc ? c : 0) + alpha * sum_r a[:, K_r] . dequant(W_r) + bias
  column-parallel (split N; q/k/v, gate/up, lm head): each rank owns its
                  columns; ``allgather_columns`` assembles [m x N] when needed.

Quantization is per (row group, column), so a shard is bit-for-bit the
quantization of the same block of the fp32 weight (``shard_host`` restates the
device kernel on host arrays, e.g. for loading shards from files).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from .quantized import Context, QuantizedTensor, _require_f32_device, _stream_of, torch

ROWS, COLUMNS = 0, 1


def shard_bounds(axis: int, extent: int, group_size: int, parts: int, index: int) -> tuple[int, int]:
    """[begin, end) of shard ``index`` of ``parts`` along rows (whole groups) or
    columns (kt_shard_bounds; host only)."""
    b, e = ctypes.c_int32(), ctypes.c_int32()
    _lib.check(_lib.load().kt_shard_bounds(axis, extent, group_size, parts, index, ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


def _int4_columns(qdata: np.ndarray, rows: int, columns: int) -> np.ndarray:
    """Unpacked nibbles [rows x columns] of an INT4 split-half packed qdata."""
    half = (columns + 1) // 2
    q = qdata.reshape(rows, half)
    out = np.empty((rows, columns), np.uint8)
    out[:, :half] = q & 15
    out[:, half:] = q[:, : columns - half] >> 4
    return out


def _pack_int4(nib: np.ndarray) -> np.ndarray:
    """Split-half packing (QuantizedTensor.kt:172-180) of nibbles [rows x columns]."""
    rows, columns = nib.shape
    half = (columns + 1) // 2
    packed = nib[:, :half].astype(np.uint8).copy()
    packed[:, : columns - half] |= (nib[:, half:].astype(np.uint8) << 4)
    return packed


def shard_host(qdata: np.ndarray, scales: np.ndarray, zeros: Optional[np.ndarray], shape, bits: int,
               group_size: int, axis: int, parts: int, index: int):
    """Shard of host arrays in the reference layout: (qdata, scales, zeros, shape)."""
    rows, columns = int(shape[0]), int(shape[1])
    groups = (rows + group_size - 1) // group_size
    extent = rows if axis == ROWS else columns
    b, e = shard_bounds(axis, extent, group_size, parts, index)
    bpr = (columns + 1) // 2 if bits == 4 else columns
    q = np.ascontiguousarray(qdata).view(np.uint8).reshape(rows, bpr)
    s = np.ascontiguousarray(scales, dtype=np.float32).reshape(groups, columns)
    z = None if zeros is None else np.ascontiguousarray(zeros).view(np.uint8).reshape(groups, columns)
    if axis == ROWS:
        g0, g1 = b // group_size, (e + group_size - 1) // group_size
        return (q[b:e].copy(), s[g0:g1].copy(), None if z is None else z[g0:g1].copy(), (e - b, columns))
    if bits == 8:
        qs = q[:, b:e].copy()
    else:
        qs = _pack_int4(_int4_columns(q, rows, columns)[:, b:e])
    return (qs, s[:, b:e].copy(), None if z is None else z[:, b:e].copy(), (rows, e - b))


def shard(qt: QuantizedTensor, axis: int, parts: int, index: int) -> QuantizedTensor:
    """Device shard of a device weight (kt_qweight_shard), built on torch's current stream."""
    import torch
    h = ctypes.c_void_p()
    stream = ctypes.c_void_p(torch.cuda.current_stream(qt.device).cuda_stream)
    _lib.check(_lib.load().kt_qweight_shard(qt._ctx.handle, qt.handle, axis, parts, index, stream, ctypes.byref(h)))
    return QuantizedTensor(h, qt._ctx)


def slice_weight(qt: QuantizedTensor, axis: int, begin: int, end: int) -> QuantizedTensor:
    """Device weight of rows (axis 0, group-aligned) or columns (axis 1) [begin, end)
    of ``qt`` (kt_qweight_slice), built on torch's current stream."""
    import torch
    h = ctypes.c_void_p()
    stream = ctypes.c_void_p(torch.cuda.current_stream(qt.device).cuda_stream)
    _lib.check(_lib.load().kt_qweight_slice(qt._ctx.handle, qt.handle, axis, int(begin), int(end), stream,
                                            ctypes.byref(h)))
    return QuantizedTensor(h, qt._ctx)


def concat_columns(weights: list) -> QuantizedTensor:
    """One weight whose columns are those of ``weights`` side by side
    (kt_qweight_concat_columns; e.g. q|k|v or gate|up fused into one matmul)."""
    import torch
    arr = (ctypes.c_void_p * len(weights))(*[w.handle.value for w in weights])
    h = ctypes.c_void_p()
    stream = ctypes.c_void_p(torch.cuda.current_stream(weights[0].device).cuda_stream)
    _lib.check(_lib.load().kt_qweight_concat_columns(weights[0]._ctx.handle, arr, len(weights), stream, ctypes.byref(h)))
    return QuantizedTensor(h, weights[0]._ctx)


class Comm:
    """One NCCL communicator per rank (kt_comm_init)."""

    ID_BYTES = 128

    def __init__(self, world: int, rank: int, unique_id: bytes, ctx: Optional[Context] = None):
        if len(unique_id) != self.ID_BYTES:
            raise ValueError(f"unique id must be {self.ID_BYTES} bytes")
        self.world, self.rank = world, rank
        self._ctx = ctx or Context.get()
        buf = ctypes.create_string_buffer(unique_id, self.ID_BYTES)
        h = ctypes.c_void_p()
        _lib.check(_lib.load().kt_comm_init(self._ctx.handle, world, rank, buf, ctypes.byref(h)))
        self._handle = h

    @classmethod
    def detached(cls, world: int, rank: int, ctx: Optional[Context] = None) -> "Comm":
        """A communicator of `world` ranks of which only `rank` exists
        (kt_comm_init_detached): every exchange area lives on this GPU, the
        other ranks never arrive, so a fused m = 1 row-parallel call runs into
        its wait limit and reports the timeout in the context's error word.
        Calls that need NCCL raise.  For testing the failure path on one GPU."""
        self = cls.__new__(cls)
        self.world, self.rank = world, rank
        self._ctx = ctx or Context.get()
        h = ctypes.c_void_p()
        _lib.check(_lib.load().kt_comm_init_detached(self._ctx.handle, world, rank, ctypes.byref(h)))
        self._handle = h
        return self

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(Comm.ID_BYTES)
        _lib.check(_lib.load().kt_comm_unique_id(buf))
        return buf.raw

    @classmethod
    def from_process_group(cls, group=None, ctx: Optional[Context] = None) -> "Comm":
        """Rank 0 of a torch.distributed group makes the id, every rank joins."""
        import torch.distributed as dist
        obj = [cls.unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        return cls(dist.get_world_size(group), dist.get_rank(group), obj[0], ctx)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def exchange_ready(self) -> bool:
        """True once the peer-memory exchange of the fused m = 1 row-parallel
        GEMV is set up and agreed by every rank."""
        out = ctypes.c_int32()
        _lib.check(_lib.load().kt_comm_exchange_ready(self.handle, ctypes.byref(out)))
        return bool(out.value)

    def set_wait_limit(self, seconds: float) -> None:
        """Limit of a fused row-parallel call's wait for the other ranks (default 2 s)."""
        _lib.check(_lib.load().kt_comm_set_wait_limit(self.handle, float(seconds)))

    def reset_exchange(self) -> None:
        """Collective: clears every rank's exchange area after a fused call
        failed (kt_comm_exchange_reset), on torch's current stream."""
        import torch
        stream = ctypes.c_void_p(torch.cuda.current_stream(self._ctx.device).cuda_stream)
        _lib.check(_lib.load().kt_comm_exchange_reset(self.handle, stream))

    def close(self) -> None:
        if self._handle:
            _lib.load().kt_comm_destroy(self._handle)
            self._handle = ctypes.c_void_p()


def matmul_row_parallel(comm: Comm, a_shard, w_shard: QuantizedTensor, c, m: int, accumulate: bool = False,
                        alpha: float = 1.0, bias=None) -> None:
    """c[m x N] = (accumulate ? c : 0) + alpha * sum over ranks of a_shard . dequant(w_shard) + bias."""
    if m < 0:
        raise ValueError(f"Negative row count {m}")
    if m == 0:
        return
    _require_f32_device("a_shard", a_shard)
    _require_f32_device("c", c)
    if a_shard.numel() < m * w_shard.rows or c.numel() < m * w_shard.columns:
        raise ValueError("a_shard / c too small for the shard")
    if bias is not None:
        _require_f32_device("bias", bias)
    _lib.check(_lib.load().kt_qmatmul_row_parallel(
        w_shard._ctx.handle, comm.handle, w_shard.handle, ctypes.c_void_p(a_shard.data_ptr()),
        ctypes.c_void_p(c.data_ptr()), m, int(bool(accumulate)), float(alpha),
        ctypes.c_void_p(bias.data_ptr()) if bias is not None else None, _stream_of(c)))


def allgather_columns(comm: Comm, y_shard, y_full, m: int) -> None:
    """y_full[m x P*ns] <- every rank's y_shard[m x ns] in rank order."""
    _require_f32_device("y_shard", y_shard)
    _require_f32_device("y_full", y_full)
    ns = y_shard.numel() // m
    if y_full.numel() < m * ns * comm.world:
        raise ValueError("y_full too small")
    _lib.check(_lib.load().kt_allgather_columns(comm.handle, ctypes.c_void_p(y_shard.data_ptr()),
                                                ctypes.c_void_p(y_full.data_ptr()), m, ns, _stream_of(y_full)))


def argmax_column_parallel(comm: Comm, logits_shard, col_begin: int, out) -> None:
    """Greedy token per row over an lm head split along N (argmaxOfLastToken,
    Transformer.kt:255-266, across shards): ``logits_shard`` [rows x n_shard]
    holds global columns [col_begin, col_begin + n_shard); ``out`` (int32,
    [rows], on the device) receives on every rank the column of the largest
    logit above -1e9 over all ranks, the lowest one among equal logits, 0 if
    none -- the single-GPU argmax of the whole row."""
    _require_f32_device("logits_shard", logits_shard)
    if out.dtype != torch.int32 or not out.is_cuda or not out.is_contiguous():
        raise ValueError("out must be a contiguous int32 CUDA tensor")
    rows, n_shard = logits_shard.shape
    if out.numel() < rows:
        raise ValueError("out too small")
    _lib.check(_lib.load().kt_argmax_column_parallel(comm.handle, ctypes.c_void_p(logits_shard.data_ptr()), rows,
                                                     n_shard, int(col_begin), ctypes.c_void_p(out.data_ptr()),
                                                     _stream_of(out)))


class RowParallelQuantizedLinear:
    """QuantizedLinear (QuantizedLinear.kt:18-25) with its weight split along K:
    ``forward_into(x_shard, out)`` takes this rank's K-columns of x."""

    def __init__(self, weight: QuantizedTensor, comm: Comm, bias=None):
        self.comm = comm
        self.k_begin, self.k_end = shard_bounds(ROWS, weight.rows, weight.group_size, comm.world, comm.rank)
        self.weight = shard(weight, ROWS, comm.world, comm.rank)
        self.bias = bias

    def forward_into(self, x_shard, out):
        m = x_shard.shape[0]
        matmul_row_parallel(self.comm, x_shard.contiguous(), self.weight, out, m, accumulate=False, bias=self.bias)
        return out


class ColumnParallelQuantizedLinear:
    """QuantizedLinear with its weight split along N: ``forward_into`` writes this
    rank's columns; ``gather_into`` assembles all columns on every rank."""

    def __init__(self, weight: QuantizedTensor, comm: Comm, bias=None):
        from .quantized import MatMul  # noqa: F401  (same entry point as QuantizedLinear)
        self.comm = comm
        self.n_begin, self.n_end = shard_bounds(COLUMNS, weight.columns, weight.group_size, comm.world, comm.rank)
        self.weight = shard(weight, COLUMNS, comm.world, comm.rank)
        self.bias = None if bias is None else bias[self.n_begin:self.n_end].contiguous()

    def forward_into(self, x, out_shard):
        from .quantized import MatMul
        m = x.shape[0]
        MatMul.multiply_quantized(x, self.weight, out_shard, m, accumulate=False, bias=self.bias)
        return out_shard

    def gather_into(self, out_shard, out_full):
        allgather_columns(self.comm, out_shard, out_full, out_shard.shape[0])
        return out_full

    def argmax_into(self, out_shard, tokens):
        """Greedy decoding when this layer is the lm head: the winning global
        column per row of the sharded logits ``out_shard``, on every rank."""
        argmax_column_parallel(self.comm, out_shard, self.n_begin, tokens)
        return tokens
