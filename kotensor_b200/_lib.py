"""ctypes binding of libkt_cuda.so (the C ABI declared in include/kt_cuda.h).

The library is built in-tree by ``kotensor_b200.build_ext``.  Loading fails
loudly when it is missing: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkt_cuda.so")

KT_OK = 0
KT_ERR_INVALID_ARGUMENT = 1
KT_ERR_NAN = 2
KT_ERR_CUDA = 3
KT_ERR_OUT_OF_MEMORY = 4
KT_ERR_UNSUPPORTED = 5
KT_ERR_NCCL = 6
KT_ERR_IO = 7

KT_PATH_GEMV, KT_PATH_GENERIC, KT_PATH_TENSOR_CORE, KT_PATH_GEMV_MMA = 0, 1, 2, 3


class KtError(RuntimeError):
    """A failure inside the CUDA library (the reference's IllegalStateException)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[kt status {status}] {message}")
        self.status = status


class KtStEntryInfo(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_char * 8), ("rank", ctypes.c_int32), ("shape", ctypes.c_int64 * 8),
        ("offset", ctypes.c_int64), ("bytes", ctypes.c_int64),
    ]


class KtStTensor(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p), ("dtype", ctypes.c_char_p), ("rank", ctypes.c_int32),
        ("shape", ctypes.POINTER(ctypes.c_int64)), ("data", ctypes.c_void_p), ("bytes", ctypes.c_int64),
        ("on_device", ctypes.c_int32),
    ]


class KtInfo(ctypes.Structure):
    _fields_ = [
        ("bits", ctypes.c_int32), ("group_size", ctypes.c_int32), ("rows", ctypes.c_int32),
        ("columns", ctypes.c_int32), ("groups", ctypes.c_int32), ("bytes_per_row", ctypes.c_int32),
        ("stored_columns", ctypes.c_int32), ("size_in_bytes", ctypes.c_int64),
        ("qdata", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("zeros", ctypes.c_void_p),
    ]


# name -> (argtypes, restype); the single source of the Python-side signatures.
P, I32, I64, F32, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
PP = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES: dict[str, tuple[list, object]] = {
    "kt_version": ([], I32),
    "kt_last_error": ([], ctypes.c_char_p),
    "kt_check_quantization": ([I32, I32], I32),
    "kt_init": ([I32, PP], I32),
    "kt_destroy": ([P], I32),
    "kt_ctx_stream": ([P, PP], I32),
    "kt_alloc": ([P, SZ, PP], I32),
    "kt_free": ([P, P], I32),
    "kt_memcpy_h2d": ([P, P, P, SZ, P], I32),
    "kt_memcpy_d2h": ([P, P, P, SZ, P], I32),
    "kt_stream_sync": ([P, P], I32),
    "kt_qweight_upload": ([P, I32, I32, I32, I32, P, P, P, PP], I32),
    "kt_qweight_from_device": ([P, I32, I32, I32, I32, P, P, P, P, PP], I32),
    "kt_quantize": ([P, I32, I32, I32, I32, P, P, PP], I32),
    "kt_qweight_info_get": ([P, ctypes.POINTER(KtInfo)], I32),
    "kt_qweight_download": ([P, P, P, P], I32),
    "kt_qweight_free": ([P], I32),
    "kt_dequantize": ([P, P, P, P], I32),
    "kt_dequantize_rows": ([P, P, P, I32, P, P, P], I32),
    "kt_qmatmul": ([P, P, P, P, I32, I32, F32, P, P], I32),
    "kt_qmatmul_noalloc": ([P, P, P, P, I32, I32, F32, P, P], I32),
    "kt_qmatmul_host": ([P, P, P, P, I32, I32, F32, P], I32),
    "kt_qmatmul_path": ([P, I32, ctypes.POINTER(I32)], I32),
    "kt_set_gemv_tuning": ([I32, I32], I32),
    "kt_set_gemv_mma_tuning": ([I32], I32),
    "kt_ctx_take_error": ([P, ctypes.POINTER(I32)], I32),
    "kt_qmatmul_t": ([P, P, P, P, I32, I32, P], I32),
    "kt_shard_bounds": ([I32, I32, I32, I32, I32, ctypes.POINTER(I32), ctypes.POINTER(I32)], I32),
    "kt_qweight_shard": ([P, P, I32, I32, I32, P, PP], I32),
    "kt_qweight_concat_columns": ([P, PP, I32, P, PP], I32),
    "kt_comm_unique_id": ([P], I32),
    "kt_comm_init": ([P, I32, I32, P, PP], I32),
    "kt_comm_destroy": ([P], I32),
    "kt_comm_init_detached": ([P, I32, I32, PP], I32),
    "kt_qmatmul_t_path": ([P, I32, ctypes.POINTER(I32)], I32),
    "kt_qmatmul_row_parallel": ([P, P, P, P, P, I32, I32, F32, P, P], I32),
    "kt_allgather_columns": ([P, P, P, I32, I32, P], I32),
    "kt_argmax_column_parallel": ([P, P, I32, I32, I32, P, P], I32),
    "kt_comm_exchange_ready": ([P, ctypes.POINTER(I32)], I32),
    "kt_comm_set_wait_limit": ([P, ctypes.c_double], I32),
    "kt_comm_exchange_reset": ([P, P], I32),
    "kt_rmsnorm": ([P, P, P, P, I32, I32, F32, P], I32),
    "kt_add_rmsnorm": ([P, P, P, P, P, I32, I32, F32, P], I32),
    "kt_rope_kv": ([P, P, I32, I32, I32, I32, P, P, P, I32, I32, P, P], I32),
    "kt_attention_scratch_floats": ([I32, I32, I32, I32], SZ),
    "kt_silu_mul_rows": ([P, P, P, I32, I32, P], I32),
    "kt_rope": ([P, P, I32, I32, I32, P, P, P], I32),
    "kt_kv_store": ([P, P, P, P, P, I32, I32, I32, I32, I32, P, P], I32),
    "kt_attention_decode": ([P, P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, F32, P, P], I32),
    "kt_attention_seqs": ([P, P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, F32, P, I32, I64, P], I32),
    "kt_rope_kv_seqs": ([P, P, I32, I32, I32, I32, P, P, P, I32, I32, P, I32, I64, P], I32),
    "kt_qmatmul_swiglu": ([P, P, P, P, P, I32, F32, P, P], I32),
    "kt_rmsnorm_qmatmul": ([P, P, P, P, F32, P, P, I32, I32, P, P], I32),
    "kt_rmsnorm_qmatmul_swiglu": ([P, P, P, P, F32, P, P, P, I32, P, P], I32),
    "kt_attention_rope_decode": ([P, P, I32, I32, I32, I32, I32, P, P, P, P, P, I32, I32, F32, P, I64, P], I32),
    "kt_silu_mul": ([P, P, P, I64, P], I32),
    "kt_add": ([P, P, P, I64, P], I32),
    "kt_argmax": ([P, P, I32, I32, P, P], I32),
    "kt_dequantize_column": ([P, P, P, I32, P, P, P], I32),
    "kt_increment": ([P, P, I32, P], I32),
    "kt_qweight_slice": ([P, P, I32, I32, I32, P, PP], I32),
    "kt_lora_project": ([P, P, I32, I32, P, I32, P, P], I32),
    "kt_lora_qmatmul": ([P, P, P, P, I32, I32, F32, P, P, P, I32, F32, P, P], I32),
    "kt_lora_backward": ([P, P, P, P, P, P, P, I32, F32, I32, P, I32, P, P, P], I32),
    "kt_gather_rows": ([P, P, P, I32, I32, P, P], I32),
    "kt_fused_cross_entropy": ([P, P, P, P, I32, P, I32, P, P, P, P], I32),
    "kt_st_open": ([ctypes.c_char_p, PP], I32),
    "kt_st_close": ([P], I32),
    "kt_st_tensor_count": ([P], I32),
    "kt_st_tensor_name": ([P, I32], ctypes.c_char_p),
    "kt_st_entry": ([P, ctypes.c_char_p, ctypes.POINTER(KtStEntryInfo)], I32),
    "kt_st_metadata_count": ([P], I32),
    "kt_st_metadata_at": ([P, I32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p)], I32),
    "kt_st_read_raw": ([P, ctypes.c_char_p, P, I64], I32),
    "kt_st_read_raw_device": ([P, P, ctypes.c_char_p, P, I64, P], I32),
    "kt_st_read_f32_device": ([P, P, ctypes.c_char_p, P, I64, P], I32),
    "kt_qweight_load": ([P, P, ctypes.c_char_p, I32, I32, I32, I32, P, PP], I32),
    "kt_st_write": ([P, ctypes.c_char_p, ctypes.POINTER(KtStTensor), I32, ctypes.POINTER(ctypes.c_char_p),
                     ctypes.POINTER(ctypes.c_char_p), I32, P], I32),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Loads libkt_cuda.so; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: build it with `python -m kotensor_b200.build_ext`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = lib
    return _lib


def check(status: int) -> None:
    """Maps a kt_status to the reference's exception convention."""
    if status == KT_OK:
        return
    msg = load().kt_last_error().decode(errors="replace")
    if status in (KT_ERR_INVALID_ARGUMENT, KT_ERR_NAN):
        raise ValueError(msg)  # IllegalArgumentException
    if status == KT_ERR_IO:
        raise OSError(msg)  # IOException
    raise KtError(status, msg)  # IllegalStateException
