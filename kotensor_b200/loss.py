"""fusedCrossEntropyLoss with a quantized head, on the GPU (kt_fused_cross_entropy).

Reference: Engine/kotensor/src/main/kotlin/Loss.kt:114-220 (IGNORE_INDEX = -100,
Loss.kt:6).  Returns the mean loss as a one-element CUDA tensor; with
``hidden_grad`` / ``bias_grad`` given, accumulates the gradients the reference's
backward adds for an upstream gradient of 1 (rows with ignored targets get none).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np

from . import _lib
from .quantized import QuantizedLinear, _require_f32_device, _stream_of

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None

IGNORE_INDEX = -100


def fused_cross_entropy_loss(hidden, head: QuantizedLinear, targets: Sequence[int], ignore_index: int = IGNORE_INDEX,
                             hidden_grad=None, bias_grad=None):
    hidden = hidden.contiguous()
    _require_f32_device("hidden", hidden)
    t = np.ascontiguousarray(np.asarray(targets, dtype=np.int32).reshape(-1))
    if t.size == 0:
        raise ValueError("targets cannot be empty")
    if hidden.numel() != t.size * head.in_size:
        raise ValueError(f"hidden has {hidden.numel()} elements, expected {t.size} × {head.in_size}")
    for name, g, n in (("hidden_grad", hidden_grad, hidden.numel()), ("bias_grad", bias_grad, head.out_size)):
        if g is not None:
            _require_f32_device(name, g)
            if g.numel() != n or not g.is_contiguous():
                raise ValueError(f"{name} must be a contiguous tensor of {n} floats")
    loss = torch.empty(1, dtype=torch.float32, device=hidden.device)
    w = head.weight

    def ptr(x: Optional["torch.Tensor"]):
        return ctypes.c_void_p(x.data_ptr()) if x is not None else None

    _lib.check(_lib.load().kt_fused_cross_entropy(w._ctx.handle, w.handle, ptr(head.bias), ptr(hidden), t.size,
                                                  t.ctypes.data_as(ctypes.c_void_p), int(ignore_index), ptr(loss),
                                                  ptr(hidden_grad), ptr(bias_grad), _stream_of(hidden)))
    return loss
