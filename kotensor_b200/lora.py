"""LoRA adapters on top of the quantized linear layer (QLoRA), on the GPU.

Reference (paths inside the Kotensor project, Engine/kotensor/src/main/kotlin/):
  LoRALinear(baseLinear, rank, alpha)    LoRA.kt:7-57
  LoRAAdapter.saveDelta / loadDelta      LoRA.kt:121-150

``forward_into`` is LoRALinear.forwardInto: the quantized matmul with the
low-rank term ``scaling * (x . A) . B`` added in the matmul's own epilogue
(kt_lora_qmatmul).  ``backward`` gives the gradients the reference's autograd
produces for LoRALinear.forward (kt_lora_backward): dx through the frozen
quantized weight and the adapter, and the adapter's grad_a / grad_b
(accumulated, like Tensor.grad).  The base weight and bias are frozen.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

from . import _lib
from .quantized import QuantizedLinear, _require_f32_device, _stream_of

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


def _p(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


class LoRALinear:
    """LoRALinear over a QuantizedLinear base (LoRA.kt:7-57)."""

    def __init__(self, base: QuantizedLinear, rank: int = 4, alpha: float = 1.0,
                 generator: Optional["torch.Generator"] = None):
        if not 1 <= rank <= 256:
            raise ValueError(f"LoRA rank must be in 1..256, got {rank}")
        self.base_linear = base
        self.rank = rank
        self.alpha = float(alpha)
        self.scaling = float(torch.tensor(alpha, dtype=torch.float32) / torch.tensor(float(rank)))
        dev = base.bias.device
        # loraA ~ U(-1, 1) / sqrt(inFeatures), loraB = 0 (LoRA.kt:16-28)
        scale_a = 1.0 / math.sqrt(base.in_size)
        u = torch.rand((base.in_size, rank), generator=generator, dtype=torch.float32, device="cpu")
        self.lora_a = ((u * 2 - 1) * scale_a).to(dev)
        self.lora_b = torch.zeros((rank, base.out_size), dtype=torch.float32, device=dev)
        self.grad_a = torch.zeros_like(self.lora_a)
        self.grad_b = torch.zeros_like(self.lora_b)
        self._projected = None

    @property
    def in_size(self) -> int:
        return self.base_linear.in_size

    @property
    def out_size(self) -> int:
        return self.base_linear.out_size

    def parameters(self) -> list:
        return [self.lora_a, self.lora_b]

    def zero_grad(self) -> None:
        self.grad_a.zero_()
        self.grad_b.zero_()

    def _projected_for(self, m: int):
        if self._projected is None or self._projected.shape[0] < m:
            self._projected = torch.empty((max(m, 1), self.rank), dtype=torch.float32, device=self.lora_a.device)
        return self._projected[:m]

    def forward_into(self, x, out):
        """out = x . deq(W) + bias + scaling * (x . A) . B; keeps x . A for backward."""
        if x.dim() != 2:
            raise ValueError(f"forwardInto takes [tokens, features] rows, got {list(x.shape)}")
        m = x.shape[0]
        x = x.contiguous()
        _require_f32_device("x", x)
        _require_f32_device("out", out)
        if x.shape[1] != self.in_size or tuple(out.shape) != (m, self.out_size):
            raise ValueError(f"x {list(x.shape)} / out {list(out.shape)} do not fit {self.in_size} -> {self.out_size}")
        p = self._projected_for(m)
        w = self.base_linear.weight
        _lib.check(_lib.load().kt_lora_qmatmul(w._ctx.handle, w.handle, _p(x), _p(out), m, 0, 1.0,
                                               _p(self.base_linear.bias), _p(self.lora_a), _p(self.lora_b),
                                               self.rank, self.scaling, _p(p), _stream_of(out)))
        return out

    def forward(self, x):
        out = torch.empty((x.shape[0], self.out_size), dtype=torch.float32, device=x.device)
        return self.forward_into(x, out)

    __call__ = forward

    def backward(self, x, dy, dx=None, accumulate_dx: bool = False):
        """Gradients of the last forward over the same x: grad_a / grad_b accumulate;
        dx (if given) receives dy . deq(W)^T + scaling * (dy . B^T) . A^T."""
        m = x.shape[0]
        x, dy = x.contiguous(), dy.contiguous()
        if tuple(dy.shape) != (m, self.out_size):
            raise ValueError(f"dy shape {list(dy.shape)} != [{m}, {self.out_size}]")
        if dx is not None and tuple(dx.shape) != (m, self.in_size):
            raise ValueError(f"dx shape {list(dx.shape)} != [{m}, {self.in_size}]")
        p = self._projected_for(m)
        w = self.base_linear.weight
        _lib.check(_lib.load().kt_lora_backward(w._ctx.handle, w.handle, _p(x), _p(dy), _p(p), _p(self.lora_a),
                                                _p(self.lora_b), self.rank, self.scaling, m, _p(dx),
                                                int(bool(accumulate_dx)), _p(self.grad_a), _p(self.grad_b),
                                                _stream_of(dy)))
        return dx

    def delta_weights(self):
        """deltaWeights(): loraA . loraB * scaling, [in x out]."""
        return (self.lora_a @ self.lora_b) * self.scaling
