"""CPU restatement of Kotensor's QLoRA pieces.  TEST INFRASTRUCTURE ONLY: the
LoRA and fused-loss parity tests use it as the checker; the product never
imports it.

Follows (paths inside the Kotensor project, Engine/kotensor/src/main/kotlin/):
  LoRALinear.forwardInto                  LoRA.kt:39-46
  LoRALinear.forward and its autograd     LoRA.kt:31-36 (matmul / scale / add nodes of Tensor.kt)
  matmulDequant's backward                Tensor.kt:171-177 -> MatMul.multiplyByQuantizedTransposed
  fusedCrossEntropyLoss (quantized head)  Loss.kt:114-220, projectRows / logitGradients Loss.kt:247-280
The quantized products are the C oracle's (oracle/kt_oracle.c); the dense
low-rank products are float64 numpy, rounded to float32 at the points where the
reference stores a float32 tensor.  Sums over the vocabulary run in float64, so
the results agree with the reference within float32 rounding, not bit for bit.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

IGNORE_INDEX = -100  # Loss.kt:6


def lora_forward(x, w, bias, lora_a, lora_b, scaling):
    """(out, projected): out = x . deq(W) + bias + scaling * (x . A) . B."""
    x = np.asarray(x, np.float32)
    base = O.multiply_quantized(x, w, threads=8) + np.asarray(bias, np.float32).reshape(1, -1)
    projected = (x.astype(np.float64) @ lora_a.astype(np.float64)).astype(np.float32)
    low = (projected.astype(np.float64) @ lora_b.astype(np.float64)) * np.float64(np.float32(scaling))
    return (base.astype(np.float64) + low).astype(np.float32), projected


def lora_backward(x, dy, w, lora_a, lora_b, scaling, projected):
    """(dx, grad_a, grad_b) of LoRALinear.forward for upstream gradient dy."""
    x64, dy64 = np.asarray(x, np.float64), np.asarray(dy, np.float64)
    s = np.float64(np.float32(scaling))
    g = dy64 @ lora_b.astype(np.float64).T                      # dP = dy . B^T
    dx = O.multiply_by_quantized_transposed(np.asarray(dy, np.float32), w, threads=8).astype(np.float64)
    dx += s * (g @ lora_a.astype(np.float64).T)
    grad_a = s * (x64.T @ g)
    grad_b = s * (np.asarray(projected, np.float64).T @ dy64)
    return dx.astype(np.float32), grad_a.astype(np.float32), grad_b.astype(np.float32)


def fused_cross_entropy(hidden, w, bias, targets, ignore_index=IGNORE_INDEX):
    """(loss, hidden_grad, bias_grad) of fusedCrossEntropyLoss with a QuantizedLinear
    head and upstream gradient 1: mean over active rows of max + ln(sum exp) - logit[target];
    hidden_grad rows of ignored targets stay zero."""
    hidden = np.asarray(hidden, np.float32)
    vocab = w.columns
    rows = [i for i, t in enumerate(targets) if t != ignore_index]
    for i in rows:
        if not 0 <= targets[i] < vocab:
            raise ValueError(f"target {targets[i]} out of bounds {vocab}")
    hidden_grad = np.zeros_like(hidden)
    bias_grad = np.zeros(vocab, np.float32)
    if not rows:
        return np.float32(0.0), hidden_grad, bias_grad
    logits = (O.multiply_quantized(hidden[rows], w, threads=8) + np.asarray(bias, np.float32).reshape(1, -1))
    l64 = logits.astype(np.float64)
    mx = np.maximum(l64.max(axis=1), -1e9)
    e = np.exp(l64 - mx[:, None])
    ssum = e.sum(axis=1)
    tgt = np.array([targets[i] for i in rows])
    loss = np.mean(mx + np.log(ssum) - l64[np.arange(len(rows)), tgt])
    scale = 1.0 / len(rows)
    grad = e / ssum[:, None]
    grad[np.arange(len(rows)), tgt] -= 1.0
    grad *= scale
    g32 = grad.astype(np.float32)
    bias_grad = grad.sum(axis=0).astype(np.float32)
    hidden_grad[rows] = O.multiply_by_quantized_transposed(g32, w, threads=8)
    return np.float32(loss), hidden_grad, bias_grad
