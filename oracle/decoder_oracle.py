"""CPU restatement of Kotensor's greedy decode step.  TEST INFRASTRUCTURE ONLY:
the decoder parity tests and bench.py's CPU legs use it as the checker; the
product never imports it.

Follows (paths inside the Kotensor project, Engine/kotensor/src/main/kotlin/):
  Transformer.decode                 Transformer.kt:141-154
  argmaxOfLastToken                  Transformer.kt:255-266
  TransformerBlock.decodeInto        TransformerBlock.kt:40-47
  Attention.decodeInto / attendHead  Attention.kt:207-239, :295-328
  RMSNorm.forwardInto                RMSNorm.kt:71-90
  RoPE invFreq / applyInPlace        RoPE.kt:3-28 (Llama-3 scaling), :39-42, :117-137
  SwiGLU.forwardInto, siluInPlace    SwiGLU.kt:19-25, Tensor.kt:231-237
  QuantizedEmbedding / TiedQuantizedEmbedding lookupInto  Embedding.kt:96-101, :129-135
  KVCache layout                     KVCache.kt:3-59
  Transformer.prefill / prefillLayers Transformer.kt:99-132 (32-row chunks, MatMul.TILE_M)
  Attention.prefillInto / attendCached Attention.kt:241-293
The projections are the C oracle's MatMul.multiplyQuantized (m = 1 schedule)
plus QuantizedLinear's bias (QuantizedLinear.kt:18-25) for quantized weights,
or a float32 product plus Linear's bias (Linear.kt) for float32 weights (the
reference's unquantized model).  Everything else is float32 numpy; summation
orders of the sums (RMSNorm, dot products, softmax) follow numpy, not the
reference's sequential loops, so results agree with the reference within
float32 rounding, not bit for bit.  The float32 mode is pinned to the
reference's own known answers: the logits its test suite holds for three tiny
Hugging Face checkpoints (GQA, q/k/v biases, tied embeddings, Llama-3 RoPE
scaling; HuggingFaceImportTest.kt:29-36, checked there at 2e-4), see
oracle/hf_oracle.py.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import oracle as O


@dataclass
class DecoderConfig:
    vocab: int
    dim: int
    layers: int
    heads: int
    kv_heads: int
    hidden: int
    eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: Optional[tuple] = None  # (factor, low, high, original max positions)
    bits: int = 4
    group_size: int = 64
    tied: bool = False
    qkv_bias: bool = False

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads


def inv_freq(head_dim: int, base: float, scaling: Optional[tuple]) -> np.ndarray:
    """RoPE.invFreq (RoPE.kt:39-42) with RoPEScaling.scale (RoPE.kt:15-27), in float32."""
    half = head_dim // 2
    out = np.empty(half, np.float32)
    for i in range(half):
        raw = np.float32(1.0) / np.float32(math.pow(float(np.float32(base)), float(np.float32(2 * i) / np.float32(head_dim))))
        if scaling is not None:
            factor, low, high, orig = (np.float32(scaling[0]), np.float32(scaling[1]), np.float32(scaling[2]),
                                       int(scaling[3]))
            low_wl = np.float32(orig) / low
            high_wl = np.float32(orig) / high
            wl = np.float32(2.0 * math.pi / float(raw))
            if wl < high_wl:
                raw = raw
            elif wl > low_wl:
                raw = raw / factor
            else:
                smooth = (np.float32(orig) / wl - low) / (high - low)
                raw = (np.float32(1.0) - smooth) * raw / factor + smooth * raw
        out[i] = np.float32(raw)
    return out


@dataclass
class DecoderWeights:
    """Host weights of a model: quantized projections in the reference layout."""
    cfg: DecoderConfig
    embedding: Optional[O.OracleQTensor]           # [vocab x dim]; None when tied to the head
    layers: list = field(default_factory=list)      # per layer: dict of OracleQTensor / float32 arrays
    final_norm: np.ndarray = None
    head: O.OracleQTensor = None                    # [dim x vocab]
    head_bias: np.ndarray = None

    @staticmethod
    def random(cfg: DecoderConfig, seed: int = 1234) -> "DecoderWeights":
        """N(0, 0.02^2) projections quantized with the reference quantizer; RMSNorm
        weights near 1 and small biases so every term is exercised."""
        rng = np.random.default_rng(seed)

        def proj(k, n):
            w = (rng.standard_normal((k, n), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            return O.quantize(w, cfg.bits, cfg.group_size)

        def vec(n, mean=0.0, sd=0.02):
            return (np.float32(mean) + rng.standard_normal(n, dtype=np.float32) * np.float32(sd)).astype(np.float32)

        kv = cfg.kv_heads * cfg.head_dim
        layers = []
        for _ in range(cfg.layers):
            layers.append({
                "norm1": vec(cfg.dim, 1.0, 0.1), "norm2": vec(cfg.dim, 1.0, 0.1),
                "wq": proj(cfg.dim, cfg.dim), "wk": proj(cfg.dim, kv), "wv": proj(cfg.dim, kv),
                "wo": proj(cfg.dim, cfg.dim),
                "bq": vec(cfg.dim) if cfg.qkv_bias else np.zeros(cfg.dim, np.float32),
                "bk": vec(kv) if cfg.qkv_bias else np.zeros(kv, np.float32),
                "bv": vec(kv) if cfg.qkv_bias else np.zeros(kv, np.float32),
                "bo": np.zeros(cfg.dim, np.float32),
                "wg": proj(cfg.dim, cfg.hidden), "wu": proj(cfg.dim, cfg.hidden), "wd": proj(cfg.hidden, cfg.dim),
                "bg": np.zeros(cfg.hidden, np.float32), "bu": np.zeros(cfg.hidden, np.float32),
                "bd": np.zeros(cfg.dim, np.float32),
            })
        head = proj(cfg.dim, cfg.vocab)
        emb = None if cfg.tied else O.quantize(
            (rng.standard_normal((cfg.vocab, cfg.dim), dtype=np.float32) * np.float32(0.5)).astype(np.float32),
            cfg.bits, cfg.group_size)
        return DecoderWeights(cfg, emb, layers, vec(cfg.dim, 1.0, 0.1), head, np.zeros(cfg.vocab, np.float32))


THREADS = 8  # host threads of the C oracle's matmul


def _linear(x: np.ndarray, w, bias: np.ndarray) -> np.ndarray:
    """QuantizedLinear.forward (quantized weight) or Linear.forward (float32
    [in x out] weight) on one row, plus the bias."""
    if isinstance(w, np.ndarray):
        y = (x.reshape(1, -1).astype(np.float32) @ w).reshape(-1).astype(np.float32)
    else:
        y = O.multiply_quantized(x.reshape(1, -1), w, threads=THREADS).reshape(-1)
    return (y + bias).astype(np.float32)


def _linear_rows(x: np.ndarray, w, bias: np.ndarray) -> np.ndarray:
    """forwardInto on [rows x in] (multiplyQuantized at m = rows), plus the bias."""
    if isinstance(w, np.ndarray):
        y = (x.astype(np.float32) @ w).astype(np.float32)
    else:
        y = O.multiply_quantized(x, w, threads=THREADS)
    return (y + bias[None, :]).astype(np.float32)


def dequantize_column(w: O.OracleQTensor, column: int) -> np.ndarray:
    """QuantizedTensor.dequantizeColumn (the value() of every row of one column,
    QuantizedTensor.kt:172-186): scale * (q - zero) in float32, vectorised."""
    rows, cols, g = w.rows, w.columns, w.group_size
    groups = (rows + g - 1) // g
    grp = np.arange(rows) // g
    scales = w.scales.reshape(groups, cols)[grp, column]
    if w.bits == 8:
        q = w.qdata.view(np.int8).reshape(rows, cols)[:, column].astype(np.int32)
        return (scales * q.astype(np.float32)).astype(np.float32)
    half = (cols + 1) // 2
    byte = w.qdata.reshape(rows, half)[:, column % half]
    q = (byte & 15) if column < half else (byte >> 4)
    zero = w.zeros.reshape(groups, cols)[grp, column].astype(np.int32)
    return (scales * (q.astype(np.int32) - zero).astype(np.float32)).astype(np.float32)


def _rmsnorm(x, w, eps):
    ss = np.float32(np.sum(x.astype(np.float32) * x.astype(np.float32), dtype=np.float32))
    r = np.float32(1.0) / np.float32(math.sqrt(float(ss / np.float32(x.size) + np.float32(eps))))
    return (x * r * w).astype(np.float32)


def _rope(v: np.ndarray, head_dim: int, freqs: np.ndarray, position: int) -> np.ndarray:
    half = head_dim // 2
    theta = (np.float32(position) * freqs).astype(np.float32)
    c = np.cos(theta.astype(np.float64)).astype(np.float32)
    s = np.sin(theta.astype(np.float64)).astype(np.float32)
    out = v.copy().reshape(-1, head_dim)
    x1, x2 = out[:, :half].copy(), out[:, half:].copy()
    out[:, :half] = x1 * c - x2 * s
    out[:, half:] = x1 * s + x2 * c
    return out.reshape(-1)


class OracleDecoder:
    """Transformer.decode on the CPU with an explicit fp32 KV cache."""

    def __init__(self, weights: DecoderWeights, max_seq: int):
        self.w = weights
        cfg = weights.cfg
        self.cfg = cfg
        self.max_seq = max_seq
        shape = (cfg.layers, cfg.kv_heads, max_seq, cfg.head_dim)
        self.keys = np.zeros(shape, np.float32)
        self.values = np.zeros(shape, np.float32)
        self.length = 0
        self.freqs = inv_freq(cfg.head_dim, cfg.rope_theta, cfg.rope_scaling)

    def embed(self, token: int) -> np.ndarray:
        cfg = self.cfg
        if cfg.tied:
            head = self.w.head  # dequantizeColumn(token): column of the [dim x vocab] head
            if isinstance(head, np.ndarray):
                return head[:, token].astype(np.float32)
            return dequantize_column(head, token)
        if isinstance(self.w.embedding, np.ndarray):  # Embedding.lookup: a row of the float32 table
            return self.w.embedding[token].astype(np.float32)
        return self.w.embedding.dequantize_row(token).astype(np.float32)

    def step(self, token: int) -> np.ndarray:
        """Logits of one decode step; advances the cache."""
        cfg, w = self.cfg, self.w
        pos = self.length
        hd, group = cfg.head_dim, cfg.heads // cfg.kv_heads
        scale = np.float32(1.0) / np.float32(math.sqrt(float(hd)))
        x = self.embed(token)
        for l, L in enumerate(w.layers):
            n1 = _rmsnorm(x, L["norm1"], cfg.eps)
            q = _rope(_linear(n1, L["wq"], L["bq"]), hd, self.freqs, pos)
            k = _rope(_linear(n1, L["wk"], L["bk"]), hd, self.freqs, pos)
            v = _linear(n1, L["wv"], L["bv"])
            self.keys[l, :, pos, :] = k.reshape(cfg.kv_heads, hd)
            self.values[l, :, pos, :] = v.reshape(cfg.kv_heads, hd)
            ctx = np.empty(cfg.dim, np.float32)
            for h in range(cfg.heads):
                qh = q[h * hd:(h + 1) * hd]
                keys = self.keys[l, h // group, :pos + 1, :]
                vals = self.values[l, h // group, :pos + 1, :]
                sc = (keys @ qh).astype(np.float32) * scale
                mx = max(np.float32(-1e9), np.float32(sc.max()))
                e = np.exp((sc - mx).astype(np.float64)).astype(np.float32)
                wts = e * (np.float32(1.0) / np.float32(np.sum(e, dtype=np.float32)))
                ctx[h * hd:(h + 1) * hd] = (wts @ vals).astype(np.float32)
            x = (x + _linear(ctx, L["wo"], L["bo"])).astype(np.float32)
            n2 = _rmsnorm(x, L["norm2"], cfg.eps)
            gate = _linear(n2, L["wg"], L["bg"])
            up = _linear(n2, L["wu"], L["bu"])
            gate = (gate / (np.float32(1.0) + np.exp(-gate.astype(np.float64)).astype(np.float32)) * up).astype(np.float32)
            x = (x + _linear(gate, L["wd"], L["bd"])).astype(np.float32)
        self.length += 1
        return _linear(_rmsnorm(x, w.final_norm, cfg.eps), w.head, w.head_bias)

    def prefill(self, tokens) -> np.ndarray:
        """Transformer.prefill: the prompt in chunks of 32 rows (prefillLayers),
        each chunk through every block at m = chunk rows (TransformerBlock /
        Attention.prefillInto: row t at position start + t attends to the cache
        up to its own position); the logits of the last token."""
        cfg, w = self.cfg, self.w
        hd, group = cfg.head_dim, cfg.heads // cfg.kv_heads
        scale = np.float32(1.0) / np.float32(math.sqrt(float(hd)))
        tokens = list(tokens)
        if not tokens:
            raise ValueError("Prompt cannot be empty")
        if self.length + len(tokens) > self.max_seq:
            raise ValueError("KV cache full")
        x = None
        for c0 in range(0, len(tokens), 32):
            chunk = tokens[c0:c0 + 32]
            T, start = len(chunk), self.length
            x = np.stack([self.embed(t) for t in chunk]).astype(np.float32)
            for l, L in enumerate(w.layers):
                n1 = np.stack([_rmsnorm(r, L["norm1"], cfg.eps) for r in x])
                q = _linear_rows(n1, L["wq"], L["bq"])
                k = _linear_rows(n1, L["wk"], L["bk"])
                v = _linear_rows(n1, L["wv"], L["bv"])
                q = np.stack([_rope(q[t], hd, self.freqs, start + t) for t in range(T)])
                k = np.stack([_rope(k[t], hd, self.freqs, start + t) for t in range(T)])
                self.keys[l, :, start:start + T, :] = k.reshape(T, cfg.kv_heads, hd).transpose(1, 0, 2)
                self.values[l, :, start:start + T, :] = v.reshape(T, cfg.kv_heads, hd).transpose(1, 0, 2)
                ctx = np.empty((T, cfg.dim), np.float32)
                end = start + T
                visible = np.arange(end)[None, :] <= (start + np.arange(T))[:, None]  # [T x end]
                for h in range(cfg.heads):
                    keys = self.keys[l, h // group, :end, :]
                    vals = self.values[l, h // group, :end, :]
                    sc = (q[:, h * hd:(h + 1) * hd] @ keys.T).astype(np.float32) * scale
                    mx = np.maximum(np.float32(-1e9), np.where(visible, sc, -np.inf).max(axis=1))
                    e = np.where(visible, np.exp((sc - mx[:, None]).astype(np.float64)), 0.0).astype(np.float32)
                    wts = e * (np.float32(1.0) / np.sum(e, axis=1, dtype=np.float32))[:, None]
                    ctx[:, h * hd:(h + 1) * hd] = (wts @ vals).astype(np.float32)
                x = (x + _linear_rows(ctx, L["wo"], L["bo"])).astype(np.float32)
                n2 = np.stack([_rmsnorm(r, L["norm2"], cfg.eps) for r in x])
                gate = _linear_rows(n2, L["wg"], L["bg"])
                up = _linear_rows(n2, L["wu"], L["bu"])
                act = (gate / (np.float32(1.0) + np.exp(-gate.astype(np.float64)).astype(np.float32)) * up)
                x = (x + _linear_rows(act.astype(np.float32), L["wd"], L["bd"])).astype(np.float32)
            self.length += T
        return _linear(_rmsnorm(x[-1], w.final_norm, cfg.eps), w.head, w.head_bias)


def argmax(logits: np.ndarray) -> int:
    """argmaxOfLastToken (Transformer.kt:255-266)."""
    best, idx = np.float32(-1e9), 0
    for v, x in enumerate(logits):
        if x > best:
            best, idx = x, v
    return idx
