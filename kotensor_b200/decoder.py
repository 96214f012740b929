"""Device-resident greedy decode step: Transformer.decode
(Engine/kotensor/src/main/kotlin/Transformer.kt:141-154) with every layer
(TransformerBlock.decodeInto, TransformerBlock.kt:40-47; Attention.decodeInto,
Attention.kt:207-239; SwiGLU.forwardInto, SwiGLU.kt:19-25) on the GPU: the
projections are the quantized matmul (kt_qmatmul, with QuantizedLinear's bias),
the rest are the decode kernels of libkt_cuda.so (kt_rmsnorm, kt_rope,
kt_kv_store, kt_attention_decode, kt_silu_mul, kt_add, kt_argmax, the
quantized / tied embedding lookups).  The token id and position live on the
device, so one step is captured into a CUDA graph and replayed per token with
no host work between tokens.  The KV cache has the reference's layout
(KVCache.kt:3-59): fp32 [layers][kvHeads][maxSeq][headDim].
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _lib
from .quantized import Context, MatMul, QuantizedTensor

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


@dataclass
class DecoderConfig:
    """Transformer(vocabularySize, dimension, numLayers, numHeads, hiddenDimension,
    numKeyValueHeads, normEps, ropeTheta, ropeScaling, quantization), Transformer.kt:3-14."""
    vocab: int
    dim: int
    layers: int
    heads: int
    kv_heads: int
    hidden: int
    eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: Optional[tuple] = None  # RoPEScaling(factor, low, high, originalMaxPositions)
    bits: int = 4
    group_size: int = 64
    tied: bool = False        # Transformer.tieEmbeddingToHead (Transformer.kt:380-386)
    qkv_bias: bool = False

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads


def rope_inv_freq(head_dim: int, base: float, scaling: Optional[tuple]) -> np.ndarray:
    """RoPE.invFreq (RoPE.kt:39-42) and RoPEScaling.scale (RoPE.kt:15-27) in float32."""
    half = head_dim // 2
    out = np.empty(half, np.float32)
    for i in range(half):
        raw = np.float32(1.0) / np.float32(math.pow(float(np.float32(base)),
                                                    float(np.float32(2 * i) / np.float32(head_dim))))
        if scaling is not None:
            factor, low, high = np.float32(scaling[0]), np.float32(scaling[1]), np.float32(scaling[2])
            orig = np.float32(int(scaling[3]))
            wl = np.float32(2.0 * math.pi / float(raw))
            if wl < orig / high:
                pass
            elif wl > orig / low:
                raw = raw / factor
            else:
                smooth = (orig / wl - low) / (high - low)
                raw = (np.float32(1.0) - smooth) * raw / factor + smooth * raw
        out[i] = np.float32(raw)
    return out


def tensor_parallel_plan(cfg: DecoderConfig, parts: int, rank: int) -> dict:
    """Rank ``rank``'s share of a decoder split over ``parts`` ranks: query and
    key/value heads (contiguous blocks), the columns [q0, q1) of the query
    projection (= the rows of the output projection), [k0, k1) of the key and
    value projections, the block [h0, h1) of whole groups of the hidden width
    (gate / up columns, down-projection rows) and the lm head's vocabulary
    columns [v0, v1).  Requires heads and kv_heads divisible by ``parts`` and
    the output projection's rows to split on group boundaries."""
    from .parallel import COLUMNS, ROWS, shard_bounds
    if parts < 1 or not 0 <= rank < parts:
        raise ValueError(f"rank {rank} of {parts}")
    if cfg.heads % parts or cfg.kv_heads % parts:
        raise ValueError(f"{cfg.heads} query / {cfg.kv_heads} key-value heads do not split over {parts} ranks")
    hd, g = cfg.head_dim, cfg.group_size
    heads, kv = cfg.heads // parts, cfg.kv_heads // parts
    q0, q1 = rank * heads * hd, (rank + 1) * heads * hd
    k0, k1 = rank * kv * hd, (rank + 1) * kv * hd
    if parts > 1 and (q0 % g or (q1 % g and q1 != cfg.dim)):
        raise ValueError(f"{q1 - q0} output-projection rows per rank is not a multiple of the group size {g}")
    hidden = shard_bounds(ROWS, cfg.hidden, g, parts, rank) if parts > 1 else (0, cfg.hidden)
    vocab = shard_bounds(COLUMNS, cfg.vocab, g, parts, rank) if parts > 1 else (0, cfg.vocab)
    return {"heads": heads, "kv_heads": kv, "q": (q0, q1), "kv": (k0, k1), "hidden": hidden, "vocab": vocab}


def _upload(w) -> QuantizedTensor:
    """A QuantizedTensor, or host arrays in the reference layout (objects with
    qdata / scales / zeros / rows / columns / bits / group_size)."""
    if isinstance(w, QuantizedTensor):
        return w
    return QuantizedTensor.from_arrays(w.qdata, w.scales, w.zeros, (w.rows, w.columns), w.bits, w.group_size)


class _Rows:
    """Activation buffers for a block of rows (one decode step, or a prefill)."""


class DeviceDecoder:
    """Greedy decoding of one sequence with weights, KV cache and buffers in HBM.

    ``max_block_rows`` (65,535, the row kernels' grid limit) bounds the rows of
    one prefill block; a batch with more prompt rows is prefilled in blocks of
    whole sequences.

    ``weights``: ``embedding`` ([vocab x dim], None when tied), ``layers`` (a list
    of dicts with wq wk wv wo wg wu wd, their biases bq bk bv bo bg bu bd and the
    RMSNorm weights norm1 norm2), ``final_norm``, ``head`` ([dim x vocab]),
    ``head_bias``.  ``batch`` sequences decode together (one KV cache each, the
    same position): every matmul of a step runs at m = batch.

    ``comm`` (a parallel.Comm over P ranks, one process per GPU, every rank
    building the decoder from the same weights): tensor parallelism
    (``tensor_parallel_plan``).  Rank r keeps its block of query heads and of
    key/value heads -- the q|k|v projection column-parallel over them,
    attention and its KV cache local -- the output projection row-parallel over
    the same rows, the gate|up projection column-parallel and the down
    projection row-parallel over one block of whole groups of the hidden width,
    and the lm head column-parallel over the vocabulary with the greedy argmax
    taken across shards (argmaxOfLastToken's rule, Transformer.kt:255-266).
    The two row-parallel products of a layer end in the only exchange: an
    all-reduce of [batch x dim] partial sums (fused into the m = 1 GEMV over
    peer memory, else NCCL), after which every rank holds the whole residual
    stream."""

    max_block_rows = 65535

    def __init__(self, cfg: DecoderConfig, weights, max_seq: int, device: Optional[int] = None, batch: int = 1,
                 comm=None):
        self.cfg = cfg
        self.max_seq = max_seq
        self.ctx = Context.get(device)
        dev = torch.device("cuda", self.ctx.device)
        f32 = dict(dtype=torch.float32, device=dev)

        def vec(a):
            if isinstance(a, torch.Tensor):
                return a.detach().to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
            return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32).reshape(-1)).to(dev)

        from .parallel import COLUMNS, ROWS, concat_columns, slice_weight
        self.comm = comm
        P = comm.world if comm is not None else 1
        plan = tensor_parallel_plan(cfg, P, comm.rank if comm is not None else 0)
        self.parts = P
        self.heads_local, self.kv_local = plan["heads"], plan["kv_heads"]
        q0, q1 = plan["q"]
        k0, k1 = plan["kv"]
        h0, h1 = plan["hidden"]
        v0, v1 = plan["vocab"]
        self.q_width, self.kv_width = q1 - q0, k1 - k0
        self.hidden_local, self.vocab_begin, self.vocab_local = h1 - h0, v0, v1 - v0

        def cols(w, b, e):
            return w if P == 1 else slice_weight(w, COLUMNS, b, e)

        self.layers = []
        for L in weights.layers:
            d = {k: (_upload(v) if k.startswith("w") else vec(v)) for k, v in L.items()}
            # q|k|v and gate|up as one matmul each: per-column quantization makes
            # the fused weight's columns exactly the separate weights' columns
            # (and a rank's column shard exactly those columns of the weight)
            d["wqkv"] = concat_columns([cols(d["wq"], q0, q1), cols(d["wk"], k0, k1), cols(d["wv"], k0, k1)])
            d["bqkv"] = torch.cat([d["bq"][q0:q1], d["bk"][k0:k1], d["bv"][k0:k1]])
            d["wgu"] = concat_columns([cols(d["wg"], h0, h1), cols(d["wu"], h0, h1)])
            d["bgu"] = torch.cat([d["bg"][h0:h1], d["bu"][h0:h1]])
            if P > 1:  # row-parallel: this rank's rows; the bias is added once, after the exchange
                d["wo"] = slice_weight(d["wo"], ROWS, q0, q1)
                d["wd"] = slice_weight(d["wd"], ROWS, h0, h1)
            for k in ("wq", "wk", "wv", "wg", "wu", "bq", "bk", "bv", "bg", "bu"):
                del d[k]
            self.layers.append(d)
        full_head = _upload(weights.head)
        self.head = cols(full_head, v0, v1)
        self.head_bias = vec(weights.head_bias)[v0:v1].contiguous()
        # tied embeddings look tokens up in the whole head (any column may be asked for)
        self.lookup_head = full_head if cfg.tied else None
        self.embedding = None if cfg.tied else _upload(weights.embedding)
        self.final_norm = vec(weights.final_norm)
        if batch < 1:
            raise ValueError(f"batch must be positive, got {batch}")
        self.batch = batch
        # one KV cache per sequence, each in the reference's layout [L][kvH][maxSeq][hd]
        # (this rank's key/value heads under tensor parallelism)
        self.keys = torch.zeros((batch, cfg.layers, self.kv_local, max_seq, cfg.head_dim), **f32)
        self.values = torch.zeros_like(self.keys)
        self.cache_stride = cfg.layers * self.kv_local * max_seq * cfg.head_dim
        self.inv_freq = vec(rope_inv_freq(cfg.head_dim, cfg.rope_theta, cfg.rope_scaling))
        self.token = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.next_token = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.position = torch.zeros(1, dtype=torch.int32, device=dev)  # shared: sequences advance together
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.logits = torch.empty((batch, self.vocab_local), **f32)  # this rank's vocabulary columns
        self._head_in = torch.empty((batch, cfg.dim), **f32)
        self._head_xn = torch.empty((batch, cfg.dim), **f32)
        self._last_rows = torch.empty(batch, dtype=torch.int32, device=dev)
        self._step_bufs = self._buffers(batch, tokens=self.token)
        self._prefill_bufs = None  # prefill buffers, allocated on first use
        self.length = 0
        self.scale = float(np.float32(1.0) / np.float32(math.sqrt(float(cfg.head_dim))))
        self._graph = None
        g_ = self.heads_local // self.kv_local
        self._fused_attention = g_ <= 8 and cfg.head_dim in (64, 128) and max_seq <= 16384
        if P > 1:
            self._warm_exchanges()

    # -- helpers
    @staticmethod
    def _p(t) -> ctypes.c_void_p:
        return ctypes.c_void_p(t.data_ptr())

    def _stream(self) -> ctypes.c_void_p:
        return ctypes.c_void_p(torch.cuda.current_stream(self.ctx.device).cuda_stream)

    def reset(self) -> None:
        self.length = 0
        self.position.zero_()

    def _buffers(self, rows: int, tokens=None) -> "_Rows":
        cfg = self.cfg
        dev = self.position.device
        f32 = dict(dtype=torch.float32, device=dev)
        kv = cfg.kv_heads * cfg.head_dim
        b = _Rows()
        b.rows = rows
        b.x = torch.empty((rows, cfg.dim), **f32)
        b.normed = torch.empty((rows, cfg.dim), **f32)
        b.qkv = torch.empty((rows, self.q_width + 2 * self.kv_width), **f32)
        b.ctx = torch.empty((rows, self.q_width), **f32)
        b.gu = torch.empty((rows, 2 * self.hidden_local), **f32)
        b.act = torch.empty((rows, self.hidden_local), **f32)
        b.tokens = tokens if tokens is not None else torch.empty(rows, dtype=torch.int32, device=dev)
        # attention scratch; zero-filled: its tail holds the fused kernel's merge counters
        b.scores = torch.zeros(_lib.load().kt_attention_scratch_floats(rows, self.heads_local, cfg.head_dim,
                                                                       self.max_seq), **f32)
        return b

    def _row_parallel(self, x, w, out, rows: int, bias, accumulate: bool = True) -> None:
        """out[rows x dim] (+)= x . W + bias (the residual add of
        TransformerBlock.decodeInto): the local product, or under tensor
        parallelism this rank's rows of W and the all-reduce of the partials."""
        if self.comm is None:
            MatMul.multiply_quantized(x, w, out, rows, accumulate=accumulate, bias=bias)
        else:
            from .parallel import matmul_row_parallel
            matmul_row_parallel(self.comm, x, w, out, rows, accumulate=accumulate, bias=bias)

    def _warm_exchanges(self) -> None:
        """Collective (every rank, at construction): each row-parallel shard
        agrees its exchange once at m = batch (the fused peer-memory GEMV at
        m = 1 is set up and agreed on its first call, and the agreement
        synchronizes the stream, which a CUDA graph capture cannot), and the
        communicator's scratch grows to the step's size, so a captured step
        neither sets up nor allocates."""
        dev = self.position.device
        m = self.batch
        x_o = torch.zeros((m, self.q_width), dtype=torch.float32, device=dev)
        x_d = torch.zeros((m, self.hidden_local), dtype=torch.float32, device=dev)
        out = torch.empty((m, self.cfg.dim), dtype=torch.float32, device=dev)
        for L in self.layers:
            self._row_parallel(x_o, L["wo"], out, m, None, accumulate=False)
            self._row_parallel(x_d, L["wd"], out, m, None, accumulate=False)
        from .parallel import argmax_column_parallel
        self.logits.zero_()
        argmax_column_parallel(self.comm, self.logits, self.vocab_begin, self.next_token)
        torch.cuda.current_stream(self.ctx.device).synchronize()

    def gather_logits(self):
        """The whole [batch x vocab] logits on every rank (an all-gather of the
        ranks' vocabulary columns; the logits themselves when not sharded)."""
        if self.comm is None:
            return self.logits
        from .parallel import allgather_columns
        if self.cfg.vocab % self.parts:
            raise ValueError("the vocabulary does not split evenly: gather the shards with their offsets")
        full = torch.empty((self.batch, self.cfg.vocab), dtype=torch.float32, device=self.logits.device)
        allgather_columns(self.comm, self.logits, full, self.batch)
        return full

    def _layers(self, b: "_Rows", rows: int, rows_per_seq: int, seq0: int = 0) -> None:
        """Embedding lookup of b.tokens[:rows] through every block; leaves the
        residual rows in b.x (the head applies the final norm).  Row r is
        sequence seq0 + r / rows_per_seq at position *position + r %
        rows_per_seq (one sequence's prompt, or one token of each of `rows`
        sequences).  Per layer: norm1 + q|k|v, RoPE / cache / attention, the
        output projection added to the residual, norm2 + gate|up + SiLU * up,
        the down projection added to the residual -- five launches at batch 1,
        where the GEMV applies each norm while staging its input row and forms
        silu(gate) * up in its epilogue."""
        L_ = _lib.load()
        cfg, h = self.cfg, self.ctx.handle
        s, p = self._stream(), self._p
        keys = ctypes.c_void_p(self.keys.data_ptr() + seq0 * self.cache_stride * self.keys.element_size())
        values = ctypes.c_void_p(self.values.data_ptr() + seq0 * self.cache_stride * self.values.element_size())
        hd, kvh = cfg.head_dim, self.kv_local
        kv = self.kv_width
        if cfg.tied:
            _lib.check(L_.kt_dequantize_column(h, self.lookup_head.handle, p(b.tokens), rows, p(b.x), p(self.status),
                                               s))
        else:
            _lib.check(L_.kt_dequantize_rows(h, self.embedding.handle, p(b.tokens), rows, p(b.x), p(self.status), s))
        for l, L in enumerate(self.layers):
            _lib.check(L_.kt_rmsnorm_qmatmul(h, L["wqkv"].handle, p(b.x), p(L["norm1"]), cfg.eps, p(b.normed),
                                             p(b.qkv), rows, 0, p(L["bqkv"]), s))
            if rows_per_seq == 1 and self._fused_attention and rows <= (16 if cfg.head_dim == 128 else 8):
                # one token per sequence: RoPE, cache store, attention and merge in one launch
                # (measured slower than the separate kernels once more sequences share a
                # step: beyond 16 at head_dim 128, beyond 8 at 64)
                _lib.check(L_.kt_attention_rope_decode(h, p(b.qkv), rows, self.q_width, self.heads_local, kvh, hd,
                                                       p(self.inv_freq), keys, values, p(b.ctx), p(b.scores),
                                                       self.max_seq, l, self.scale, p(self.position),
                                                       self.cache_stride, s))
            else:
                _lib.check(L_.kt_rope_kv_seqs(h, p(b.qkv), rows, self.q_width, kvh, hd, p(self.inv_freq), keys,
                                              values, self.max_seq, l, p(self.position), rows_per_seq,
                                              self.cache_stride, s))
                _lib.check(L_.kt_attention_seqs(h, p(b.qkv), keys, values, p(b.ctx), p(b.scores), rows,
                                                self.q_width + 2 * kv, self.heads_local, kvh, hd, self.max_seq, l,
                                                self.scale, p(self.position), rows_per_seq, self.cache_stride, s))
            self._row_parallel(b.ctx[:rows], L["wo"], b.x[:rows], rows, L["bo"])  # x += attention output
            _lib.check(L_.kt_rmsnorm_qmatmul_swiglu(h, L["wgu"].handle, p(b.x), p(L["norm2"]), cfg.eps,
                                                    p(b.normed), p(b.gu), p(b.act), rows, p(L["bgu"]), s))
            self._row_parallel(b.act[:rows], L["wd"], b.x[:rows], rows, L["bd"])  # x += feed-forward output

    def _head(self, x_rows, advance: int) -> None:
        """The final norm and the head on `batch` residual rows, greedy argmax
        per row, position += advance."""
        L_ = _lib.load()
        h, s, p = self.ctx.handle, self._stream(), self._p
        _lib.check(L_.kt_rmsnorm_qmatmul(h, self.head.handle, p(x_rows), p(self.final_norm), self.cfg.eps,
                                         p(self._head_xn), p(self.logits), self.batch, 0, p(self.head_bias), s))
        if self.comm is None:
            _lib.check(L_.kt_argmax(h, p(self.logits), self.batch, self.cfg.vocab, p(self.next_token), s))
        else:  # every rank's best column, merged across ranks: the same token everywhere
            from .parallel import argmax_column_parallel
            argmax_column_parallel(self.comm, self.logits, self.vocab_begin, self.next_token)
        _lib.check(L_.kt_increment(h, p(self.position), advance, s))
        self.token.copy_(self.next_token)

    def _launch_step(self) -> None:
        """One decode step on the current stream: reads self.token and
        self.position, writes self.logits and self.next_token, advances
        the position and feeds the next tokens back."""
        b = self._step_bufs
        self._layers(b, self.batch, 1)
        self._head(b.x, 1)

    def _result(self):
        return self.logits[0] if self.batch == 1 else self.logits

    def prefill(self, prompts):
        """Transformer.prefill (Transformer.kt:99-132) for every sequence: each
        prompt (a list of token ids; one per sequence, equal lengths) runs as one
        block of rows through every layer (the matmuls at m = batch x T on the
        tensor-core GEMM, causal attention over each sequence's cache); returns
        the last tokens' logits and leaves their greedy successors in
        next_token / token."""
        if len(prompts) > 0 and not isinstance(prompts[0], (list, tuple, np.ndarray)):
            prompts = [prompts]
        if len(prompts) != self.batch:
            raise ValueError(f"{len(prompts)} prompts for a batch of {self.batch}")
        T = len(prompts[0])
        if T == 0:
            raise ValueError("Prompt cannot be empty")
        if any(len(pr) != T for pr in prompts):
            raise ValueError("prompts of one batch must have equal lengths")
        if any(not 0 <= t < self.cfg.vocab for pr in prompts for t in pr):
            raise ValueError("token out of vocab bounds")
        if self.length + T > self.max_seq:
            raise ValueError(f"KV cache full: {self.length} + {T} positions exceed maxSequenceLength {self.max_seq}")
        if T > self.max_block_rows:
            raise ValueError(f"{T} prompt tokens exceed {self.max_block_rows} rows of one prefill block")
        # whole sequences per block: a block holds at most max_block_rows rows (the
        # kernels' grid rows); larger batches are prefilled in several blocks
        per = min(self.batch, self.max_block_rows // T)
        if self._prefill_bufs is None or self._prefill_bufs.rows < per * T:
            self._prefill_bufs = self._buffers(per * T)
        if self.comm is not None:
            # a larger block may replace the communicator's scratch that a
            # captured step refers to: capture again before the next replay
            self._graph = None
        b = self._prefill_bufs
        flat = torch.tensor([t for pr in prompts for t in pr], dtype=torch.int32)
        L_ = _lib.load()
        for s0 in range(0, self.batch, per):
            s1 = min(self.batch, s0 + per)
            rows = (s1 - s0) * T
            b.tokens[:rows].copy_(flat[s0 * T:s1 * T])
            self._layers(b, rows, T, seq0=s0)
            # the head only on each sequence's last row
            self._last_rows[:s1 - s0].copy_(torch.tensor([q * T + T - 1 for q in range(s1 - s0)], dtype=torch.int32))
            dst = ctypes.c_void_p(self._head_in.data_ptr() + s0 * self.cfg.dim * self._head_in.element_size())
            _lib.check(L_.kt_gather_rows(self.ctx.handle, self._p(b.x), self._p(self._last_rows), s1 - s0,
                                         self.cfg.dim, dst, self._stream()))
        self._head(self._head_in, T)
        self.length += T
        return self._result()

    def step(self, tokens):
        """Transformer.decode(token) for every sequence (an int when batch == 1):
        the logits of this step (device tensor)."""
        tokens = [tokens] if isinstance(tokens, (int, np.integer)) else list(tokens)
        if len(tokens) != self.batch:
            raise ValueError(f"{len(tokens)} tokens for a batch of {self.batch}")
        for t in tokens:
            if not 0 <= t < self.cfg.vocab:
                raise ValueError(f"{t} out of vocab bounds {self.cfg.vocab}")
        if self.length >= self.max_seq:
            raise ValueError(f"KV cache full: maxSequenceLength {self.max_seq}")
        self.token.copy_(torch.tensor(tokens, dtype=torch.int32))
        self._launch_step()
        self.length += 1
        return self._result()

    def capture(self) -> None:
        """Records one step (from the current self.token / self.position) into a CUDA graph."""
        torch.cuda.synchronize()
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph):
            self._launch_step()

    def generate(self, prompt: list[int], max_tokens: int) -> list[int]:
        """Greedy continuation of one sequence (batch 1): the prompt fed step by
        step (eager), then ``max_tokens`` replays of the captured step."""
        if self.batch != 1:
            raise ValueError("generate is for batch 1; use generate_batch")
        if len(prompt) + max_tokens > self.max_seq:
            raise ValueError("prompt + max_tokens exceed max_seq")
        for t in prompt:
            self.step(t)
        out = [int(self.next_token[0].item())]
        if self._graph is None:
            self.capture()  # captures the position reached after the prompt
        for _ in range(max_tokens - 1):
            self._graph.replay()
            self.length += 1
            out.append(int(self.next_token[0].item()))
        return out

    def generate_batch(self, prompts, max_tokens: int) -> list:
        """Greedy continuation of every sequence: the prompts prefilled as blocks,
        then ``max_tokens`` - 1 replays of the captured batched step."""
        if len(prompts[0]) + max_tokens > self.max_seq:
            raise ValueError("prompt + max_tokens exceed max_seq")
        self.prefill(prompts)
        out = [self.next_token.cpu().tolist()]
        if self._graph is None:
            self.capture()
        for _ in range(max_tokens - 1):
            self._graph.replay()
            self.length += 1
            out.append(self.next_token.cpu().tolist())
        return [[row[q] for row in out] for q in range(self.batch)]

    # -- files (Transformer.saveQuantized / loadQuantized, Transformer.kt:402-471)
    def save_quantized(self, path) -> None:
        """Transformer.saveQuantized: the reference's file, byte for byte, written
        from HBM (q|k|v and gate|up are split back into their projections)."""
        from .parallel import COLUMNS, slice_weight
        if self.comm is not None:
            raise ValueError("save_quantized needs the whole model: save from an unsharded decoder")
        from .safetensors import SafeTensorsEntry, quantized_entries, save_entries
        cfg = self.cfg
        kv = cfg.kv_heads * cfg.head_dim
        meta = quantized_metadata(cfg)
        entries, keep = [], []

        def f32(name, t, n):
            entries.append(SafeTensorsEntry(name, "F32", [1, n], t.contiguous()))

        for l, L in enumerate(self.layers):
            f32(f"block.{l}.norm1.weight", L["norm1"], cfg.dim)
            f32(f"block.{l}.norm2.weight", L["norm2"], cfg.dim)
        f32("finalNorm.weight", self.final_norm, cfg.dim)
        q_cols = [(0, cfg.dim), (cfg.dim, cfg.dim + kv), (cfg.dim + kv, cfg.dim + 2 * kv)]
        g_cols = [(0, cfg.hidden), (cfg.hidden, 2 * cfg.hidden)]
        projections = []
        for l, L in enumerate(self.layers):
            parts = {}
            for key, (b, e) in zip(("wq", "wk", "wv"), q_cols):
                parts[key] = (slice_weight(L["wqkv"], COLUMNS, b, e), L["bqkv"][b:e])
            parts["wo"] = (L["wo"], L["bo"])
            for key, (b, e) in zip(("wg", "wu"), g_cols):
                parts[key] = (slice_weight(L["wgu"], COLUMNS, b, e), L["bgu"][b:e])
            parts["wd"] = (L["wd"], L["bd"])
            for suffix, key in PROJECTION_NAMES:
                projections.append((f"block.{l}.{suffix}",) + parts[key])
        projections.append(("lmHead", self.head, self.head_bias))
        for name, w, b in projections:
            f32(f"{name}.bias", b, w.columns)
        quantized = ([] if cfg.tied else [("embedding", self.embedding)]) + [(n, w) for n, w, _ in projections]
        for name, w in quantized:
            entries += quantized_entries(name, w)
            keep.append(w)  # the slices stay alive until the file is written
        save_entries(path, entries, meta)

    @staticmethod
    def load_quantized(path, max_seq: int, device: Optional[int] = None) -> "DeviceDecoder":
        """Transformer.loadQuantized: a decoder whose weights go from the file
        straight into HBM."""
        cfg, weights = load_quantized_weights(path, device)
        return DeviceDecoder(cfg, weights, max_seq, device)


# (file name suffix, decoder weight key) in Transformer.namedProjections order (Transformer.kt:268-282)
PROJECTION_NAMES = [("attention.wQ", "wq"), ("attention.wK", "wk"), ("attention.wV", "wv"),
                    ("attention.wOut", "wo"), ("ffn.wGate", "wg"), ("ffn.wUp", "wu"), ("ffn.wDown", "wd")]


def quantized_metadata(cfg: DecoderConfig) -> dict:
    """The kotensor.* metadata of Transformer.saveQuantized (Transformer.kt:403-419)."""
    from .safetensors import java_float_string as js
    meta = {
        "kotensor.vocabularySize": str(cfg.vocab),
        "kotensor.dimension": str(cfg.dim),
        "kotensor.numLayers": str(cfg.layers),
        "kotensor.numHeads": str(cfg.heads),
        "kotensor.hiddenDimension": str(cfg.hidden),
        "kotensor.numKeyValueHeads": str(cfg.kv_heads),
        "kotensor.normEps": js(cfg.eps),
        "kotensor.ropeTheta": js(cfg.rope_theta),
    }
    if cfg.rope_scaling is not None:
        f, lo, hi, orig = cfg.rope_scaling
        meta["kotensor.ropeScaling"] = f"{js(f)},{js(lo)},{js(hi)},{int(orig)}"
    meta["kotensor.quantization.bits"] = str(cfg.bits)
    meta["kotensor.quantization.groupSize"] = str(cfg.group_size)
    if cfg.tied:
        meta["kotensor.tiedEmbedding"] = "true"
    return meta


class LoadedWeights:
    """Device weights read from a file, in DeviceDecoder's ``weights`` shape."""

    def __init__(self):
        self.embedding = None
        self.layers = []
        self.final_norm = None
        self.head = None
        self.head_bias = None


def load_quantized_weights(path, device: Optional[int] = None):
    """(config, weights) of a file written by Transformer.saveQuantized
    (Transformer.loadQuantized, Transformer.kt:433-471), weights in HBM."""
    from .quantized import Quantization
    from .safetensors import SafeTensorsFile
    with SafeTensorsFile(path) as f:
        meta = f.metadata

        def value(key):
            if key not in meta:
                raise ValueError(f"{path} has no {key} metadata; was it written by saveQuantized?")
            return meta[key]

        scaling = None
        if "kotensor.ropeScaling" in meta:
            p = meta["kotensor.ropeScaling"].split(",")
            scaling = (float(np.float32(p[0])), float(np.float32(p[1])), float(np.float32(p[2])), int(p[3]))
        q = Quantization(int(value("kotensor.quantization.bits")), int(value("kotensor.quantization.groupSize")))
        cfg = DecoderConfig(vocab=int(value("kotensor.vocabularySize")), dim=int(value("kotensor.dimension")),
                            layers=int(value("kotensor.numLayers")), heads=int(value("kotensor.numHeads")),
                            kv_heads=int(value("kotensor.numKeyValueHeads")),
                            hidden=int(value("kotensor.hiddenDimension")),
                            eps=float(np.float32(value("kotensor.normEps"))),
                            rope_theta=float(np.float32(value("kotensor.ropeTheta"))), rope_scaling=scaling,
                            bits=q.bits, group_size=q.group_size, tied=meta.get("kotensor.tiedEmbedding") == "true")
        kv = cfg.kv_heads * cfg.head_dim
        shapes = {"wq": (cfg.dim, cfg.dim), "wk": (cfg.dim, kv), "wv": (cfg.dim, kv), "wo": (cfg.dim, cfg.dim),
                  "wg": (cfg.dim, cfg.hidden), "wu": (cfg.dim, cfg.hidden), "wd": (cfg.hidden, cfg.dim)}

        def param(name):
            if name not in f:
                raise ValueError(f"{path} is missing {name}")
            return f.load(name, device).reshape(-1)

        w = LoadedWeights()
        for l in range(cfg.layers):
            L = {"norm1": param(f"block.{l}.norm1.weight"), "norm2": param(f"block.{l}.norm2.weight")}
            for suffix, key in PROJECTION_NAMES:
                name = f"block.{l}.{suffix}"
                L["b" + key[1]] = param(f"{name}.bias")
                L[key] = f.load_quantized(name, q, *shapes[key], device=device)
            w.layers.append(L)
        w.final_norm = param("finalNorm.weight")
        w.head_bias = param("lmHead.bias")
        w.head = f.load_quantized("lmHead", q, cfg.dim, cfg.vocab, device=device)
        if not cfg.tied:
            w.embedding = f.load_quantized("embedding", q, cfg.vocab, cfg.dim, device=device)
        torch.cuda.current_stream(w.head.device).synchronize()  # the file's staging buffers are released on close
    return cfg, w
