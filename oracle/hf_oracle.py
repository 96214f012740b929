"""CPU restatement of Kotensor's Hugging Face checkpoint import.  TEST
INFRASTRUCTURE ONLY: the decoder parity tests use it to turn the reference's
tiny checkpoints into oracle (and device) decoder weights; the product never
imports it.

Follows (paths inside the Kotensor project, Engine/kotensor/src/main/kotlin/):
  HuggingFaceConfig.fromJson (defaults, head_dim check, rope_scaling "llama3")
                                             HuggingFaceModelLoader.kt:33-82
  weightMapping / kotensorName / isTransposedOnImport
                                             HuggingFaceModelLoader.kt:93-122
  weightFiles (single file or sharded index) HuggingFaceModelLoader.kt:146-159
  loadWeights (tied lm head = transposed embedding table, missing biases = 0,
               quantized projections quantized from the transposed fp32 weight)
                                             HuggingFaceModelLoader.kt:168-233
The tensors are read with oracle/safetensors_oracle.py (SafeTensors.kt's
reader and readInto conversion).  ``load(directory)`` gives the reference's
unquantized model (float32 weights, Linear projections); ``load(directory,
bits, group_size)`` the model HuggingFaceModelLoader.load(directory,
Quantization(bits, groupSize)) builds: every projection and the lm head
quantized from its transposed weight, the embedding table quantized as
[vocab x dim] (QuantizedEmbedding).
"""
from __future__ import annotations

import json
import os
import re
from typing import Optional

import numpy as np

from . import decoder_oracle as DO
from . import oracle as O
from . import safetensors_oracle as SO

_MAPPING = [
    (r"^model\.embed_tokens\.weight$", "embedding.weight"),
    (r"^model\.norm\.weight$", "finalNorm.weight"),
    (r"^lm_head\.weight$", "lmHead.weight"),
    (r"^model\.layers\.(\d+)\.input_layernorm\.weight$", r"block.\1.norm1.weight"),
    (r"^model\.layers\.(\d+)\.post_attention_layernorm\.weight$", r"block.\1.norm2.weight"),
    (r"^model\.layers\.(\d+)\.self_attn\.q_proj\.(weight|bias)$", r"block.\1.attention.wQ.\2"),
    (r"^model\.layers\.(\d+)\.self_attn\.k_proj\.(weight|bias)$", r"block.\1.attention.wK.\2"),
    (r"^model\.layers\.(\d+)\.self_attn\.v_proj\.(weight|bias)$", r"block.\1.attention.wV.\2"),
    (r"^model\.layers\.(\d+)\.self_attn\.o_proj\.(weight|bias)$", r"block.\1.attention.wOut.\2"),
    (r"^model\.layers\.(\d+)\.mlp\.gate_proj\.(weight|bias)$", r"block.\1.ffn.wGate.\2"),
    (r"^model\.layers\.(\d+)\.mlp\.up_proj\.(weight|bias)$", r"block.\1.ffn.wUp.\2"),
    (r"^model\.layers\.(\d+)\.mlp\.down_proj\.(weight|bias)$", r"block.\1.ffn.wDown.\2"),
]
_TRANSPOSED = re.compile(r"^(block\.\d+\.(attention\.w(Q|K|V|Out)|ffn\.w(Gate|Up|Down))|lmHead)\.weight$")
# decoder weight key of each projection name (Transformer.namedProjections order)
_KEYS = {"attention.wQ": "q", "attention.wK": "k", "attention.wV": "v", "attention.wOut": "o",
         "ffn.wGate": "g", "ffn.wUp": "u", "ffn.wDown": "d"}


def kotensor_name(hf_name: str) -> Optional[str]:
    """HuggingFaceModelLoader.kotensorName."""
    for pattern, repl in _MAPPING:
        if re.search(pattern, hf_name):
            return re.sub(pattern, repl, hf_name)
    return None


def is_transposed_on_import(name: str) -> bool:
    return _TRANSPOSED.match(name) is not None


def load_config(directory: str) -> DO.DecoderConfig:
    """HuggingFaceConfig.fromJson as the decoder configuration."""
    with open(os.path.join(directory, "config.json"), encoding="utf-8") as f:
        root = json.load(f)
    model_type = root.get("model_type", "llama")
    if model_type not in ("llama", "qwen2", "mistral"):
        raise ValueError(f"Unsupported model_type '{model_type}'")
    hidden, heads = int(root["hidden_size"]), int(root["num_attention_heads"])
    head_dim = root.get("head_dim")
    if head_dim is not None and int(head_dim) * heads != hidden:
        raise ValueError("head_dim x num_attention_heads must equal hidden_size")
    kv = int(root.get("num_key_value_heads", heads))
    if hidden % heads != 0 or heads % kv != 0:
        raise ValueError("inconsistent head counts")
    scaling = None
    rs = root.get("rope_scaling")
    if isinstance(rs, dict):
        kind = rs.get("rope_type", rs.get("type", "default"))
        if kind == "llama3":
            scaling = (float(np.float32(rs.get("factor", 8.0))), float(np.float32(rs.get("low_freq_factor", 1.0))),
                       float(np.float32(rs.get("high_freq_factor", 4.0))),
                       int(rs.get("original_max_position_embeddings", 8192)))
        elif kind != "default":
            raise ValueError(f"Unsupported rope_scaling type '{kind}'")
    return DO.DecoderConfig(vocab=int(root["vocab_size"]), dim=hidden, layers=int(root["num_hidden_layers"]),
                            heads=heads, kv_heads=kv, hidden=int(root["intermediate_size"]),
                            eps=float(np.float32(root.get("rms_norm_eps", 1e-6))),
                            rope_theta=float(np.float32(root.get("rope_theta", 10000.0))), rope_scaling=scaling,
                            tied=False, qkv_bias=False)


def weight_files(directory: str) -> list[str]:
    """HuggingFaceModelLoader.weightFiles: the index's shards in first-mention order, or model.safetensors."""
    index = os.path.join(directory, "model.safetensors.index.json")
    if os.path.isfile(index):
        with open(index, encoding="utf-8") as f:
            weight_map = json.load(f)["weight_map"]
        shards = []
        for shard in weight_map.values():
            if shard not in shards:
                shards.append(shard)
        return [os.path.join(directory, s) for s in shards]
    single = os.path.join(directory, "model.safetensors")
    if not os.path.isfile(single):
        raise ValueError(f"No model.safetensors or model.safetensors.index.json in {directory}")
    return [single]


def _read_tensors(directory: str) -> dict:
    """Kotensor name -> float32 array (readInto conversion), over every shard."""
    out = {}
    for path in weight_files(directory):
        entries, _, _ = SO.parse(path)
        for hf_name, (dtype, shape, _, _) in entries.items():
            name = kotensor_name(hf_name)
            if name is None:
                continue  # ignored (e.g. rotary_emb.inv_freq)
            with np.errstate(over="ignore"):
                arr = SO.to_float32(dtype, SO.read_raw(path, hf_name)).reshape(shape)
            out[name] = arr
    return out


def load(directory: str, bits: Optional[int] = None, group_size: int = 64) -> DO.DecoderWeights:
    """The reference's model of a checkpoint directory as oracle decoder weights:
    float32 (bits None) or quantized (bits 4 / 8, group_size)."""
    cfg = load_config(directory)
    t = _read_tensors(directory)
    if "lmHead.weight" not in t:
        with open(os.path.join(directory, "config.json"), encoding="utf-8") as f:
            if json.load(f).get("tie_word_embeddings") is not True:
                raise ValueError("lm_head.weight is missing and tie_word_embeddings is false")
        t["lmHead.weight"] = t["embedding.weight"]  # transposed below like lm_head.weight [vocab, dim]
    kv = cfg.kv_heads * cfg.head_dim
    shapes = {"q": (cfg.dim, cfg.dim), "k": (cfg.dim, kv), "v": (cfg.dim, kv), "o": (cfg.dim, cfg.dim),
              "g": (cfg.dim, cfg.hidden), "u": (cfg.dim, cfg.hidden), "d": (cfg.hidden, cfg.dim)}
    if bits is not None:
        cfg.bits, cfg.group_size = bits, group_size

    def projection(name, k_in, n_out):
        w = t[name]
        if w.shape != (n_out, k_in):
            raise ValueError(f"{name} has shape {list(w.shape)}, expected [{n_out}, {k_in}]")
        wt = np.ascontiguousarray(w.T, dtype=np.float32)  # [in x out]
        return wt if bits is None else O.quantize(wt, bits, group_size)

    def vector(name, n):
        return np.ascontiguousarray(t[name], np.float32).reshape(n) if name in t else np.zeros(n, np.float32)

    layers = []
    for l in range(cfg.layers):
        L = {"norm1": vector(f"block.{l}.norm1.weight", cfg.dim), "norm2": vector(f"block.{l}.norm2.weight", cfg.dim)}
        for proj, key in _KEYS.items():
            k_in, n_out = shapes[key]
            L["w" + key] = projection(f"block.{l}.{proj}.weight", k_in, n_out)
            L["b" + key] = vector(f"block.{l}.{proj}.bias", n_out)
        layers.append(L)
    if any(np.any(L["bq"]) or np.any(L["bk"]) or np.any(L["bv"]) for L in layers):
        cfg.qkv_bias = True
    emb = np.ascontiguousarray(t["embedding.weight"], np.float32).reshape(cfg.vocab, cfg.dim)
    embedding = emb if bits is None else O.quantize(emb, bits, group_size)
    head = projection("lmHead.weight", cfg.dim, cfg.vocab)
    return DO.DecoderWeights(cfg, embedding, layers, vector("finalNorm.weight", cfg.dim), head,
                             vector("lmHead.bias", cfg.vocab))


def expected(directory: str):
    """(input ids, logits [T x vocab]) of the checkpoint's expected.json (HuggingFaceImportTest.expected)."""
    with open(os.path.join(directory, "expected.json"), encoding="utf-8") as f:
        root = json.load(f)
    return [int(v) for v in root["input_ids"]], np.array(root["logits"], np.float32)
