"""The decoder oracle pinned to the reference's own known answers (no GPU).

The Kotensor suite holds three tiny Hugging Face checkpoints with the logits
Hugging Face computed for every position of a 7-token input
(tests/golden/hf/, copied by tests/golden/make_hf_golden.py).  The reference
checks its float32 decoder against them at 2e-4 absolute
(HuggingFaceImportTest.kt:29-36 full forward, :52-61 decode steps; :84 and
:100 for the Qwen and Llama-3 checkpoints).  Here the oracle's restatement of
Transformer.decode (oracle/decoder_oracle.py), fed the reference's float32
import of each checkpoint (oracle/hf_oracle.py), must meet the same bound at
every step.  Together the three cover grouped-query attention (2 and 1 kv
heads), q/k/v biases, a tied lm head, an explicit head_dim and Llama-3 RoPE
scaling -- every non-matmul piece of the decode step the device kernels are
checked against.
"""
import os

import numpy as np
import pytest

from oracle import decoder_oracle as DO
from oracle import hf_oracle as H

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HF = os.path.join(ROOT, "tests", "golden", "hf")
CHECKPOINTS = ["llama_tiny", "llama3_tiny", "qwen_tiny_sharded"]
TOL = 2e-4  # HuggingFaceImportTest's bound


@pytest.mark.parametrize("name", CHECKPOINTS)
def test_oracle_decode_matches_reference_logits(name):
    d = os.path.join(HF, name)
    weights = H.load(d)
    ids, logits = H.expected(d)
    dec = DO.OracleDecoder(weights, max_seq=len(ids))
    for t, tok in enumerate(ids):
        got = dec.step(tok)
        assert got.shape == (weights.cfg.vocab,)
        err = float(np.abs(got - logits[t]).max())
        assert err <= TOL, f"{name} position {t}: {err}"


def test_checkpoint_configs_are_read_like_the_reference():
    """HuggingFaceImportTest.kt:40-45, :67-79, :91-95."""
    llama = H.load_config(os.path.join(HF, "llama_tiny"))
    assert (llama.kv_heads, llama.head_dim, llama.rope_scaling) == (2, 8, None)
    assert np.float32(llama.eps) == np.float32(1e-5)
    qwen = H.load(os.path.join(HF, "qwen_tiny_sharded"))
    assert qwen.cfg.kv_heads == 1 and qwen.cfg.qkv_bias
    assert np.any(qwen.layers[0]["bq"] != 0) and np.all(qwen.layers[0]["bo"] == 0)
    # tied: the lm head is the transposed embedding table
    assert np.array_equal(qwen.head, qwen.embedding.T)
    l3 = H.load_config(os.path.join(HF, "llama3_tiny"))
    assert np.float32(l3.rope_theta) == np.float32(500000.0) and l3.rope_scaling[0] == 8.0
    assert H.weight_files(os.path.join(HF, "qwen_tiny_sharded"))[0].endswith("model-00001-of-00002.safetensors")


def test_weight_name_mapping():
    """HuggingFaceImportTest.testWeightNameMapping."""
    assert H.kotensor_name("model.embed_tokens.weight") == "embedding.weight"
    assert H.kotensor_name("model.layers.12.self_attn.q_proj.weight") == "block.12.attention.wQ.weight"
    assert H.kotensor_name("model.layers.3.self_attn.k_proj.bias") == "block.3.attention.wK.bias"
    assert H.kotensor_name("model.layers.0.mlp.gate_proj.weight") == "block.0.ffn.wGate.weight"
    assert H.kotensor_name("model.layers.7.post_attention_layernorm.weight") == "block.7.norm2.weight"
    assert H.kotensor_name("model.norm.weight") == "finalNorm.weight"
    assert H.kotensor_name("lm_head.weight") == "lmHead.weight"
    assert H.kotensor_name("model.layers.0.self_attn.rotary_emb.inv_freq") is None
    assert H.kotensor_name("transformer.h.0.attn.c_attn.weight") is None
    assert H.is_transposed_on_import("block.1.attention.wOut.weight")
    assert H.is_transposed_on_import("lmHead.weight")
    assert not H.is_transposed_on_import("block.1.attention.wOut.bias")
    assert not H.is_transposed_on_import("embedding.weight")
    assert not H.is_transposed_on_import("block.1.norm1.weight")


def test_oracle_detects_a_planted_error():
    """The comparison has teeth: a RoPE base off by 1 % moves the logits past the bound."""
    d = os.path.join(HF, "llama_tiny")
    weights = H.load(d)
    ids, logits = H.expected(d)
    weights.cfg.rope_theta *= 1.01
    dec = DO.OracleDecoder(weights, max_seq=len(ids))
    worst = max(float(np.abs(dec.step(t) - logits[i]).max()) for i, t in enumerate(ids))
    assert worst > TOL


@pytest.mark.parametrize("name", CHECKPOINTS)
def test_oracle_prefill_matches_reference_logits(name):
    """Transformer.prefill's restatement (32-row chunks) on the same checkpoints:
    the last position's logits within the reference's bound."""
    d = os.path.join(HF, name)
    ids, logits = H.expected(d)
    dec = DO.OracleDecoder(H.load(d), max_seq=len(ids))
    assert float(np.abs(dec.prefill(ids) - logits[-1]).max()) <= TOL


@pytest.mark.parametrize("bits", [4, 8])
def test_oracle_prefill_matches_its_steps_on_quantized_checkpoints(bits):
    """The quantized import (HuggingFaceModelLoader.load with a Quantization):
    prefill of the whole input and the token-by-token decode steps agree."""
    d = os.path.join(HF, "qwen_tiny_sharded")
    ids, _ = H.expected(d)
    w = H.load(d, bits, 32)
    a, b = DO.OracleDecoder(w, 16), DO.OracleDecoder(w, 16)
    pa = a.prefill(ids)
    for t in ids:
        pb = b.step(t)
    assert float(np.abs(pa - pb).max()) <= 1e-4 * float(np.abs(pb).max())


@pytest.mark.parametrize("bits", [4, 8])
def test_vectorised_dequantize_column_equals_value(bits):
    cfg = DO.DecoderConfig(vocab=51, dim=96, layers=1, heads=2, kv_heads=1, hidden=64, bits=bits, group_size=32,
                           tied=True)
    w = DO.DecoderWeights.random(cfg, 3)
    for c in (0, 7, 25, 26, 50):
        ref = np.array([w.head.value(k, c) for k in range(cfg.dim)], np.float32)
        assert np.array_equal(ref.view(np.uint32), DO.dequantize_column(w.head, c).view(np.uint32))
