"""Greedy decode on the device against the pinned oracle, on the reference's
own checkpoints and on BASELINE's named model shapes.

1. The three tiny Hugging Face checkpoints of the reference's suite
   (tests/golden/hf/), imported as HuggingFaceModelLoader.load(dir,
   Quantization(bits, 32)) does (oracle/hf_oracle.py).  The oracle's float32
   restatement of the same decode step meets the reference's own 2e-4 bound on
   Hugging Face's logits for them (tests/test_hf_golden_cpu.py); here the
   device decoder must track the oracle on the quantized import, step by step
   and through a prefill.
2. BASELINE config 3 (the INT8 ~163M Llama-style decoder, 128-token prompt +
   256 greedy steps), config 4 (Qwen2-0.5B-shaped INT4, 512-token prompt + 16
   steps, batch 1) and config 5 (Llama-3-8B-shaped INT4, short prompt + 4
   steps): random N(0, 0.02^2) weights quantized on the device (bit-exact with
   the reference quantizer, checked elsewhere) and downloaded for the oracle.

Per step: the logits within the tolerance of the kernels that ran (1e-3 of
max|logit| on the fp32-accumulate paths, 2e-2 once a bf16 tensor-core prefill
filled the cache), and the device's greedy token equal to the oracle's
argmaxOfLastToken (Transformer.kt:255-266) unless the oracle's best and the
chosen logit lie within twice the measured error of that step (a tie at this
precision).  Both sides consume the device's tokens, so a tie cannot derail the
comparison.
"""
import os
from types import SimpleNamespace

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HF = os.path.join(ROOT, "tests", "golden", "hf")
TOL_FP32 = 1e-3
TOL_BF16 = 2e-2


def _device_cfg(cfg_o):
    from kotensor_b200 import decoder as D
    return D.DecoderConfig(vocab=cfg_o.vocab, dim=cfg_o.dim, layers=cfg_o.layers, heads=cfg_o.heads,
                           kv_heads=cfg_o.kv_heads, hidden=cfg_o.hidden, eps=cfg_o.eps, rope_theta=cfg_o.rope_theta,
                           rope_scaling=cfg_o.rope_scaling, bits=cfg_o.bits, group_size=cfg_o.group_size,
                           tied=cfg_o.tied, qkv_bias=cfg_o.qkv_bias)


class StepChecker:
    """Compares one step's logits and greedy token with the oracle's."""

    def __init__(self):
        self.ties = 0
        self.steps = 0
        self.worst = 0.0

    def __call__(self, logits, ref_logits, chosen, tol, where=""):
        from oracle import decoder_oracle as DO
        scale = float(np.abs(ref_logits).max())
        err = float(np.abs(logits.astype(np.float64) - ref_logits).max())
        self.worst = max(self.worst, err / scale)
        assert err <= tol * scale, f"{where}: error {err / scale:.3g} of max|logit|"
        best = DO.argmax(ref_logits)
        if chosen != best:
            gap = float(ref_logits[best]) - float(ref_logits[chosen])
            assert gap <= 2 * err, f"{where}: token {chosen}, oracle {best} (gap {gap:.3g}, error {err:.3g})"
            self.ties += 1
        self.steps += 1


@pytest.mark.parametrize("name", ["llama_tiny", "llama3_tiny", "qwen_tiny_sharded"])
@pytest.mark.parametrize("bits", [4, 8])
def test_reference_checkpoints_decode_like_the_oracle(kt, oracle, name, bits):
    from oracle import decoder_oracle as DO
    from oracle import hf_oracle as H
    from kotensor_b200 import decoder as D
    d = os.path.join(HF, name)
    ids, _ = H.expected(d)
    weights = H.load(d, bits, 32)
    cfg = _device_cfg(weights.cfg)
    check = StepChecker()
    # token by token (m = 1 kernels), then greedy continuation
    ref = DO.OracleDecoder(weights, max_seq=32)
    dev = D.DeviceDecoder(cfg, weights, max_seq=32)
    for t in ids:
        check(dev.step(t).cpu().numpy(), ref.step(t), int(dev.next_token.item()), TOL_FP32, f"{name} prompt")
    for _ in range(8):
        tok = int(dev.next_token.item())
        check(dev.step(tok).cpu().numpy(), ref.step(tok), int(dev.next_token.item()), TOL_FP32, f"{name} decode")
    # the 7 ids as one prefill block (m = 7: the m <= 8 kernels), then steps from that cache
    ref2 = DO.OracleDecoder(weights, max_seq=32)
    dev2 = D.DeviceDecoder(cfg, weights, max_seq=32)
    check(dev2.prefill(ids).cpu().numpy(), ref2.prefill(ids), int(dev2.next_token.item()), TOL_FP32, "prefill")
    for _ in range(4):
        tok = int(dev2.next_token.item())
        check(dev2.step(tok).cpu().numpy(), ref2.step(tok), int(dev2.next_token.item()), TOL_FP32, "after prefill")
    assert int(dev.status.item()) == 0 and int(dev2.status.item()) == 0
    assert kt.Context.get().take_error() == 0


# BASELINE.json configs 3, 4, 5 (the shapes bench.py times)
LLAMA_163M_INT8 = dict(vocab=32000, dim=768, layers=12, heads=12, kv_heads=12, hidden=2048, eps=1e-6,
                       rope_theta=10000.0, bits=8, group_size=64, tied=False, qkv_bias=False)
QWEN2_05B_INT4 = dict(vocab=151936, dim=896, layers=24, heads=14, kv_heads=2, hidden=4864, eps=1e-6,
                      rope_theta=1000000.0, bits=4, group_size=64, tied=True, qkv_bias=True)
LLAMA3_8B_INT4 = dict(vocab=128256, dim=4096, layers=32, heads=32, kv_heads=8, hidden=14336, eps=1e-5,
                      rope_theta=500000.0, rope_scaling=(8.0, 1.0, 4.0, 8192), bits=4, group_size=64, tied=False,
                      qkv_bias=False)


def _random_model(kt, spec, seed):
    """Device weights (quantized on the GPU) and the same bytes on the host for the oracle."""
    from oracle import decoder_oracle as DO
    from oracle import oracle as O
    cfg_o = DO.DecoderConfig(**spec)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    rng = np.random.default_rng(seed)
    q = kt.Quantization(cfg_o.bits, cfg_o.group_size)

    def proj(k, n, sd=0.02):
        w = torch.randn((k, n), generator=gen, device="cuda") * sd
        qt = kt.QuantizedTensor.quantize(w, q)
        del w
        qd, s, z = qt.download()
        host = O.OracleQTensor(np.ascontiguousarray(qd).reshape(-1).view(np.uint8), s.reshape(-1),
                               None if z is None else z.reshape(-1), k, n, cfg_o.bits, cfg_o.group_size)
        return qt, host

    def vec(n, mean=0.0, sd=0.0):
        return (np.float32(mean) + rng.standard_normal(n).astype(np.float32) * np.float32(sd)).astype(np.float32)

    kv = cfg_o.kv_heads * cfg_o.head_dim
    dev_layers, host_layers = [], []
    for _ in range(cfg_o.layers):
        dl, hl = {}, {}
        for key, (k, n) in {"wq": (cfg_o.dim, cfg_o.dim), "wk": (cfg_o.dim, kv), "wv": (cfg_o.dim, kv),
                            "wo": (cfg_o.dim, cfg_o.dim), "wg": (cfg_o.dim, cfg_o.hidden),
                            "wu": (cfg_o.dim, cfg_o.hidden), "wd": (cfg_o.hidden, cfg_o.dim)}.items():
            dl[key], hl[key] = proj(k, n)
        sd = 0.02 if cfg_o.qkv_bias else 0.0
        for key, n in (("bq", cfg_o.dim), ("bk", kv), ("bv", kv)):
            dl[key] = hl[key] = vec(n, 0.0, sd)
        for key, n in (("bo", cfg_o.dim), ("bg", cfg_o.hidden), ("bu", cfg_o.hidden), ("bd", cfg_o.dim)):
            dl[key] = hl[key] = vec(n)
        dl["norm1"] = hl["norm1"] = vec(cfg_o.dim, 1.0, 0.1)
        dl["norm2"] = hl["norm2"] = vec(cfg_o.dim, 1.0, 0.1)
        dev_layers.append(dl)
        host_layers.append(hl)
    head_d, head_h = proj(cfg_o.dim, cfg_o.vocab)
    emb_d, emb_h = (None, None) if cfg_o.tied else proj(cfg_o.vocab, cfg_o.dim, 0.5)
    final = vec(cfg_o.dim, 1.0, 0.1)
    bias = np.zeros(cfg_o.vocab, np.float32)
    dev_w = SimpleNamespace(embedding=emb_d, layers=dev_layers, final_norm=final, head=head_d, head_bias=bias)
    host_w = DO.DecoderWeights(cfg_o, emb_h, host_layers, final, head_h, bias)
    return cfg_o, dev_w, host_w


def _run(kt, spec, seed, prompt_len, steps, prefill, max_seq):
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    DO.THREADS = max(8, os.cpu_count() or 8)
    cfg_o, dev_w, host_w = _random_model(kt, spec, seed)
    dev = D.DeviceDecoder(_device_cfg(cfg_o), dev_w, max_seq=max_seq)
    del dev_w
    ref = DO.OracleDecoder(host_w, max_seq=max_seq)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg_o.vocab, size=prompt_len).tolist()
    check = StepChecker()
    if prefill:
        tol = TOL_BF16 if prompt_len > 8 else TOL_FP32  # m > 8: the bf16 tensor-core GEMM
        check(dev.prefill(prompt).cpu().numpy(), ref.prefill(prompt), int(dev.next_token.item()), tol, "prefill")
    else:
        tol = TOL_FP32
        for i, t in enumerate(prompt):
            check(dev.step(t).cpu().numpy(), ref.step(t), int(dev.next_token.item()), tol, f"prompt {i}")
    generated = []
    for i in range(steps):
        tok = int(dev.next_token.item())
        generated.append(tok)
        check(dev.step(tok).cpu().numpy(), ref.step(tok), int(dev.next_token.item()), tol, f"step {i}")
    assert int(dev.status.item()) == 0
    assert kt.Context.get().take_error() == 0
    print(f"{check.steps} steps, worst error {check.worst:.3g} of max|logit|, {check.ties} ties")
    return check, generated


def test_config3_int8_163m_full_run_matches_the_oracle(kt, oracle):
    """BASELINE config 3 in full: the 128-token prompt decoded token by token
    (every matmul at m = 1), then 256 greedy steps; every one of the 384 steps
    checked."""
    check, generated = _run(kt, LLAMA_163M_INT8, seed=3, prompt_len=128, steps=256, prefill=False, max_seq=400)
    assert check.steps == 384 and len(generated) == 256


def test_config3_int8_163m_prefill_then_steps(kt, oracle):
    """The same model with the 128-token prompt as one prefill block (bf16
    tensor-core GEMM), then 32 greedy steps."""
    _run(kt, LLAMA_163M_INT8, seed=3, prompt_len=128, steps=32, prefill=True, max_seq=200)


def test_config4_qwen2_05b_prefill_512_then_steps(kt, oracle):
    """BASELINE config 4 at batch 1: the 512-token prompt prefilled, then 16 greedy steps."""
    _run(kt, QWEN2_05B_INT4, seed=4, prompt_len=512, steps=16, prefill=True, max_seq=544)


def test_config5_llama3_8b_short_prompt_then_steps(kt, oracle):
    """BASELINE config 5 on one GPU: an 8-token prompt prefilled (m = 8 kernels),
    then 4 greedy steps; the oracle holds the 4.3 GB of packed weights."""
    _run(kt, LLAMA3_8B_INT4, seed=5, prompt_len=8, steps=4, prefill=True, max_seq=16)
