"""The device decode step (kotensor_b200/decoder.py) against the CPU
restatement of Transformer.decode (oracle/decoder_oracle.py) on small random
models: logits of every step within the fp32 tolerance, and each greedy token
the oracle's best up to that tolerance (teacher-forced with the device's own
choices, so a near tie cannot derail the comparison)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL = 1e-3

CONFIGS = {
    "int4_gqa_bias_scaled_rope": dict(vocab=1000, dim=256, layers=2, heads=4, kv_heads=2, hidden=512,
                                      rope_theta=500000.0, rope_scaling=(8.0, 1.0, 4.0, 8192), bits=4,
                                      group_size=64, tied=False, qkv_bias=True),
    "int8_tied_mha": dict(vocab=768, dim=192, layers=2, heads=3, kv_heads=3, hidden=384, rope_theta=10000.0,
                          bits=8, group_size=64, tied=True, qkv_bias=False),
    "int4_tied_qwen_like": dict(vocab=2048, dim=128, layers=3, heads=2, kv_heads=1, hidden=256,
                                rope_theta=1000000.0, bits=4, group_size=32, tied=True, qkv_bias=True),
}


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_decode_steps_match_the_oracle(kt, oracle, name):
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    cfg_o = DO.DecoderConfig(**CONFIGS[name])
    cfg_d = D.DecoderConfig(**CONFIGS[name])
    assert np.array_equal(D.rope_inv_freq(cfg_d.head_dim, cfg_d.rope_theta, cfg_d.rope_scaling),
                          DO.inv_freq(cfg_o.head_dim, cfg_o.rope_theta, cfg_o.rope_scaling))
    weights = DO.DecoderWeights.random(cfg_o, seed=len(name))
    ref = DO.OracleDecoder(weights, max_seq=40)
    dev = D.DeviceDecoder(cfg_d, weights, max_seq=40)
    token = 3
    for step in range(24):
        logits = dev.step(token).cpu().numpy()
        ref_logits = ref.step(token)
        scale = np.abs(ref_logits).max()
        assert np.abs(logits - ref_logits).max() <= TOL * scale, (step, np.abs(logits - ref_logits).max() / scale)
        chosen = int(dev.next_token.item())
        assert chosen == int(np.argmax(logits)) or logits[chosen] == logits.max()
        assert ref_logits[chosen] >= ref_logits.max() - TOL * scale
        token = chosen
    assert int(dev.status.item()) == 0
    assert kt.Context.get().take_error() == 0


def test_captured_step_replays_like_eager_steps(kt, oracle):
    """The CUDA-graph replay of one step gives the same tokens and logits as
    the eager steps (identical kernels, identical order)."""
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    params = CONFIGS["int4_gqa_bias_scaled_rope"]
    weights = DO.DecoderWeights.random(DO.DecoderConfig(**params), seed=5)
    a = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=64)
    b = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=64)
    prompt = [5, 17, 99, 4]
    out_graph = a.generate(prompt, 20)
    for t in prompt:
        b.step(t)
    out_eager = [int(b.next_token.item())]
    for _ in range(19):
        b.step(out_eager[-1])
        out_eager.append(int(b.next_token.item()))
    assert out_graph == out_eager
    assert torch.equal(a.logits, b.logits)
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("name", sorted(CONFIGS))
@pytest.mark.parametrize("prompt_len", [5, 37])
def test_prefill_matches_stepwise_oracle(kt, oracle, name, prompt_len):
    """Transformer.prefill on the device (the prompt as one block, matmuls at
    m = prompt length on the tensor-core GEMM when m >= 9, bf16 tolerance)
    against the oracle fed the prompt token by token; then decode steps from
    the prefilled cache stay within the fp32 step tolerance of the oracle's."""
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    cfg_o, cfg_d = DO.DecoderConfig(**CONFIGS[name]), D.DecoderConfig(**CONFIGS[name])
    weights = DO.DecoderWeights.random(cfg_o, seed=100 + prompt_len)
    ref = DO.OracleDecoder(weights, max_seq=64)
    dev = D.DeviceDecoder(cfg_d, weights, max_seq=64)
    rng = np.random.default_rng(prompt_len)
    prompt = rng.integers(0, cfg_o.vocab, size=prompt_len).tolist()
    for t in prompt:
        ref_logits = ref.step(t)
    logits = dev.prefill(prompt).cpu().numpy()
    tol = 2e-2 if prompt_len >= 9 else TOL
    scale = np.abs(ref_logits).max()
    assert np.abs(logits - ref_logits).max() <= tol * scale
    token = int(dev.next_token.item())
    for _ in range(4):
        logits = dev.step(token).cpu().numpy()
        ref_logits = ref.step(token)
        scale = np.abs(ref_logits).max()
        assert np.abs(logits - ref_logits).max() <= tol * scale
        token = int(dev.next_token.item())
    assert int(dev.status.item()) == 0
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("batch", [3, 12])
def test_batched_decode_matches_single_sequences(kt, oracle, batch):
    """`batch` sequences decoding together (one KV cache each, every matmul at
    m = batch, the prompts prefilled as one block of batch x T rows) give each
    sequence the logits its own batch-1 decoder gives (teacher-forced with the
    batched greedy tokens); bf16 tensor-core tolerance wherever a matmul of
    either side takes the tcgen05 GEMM."""
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    params = CONFIGS["int4_gqa_bias_scaled_rope"]
    weights = DO.DecoderWeights.random(DO.DecoderConfig(**params), seed=11)
    rng = np.random.default_rng(batch)
    T = 6
    prompts = [rng.integers(0, params["vocab"], T).tolist() for _ in range(batch)]
    dec = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=32, batch=batch)
    singles = [D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=32) for _ in range(batch)]
    tol = 3e-2
    got = dec.prefill(prompts).cpu().numpy()
    for q, single in enumerate(singles):
        want = single.prefill(prompts[q]).cpu().numpy()
        assert np.abs(got[q] - want).max() <= tol * np.abs(want).max(), q
    for _ in range(4):
        tokens = dec.next_token.cpu().tolist()
        got = dec.step(tokens).cpu().numpy()
        for q, single in enumerate(singles):
            want = single.step(tokens[q]).cpu().numpy()
            assert np.abs(got[q] - want).max() <= tol * np.abs(want).max(), q
    assert int(dec.status.item()) == 0
    assert kt.Context.get().take_error() == 0


def test_prefill_in_several_blocks_matches_one_block(kt, oracle):
    """A batch whose prompt rows exceed one prefill block is prefilled in blocks
    of whole sequences (here the block limit is lowered to 2 sequences of 7 rows
    so a batch of 5 takes 3 blocks); every sequence gets the logits, cache and
    next steps of the one-block prefill (bf16 tolerance: the blocks' matmuls run
    at other m)."""
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    params = CONFIGS["int4_gqa_bias_scaled_rope"]
    weights = DO.DecoderWeights.random(DO.DecoderConfig(**params), seed=23)
    rng = np.random.default_rng(23)
    batch, T = 5, 7
    prompts = [rng.integers(0, params["vocab"], T).tolist() for _ in range(batch)]
    whole = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=24, batch=batch)
    split = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=24, batch=batch)
    split.max_block_rows = 2 * T + 3
    tol = 3e-2
    want = whole.prefill(prompts).cpu().numpy()
    got = split.prefill(prompts).cpu().numpy()
    assert np.abs(got - want).max() <= tol * np.abs(want).max()
    for _ in range(3):
        tokens = whole.next_token.cpu().tolist()
        want = whole.step(tokens).cpu().numpy()
        got = split.step(tokens).cpu().numpy()
        assert np.abs(got - want).max() <= tol * np.abs(want).max()
    tiny = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=24)
    tiny.max_block_rows = T - 1  # one prompt longer than a block
    with pytest.raises(ValueError):
        tiny.prefill(prompts[0])
    assert int(split.status.item()) == 0
    assert kt.Context.get().take_error() == 0


def test_batched_graph_replay_matches_eager_steps(kt, oracle):
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    params = CONFIGS["int8_tied_mha"]
    weights = DO.DecoderWeights.random(DO.DecoderConfig(**params), seed=4)
    prompts = [[5, 17, 99, 4], [1, 2, 3, 4], [700, 8, 9, 10], [42, 42, 42, 42]]
    a = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=40, batch=4)
    b = D.DeviceDecoder(D.DecoderConfig(**params), weights, max_seq=40, batch=4)
    out_graph = a.generate_batch(prompts, 10)
    b.prefill(prompts)
    out_eager = [[t] for t in b.next_token.cpu().tolist()]
    for _ in range(9):
        b.step(b.next_token.cpu().tolist())
        for q, t in enumerate(b.next_token.cpu().tolist()):
            out_eager[q].append(t)
    assert out_graph == out_eager
    assert torch.equal(a.logits, b.logits)
    assert kt.Context.get().take_error() == 0


@pytest.mark.parametrize("heads,kv_heads,head_dim", [(12, 12, 64), (14, 2, 64), (32, 8, 128), (8, 1, 64), (7, 7, 128)])
@pytest.mark.parametrize("position", [0, 63, 64, 200])
def test_fused_decode_attention_matches_the_separate_kernels(kt, heads, kv_heads, head_dim, position):
    """kt_attention_rope_decode (RoPE, cache store, attention and merge in one
    launch) against kt_rope_kv_seqs + kt_attention_seqs on the same rows: the
    same cache entries and the same context within float32 rounding, on three
    sequences with caches cache_stride apart; twice in a row (the merge
    counters are left at zero)."""
    import ctypes
    from kotensor_b200 import _lib
    from kotensor_b200 import decoder as D
    lib = kt.load_library()
    h = kt.Context.get().handle
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rows, layers, max_seq, layer = 3, 2, 256, 1
    q_width, kv = heads * head_dim, kv_heads * head_dim
    gen = torch.Generator(device="cuda")
    gen.manual_seed(heads * 1000 + position)
    qkv = torch.randn((rows, q_width + 2 * kv), generator=gen, device="cuda")
    cache = torch.randn((2, rows, layers, kv_heads, max_seq, head_dim), generator=gen, device="cuda")
    stride = layers * kv_heads * max_seq * head_dim
    inv = torch.as_tensor(D.rope_inv_freq(head_dim, 500000.0, (8.0, 1.0, 4.0, 8192))).cuda()
    pos = torch.tensor([position], dtype=torch.int32, device="cuda")
    scale = float(1.0 / np.sqrt(head_dim))
    nsc = lib.kt_attention_scratch_floats(rows, heads, head_dim, max_seq)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    # the separate kernels
    ref_cache = cache.clone()
    ref_qkv = qkv.clone()
    ref_ctx = torch.empty((rows, q_width), device="cuda")
    sc = torch.zeros(nsc, device="cuda")
    _lib.check(lib.kt_rope_kv_seqs(h, p(ref_qkv), rows, q_width, kv_heads, head_dim, p(inv), p(ref_cache[0]),
                                   p(ref_cache[1]), max_seq, layer, p(pos), 1, stride, s))
    _lib.check(lib.kt_attention_seqs(h, p(ref_qkv), p(ref_cache[0]), p(ref_cache[1]), p(ref_ctx), p(sc), rows,
                                     q_width + 2 * kv, heads, kv_heads, head_dim, max_seq, layer, scale, p(pos), 1,
                                     stride, s))
    fused_sc = torch.zeros(nsc, device="cuda")
    for _ in range(2):
        got_cache = cache.clone()
        got_ctx = torch.full((rows, q_width), float("nan"), device="cuda")
        _lib.check(lib.kt_attention_rope_decode(h, p(qkv), rows, q_width, heads, kv_heads, head_dim, p(inv),
                                                p(got_cache[0]), p(got_cache[1]), p(got_ctx), p(fused_sc), max_seq,
                                                layer, scale, p(pos), stride, s))
        torch.cuda.synchronize()
        assert torch.allclose(got_cache, ref_cache, rtol=1e-6, atol=1e-6)
        err = (got_ctx - ref_ctx).abs().max().item() / ref_ctx.abs().max().item()
        assert err <= 1e-5, err
        ntick = rows * heads
        assert not torch.any(fused_sc[nsc - ntick:].view(torch.int32)).item()  # counters back at zero
    assert kt.Context.get().take_error() == 0


def test_fused_decode_attention_rejects_other_head_dims(kt):
    """The fused kernel is built for head_dim 64 and 128; other shapes are
    refused (the decoder then runs the separate kernels)."""
    import ctypes
    from kotensor_b200 import _lib
    lib = kt.load_library()
    t = torch.zeros(4096, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = ctypes.c_void_p(t.data_ptr())
    st = lib.kt_attention_rope_decode(kt.Context.get().handle, p, 1, 32, 4, 1, 8, p, p, p, p, p, 16, 0, 0.1,
                                      ctypes.c_void_p(pos.data_ptr()), 0, None)
    assert st == _lib.KT_ERR_UNSUPPORTED


def _causal_attention_ref(q, kc, vc, heads, kv_heads, head_dim, rows_per_seq, p0, scale):
    """Attention.prefillInto / attendHead (Attention.kt:241-293, :295-328) in
    float64: row r of sequence r // rows_per_seq at position p0 + r % rows_per_seq
    attends to positions 0 .. its own of its sequence's cache (layer 0)."""
    rows = q.shape[0]
    g = heads // kv_heads
    out = np.zeros((rows, heads * head_dim))
    for r in range(rows):
        seq, pos = r // rows_per_seq, p0 + r % rows_per_seq
        for h in range(heads):
            kv = h // g
            qv = q[r, h * head_dim:(h + 1) * head_dim].astype(np.float64)
            k = kc[seq, 0, kv, :pos + 1].astype(np.float64)
            v = vc[seq, 0, kv, :pos + 1].astype(np.float64)
            s = k @ qv * scale
            e = np.exp(s - s.max())
            out[r, h * head_dim:(h + 1) * head_dim] = (e / e.sum()) @ v
    return out


@pytest.mark.parametrize("heads,kv_heads,head_dim", [(32, 8, 128), (14, 2, 64), (12, 12, 64), (8, 1, 128)])
@pytest.mark.parametrize("seqs,rows_per_seq,p0", [(1, 200, 0), (2, 37, 0), (1, 70, 50), (3, 5, 3), (1, 9, 120),
                                                 (2, 160, 96)])
def test_prefill_attention_matches_float64(kt, heads, kv_heads, head_dim, seqs, rows_per_seq, p0):
    """kt_attention_seqs on prompt blocks (rows_per_seq > 1) against a float64
    restatement of causal attention: blocks of 9 rows or more run the flash
    kernel on TF32 tensor cores (within 5e-3 of max|context|, inside the bf16
    prefill tolerance), smaller ones the fp32 kernel and merge (1e-5); group
    sizes 1, 4, 7, 8, head_dim 64 and 128, several sequences, partial query
    tiles, a block starting after earlier positions (p0 > 0) and spans of 64
    positions crossed."""
    import ctypes
    from kotensor_b200 import _lib
    lib = kt.load_library()
    h = kt.Context.get().handle
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rows, max_seq = seqs * rows_per_seq, 256
    q_width, kv = heads * head_dim, kv_heads * head_dim
    gen = torch.Generator(device="cuda")
    gen.manual_seed(heads + 7 * rows + p0)
    qkv = torch.randn((rows, q_width + 2 * kv), generator=gen, device="cuda")
    cache = torch.randn((2, seqs, 1, kv_heads, max_seq, head_dim), generator=gen, device="cuda")
    stride = kv_heads * max_seq * head_dim
    pos = torch.tensor([p0], dtype=torch.int32, device="cuda")
    scale = float(1.0 / np.sqrt(head_dim))
    sc = torch.zeros(lib.kt_attention_scratch_floats(rows, heads, head_dim, max_seq), device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    ctx = torch.full((rows, q_width), float("nan"), device="cuda")
    _lib.check(lib.kt_attention_seqs(h, p(qkv), p(cache[0]), p(cache[1]), p(ctx), p(sc), rows, q_width + 2 * kv,
                                     heads, kv_heads, head_dim, max_seq, 0, scale, p(pos), rows_per_seq, stride, s))
    torch.cuda.synchronize()
    ref = _causal_attention_ref(qkv[:, :q_width].cpu().numpy(), cache[0].cpu().numpy(), cache[1].cpu().numpy(),
                                heads, kv_heads, head_dim, rows_per_seq, p0, scale)
    got = ctx.cpu().numpy().astype(np.float64)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= (5e-3 if rows >= 9 else 1e-5), err
    assert kt.Context.get().take_error() == 0
