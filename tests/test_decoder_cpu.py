"""CPU checks of the decode-step restatement and of the product's host-side
RoPE frequencies (both follow RoPE.kt:3-42)."""
import math

import numpy as np


def test_rope_frequencies_follow_the_reference_formula(kt, oracle):
    from oracle import decoder_oracle as DO
    from kotensor_b200 import decoder as D
    for hd, base, scaling in [(64, 10000.0, None), (128, 500000.0, (8.0, 1.0, 4.0, 8192)), (64, 1e6, None)]:
        a = D.rope_inv_freq(hd, base, scaling)
        assert np.array_equal(a, DO.inv_freq(hd, base, scaling))
        assert a[0] == np.float32(1.0)
        if scaling is None:
            i = hd // 4
            assert abs(float(a[i]) - 1.0 / base ** (2 * i / hd)) <= 1e-6 * float(a[i])
        else:  # the lowest frequencies are divided by the factor
            assert a[-1] < np.float32(1.0) / np.float32(math.pow(base, (hd - 2) / hd)) / np.float32(7.9)


def test_oracle_decode_is_causal_and_deterministic(kt, oracle):
    """A step's logits depend only on the tokens so far (the KV cache), and two
    runs agree exactly."""
    from oracle import decoder_oracle as DO
    cfg = DO.DecoderConfig(vocab=300, dim=64, layers=2, heads=2, kv_heads=1, hidden=128, bits=4, group_size=32,
                           qkv_bias=True)
    w = DO.DecoderWeights.random(cfg, seed=9)
    a, b = DO.OracleDecoder(w, 16), DO.OracleDecoder(w, 16)
    la = [a.step(t) for t in (1, 2, 3)]
    lb = [b.step(t) for t in (1, 2, 4)]
    assert np.array_equal(la[0], lb[0]) and np.array_equal(la[1], lb[1])
    assert not np.array_equal(la[2], lb[2])
    c = DO.OracleDecoder(w, 16)
    assert np.array_equal([c.step(t) for t in (1, 2, 3)][2], la[2])
    assert DO.argmax(np.array([-2e9, 5.0, 5.0, 1.0], np.float32)) == 1
    assert DO.argmax(np.array([-2e9, -3e9], np.float32)) == 0
