"""kt_qmatmul_chain: consecutive one-token products in one persistent launch.

Each step is MatMul.multiplyQuantized at m = 1 (with QuantizedLinear's bias,
an optional RMSNorm of the input and an optional SwiGLU epilogue), fed either
a tensor or an earlier step's output.  The chain must give what the same
steps give as separate calls (kt_qmatmul, kt_rmsnorm_qmatmul_swiglu) -- the
same integer tensor-core arithmetic, so within 1e-6 of max|y| -- and stay
within the fp32 tolerance of the oracle; replays of a captured CUDA graph of a
chain must give the eager results (the step counters are back at zero after
every launch).
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-3
TOL_SAME = 1e-6


def rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def quantized(kt, oracle, rng, k, n, bits):
    w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
    ref = oracle.quantize(w, bits, 64)
    return kt.QuantizedTensor.from_arrays(ref.qdata, ref.scales, ref.zeros, (k, n), bits, 64), ref


def test_chain_of_ffn_pairs_equals_separate_calls_and_the_oracle(kt, oracle):
    """The bench step: up (2048 x 5632) -> down (5632 x 2048), up (4096 x 14336)
    -> down (14336 x 4096), INT4 g64, one launch."""
    rng = np.random.default_rng(11)
    shapes = [(2048, 5632), (5632, 2048), (4096, 14336), (14336, 4096)]
    ws = [quantized(kt, oracle, rng, k, n, 4) for k, n in shapes]
    x0 = torch.randn(2048, device="cuda")
    x2 = torch.randn(4096, device="cuda")
    ys = [torch.full((n,), float("nan"), device="cuda") for _, n in shapes]
    steps = [dict(weight=ws[0][0], a=x0, c=ys[0]), dict(weight=ws[1][0], input=0, c=ys[1]),
             dict(weight=ws[2][0], a=x2, c=ys[2]), dict(weight=ws[3][0], input=2, c=ys[3])]
    kt.MatMul.multiply_chain(steps)
    # the same products one call at a time
    want = [torch.empty((n,), device="cuda") for _, n in shapes]
    kt.MatMul.multiply_quantized(x0, ws[0][0], want[0], 1, accumulate=False)
    kt.MatMul.multiply_quantized(want[0], ws[1][0], want[1], 1, accumulate=False)
    kt.MatMul.multiply_quantized(x2, ws[2][0], want[2], 1, accumulate=False)
    kt.MatMul.multiply_quantized(want[2], ws[3][0], want[3], 1, accumulate=False)
    torch.cuda.synchronize()
    for i in range(4):
        assert rel(ys[i], want[i]) <= TOL_SAME, i
    # the first pair against the oracle, the down product fed the chain's own up output
    up = oracle.multiply_quantized(x0.cpu().numpy()[None, :], ws[0][1], threads=8)
    assert rel(ys[0], torch.from_numpy(up[0])) <= TOL_FP32
    down = oracle.multiply_quantized(ys[0].cpu().numpy()[None, :], ws[1][1], threads=8)
    assert rel(ys[1], torch.from_numpy(down[0])) <= TOL_FP32
    assert kt.Context.get().take_error() == 0


def test_chain_int8_with_bias_alpha_and_accumulate(kt, oracle):
    rng = np.random.default_rng(12)
    (w0, r0), (w1, r1) = quantized(kt, oracle, rng, 2048, 2048, 8), quantized(kt, oracle, rng, 2048, 2048, 8)
    x = torch.randn(2048, device="cuda")
    bias = torch.randn(2048, device="cuda") * 0.1
    y0 = torch.empty(2048, device="cuda")
    y1 = torch.randn(2048, device="cuda")
    c1 = y1.clone()
    kt.MatMul.multiply_chain([dict(weight=w0, a=x, c=y0, bias=bias),
                              dict(weight=w1, input=0, c=y1, accumulate=True, alpha=0.5)])
    want0 = torch.empty(2048, device="cuda")
    kt.MatMul.multiply_quantized(x, w0, want0, 1, accumulate=False, bias=bias)
    want1 = c1.clone()
    kt.MatMul.multiply_quantized(want0, w1, want1, 1, accumulate=True, alpha=0.5)
    torch.cuda.synchronize()
    assert rel(y0, want0) <= TOL_SAME and rel(y1, want1) <= TOL_SAME
    ref0 = oracle.multiply_quantized(x.cpu().numpy()[None, :], r0, threads=8)[0] + bias.cpu().numpy()
    assert rel(y0, torch.from_numpy(ref0)) <= TOL_FP32
    assert kt.Context.get().take_error() == 0


def test_chain_of_a_swiglu_ffn_into_the_residual(kt, oracle):
    """TransformerBlock.decodeInto's second half (TransformerBlock.kt:44-46) as one
    chain: h = silu(g) * u with [g | u] = RMSNorm(x) . W_gu (norm and SwiGLU in
    the first step), then x += h . W_down -- the second step writes the row the
    first one read."""
    from kotensor_b200 import _lib
    rng = np.random.default_rng(13)
    d, hid = 896, 4864
    wgu, _ = quantized(kt, oracle, rng, d, 2 * hid, 4)
    wd, _ = quantized(kt, oracle, rng, hid, d, 4)
    nw = torch.from_numpy((1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)).cuda()
    x0 = torch.randn(d, device="cuda") * 3
    x = x0.clone()
    h = torch.empty(hid, device="cuda")
    kt.MatMul.multiply_chain([dict(weight=wgu, a=x, c=h, norm_weight=nw, norm_eps=1e-6, swiglu=True),
                              dict(weight=wd, input=0, c=x, accumulate=True)])
    lib = kt.load_library()
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    hh = kt.Context.get().handle
    want_h = torch.empty(hid, device="cuda")
    want_x = x0.clone()
    _lib.check(lib.kt_rmsnorm_qmatmul_swiglu(hh, wgu.handle, p(want_x), p(nw), 1e-6, None, None, p(want_h), 1,
                                             None, s))
    _lib.check(lib.kt_qmatmul(hh, wd.handle, p(want_h), p(want_x), 1, 1, 1.0, None, s))
    torch.cuda.synchronize()
    assert rel(h, want_h) <= TOL_SAME
    assert rel(x, want_x) <= TOL_SAME
    assert kt.Context.get().take_error() == 0


def test_chain_replays_in_a_cuda_graph(kt, oracle):
    """Captured once, replayed with new inputs: every replay equals an eager chain."""
    rng = np.random.default_rng(14)
    (w0, _), (w1, _) = quantized(kt, oracle, rng, 4096, 14336, 4), quantized(kt, oracle, rng, 14336, 4096, 4)
    x = torch.empty(4096, device="cuda")
    y0 = torch.empty(14336, device="cuda")
    y1 = torch.empty(4096, device="cuda")
    steps = [dict(weight=w0, a=x, c=y0), dict(weight=w1, input=0, c=y1)]
    x.copy_(torch.randn(4096, device="cuda"))
    kt.MatMul.multiply_chain(steps)  # warm-up: workspace and kernel attributes before the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=st):
        kt.MatMul.multiply_chain(steps)
    for i in range(3):
        x.copy_(torch.randn(4096, device="cuda"))
        g.replay()
        torch.cuda.synchronize()
        got0, got1 = y0.clone(), y1.clone()
        kt.MatMul.multiply_chain(steps)
        torch.cuda.synchronize()
        assert torch.equal(got0, y0) and torch.equal(got1, y1), i
    del g
    assert kt.Context.get().take_error() == 0


def test_chain_rejects_what_it_cannot_run(kt, oracle):
    from kotensor_b200 import _lib
    rng = np.random.default_rng(15)
    w, _ = quantized(kt, oracle, rng, 1024, 2048, 4)
    x = torch.randn(1024, device="cuda")
    y = torch.empty(2048, device="cuda")
    with pytest.raises(ValueError):  # a step may only read an earlier one
        kt.MatMul.multiply_chain([dict(weight=w, input=0, c=y)])
    with pytest.raises(ValueError):  # widths must chain
        kt.MatMul.multiply_chain([dict(weight=w, a=x, c=y), dict(weight=w, input=0, c=x)])
    wide, _ = quantized(kt, oracle, rng, 256, 256 * 200, 4)  # 200 column tiles of 256: fits
    big, _ = quantized(kt, oracle, rng, 256, 256 * 600, 4)   # 600 tiles: more than the GPU holds at once
    yb = torch.empty(256 * 600, device="cuda")
    with pytest.raises(_lib.KtError) as e:
        kt.MatMul.multiply_chain([dict(weight=big, a=torch.randn(256, device="cuda"), c=yb)])
    assert e.value.status == _lib.KT_ERR_UNSUPPORTED
    yw = torch.empty(256 * 200, device="cuda")
    kt.MatMul.multiply_chain([dict(weight=wide, a=torch.randn(256, device="cuda"), c=yw)])
    torch.cuda.synchronize()
    assert kt.Context.get().take_error() == 0
